"""Host-side constant builders and the int32 overflow proof (no device code, no oracle).

Restates the numeric primitives of the reference quantizer, anvil/frontend/quantize.py:
    fixed_point :40-56, rsqrt_kmax :67-69, rmsnorm_lut :72-80, ss_shift_for :85-91, rms_xmax_table :99-113,
    rms_wide_bounds :116-119, rmsnorm_lut_wide :122-144, silu_lut :147-152, exp_bits :155-157, exp_lut :160-162,
    prove_no_overflow :175-253
and adds the builders of the nanoGPT extensions: gelu_lut (the silu_lut recipe with GELU), layernorm bounds in
prove_no_overflow (a mean-centred row has entries up to twice the input magnitude), the qlinear bias and embed.
tests/golden/reference_quantize.json.gz pins these against the reference's own code.
"""
from __future__ import annotations

import math

import numpy as np

from ..ir import graph as g

INT32_MAX = (1 << 31) - 1
RSQRT_LEN = 1024
SOFTMAX_ONE = 127
HEADROOM = 1.5
QMAX = {"i8": 127, "i16": (1 << 15) - 1}


def _rnd(s):
    return (1 << (s - 1)) if s else 0


def rsqrt_index(ss, n):
    """(idx, k): idx = ss; while idx >= n: idx >>= 2, k += 1 (element-wise)."""
    idx = np.array(ss, dtype=np.int64, copy=True)
    k = np.zeros_like(idx)
    while True:
        big = idx >= n
        if not big.any():
            return idx, k
        idx = np.where(big, idx >> 2, idx)
        k += big


def fixed_point(ms, bounds, k=0, *, max_shift=31):
    """(M_i, s): the largest s in [0, max_shift - k] with M_i = round(m_i 2^s) and
    sum(bound_i M_i) + 2^(s+k-1) <= INT32_MAX; ValueError if a multiplier vanishes, OverflowError if no s fits."""
    if len(ms) != len(bounds) or not ms:
        raise ValueError("fixed_point needs one bound per multiplier")
    if any(m <= 0 for m in ms) or any(b < 0 for b in bounds):
        raise ValueError(f"multipliers must be positive and bounds non-negative: {ms}, {bounds}")
    for s in range(max_shift - k, -1, -1):
        mi = [round(m * (1 << s)) for m in ms]
        if sum(int(b) * m for b, m in zip(bounds, mi)) + _rnd(s + k) <= INT32_MAX:
            if min(mi) < 1:
                raise ValueError(f"multipliers {ms} vanish at shift {s}")
            return mi, s
    raise OverflowError(f"bounds {bounds} leave no room for multipliers {ms}")


def maxabs_scale(x) -> float:
    return float(np.abs(np.asarray(x)).max()) / 127


def quantize_array(x, scale, dtype="i8"):
    q = QMAX[dtype]
    return np.clip(np.rint(np.asarray(x, dtype=np.float64) / scale), -q - 1, q).astype(np.int64)


def rsqrt_kmax(d, n=RSQRT_LEN, mag=128):
    return int(rsqrt_index(d * mag * mag, n)[1])


def rmsnorm_lut(sx, sw, sh, wmax, d, eps, n=RSQRT_LEN, mag=128):
    """(rsqrt_lut, s): lut[i] = round(rsqrt(sx^2 i / d + eps) sx sw / sh 2^s), lut[0] = 0. `mag` bounds |x| (128 for
    int8 rows; a layernorm passes its centred magnitude)."""
    ss = np.arange(1, n)
    r = np.r_[0, 1 / np.sqrt(sx ** 2 * ss / d + eps) * sx * sw / sh]
    (rmax,), s = fixed_point([r.max()], [mag * wmax], rsqrt_kmax(d, n, mag))
    lut = np.rint(r * (1 << s)).astype(np.int64)
    return lut, s


def ss_shift_for(d, mag):
    for c in range(31):
        if d * ((mag * mag + _rnd(c)) >> c) <= INT32_MAX:
            return c
    raise OverflowError(f"no square shift fits {d} entries of magnitude {mag}")


def _xmax(ss_max, c, mag):
    return min(mag, math.isqrt(max(0, (ss_max + 1) * (1 << c) - _rnd(c) - 1)))


def rms_xmax_table(d, n, c, mag, e=0):
    ss_top = d * ((mag * mag + _rnd(c)) >> c) + e
    kmax = int(rsqrt_index(ss_top, n)[1])
    out = {}
    for k in range(kmax + 1):
        hi = np.minimum((np.arange(n, dtype=object) + 1) * (4 ** k) - 1, ss_top)
        xm = np.array([_xmax(int(v) - e, c, mag) if v >= e else 0 for v in hi], dtype=np.int64)
        if k:
            xm[: n // 4] = 0
        out[k] = xm
    return out


def rms_wide_bounds(lut, wmax, M, s, xm_table):
    lut = np.asarray(lut, dtype=np.int64)
    return {k: int((xm * wmax * lut).max()) * M + _rnd(s + k) for k, xm in xm_table.items()}


def rmsnorm_lut_wide(sx, sw, sh, wmax, d, eps, mag, n=RSQRT_LEN):
    """(rsqrt_lut, s, c, e) for a wide (i16) row: eps folded into the sum as e, squares shifted by c."""
    c = ss_shift_for(d, mag)
    unit = sx ** 2 * (1 << c) / d
    e = max(1, int(round(eps / unit)))
    if d * ((mag * mag + _rnd(c)) >> c) + e > INT32_MAX:
        raise OverflowError(f"eps folds to {e}: the rmsnorm sum of squares cannot stay in int32 at scale {sx}")
    ss = np.arange(1, n)
    r = np.r_[0, 1 / np.sqrt(unit * ss) * sx * sw / sh]
    xm = rms_xmax_table(d, n, c, mag, e)
    kmax = max(xm)
    for s in range(31 - kmax, -1, -1):
        lut = np.rint(r * (1 << s)).astype(np.int64)
        if max(rms_wide_bounds(lut, wmax, 1, s, xm).values()) <= INT32_MAX:
            if lut[n // 4:].min() < 64:
                raise ValueError(f"rsqrt LUT too coarse at shift {s} (min entry {lut[n // 4:].min()})")
            return lut, s, c, e
    raise OverflowError("no rsqrt LUT shift fits a wide rmsnorm")


def silu_lut(s_in):
    x = np.arange(-128, 128) * s_in
    y = x / (1 + np.exp(-x))
    s = maxabs_scale(y)
    return quantize_array(y, s), s


def gelu(x):
    """GELU, exact erf form (torch.nn.functional.gelu's default)."""
    from math import erf
    x = np.asarray(x, dtype=np.float64)
    return 0.5 * x * (1.0 + np.vectorize(erf)(x / math.sqrt(2.0)))


def gelu_lut(s_in, s_out=None, approximate="none"):
    """(lut, scale): GELU of every int8 input at scale s_in, quantized at s_out (default: its own max-abs)."""
    x = np.arange(-128, 128) * s_in
    if approximate == "tanh":
        y = 0.5 * x * (1 + np.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))
    else:
        y = gelu(x)
    s = maxabs_scale(y) if s_out is None else s_out
    return quantize_array(y, s), s


def exp_bits(t, one=SOFTMAX_ONE):
    return max(e for e in range(31) if (one + t // 2) << e <= INT32_MAX and t << e <= INT32_MAX)


def exp_lut(score_scale, t, one=SOFTMAX_ONE):
    return np.rint(np.exp(np.arange(-255, 1) * score_scale) * (1 << exp_bits(t, one))).astype(np.int64)


# ------------------------------------------------------------------------------------------ overflow proof

def _rms_checks(name, d, n, mag_x, mag_w, lut_val, lut_mag, M, s, c, e, dtype_is_i8, bad):
    if dtype_is_i8 and c == 0 and e == 0:
        kmax = rsqrt_kmax(d, n, mag_x)
        xwr = mag_x * mag_w * lut_mag
        checks = {"sum x^2": d * mag_x ** 2, "x*w*r": xwr, "x*w*r*M + round": xwr * M + _rnd(s + kmax)}
    else:
        if lut_val is None:
            raise ValueError(f"{name}: the wide norm bound needs the rsqrt LUT's values")
        xm = rms_xmax_table(d, n, c, mag_x, e)
        kmax = max(xm)
        xwr = max(int((v * mag_w * lut_val).max()) for v in xm.values())
        checks = {"x^2 + round": mag_x ** 2 + _rnd(c), "sum x^2": d * ((mag_x ** 2 + _rnd(c)) >> c) + e,
                  "x*w": mag_x * mag_w, "x*w*r": xwr,
                  "x*w*r*M + round": max(rms_wide_bounds(lut_val, mag_w, M, s, xm).values())}
    if s + kmax > 31:
        bad.append(f"{name}: shift s + kmax = {s + kmax} > 31")
    return checks


def prove_no_overflow(module, consts=None) -> dict:
    """Propagate a magnitude bound for every value (int8 inputs 128, i16 2^15, softmax outputs `one`, LUT outputs
    max|table|) and bound every int32 intermediate of every op; {op sym: worst |intermediate|}, or OverflowError
    naming each op whose bound can exceed INT32_MAX (anvil/frontend/quantize.py:175-253, plus the extensions)."""
    consts = consts or {}
    mag, cval, worst, bad = {}, {}, {}, []
    for op in g.func_of(module).ops:
        if isinstance(op, g.OutputOp):
            continue
        r = id(op.result)
        name = op.sym_str or op.name
        checks = {}
        if isinstance(op, g.InputOp):
            m = {"i8": 128, "i16": 1 << 15}.get(g.qt(op.result).dtype, 1 << 31)
        elif isinstance(op, g.ConstOp):
            v = op.value if op.value is not None else np.asarray(consts[op.sym_str], dtype=np.int64)
            v = np.asarray(v, dtype=np.int64).reshape(g.qt(op.result).dims)
            cval[r] = v
            m = int(np.abs(v).max()) if v.size else 0
        elif isinstance(op, (g.QMatmulOp, g.QLinearOp)):
            M, s = op.M, op.s
            if id(op.b) in cval:
                acc = mag[id(op.a)] * int(np.abs(cval[id(op.b)]).sum(axis=-2).max())
            else:
                acc = g.qt(op.a).dims[-1] * mag[id(op.a)] * mag[id(op.b)]
            if op.bias is not None:
                acc += int(np.abs(cval[id(op.bias)]).max())
            checks = {"acc": acc, "acc*M + round": acc * M + _rnd(s)}
            m = mag[id(op.lut)] if op.lut is not None else (128 if g.qt(op.result).dtype == "i8" else 1 << 15)
        elif isinstance(op, g.LutOp):
            m = mag[id(op.table)]
        elif isinstance(op, g.LutMulOp):
            prod = mag[id(op.table)] * mag[id(op.y)]
            checks = {"lut*y": prod, "lut*y*M + round": prod * op.M + _rnd(op.s)}
            m = 128
        elif isinstance(op, (g.RmsNormIntOp, g.LayerNormIntOp)):
            d, n = g.qt(op.x).dims[-1], g.qt(op.lut).dims[0]
            mx = mag[id(op.x)]
            center = isinstance(op, g.LayerNormIntOp)
            if center:
                checks_c = {"row sum": d * mx}
                mx = 2 * mx                    # x - mean: both in [-mag, mag)
            i8_fast = g.qt(op.x).dtype == "i8" and not center
            checks = _rms_checks(name, d, n, mx, mag[id(op.w)], cval.get(id(op.lut)), mag[id(op.lut)], op.M, op.s,
                                 op.ss_shift_int, op.ss_init_int, i8_fast, bad)
            if center:
                checks.update(checks_c)
            m = 128
        elif isinstance(op, g.SoftmaxLutOp):
            one, emax, t = op.one, mag[id(op.lut)], g.qt(op.x).dims[-1]
            checks = {"exp sum": t * emax, "e*one + S/2": emax * one + t * emax // 2}
            m = one
        elif isinstance(op, g.AddRequantOp):
            checks = {"a*Ma + b*Mb + round": mag[id(op.a)] * op.Ma + mag[id(op.b)] * op.Mb + _rnd(op.s)}
            m = 128 if g.qt(op.result).dtype == "i8" else 1 << 15
        elif isinstance(op, g.EmbedOp):
            checks = {"a*Ma + b*Mb + round": mag[id(op.wte)] * op.Ma + mag[id(op.wpe)] * op.Mb + _rnd(op.s)}
            m = 128
        elif isinstance(op, (g.TransposeOp, g.ReshapeOp)):
            m = mag[id(op.x)]
            if id(op.x) in cval:
                x = cval[id(op.x)]
                cval[r] = (np.transpose(x, op.perm_list) if isinstance(op, g.TransposeOp)
                           else x.reshape(g.qt(op.result).dims))
        else:
            raise NotImplementedError(f"prove_no_overflow: {op.name}")
        mag[r] = m
        if checks:
            worst[name] = max(checks.values())
            bad += [f"{name}: {k} reaches {v} > {INT32_MAX}" for k, v in checks.items() if v > INT32_MAX]
    if bad:
        raise OverflowError("int32 overflow possible: " + "; ".join(bad))
    return worst
