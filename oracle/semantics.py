"""CPU oracle (test infrastructure only): numpy restatement of Anvil's checked int32 op semantics.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may import this package; the product path
(the anvil package and libanvil_cuda.so) never does.

What is restated, and from where
--------------------------------
* The golden base ops live in the third-party module `xf.golden` of the `sim/` submodule
  Ashtonantony28/Didactic_GPU_Simulator, pinned at commit 096c6ef (reference .gitmodules, docs/design.md:5-6,
  PLAN.md:42). That submodule is not vendored in the reference checkout, so its source is absent. The base ops
  below are restated from the reference's own descriptions and from its three independent in-repo restatements:
    - requant:      anvil/semantics.py:146-155 (requant_dtype, identical for i8), anvil/backend/idioms.py:150-163,
                    anvil/vortexv/codegen.py:10-13 (rqs of the exact 64-bit product)
    - rsqrt_index:  anvil/lower/graph_to_tensor.py:319-349, anvil/codegen/lower.py:791-803,
                    anvil/vortexv/codegen.py:512-519 (while idx >= n: idx >>= 2; k += 1)
    - rmsnorm_int:  anvil/semantics.py:164-182 (rmsnorm_wide with c = e = 0), anvil/lower/graph_to_tensor.py:319-349
    - softmax_lut:  anvil/lower/graph_to_tensor.py:352-398, anvil/vortexv/codegen.py:545-615
    - swiglu_lut:   anvil/lower/graph_to_tensor.py:297-300 (requant(table[x + 128] * y, M, s))
    - residual_add: anvil/semantics.py:106-115 (add_requant with i8 operands and result)
    - matmul_i8:    checked int32 a @ b (anvil/semantics.py:95-103 uses it; anvil/lower/graph_to_tensor.py:243-266)
* The generalized ops (requant_var, lut_i8, qmatmul, add_requant, requant_dtype, sq_shift, rmsnorm_wide, ...)
  follow anvil/semantics.py line by line (cited per function).
* Extensions with no reference code (the nanoGPT family): qmatmul bias, layernorm_int, embed. Each reduces to a
  reference op in a degenerate case (bias = 0; rows with sum 0 and no bias; embed = residual_add of two
  gathered rows).

Discipline: every value is an int64 numpy array; every intermediate the reference checks must fit int32 and raises
OverflowError otherwise; int8 operands outside int8 raise ValueError; LUT indices outside the table raise
IndexError; shifts outside [0, 31] raise ValueError.
"""
from __future__ import annotations

import numpy as np

I8 = (-128, 127)
I16 = (-(1 << 15), (1 << 15) - 1)
I32 = (-(1 << 31), (1 << 31) - 1)
DT_RANGE = {"i8": I8, "i16": I16, "i32": I32}


# ---------------------------------------------------------------------------------------------- checked ints

def check_i32(x, what="value"):
    """x as int64 numpy, OverflowError if any element leaves int32 (anvil/semantics.py:47-49, golden._i32)."""
    x = np.asarray(x, dtype=np.int64)
    if x.size and (x.min() < I32[0] or x.max() > I32[1]):
        raise OverflowError(f"{what} leaves int32")
    return x


def check_i8(x, what="value"):
    """x as int64 numpy, ValueError if any element leaves int8 (anvil/semantics.py:52-54, golden._i8)."""
    x = np.asarray(x, dtype=np.int64)
    if x.size and (x.min() < I8[0] or x.max() > I8[1]):
        raise ValueError(f"{what} is not int8")
    return x


def check_dtype(x, dtype, what="value"):
    """anvil/semantics.py:129-139: ValueError outside i8/i16, OverflowError outside i32."""
    if dtype == "i32":
        return check_i32(x, what)
    if dtype == "i8":
        return check_i8(x, what)
    lo, hi = DT_RANGE[dtype]
    x = np.asarray(x, dtype=np.int64)
    if x.size and (x.min() < lo or x.max() > hi):
        raise ValueError(f"{what} is not int{dtype[1:]}")
    return x


def clamp_i8(x):
    return np.clip(np.asarray(x, dtype=np.int64), *I8)


def clamp_dtype(x, dtype):
    return np.clip(np.asarray(x, dtype=np.int64), *DT_RANGE[dtype])


def _is_i8(x):
    return not x.size or (x.min() >= I8[0] and x.max() <= I8[1])


def round_term(s):
    """2^(s-1), 0 when s == 0 (anvil/semantics.py:57-62)."""
    s = int(s)
    if not 0 <= s <= 31:
        raise ValueError(f"shift {s} outside [0, 31]")
    return (1 << (s - 1)) if s else 0


# ---------------------------------------------------------------------------------------------- golden base

def requant_dtype(acc, m, s, dtype="i8"):
    """clamp_dtype((acc*M + 2^(s-1)) >> s): acc, acc*M and acc*M + round each checked int32, `>>` arithmetic
    (floor). i8 is golden.requant (anvil/semantics.py:146-155; anvil/backend/idioms.py:150-163)."""
    s = int(s)
    if not 0 <= s <= 31:
        raise ValueError(f"shift {s} outside [0, 31]")
    acc = check_i32(acc, "acc")
    prod = check_i32(acc * int(m), "acc*M")
    rounded = check_i32(prod + round_term(s), "acc*M + round")
    return clamp_dtype(rounded >> s, dtype)


def requant(acc, m, s):
    """golden.requant: requant_dtype with an int8 clamp."""
    return requant_dtype(acc, m, s, "i8")


EXACT_F64_K = 1 << 38          # K * 128 * 128 < 2^52: every partial sum of int8 products is exact in float64


def matmul_i8(a, b):
    """golden.matmul_i8: int8 operands, exact product summed, the result checked int32. Batched as numpy matmul
    broadcasts ((..., M, K) @ (K, N) or (..., M, K) @ (..., K, N)). The sums are formed in float64 BLAS when K is
    small enough that every partial sum of int8 products is an integer below 2^53 (always, in practice), which is
    exact and equal to the int64 sum; otherwise in int64."""
    a, b = check_i8(a, "a"), check_i8(b, "b")
    if a.shape[-1] < EXACT_F64_K:
        out = np.rint(np.matmul(a.astype(np.float64), b.astype(np.float64))).astype(np.int64)
    else:
        out = np.matmul(a, b)
    return check_i32(out, "a @ b")


def rsqrt_index(ss, n):
    """golden.rsqrt_index: idx = ss, k = 0; while idx >= n: idx >>= 2; k += 1 (element-wise; ss >= 0).
    Restated from anvil/vortexv/codegen.py:512-519 and anvil/codegen/lower.py:791-803."""
    idx = np.array(ss, dtype=np.int64, copy=True)
    if idx.size and idx.min() < 0:
        raise ValueError("rsqrt_index needs a non-negative sum")
    k = np.zeros_like(idx)
    while True:
        big = idx >= n
        if not big.any():
            break
        idx = np.where(big, idx >> 2, idx)
        k += big
    return idx, k


def residual_add(a, b, ma, mb, s):
    """golden.residual_add: clamp_i8((a*Ma + b*Mb + 2^(s-1)) >> s) with int8 operands, every intermediate checked
    (anvil/semantics.py:106-115 on its all-i8 path)."""
    a, b = check_i8(a, "a"), check_i8(b, "b")
    acc = check_i32(check_i32(a * int(ma), "a*Ma") + check_i32(b * int(mb), "b*Mb"), "a*Ma + b*Mb")
    return requant(acc, 1, s)


def swiglu_lut(x, y, table, m, s):
    """golden.swiglu_lut: requant(table[x + 128] * y, M, s) (anvil/lower/graph_to_tensor.py:297-300)."""
    x, y, table = check_i8(x, "x"), check_i8(y, "y"), check_i8(table, "lut")
    if table.shape != (256,):
        raise ValueError("int8 LUT must have 256 entries")
    return requant(check_i32(table[x + 128] * y, "lut*y"), m, s)


def rmsnorm_int(x, w, rsqrt_lut, m, s):
    """golden.rmsnorm_int on int8 rows: ss = sum x^2, (idx, k) = rsqrt_index(ss, len(lut)),
    out = requant(x*w*lut[idx], M, s + k) (anvil/semantics.py:164-182 with c = e = 0)."""
    return _rms_core(check_i8(x, "x"), w, rsqrt_lut, m, s, 0, 0)


def softmax_lut(x, lut, one, causal=True):
    """golden.softmax_lut over the last axis (anvil/lower/graph_to_tensor.py:352-398,
    anvil/vortexv/codegen.py:545-615). Row i of (..., T1, T2) keeps j <= i when causal, else every j:
        m = max(-128, max kept x_j);  e_j = lut[x_j - m + 255];  S = sum kept e_j   (checked int32)
        p_j = (e_j*one + S//2) // S  (floor, operands non-negative);  masked p_j = 0."""
    x = check_i8(x, "x")
    lut = check_i32(lut, "exp_lut")
    if lut.shape != (256,):
        raise ValueError("exp LUT must have 256 entries")
    if x.ndim < 2:
        raise ValueError("softmax_lut needs rank >= 2")
    t1, t2 = x.shape[-2:]
    keep = np.ones((t1, t2), dtype=bool)
    if causal:
        keep = np.arange(t2)[None, :] <= np.arange(t1)[:, None]
    keep = np.broadcast_to(keep, x.shape)
    mx = np.maximum(np.where(keep, x, I8[0]).max(axis=-1, keepdims=True), I8[0])
    idx = np.where(keep, x - mx + 255, 255)
    e = np.where(keep, lut[idx], 0)
    tot = check_i32(e.sum(axis=-1, keepdims=True), "exp sum")
    num = check_i32(check_i32(e * int(one), "e*one") + tot // 2, "e*one + S/2")
    if (tot <= 0).any() or (num < 0).any():
        raise ValueError("softmax division needs a non-negative numerator and a positive sum")
    return np.where(keep, num // tot, 0)


# ------------------------------------------------------------------------------------------ generalized ops

def requant_var(acc, m, s):
    """requant with a per-element shift broadcast against acc (anvil/semantics.py:65-73)."""
    acc = check_i32(acc, "acc")
    s = np.broadcast_to(np.asarray(s, dtype=np.int64), acc.shape)
    out = np.empty(acc.shape, dtype=np.int64)
    for sv in np.unique(s):
        sel = s == sv
        out[sel] = requant(acc[sel], m, int(sv))
    return out


def lut_lookup(table, idx, offset=0):
    """table[idx + offset] with an explicit bounds check (anvil/semantics.py:76-84)."""
    table = np.asarray(table, dtype=np.int64)
    i = np.asarray(idx, dtype=np.int64) + int(offset)
    if table.ndim != 1:
        raise ValueError("LUT must be 1-D")
    if i.size and (i.min() < 0 or i.max() >= len(table)):
        raise IndexError(f"LUT index outside [0, {len(table)})")
    return table[i]


def lut_i8(x, table):
    """Unary int8 LUT table[x + 128] (anvil/semantics.py:87-92)."""
    x, table = check_i8(x, "x"), check_i8(table, "lut")
    if table.shape != (256,):
        raise ValueError("int8 LUT must have 256 entries")
    return table[x + 128]


def qmatmul(a, b, m, s, lut=None, dtype="i8", bias=None):
    """requant(a @ b, M, s) then the optional LUT epilogue; an i16 result clamps to int16
    (anvil/semantics.py:95-103). Extension: `bias` (int32 per output column) is added to the accumulator, checked,
    before the requant; bias = None or 0 is the reference op."""
    if dtype != "i8" and lut is not None:
        raise ValueError("a LUT epilogue needs an i8 result")
    acc = matmul_i8(a, b)
    if bias is not None:
        acc = check_i32(acc + check_i32(bias, "bias"), "acc + bias")
    out = requant_dtype(acc, m, s, dtype)
    return out if lut is None else lut_i8(out, lut)


def add_requant(a, b, ma, mb, s, dtype="i8"):
    """clamp((a*Ma + b*Mb + 2^(s-1)) >> s) to `dtype`; all-i8 is golden.residual_add, otherwise a and b may be
    i8 or i16 (anvil/semantics.py:106-115)."""
    a, b = np.asarray(a, dtype=np.int64), np.asarray(b, dtype=np.int64)
    if dtype == "i8" and _is_i8(a) and _is_i8(b):
        return residual_add(a, b, ma, mb, s)
    a, b = check_dtype(a, "i16", "a"), check_dtype(b, "i16", "b")
    acc = check_i32(check_i32(a * int(ma), "a*Ma") + check_i32(b * int(mb), "b*Mb"), "a*Ma + b*Mb")
    return requant_dtype(acc, 1, s, dtype)


def sq_shift(x, c):
    """(x*x + 2^(c-1)) >> c, checked (anvil/semantics.py:158-161)."""
    sq = check_i32(np.asarray(x, dtype=np.int64) ** 2, "x*x")
    return check_i32(sq + round_term(c), "x*x + round") >> int(c)


def _rms_core(x, w, rsqrt_lut, m, s, c, e, bias=None):
    """The shared row body of rmsnorm_wide / layernorm_int on an already-checked row tensor x."""
    w = check_i8(w, "w")
    lut = check_i32(rsqrt_lut, "rsqrt_lut")
    if lut.ndim != 1 or (lut.size and lut.min() < 0):
        raise ValueError("rsqrt_lut must be a non-negative 1-D table")
    ss = check_i32(sq_shift(x, c).sum(axis=-1) + int(e), "sum of squares")
    idx, k = rsqrt_index(ss, len(lut))
    xwr = check_i32(check_i32(x * w, "x*w") * lut[idx][..., None], "x*w*r")
    if bias is None:
        out = np.empty_like(xwr)
        kk = np.broadcast_to(k[..., None], xwr.shape)
        for kv in np.unique(k):
            out[kk == kv] = requant(xwr[kk == kv], m, int(s) + int(kv))
        return out
    # layernorm bias: the same requant numerator and shift, + bias, then one int8 clamp
    b = check_i8(bias, "bias")
    out = np.empty_like(xwr)
    kk = np.broadcast_to(k[..., None], xwr.shape)
    for kv in np.unique(k):
        sh = int(s) + int(kv)
        if not 0 <= sh <= 31:
            raise ValueError(f"shift {sh} outside [0, 31]")
        sel = kk == kv
        num = check_i32(check_i32(xwr[sel] * int(m), "acc*M") + round_term(sh), "acc*M + round") >> sh
        out[sel] = num
    return clamp_i8(check_i32(out + b, "norm + bias"))


def rmsnorm_wide(x, w, rsqrt_lut, m, s, ss_shift=0, ss_init=0, xdtype="i8"):
    """rmsnorm_int on an i8 or i16 row with ss = e + sum((x^2 + 2^(c-1)) >> c) (anvil/semantics.py:164-182)."""
    x = np.asarray(x, dtype=np.int64)
    if xdtype == "i8" and int(ss_shift) == 0 and int(ss_init) == 0:
        return rmsnorm_int(x, w, rsqrt_lut, m, s)
    return _rms_core(check_dtype(x, xdtype, "x"), w, rsqrt_lut, m, s, int(ss_shift), int(ss_init))


def layernorm_int(x, w, rsqrt_lut, m, s, ss_shift=0, ss_init=0, xdtype="i8", bias=None):
    """Extension (no reference code). Per row of d entries:
        mean = floor((sum x + d // 2) / d)     (sum checked int32)
        xc   = x - mean
        then rmsnorm_wide's body on xc: ss = e + sum((xc^2 + 2^(c-1)) >> c), (idx, k) = rsqrt_index(ss, n),
        v = (xc*w*lut[idx]*M + 2^(s+k-1)) >> (s+k), out = clamp_i8(v + bias)   (bias absent = 0)
    Without a bias this is requant(xc*w*lut[idx], M, s + k); on rows with sum 0 it is rmsnorm_wide exactly."""
    x = check_dtype(np.asarray(x, dtype=np.int64), xdtype, "x")
    d = x.shape[-1]
    tot = check_i32(x.sum(axis=-1, keepdims=True), "row sum")
    mean = (tot + d // 2) // d
    xc = x - mean
    return _rms_core(xc, w, rsqrt_lut, m, s, int(ss_shift), int(ss_init), bias)


def embed(ids, wte, wpe, ma, mb, s):
    """Extension: x[..., t, :] = residual_add(wte[ids[..., t]], wpe[t], Ma, Mb, s); ids outside [0, V) raise
    IndexError like lut_lookup."""
    ids = np.asarray(ids, dtype=np.int64)
    wte, wpe = check_i8(wte, "wte"), check_i8(wpe, "wpe")
    if ids.size and (ids.min() < 0 or ids.max() >= wte.shape[0]):
        raise IndexError(f"token id outside [0, {wte.shape[0]})")
    t = ids.shape[-1]
    if t > wpe.shape[0]:
        raise IndexError(f"{t} positions > {wpe.shape[0]} wpe rows")
    return residual_add(wte[ids], np.broadcast_to(wpe[:t], ids.shape + (wte.shape[1],)), ma, mb, s)
