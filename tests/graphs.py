"""Seeded random anvil.graph cases for cuda-vs-oracle fuzzing.

Modelled on the reference's fuzz strategy (tests/vortexv/vv_graphs.py:49-123: draw a transformer-shaped graph,
redraw while the golden interpreter rejects it) but drawn here independently. Coverage per draw:
multi-head head-batched matmuls with T1 != T2, a kT made by one transpose or by two, LUT epilogues, causal and
non-causal softmax with an i8 or i32 result, i8 or i16 residual streams (an i16 rmsnorm with ss_shift/ss_init),
lut_mul, and the nanoGPT extensions (layernorm_int with bias, qlinear bias, embed) when `ext` is set.
Sizes are small so the oracle finishes in milliseconds; `big=True` draws shapes large enough for the
tcgen05 GEMM path (K a multiple of 16, hundreds of rows).
"""
from __future__ import annotations

import numpy as np

from anvil.ir.graph import GraphBuilder
from oracle import interp


def rsqrt_lut(n, scale=1 << 15):
    return np.round(scale / np.sqrt(np.arange(n) + 1)).astype(np.int64)


def exp_lut(tau=24.0, e=14):
    return np.round((1 << e) * np.exp((np.arange(256) - 255) / tau)).astype(np.int64)


def mult_shift(rng, gain, lo=8, hi=20):
    """(M, s) with M / 2^s close to `gain` (times a random factor in [0.5, 2])."""
    s = int(rng.integers(lo, hi + 1))
    m = max(1, int(round(gain * (1 << s) * rng.uniform(0.5, 2.0))))
    return min(m, (1 << 31) - 1), s


ACT = 50.0                  # typical |int8 activation| in these graphs


def mm_params(rng, k, out=40.0):
    return mult_shift(rng, out / (ACT * ACT * np.sqrt(k)))


def draw(rng, big=False, ext=True):
    """(module, consts, inputs) for one random transformer-style graph."""
    if big:
        T = int(rng.choice([128, 192, 256]))
        T2 = T
        H = int(rng.choice([1, 2]))
        dh = int(rng.choice([16, 32, 64]))
        d = int(rng.choice([64, 128]))
        ff = int(rng.choice([128, 256]))
    else:
        T = int(rng.integers(2, 9))
        T2 = T if rng.random() < 0.7 else int(rng.integers(2, 9))
        H = int(rng.integers(1, 4))
        dh = int(rng.integers(2, 10))
        d = int(rng.integers(3, 21))
        ff = int(rng.integers(3, 25))
    wide = rng.random() < 0.4
    use_ln = ext and rng.random() < 0.5
    use_bias = ext and rng.random() < 0.5
    use_embed = ext and rng.random() < 0.3 and not wide
    g = GraphBuilder("fuzz")
    consts = {}

    def const(name, shape, dtype="i8", value=None):
        v = rng.integers(-128, 128, shape) if value is None else np.asarray(value)
        consts[name] = np.asarray(v, dtype=np.int64)
        return g.const(name, list(np.shape(v)), dtype)

    inputs = {}
    if use_embed:
        V = int(rng.integers(5, 40))
        ids = g.input("ids", [T], "i32")
        ema, emb = int(rng.integers(1, 1 << 11)), int(rng.integers(1, 1 << 11))
        x = g.embed("x", ids, const("wte", [V, d]), const("wpe", [T + int(rng.integers(0, 3)), d]), ema, emb, 12)
        inputs["ids"] = rng.integers(0, V, T)
    else:
        x = g.input("x", [T, d], "i16" if wide else "i8")
        inputs["x"] = rng.integers(-(1 << 15), 1 << 15, (T, d)) if wide else rng.integers(-128, 128, (T, d))
    xk = g.input("xk", [T2, d])
    inputs["xk"] = rng.integers(-128, 128, (T2, d))
    nl = int(rng.choice([64, 256, 1024]))
    rs = const("rsqrt", [nl], "i32", rsqrt_lut(nl))
    norm_gain = 40.0 / (ACT * (1 << 15) / (ACT * np.sqrt(d)))
    if use_ln and not wide:
        h = g.layernorm_int("h", x, const("nw", [d]), rs, *mult_shift(rng, norm_gain, 4, 14),
                            bias=const("nb", [d], value=rng.integers(-20, 21, d)) if rng.random() < 0.6 else None)
    elif wide:
        h = g.rmsnorm_int("h", x, const("nw", [d]), rs, 1, int(rng.integers(12, 20)),
                          ss_shift=int(rng.integers(4, 9)), ss_init=int(rng.integers(0, 64)))
    else:
        h = g.rmsnorm_int("h", x, const("nw", [d]), rs, *mult_shift(rng, norm_gain, 4, 14))
    hk = g.rmsnorm_int("hk", xk, const("nwk", [d]), rs, *mult_shift(rng, norm_gain, 4, 14))

    def bias(name, n):
        if not use_bias or rng.random() < 0.3:
            return None
        return const(name, [n], "i32", rng.integers(-3000, 3001, n))

    q = g.qlinear("q", h, const("wq", [d, H * dh]), *mm_params(rng, d), bias=bias("bq", H * dh))
    k = g.qlinear("k", hk, const("wk", [d, H * dh]), *mm_params(rng, d), bias=bias("bk", H * dh))
    v = g.qlinear("v", hk, const("wv", [d, H * dh]), *mm_params(rng, d))
    qh = g.transpose("qh", g.reshape("q3", q, [T, H, dh]), [1, 0, 2])
    k3 = g.reshape("k3", k, [T2, H, dh])
    if rng.random() < 0.5:
        kT = g.transpose("kT", k3, [1, 2, 0])
    else:
        kT = g.transpose("kT", g.transpose("kh", k3, [1, 0, 2]), [0, 2, 1])
    sc = g.qmatmul("scores", qh, kT, *mm_params(rng, dh))
    causal = bool(rng.random() < 0.6)
    ex = const("exp", [256], "i32", exp_lut())
    p = g.softmax_lut("p", sc, ex, int(rng.integers(32, 128)), causal)
    vh = g.transpose("vh", g.reshape("v3", v, [T2, H, dh]), [1, 0, 2])
    o = g.qmatmul("o", p, vh, *mm_params(rng, T2))
    o2 = g.reshape("o2", g.transpose("ot", o, [1, 0, 2]), [T, H * dh])
    y = g.qlinear("y", o2, const("wo", [H * dh, d]), *mm_params(rng, H * dh), bias=bias("bo", d))
    rdt = "i16" if wide else "i8"
    rt = 2000.0 if wide else 40.0
    base = 1 << 15 if wide else ACT
    ma, s1 = mult_shift(rng, rt / 2 / base, 8, 16)
    mb = max(1, int(round(rt / 2 / ACT * (1 << s1))))
    r1 = g.add_requant("r1", x, y, ma, mb, s1, dtype=rdt)
    if wide:
        h2 = g.rmsnorm_int("h2", r1, const("nw2", [d]), rs, 1, int(rng.integers(12, 20)),
                           ss_shift=int(rng.integers(4, 9)), ss_init=int(rng.integers(0, 64)))
    else:
        h2 = g.rmsnorm_int("h2", r1, const("nw2", [d]), rs, *mult_shift(rng, norm_gain, 4, 14))
    gate = g.qlinear("gate", h2, const("wg", [d, ff]), *mm_params(rng, d),
                     lut=const("glut", [256]) if rng.random() < 0.5 else None)
    up = g.qlinear("up", h2, const("wu", [d, ff]), *mm_params(rng, d))
    act = g.lut_mul("act", gate, up, const("silu", [256]), *mult_shift(rng, 40.0 / (ACT * ACT)))
    act = g.lut("act2", act, const("lut2", [256]))
    dn = g.qlinear("down", act, const("wd", [ff, d]), *mm_params(rng, ff, 2000.0 if wide else 40.0), dtype=rdt)
    ma, s2 = mult_shift(rng, 20.0 / (2000.0 if wide else ACT), 8, 18)
    mb2 = max(1, int(round(20.0 / (2000.0 if wide else ACT) * (1 << s2) * rng.uniform(0.5, 2))))
    out = g.add_requant("out", r1, dn, ma, mb2, s2)
    p32 = g.softmax_lut("p32", sc, ex, int(rng.integers(1, 1 << 12)), not causal, dtype="i32")
    g.output(out, p32)
    return g.module(), consts, inputs


def random_case(seed, big=False, ext=True, tries=60, batch=None):
    """(module, consts, inputs, oracle GraphResult) redrawn until the oracle accepts it. With `batch`, inputs get
    a leading batch dim of that size and the oracle runs batched."""
    rng = np.random.default_rng(seed)
    for _ in range(tries):
        m, c, x = draw(rng, big, ext)
        if batch:
            xb = {}
            for k, v in x.items():
                extra = [v] + [(rng.integers(0, int(c["wte"].shape[0]), v.shape) if k == "ids" else
                                rng.integers(v.min(), v.max() + 1, v.shape)) for _ in range(batch - 1)]
                xb[k] = np.stack(extra)
            x = xb
        try:
            return m, c, x, interp.run(m, x, c, batch=bool(batch))
        except (OverflowError, ValueError, ZeroDivisionError, IndexError):
            continue
    raise RuntimeError(f"seed {seed}: no in-contract draw in {tries} tries")


def attention_graph(seed, T, C, nh, causal=True, T2=None):
    """(module, consts, x) for x -> q/k/v projections -> heads -> qk^T -> softmax_lut -> p@v -> merged heads ->
    projection: the chain the fused attention kernel runs (self-attention when T2 is None)."""
    rng = np.random.default_rng(seed)
    T2 = T if T2 is None else T2
    hd = C // nh
    g = GraphBuilder("attn")
    consts = {}

    def const(name, shape, dtype="i8", value=None):
        v = rng.integers(-128, 128, shape) if value is None else np.asarray(value)
        consts[name] = np.asarray(v, dtype=np.int64)
        return g.const(name, list(np.shape(v)), dtype)

    from anvil.frontend.numerics import fixed_point

    def fp(gain, bound):                       # (M, s) that the static int32 proof accepts
        (m,), s = fixed_point([gain * rng.uniform(0.7, 1.4)], [bound])
        return m, s

    def lin(name, x_, w_):
        wv = rng.integers(-127, 128, (C, C))
        return g.qlinear(name, x_, const(w_, [C, C], value=wv),
                         *fp(40.0 / (ACT * 73 * np.sqrt(C)), 128 * int(np.abs(wv).sum(axis=0).max())))

    x = g.input("x", [T, C])
    xk = g.input("xk", [T2, C]) if T2 != T else x
    q = lin("q", x, "wq")
    k = lin("k", xk, "wk")
    v = lin("v", xk, "wv")
    qh = g.transpose("qh", g.reshape("q3", q, [T, nh, hd]), [1, 0, 2])
    kh = g.transpose("kh", g.reshape("k3", k, [T2, nh, hd]), [1, 0, 2])
    kT = g.transpose("kT", kh, [0, 2, 1])
    sc = g.qmatmul("scores", qh, kT, *fp(30.0 / (40.0 * 40.0 * np.sqrt(hd)), hd * 128 * 128))
    p = g.softmax_lut("p", sc, const("exp", [256], "i32", exp_lut(tau=12.0, e=14)), 127, causal)
    vh = g.transpose("vh", g.reshape("v3", v, [T2, nh, hd]), [1, 0, 2])
    o = g.qmatmul("o", p, vh, *fp(40.0 / (127 * 40.0 / np.sqrt(max(T2, 1)) * 3), T2 * 127 * 128))
    om = g.reshape("om", g.transpose("om.t", o, [1, 0, 2]), [T, C])
    y = lin("y", om, "wo")
    g.output(y)
    xs = {"x": rng.integers(-128, 128, (T, C))}
    if T2 != T:
        xs["xk"] = rng.integers(-128, 128, (T2, C))
    return g.module(), consts, xs
