"""CPU emulator of a lowered launch list (test infrastructure only).

Executes the anvil_op records of anvil.runtime.program on a numpy byte arena and const blob, one numpy routine per
op kind with the kernels' arithmetic (64-bit products, arithmetic shifts, clamps). It exists to test the host-side
lowering (views, strided copies, B^T operands, fusion, liveness offsets) on machines without a GPU: if the
emulated launch list matches the oracle, the offsets and shapes handed to the GPU are right. It is never used by
the product path.
"""
from __future__ import annotations

import numpy as np

from anvil.runtime import cuda as C

DT = {1: np.int8, 2: np.int16, 4: np.int32}
RANGE = {1: (-128, 127), 2: (-(1 << 15), (1 << 15) - 1), 4: (-(1 << 31), (1 << 31) - 1)}


def _rnd(s):
    return (1 << (s - 1)) if s else 0


class Emu:
    def __init__(self, blob: np.ndarray, arena_bytes: int):
        self.blob = np.asarray(blob, dtype=np.uint8)
        self.arena = np.zeros(max(arena_bytes, 1), dtype=np.uint8)

    def _mem(self, loc):
        if loc & C.LOC_CONST:
            return self.blob, loc & ~C.LOC_CONST
        return self.arena, loc

    def get(self, loc, n, isz):
        mem, off = self._mem(loc)
        assert off + n * isz <= mem.size, "read outside region"
        return mem[off:off + n * isz].view(DT[isz]).astype(np.int64)

    def put(self, loc, vals, isz):
        mem, off = self._mem(loc)
        assert not loc & C.LOC_CONST, "write into the const region"
        vals = np.asarray(vals, dtype=np.int64).ravel()
        assert off + vals.size * isz <= mem.size, "write outside region"
        mem[off:off + vals.size * isz] = vals.astype(DT[isz]).view(np.uint8)

    def run(self, ops):
        for o in ops:
            getattr(self, "k%d" % o.kind)(o)

    def k1(self, o):                                    # GEMM
        if o.flags & C.F_SPLIT:
            return self._split_gemm(o)
        batch, M, N, K = (int(o.dims[i]) for i in range(4))
        abs_, bbs, obs, ors = (int(o.strides[i]) for i in range(4))
        grp, gst, cst = int(o.strides[4]) or M, int(o.strides[5]), int(o.strides[6]) or 1
        lo, hi = RANGE[o.out_bytes]
        lut = self.get(o.off[3], 256, 1) if o.flags & C.F_LUT else None
        bias = self.get(o.off[4], N, 4) if o.flags & C.F_BIAS else None
        for b in range(batch):
            a = self.get(o.off[0] + b * abs_, M * K, 1).reshape(M, K)
            bt = self.get(o.off[1] + (b * bbs if bbs else 0), N * K, 1).reshape(N, K)
            acc = a @ bt.T
            if bias is not None and o.flags & C.F_BIAS_RND:        # folded bias*M + 2^(s-1)
                v = np.clip((acc * int(o.mult) + bias) >> int(o.shift), lo, hi)
            else:
                if bias is not None:
                    acc = acc + bias
                v = np.clip((acc * int(o.mult) + _rnd(int(o.shift))) >> int(o.shift), lo, hi)
            if lut is not None:
                v = lut[v + 128]
            if o.flags & C.F_RESIDUAL:                                  # y clamped to its dtype, then the add
                y = np.clip(np.clip((acc * int(o.mult) + (bias if bias is not None and o.flags & C.F_BIAS_RND
                                                          else _rnd(int(o.shift)))) >> int(o.shift),
                                    *RANGE[o.in_bytes]), *RANGE[o.in_bytes])
                res = self.get(o.off[5], M * N, o.in2_bytes).reshape(M, N)
                s2 = int(o.shift2)
                v = np.clip((res * int(o.ma) + y * int(o.mb) + _rnd(s2)) >> s2, lo, hi)
            mem, base = self._mem(o.off[2])
            idx = (b * obs + (np.arange(M)[:, None] // grp) * gst + (np.arange(M)[:, None] % grp) * ors
                   + np.arange(N)[None, :] * cst)
            flat = mem[base:].view(DT[o.out_bytes])
            assert idx.max() < flat.size, "write outside region"
            flat[idx] = v.astype(DT[o.out_bytes])

    def _split_gemm(self, o):
        """Several linears as one GEMM: chunk c of dims[4] columns requantised with aux[c]; columns below dims[5]
        row-major to off[2] (row stride strides[3]), the rest head-major transposed (group dims[6]) to off[6]."""
        M, N, K, Cw, R, T = (int(o.dims[i]) for i in (1, 2, 3, 4, 5, 6))
        a = self.get(o.off[0], M * K, 1).reshape(M, K)
        bt = self.get(o.off[1], N * K, 1).reshape(N, K)
        acc = a @ bt.T
        bias = self.get(o.off[4], N, 4) if o.flags & C.F_BIAS else None
        v = np.empty_like(acc)
        for c in range(N // Cw):
            m, s = int(o.aux[c]) >> 8, int(o.aux[c]) & 255
            cols = slice(c * Cw, (c + 1) * Cw)
            add = bias[cols] if bias is not None else _rnd(s)
            v[:, cols] = np.clip((acc[:, cols] * m + add) >> s, -128, 127)
        mem, base = self._mem(o.off[2])
        ors = int(o.strides[3])
        for r in range(M):
            mem[base + r * ors: base + r * ors + R] = v[r, :R].astype(np.int8).view(np.uint8)
        if R < N:
            N2 = N - R
            mem2, base2 = self._mem(o.off[6])
            r = np.arange(M)[:, None]
            idx = (r // T) * (N2 * T) + np.arange(N2)[None, :] * T + r % T
            flat = mem2[base2:].view(np.int8)
            assert idx.max() < flat.size, "write outside region"
            flat[idx] = v[:, R:].astype(np.int8)

    def k2(self, o):                                    # LUT
        n = int(o.dims[0])
        self.put(o.off[2], self.get(o.off[1], 256, 1)[self.get(o.off[0], n, 1) + 128], 1)

    def k3(self, o):                                    # LUT_MUL
        n = int(o.dims[0])
        t = self.get(o.off[2], 256, 1)[self.get(o.off[0], n, 1) + 128] * self.get(o.off[1], n, 1)
        self.put(o.off[3], np.clip((t * int(o.mult) + _rnd(int(o.shift))) >> int(o.shift), -128, 127), 1)

    def k4(self, o):                                    # ADD_REQUANT
        n = int(o.dims[0])
        a, b = self.get(o.off[0], n, o.in_bytes), self.get(o.off[1], n, o.in2_bytes)
        s = int(o.shift)
        self.put(o.off[2], np.clip((a * int(o.ma) + b * int(o.mb) + _rnd(s)) >> s, *RANGE[o.out_bytes]), o.out_bytes)

    def k5(self, o):                                    # NORM
        rows, d, n = (int(o.dims[i]) for i in range(3))
        x = self.get(o.off[0], rows * d, o.in_bytes).reshape(rows, d)
        w = self.get(o.off[1], d, 1)
        lut = self.get(o.off[2], n, 4)
        if o.flags & C.F_CENTER:
            x = x - (x.sum(axis=1, keepdims=True) + d // 2) // d
        c, e = int(o.ss_shift), int(o.ss_init)
        ss = ((x * x + _rnd(c)) >> c).sum(axis=1) + e
        idx, k = ss.copy(), np.zeros_like(ss)
        while (idx >= n).any():
            big = idx >= n
            idx = np.where(big, idx >> 2, idx)
            k += big
        sh = int(o.shift) + k[:, None]
        num = x * w * lut[idx][:, None] * int(o.mult)
        v = (num + np.where(sh > 0, 1 << np.maximum(sh - 1, 0), 0)) >> sh
        if o.flags & C.F_BIAS:
            v = v + self.get(o.off[4], d, 1)
        self.put(o.off[3], np.clip(v, -128, 127), 1)

    def k6(self, o):                                    # SOFTMAX
        b, t1, t2 = (int(o.dims[i]) for i in range(3))
        x = self.get(o.off[0], b * t1 * t2, 1).reshape(b, t1, t2)
        lut = self.get(o.off[1], 256, 4)
        keep = np.ones((t1, t2), bool)
        if o.flags & C.F_CAUSAL:
            keep = np.arange(t2)[None, :] <= np.arange(t1)[:, None]
        keep = np.broadcast_to(keep, x.shape)
        mx = np.maximum(np.where(keep, x, -128).max(axis=-1, keepdims=True), -128)
        e = np.where(keep, lut[np.where(keep, x - mx + 255, 255)], 0)
        tot = e.sum(axis=-1, keepdims=True)
        p = np.where(keep, (e * int(o.one) + tot // 2) // np.maximum(tot, 1), 0)
        self.put(o.off[2], p, o.out_bytes)

    def k7(self, o):                                    # TRANSPOSE (strided gather)
        rank = int(o.dims[0])
        shape = [int(o.dims[1 + i]) for i in range(rank)]
        st = [int(o.strides[i]) for i in range(rank)]
        span = sum((d - 1) * s for d, s in zip(shape, st)) + 1
        src = self.get(o.off[0], span, o.in_bytes)
        idx = np.zeros(shape, dtype=np.int64)
        for i, (d, s) in enumerate(zip(shape, st)):
            sh = [1] * rank
            sh[i] = d
            idx = idx + (np.arange(d) * s).reshape(sh)
        self.put(o.off[1], src[idx], o.in_bytes)

    def k8(self, o):                                    # EMBED
        b, t, d, vocab = (int(o.dims[i]) for i in range(4))
        ids = self.get(o.off[0], b * t, 4).reshape(b, t)
        assert ids.min() >= 0 and ids.max() < vocab
        wte = self.get(o.off[1], vocab * d, 1).reshape(vocab, d)
        wpe = self.get(o.off[2], t * d, 1).reshape(t, d)
        s = int(o.shift)
        v = (wte[ids] * int(o.ma) + wpe[None] * int(o.mb) + _rnd(s)) >> s
        self.put(o.off[3], np.clip(v, -128, 127), 1)

    def k9(self, o):                                    # ATTENTION
        B, H, T1, T2, hd = (int(o.dims[i]) for i in range(5))
        st = [int(o.strides[i]) for i in range(8)]
        lut = self.get(o.off[4], 256, 4)
        mq, mk = self._mem(o.off[0]), self._mem(o.off[1])
        vt = self.get(o.off[2], B * H * hd * T2, 1).reshape(B, H, hd, T2)
        qv = mq[0][mq[1]:].view(np.int8)
        kv = mk[0][mk[1]:].view(np.int8)
        bi, hi, ti, di = np.ix_(np.arange(B), np.arange(H), np.arange(T1), np.arange(hd))
        q = qv[bi * st[0] + hi * st[1] + ti * st[2] + di].astype(np.int64)
        bi, hi, ti, di = np.ix_(np.arange(B), np.arange(H), np.arange(T2), np.arange(hd))
        k = kv[bi * st[3] + hi * st[4] + ti * st[5] + di].astype(np.int64)
        s1, s2 = int(o.shift), int(o.shift2)
        sc = np.clip((q @ np.swapaxes(k, -1, -2) * int(o.mult) + _rnd(s1)) >> s1, -128, 127)
        keep = np.ones((T1, T2), bool)
        if o.flags & C.F_CAUSAL:
            keep = np.arange(T2)[None, :] <= np.arange(T1)[:, None]
        keep = np.broadcast_to(keep, sc.shape)
        mx = np.maximum(np.where(keep, sc, -128).max(axis=-1, keepdims=True), -128)
        e = np.where(keep, lut[np.where(keep, sc - mx + 255, 255)], 0)
        tot = e.sum(axis=-1, keepdims=True)
        p = np.where(keep, (e * int(o.one) + tot // 2) // np.maximum(tot, 1), 0)
        out = np.clip((p @ np.swapaxes(vt, -1, -2) * int(o.mult2) + _rnd(s2)) >> s2, -128, 127)   # (B, H, T1, hd)
        mem, base = self._mem(o.off[3])
        bi, hi, ti, di = np.ix_(np.arange(B), np.arange(H), np.arange(T1), np.arange(hd))
        flat = mem[base:].view(np.int8)
        flat[bi * st[6] + ti * st[7] + hi * hd + di] = out.astype(np.int8)

    def k10(self, o):                                   # COPY
        n = int(o.dims[0])
        self.put(o.off[1], self.get(o.off[0], n, 1), 1)


def run_program(cm, inputs: dict, keep="outputs"):
    """Lower `cm` for the batch of `inputs` (each with a leading batch dim), emulate it, return {sym: ints}."""
    from anvil.driver import _apply_view
    batch = next(iter(inputs.values())).shape[0]
    prog = cm.program(batch, keep)
    emu = Emu(cm._pool.blob(), prog.plan.arena)
    for sym, (off, shape, dtype) in prog.inputs.items():
        emu.put(off, np.asarray(inputs[sym]).ravel(), {"i8": 1, "i16": 2, "i32": 4}[dtype])
    emu.run(prog.ops)
    out = {}
    for sym, v in cm._readable(prog, keep).items():
        out[sym] = _apply_view(emu.arena[prog.plan.addresses[v.root]:], v)
    return out
