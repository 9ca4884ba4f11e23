"""CPU oracle (test infrastructure only): scalar loop-nest restatements of the row ops, for cross-checking
oracle.semantics on small shapes.

These follow the reference's two other restatements of the golden arithmetic, element by element in Python ints:
    - the loop-nest lowering anvil/lower/graph_to_tensor.py (matmul :243-266, rmsnorm :319-349, softmax :352-398,
      lut_mul :297-300, add_requant :303-307), with requant as the ISA idiom anvil/backend/idioms.py:150-163
      (clamp_i8((acc*m + rnd) >>> s)) and rsqrt_index as the counted, branch-free form of anvil/codegen/lower.py:
      791-803 (each trip: f = (idx >= n); k += f; idx >>= 2f);
    - the Vortex-V codegen anvil/vortexv/codegen.py:10-13,480-615, whose requant is rqs of the exact 64-bit product,
      clamp((acc*M + 2^(s-1)) >> s), and whose softmax divides (e*one + S/2) by S unsigned.
They raise nothing: callers use them only where oracle.semantics accepted the inputs, and compare results.
"""
from __future__ import annotations

import numpy as np

RSQRT_TRIPS = 16            # enough trips for any int32 sum and any LUT of >= 2 entries


def _clamp(v, lo=-128, hi=127):
    return lo if v < lo else hi if v > hi else v


def requant_idiom(acc, m, s, lo=-128, hi=127):
    """anvil/backend/idioms.py:150-163: clamp((acc*m + rnd) >> s), rnd = 2^(s-1) or 0."""
    rnd = (1 << (s - 1)) if s else 0
    return _clamp((int(acc) * int(m) + rnd) >> s, lo, hi)


def rqs(x64, s):
    """anvil/vortexv/codegen.py:10-13: Vortex-V mlacc.rqs on an exact 64-bit product."""
    return _clamp((int(x64) + ((1 << (s - 1)) if s else 0)) >> s)


def rsqrt_index_counted(ss, n):
    """anvil/codegen/lower.py:791-803, branch-free trips."""
    idx, k = int(ss), 0
    for _ in range(RSQRT_TRIPS):
        f = 1 if idx - (n - 1) > 0 else 0
        k += f
        idx >>= 2 * f
    return idx, k


def qmatmul_loops(a, b, m, s, lut=None, lo=-128, hi=127, bias=None):
    """2-D (M, K) @ (K, N): acc over k, requant, optional LUT gather (graph_to_tensor.py:243-266)."""
    a, b = np.asarray(a), np.asarray(b)
    M, K = a.shape
    N = b.shape[1]
    out = np.zeros((M, N), dtype=np.int64)
    for i in range(M):
        for j in range(N):
            acc = 0
            for k in range(K):
                acc += int(a[i, k]) * int(b[k, j])
            if bias is not None:
                acc += int(bias[j])
            r = requant_idiom(acc, m, s, lo, hi)
            out[i, j] = r if lut is None else int(lut[r + 128])
    return out


def softmax_loops(x, lut, one, causal):
    """Three stages per row as graph_to_tensor.py:352-398: max (init -128), sum of lut[x - max + 255] over kept j,
    then (e*one + S//2) // S, masked entries 0. x is (T1, T2)."""
    x = np.asarray(x)
    t1, t2 = x.shape
    out = np.zeros((t1, t2), dtype=np.int64)
    for i in range(t1):
        kept = [j for j in range(t2) if (j <= i or not causal)]
        mx = -128
        for j in kept:
            mx = max(mx, int(x[i, j]))
        tot = 0
        for j in kept:
            tot += int(lut[int(x[i, j]) - mx + 255])
        for j in kept:
            e = int(lut[int(x[i, j]) - mx + 255])
            out[i, j] = (e * one + tot // 2) // tot
    return out


def rmsnorm_loops(x, w, lut, m, s, c=0, e=0):
    """Stat then norm stage per row (graph_to_tensor.py:319-349; vortexv/codegen.py:480-543). x is (T, D)."""
    x = np.asarray(x)
    t, d = x.shape
    n = len(lut)
    out = np.zeros((t, d), dtype=np.int64)
    for i in range(t):
        ss = 0
        for j in range(d):
            sq = int(x[i, j]) * int(x[i, j])
            if c:
                sq = (sq + (1 << (c - 1))) >> c
            ss += sq
        ss += e
        idx, k = rsqrt_index_counted(ss, n)
        r = int(lut[idx])
        for j in range(d):
            out[i, j] = rqs(int(x[i, j]) * int(w[j]) * r * int(m), s + k)      # vortexv: x*w, then *(r*M), rqs
    return out


def lut_mul_loops(x, y, table, m, s):
    x, y = np.asarray(x).ravel(), np.asarray(y).ravel()
    return np.array([requant_idiom(int(table[int(a) + 128]) * int(b), m, s) for a, b in zip(x, y)])


def add_requant_loops(a, b, ma, mb, s, lo=-128, hi=127):
    """graph_to_tensor.py:303-307 / _requant :269-278: (a*Ma + b*Mb) requantized with M = 1."""
    a, b = np.asarray(a).ravel(), np.asarray(b).ravel()
    return np.array([requant_idiom(int(p) * int(ma) + int(q) * int(mb), 1, s, lo, hi) for p, q in zip(a, b)])
