"""Integer identities the CUDA kernels rely on, restated in Python and checked exhaustively or on dense samples
against the plain definitions (CPU). Each test names the kernel code that uses the identity.

- norm_row_kernel / norm_vec_kernel (rowops.cuh): the rsqrt-table index k, the smallest k with (ss >> 2k) < n,
  in closed form from bit lengths instead of the shift loop of the reference's semantics
  (anvil/semantics.py, rmsnorm: while idx >= n: idx >>= 2; k += 1), and floor((sum + d/2) / d) by an unsigned
  division after a 128 d offset.
- tile_div (common.cuh) with the host's div_magic (anvil_abi.cu): x / d for 0 <= x < 2^31 as a 32 x 32 -> high
  32 multiply and a shift.
- ceil_pow2_div (attention.cuh): ceil(2^(31 + lg) / S) from a correctly rounded double quotient and two exact
  64-bit checks; and the pass-B division floor(n / S) = umulhi(n, m) >> (lg - 1) it feeds.
"""
import random

import numpy as np


def _k_loop(ss, n):
    idx, k = ss, 0
    while idx >= n:
        idx >>= 2
        k += 1
    return k


def _k_closed(ss, n):
    if ss < n:
        return 0
    ka = max(0, (ss.bit_length() - n.bit_length() + 1) >> 1)
    return ka + int((ss >> (2 * ka)) >= n)


def test_rsqrt_index_closed_form_equals_the_shift_loop():
    rng = random.Random(0)
    ns = list(range(1, 300)) + [511, 512, 513, 1023, 1024, 4095, 4096, 65536, 2 ** 20, 2 ** 30, 2 ** 31 - 1]
    for n in ns:
        sss = list(range(0, 3000, 7)) + [rng.randrange(0, 2 ** 31) for _ in range(300)]
        sss += [2 ** j + e for j in range(31) for e in (-1, 0, 1) if 0 <= 2 ** j + e < 2 ** 31]
        for ss in sss:
            assert _k_closed(ss, n) == _k_loop(ss, n), (ss, n)


def test_floor_mean_by_offset_unsigned_division():
    for d in (32, 64, 256, 400, 768, 1024, 2048):
        for s in list(range(-128 * d, -128 * d + 50)) + list(range(127 * d - 50, 127 * d + 1)) + \
                [random.Random(d).randrange(-128 * d, 127 * d + 1) for _ in range(2000)]:
            num = s + d // 2
            want = num // d                                   # Python floors
            got = (num + 128 * d) // d - 128                  # dividend positive: unsigned division
            assert got == want, (d, s)


def _div_magic(d):
    if d <= 1:
        return 0, 0
    lg = (d - 1).bit_length()                                 # ceil(log2 d)
    return ((1 << (31 + lg)) + d - 1) // d, lg - 1


def _tile_div(x, d, m, s):
    return x if d == 1 else ((x * m) >> 32) >> s


def test_tile_div_by_host_magic_equals_floor_division():
    rng = random.Random(1)
    ds = list(range(1, 2000)) + [rng.randrange(1, 2 ** 31) for _ in range(1000)]
    ds += [2 ** k + e for k in range(1, 31) for e in (-1, 0, 1)]
    for d in ds:
        m, s = _div_magic(d)
        assert m < 2 ** 32
        for x in [0, 1, d - 1, d, d + 1, 2 ** 31 - 1, 2 ** 31 - d] + [rng.randrange(0, 2 ** 31) for _ in range(100)]:
            if 0 <= x < 2 ** 31:
                assert _tile_div(x, d, m, s) == x // d, (x, d)


def _ceil_pow2_div(S, lg):
    n = 1 << (31 + lg)
    m = int(float(n) / float(S)) + 1                          # IEEE double quotient, truncated, + 1
    if (m - 1) * S >= n:
        m -= 1
    if m * S < n:
        m += 1
    return m


def test_ceil_pow2_div_equals_the_exact_ceiling_and_divides_exactly():
    rng = random.Random(2)
    Ss = list(range(2, 50000)) + [rng.randrange(2, 2 ** 31) for _ in range(50000)]
    Ss += [2 ** k + e for k in range(1, 31) for e in (-2, -1, 0, 1, 2) if 2 <= 2 ** k + e < 2 ** 31]
    for S in Ss:
        lg = (S - 1).bit_length()
        m = _ceil_pow2_div(S, lg)
        assert m == -(-(1 << (31 + lg)) // S) and m < 2 ** 32, S
    # the pass-B division it feeds: floor(n / S) = umulhi(n, m) >> (lg - 1) for 0 <= n < 2^31
    for S in [2, 3, 5, 127, 1000, 16384, 2 ** 20 + 7, 2 ** 24 - 1, 2 ** 30 + 3]:
        lg = (S - 1).bit_length()
        m = _ceil_pow2_div(S, lg)
        ns = np.concatenate([np.arange(0, 5000), np.array([rng.randrange(0, 2 ** 31) for _ in range(5000)]),
                             np.array([2 ** 31 - 1, S * 7 - 1, S * 7, S * 7 + 1])]).astype(object)
        for n in ns:
            if 0 <= n < 2 ** 31:
                assert ((n * m) >> 32) >> (lg - 1) == n // S, (n, S)



def _div_magic(d):
    if d <= 1:
        return 0, 0
    l = (d - 1).bit_length()
    return ((1 << (31 + l)) + d - 1) // d, l - 1


def _tile_div(x, d, m, s):
    return x if d == 1 else (x * m >> 32) >> s


def test_attention_work_blocks_cover_every_item_once():
    """attn_tile (attention.cuh) with the host's block size (anvil_abi.cu prepare_attention): the items
    0 .. B*H*nqt - 1 map one to one onto (batch-head, query tile) pairs, heaviest tile first inside each block of
    hb pairs, for full and partial last blocks."""
    for BH, nqt, sms in [(768, 8, 148), (24, 8, 148), (5, 3, 148), (64, 1, 148), (37, 8, 148), (1, 1, 148)]:
        grid = min(BH * nqt, sms)
        hb = min(max(1, (2 * grid + nqt // 2) // nqt), BH)
        last = BH - (BH - 1) // hb * hb
        bm, bs = _div_magic(hb * nqt)
        hm, hs = _div_magic(hb)
        lm, ls = _div_magic(last)
        seen = set()
        for t in range(BH * nqt):
            blk = _tile_div(t, hb * nqt, bm, bs)
            wi = t - blk * hb * nqt
            base = blk * hb
            heads = last if base + hb > BH else hb
            r = _tile_div(wi, heads, lm, ls) if base + hb > BH else _tile_div(wi, heads, hm, hs)
            assert r == wi // heads
            bh, qt = base + wi - r * heads, nqt - 1 - r
            assert 0 <= bh < BH and 0 <= qt < nqt
            seen.add((bh, qt))
        assert len(seen) == BH * nqt



def _dp4a_s32_u32(a, b, c):
    """PTX dp4a.s32.u32: the four bytes of a signed, of b unsigned, products summed into c (mod 2^32)."""
    tot = c
    for i in range(4):
        x = (a >> (8 * i)) & 255
        x = x - 256 if x >= 128 else x
        tot += x * ((b >> (8 * i)) & 255)
    return tot & 0xFFFFFFFF


def test_lut_address_by_dp4a():
    """attention.cuh lut_byte: dp4a.s32.u32(w, stride << 8q, base) is base + stride * (signed byte q of w), the
    shared address of that byte's exp-LUT entry, for both entry strides the kernel uses (32 and 128 bytes)."""
    rng = random.Random(11)
    for stride in (32, 128):
        for _ in range(2000):
            w = rng.randrange(0, 1 << 32)
            base = rng.randrange(16384, 1 << 18)
            for q in range(4):
                x = (w >> (8 * q)) & 255
                x = x - 256 if x >= 128 else x
                assert _dp4a_s32_u32(w, stride << (8 * q), base) == base + stride * x
