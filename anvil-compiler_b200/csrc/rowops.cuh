// Memory-bound kernels: lut, lut_mul, add_requant, rmsnorm_int / layernorm_int, softmax_lut, transpose, embed.
//
// All are grid-stride over 16-byte vectors where the data allows it (arena buffers start 256-byte aligned), hold
// the small tables (256 x i8 LUT, 256 x i32 exp LUT) in shared memory, and reduce rows with warp shuffles. Each
// follows the oracle's arithmetic exactly (cited per kernel); CHECK adds the int32 range checks the reference
// raises on, reported through the model's flag words.
#pragma once

#include "common.cuh"

namespace anvil {

__host__ __device__ inline void dt_range(int bytes, int &lo, int &hi) {
  if (bytes == 1) { lo = -128; hi = 127; }
  else if (bytes == 2) { lo = -32768; hi = 32767; }
  else { lo = (int)0x80000000; hi = 0x7fffffff; }
}

// ------------------------------------------------------------------------------------------------------ lut
// table[x + 128] (anvil/semantics.py:87-92)
__global__ void lut_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ table, int8_t *__restrict__ out,
                           int64_t n) {
  __shared__ int8_t t[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) t[i] = table[i];
  __syncthreads();
  const int64_t nv = n / 16;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv; v += stride) {
    uint4 in = reinterpret_cast<const uint4 *>(x)[v];
    uint32_t w[4] = {in.x, in.y, in.z, in.w};
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint32_t o = 0;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        int xv = (int8_t)((w[q] >> (8 * b)) & 0xff);
        o |= ((uint32_t)(uint8_t)t[xv + 128]) << (8 * b);
      }
      w[q] = o;
    }
    reinterpret_cast<uint4 *>(out)[v] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (int64_t i = nv * 16 + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride)
    out[i] = t[x[i] + 128];
}

// ------------------------------------------------------------------------------------------------- lut_mul
// requant(table[x + 128] * y, M, s) (golden.swiglu_lut; anvil/lower/graph_to_tensor.py:297-300)
template <bool CHECK>
__global__ void lut_mul_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ y,
                               const int8_t *__restrict__ table, int8_t *__restrict__ out, int64_t n, long long m,
                               int s, uint32_t *flags, int op_index) {
  __shared__ int8_t t[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) t[i] = table[i];
  __syncthreads();
  bool bad = false;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    long long prod = (long long)t[x[i] + 128] * (long long)y[i];
    out[i] = (int8_t)requant64<CHECK>(prod, m, s, -128, 127, bad);
  }
  if (CHECK && __any_sync(0xffffffffu, bad) && bad) raise_flag(flags, FLAG_OVERFLOW, op_index);
}

// --------------------------------------------------------------------------------------------- add_requant
// clamp((a*Ma + b*Mb + 2^(s-1)) >> s) to the result dtype (anvil/semantics.py:106-115; residual_add for i8)
template <int AB, int BB, int OB, bool CHECK>
__global__ void add_requant_kernel(const void *__restrict__ a_, const void *__restrict__ b_, void *__restrict__ o_,
                                   int64_t n, long long ma, long long mb, int s, uint32_t *flags, int op_index) {
  using TA = typename IntOf<AB>::T;
  using TB = typename IntOf<BB>::T;
  using TO = typename IntOf<OB>::T;
  const TA *a = reinterpret_cast<const TA *>(a_);
  const TB *b = reinterpret_cast<const TB *>(b_);
  TO *o = reinterpret_cast<TO *>(o_);
  int lo, hi;
  dt_range(OB, lo, hi);
  bool bad = false;
  const long long rnd = round_term(s);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  constexpr int V = 8;                        // 8 elements per step: 8 B (i8) or 16 B (i16) per operand
  const int64_t nv = n / V;
  for (int64_t v = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; v < nv; v += stride) {
    TA av[V];
    TB bv[V];
    TO ov[V];
    if (AB == 1) *reinterpret_cast<uint2 *>(av) = reinterpret_cast<const uint2 *>(a)[v];
    else *reinterpret_cast<uint4 *>(av) = reinterpret_cast<const uint4 *>(a)[v];
    if (BB == 1) *reinterpret_cast<uint2 *>(bv) = reinterpret_cast<const uint2 *>(b)[v];
    else *reinterpret_cast<uint4 *>(bv) = reinterpret_cast<const uint4 *>(b)[v];
#pragma unroll
    for (int q = 0; q < V; ++q) {
      long long pa = (long long)av[q] * ma, pb = (long long)bv[q] * mb;
      long long acc = pa + pb, r = acc + rnd;
      if (CHECK) bad |= !fits_i32(pa) | !fits_i32(pb) | !fits_i32(acc) | !fits_i32(r);
      ov[q] = (TO)clampi(r >> s, lo, hi);
    }
    if (OB == 1) reinterpret_cast<uint2 *>(o)[v] = *reinterpret_cast<uint2 *>(ov);
    else reinterpret_cast<uint4 *>(o)[v] = *reinterpret_cast<uint4 *>(ov);
  }
  for (int64_t i = nv * V + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    long long pa = (long long)a[i] * ma, pb = (long long)b[i] * mb;
    long long acc = pa + pb, r = acc + rnd;
    if (CHECK) bad |= !fits_i32(pa) | !fits_i32(pb) | !fits_i32(acc) | !fits_i32(r);
    o[i] = (TO)clampi(r >> s, lo, hi);
  }
  if (CHECK && __any_sync(0xffffffffu, bad) && bad) raise_flag(flags, FLAG_OVERFLOW, op_index);
}

// -------------------------------------------------------------------------------------------------- norms
// rmsnorm_int / rmsnorm_wide (anvil/semantics.py:164-182) and the layernorm_int extension, one warp per row:
//   [CENTER] mean = floor((sum x + d/2) / d), xc = x - mean       (else xc = x)
//   ss = e + sum((xc^2 + 2^(c-1)) >> c);  idx, k = rsqrt_index(ss, n)  (while idx >= n: idx >>= 2, k++)
//   out = clamp_i8(((xc*w*lut[idx])*M + 2^(s+k-1)) >> (s+k) [+ bias])
template <int XB, bool CHECK>
__global__ void norm_kernel(const void *__restrict__ x_, const int8_t *__restrict__ w,
                            const int32_t *__restrict__ lut, const int8_t *__restrict__ bias,
                            int8_t *__restrict__ out, int64_t rows, int d, int n, long long m, int s, int c,
                            long long e, int center, uint32_t *flags, int op_index) {
  using TX = typename IntOf<XB>::T;
  const TX *x = reinterpret_cast<const TX *>(x_);
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  bool bad = false, badidx = false;
  const long long rc = round_term(c);
  for (int64_t row = warp; row < rows; row += nwarps) {
    const TX *xr = x + row * d;
    long long mean = 0;
    if (center) {
      long long sum = 0;
      for (int j = lane; j < d; j += 32) sum += xr[j];
#pragma unroll
      for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      if (CHECK) bad |= !fits_i32(sum);
      long long num = sum + d / 2;                        // floor division by d > 0
      mean = num >= 0 ? num / d : -((-num + d - 1) / d);
    }
    long long ss = 0;
    for (int j = lane; j < d; j += 32) {
      long long xc = (long long)xr[j] - mean;
      long long sq = xc * xc, sr = sq + rc;
      if (CHECK) bad |= !fits_i32(sq) | !fits_i32(sr);
      ss += sr >> c;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    ss += e;
    if (CHECK) bad |= !fits_i32(ss);
    long long idx = ss;
    int k = 0;
    while (idx >= n) { idx >>= 2; ++k; }
    if (idx < 0) { badidx = true; idx = 0; }
    const long long r = lut[idx];
    const int sh = s + k;
    if (sh > 31) bad = true;
    const int shc = sh > 62 ? 62 : sh;
    const long long rnd = round_term(shc > 31 ? 31 : shc);
    int8_t *orow = out + row * d;
    for (int j = lane; j < d; j += 32) {
      long long xc = (long long)xr[j] - mean;
      long long xw = xc * (long long)w[j];
      long long xwr = xw * r;
      long long p = xwr * m, q = p + rnd;
      if (CHECK) bad |= !fits_i32(xw) | !fits_i32(xwr) | !fits_i32(p) | !fits_i32(q);
      long long v = q >> shc;
      if (bias) {
        v += bias[j];
      }
      orow[j] = (int8_t)clampi(v, -128, 127);
    }
  }
  if (CHECK && __any_sync(0xffffffffu, bad) && bad) raise_flag(flags, FLAG_OVERFLOW, op_index);
  if (__any_sync(0xffffffffu, badidx) && badidx) raise_flag(flags, FLAG_INDEX, op_index);
}

// Vectorised form for int8 rows with d % 16 == 0 and d <= 512 * NV, when the static int32 proof holds (no
// device checks): one warp per row, the row, the weights and the bias held in registers as 16-byte vectors
// (NV per lane), one read and one write of the row, 32-bit arithmetic (every intermediate is proven to fit).
__device__ __forceinline__ int sext8(uint32_t w, int q) { return (int)(int8_t)(w >> (8 * q)); }

template <int NV>
__global__ void __launch_bounds__(256) norm_vec_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ w,
                                                       const int32_t *__restrict__ lut,
                                                       const int8_t *__restrict__ bias, int8_t *__restrict__ out,
                                                       int64_t rows, int d, int n, int m, int s, int c, int e,
                                                       int center) {
  const int lane = threadIdx.x & 31;
  const int nvec = d >> 4;
  uint4 wv[NV], bv[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int iv = lane + 32 * v;
    wv[v] = iv < nvec ? reinterpret_cast<const uint4 *>(w)[iv] : make_uint4(0, 0, 0, 0);
    bv[v] = (bias && iv < nvec) ? reinterpret_cast<const uint4 *>(bias)[iv] : make_uint4(0, 0, 0, 0);
  }
  const int rc = c ? 1 << (c - 1) : 0;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t row = warp; row < rows; row += nwarps) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * d);
    uint4 xv[NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int iv = lane + 32 * v;
      xv[v] = iv < nvec ? xr[iv] : make_uint4(0, 0, 0, 0);
    }
    int mean = 0;
    if (center) {
      int sum = 0;
#pragma unroll
      for (int v = 0; v < NV; ++v) {
        const uint32_t ws[4] = {xv[v].x, xv[v].y, xv[v].z, xv[v].w};
#pragma unroll
        for (int q = 0; q < 16; ++q) sum += sext8(ws[q >> 2], q & 3);
      }
      sum = __reduce_add_sync(0xffffffffu, sum);
      // floor((sum + d/2) / d): |sum| <= 128 d, so the offset of 128 d makes the dividend positive
      mean = (int)((unsigned)(sum + d / 2 + 128 * d) / (unsigned)d) - 128;
    }
    int ss = 0;
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      if (lane + 32 * v >= nvec) continue;
      const uint32_t ws[4] = {xv[v].x, xv[v].y, xv[v].z, xv[v].w};
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const int xc = sext8(ws[q >> 2], q & 3) - mean;
        ss += (xc * xc + rc) >> c;
      }
    }
    ss = __reduce_add_sync(0xffffffffu, ss);
    ss += e;
    int k = 0;
    if (ss >= n) {
      // the smallest k with (ss >> 2k) < n: bit lengths give it to within one step
      const int ka = max(0, (32 - __clz(ss) - (32 - __clz(n)) + 1) >> 1);
      k = ka + ((ss >> (2 * ka)) >= n);
    }
    const int r = lut[ss >> (2 * k)];
    const int sh = s + k;
    const int rnd = sh ? 1 << (sh - 1) : 0;
    uint4 *orow = reinterpret_cast<uint4 *>(out + row * d);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const int iv = lane + 32 * v;
      if (iv >= nvec) continue;
      const uint32_t ws[4] = {xv[v].x, xv[v].y, xv[v].z, xv[v].w};
      const uint32_t ww[4] = {wv[v].x, wv[v].y, wv[v].z, wv[v].w};
      const uint32_t bb[4] = {bv[v].x, bv[v].y, bv[v].z, bv[v].w};
      uint32_t o4[4] = {0, 0, 0, 0};
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        const int xc = sext8(ws[q >> 2], q & 3) - mean;
        int y = mad_wrap(mad_wrap(mad_wrap(xc, sext8(ww[q >> 2], q & 3), 0), r, 0), m, rnd) >> sh;
        y += sext8(bb[q >> 2], q & 3);
        y = min(127, max(-128, y));
        o4[q >> 2] |= ((uint32_t)(uint8_t)y) << (8 * (q & 3));
      }
      orow[iv] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
    }
  }
}


// norm_vec for rows of d = 256 * NV8 int8 values (unchecked, static int32 proof). One warp per row, every lane
// NV8 8-byte vectors (lane + 32 v); the weights (as dp2a byte pairs) and the bias held in registers once per
// thread; the next row's vectors loaded before the current row is computed (two rows in flight per warp). Row
// statistics come from dp4a and redux.sync (sum and sum of squares, exact in int32 for d <= 2048); with no
// per-element shift (c == 0) the centered sum of squares is sum(x^2) - 2 mean sum(x) + d mean^2, the same integer.
// Each output element takes one byte permute ({x_q, -mean} as 16-bit halves) and one dp2a for (x_q - mean) * w_q;
// that times r * M is equal mod 2^32 to ((x - mean) * w * r) * M, exact because the proof bounds the true value.
// The launch bounds keep the register budget that gives 5/4/3 (4 without a bias)/2 resident blocks for
// 256/512/768/1024-wide rows.
template <int NV8, bool BIAS>
__global__ void __launch_bounds__(256, NV8 == 1 ? 5 : NV8 == 2 ? 4 : NV8 == 3 ? (BIAS ? 3 : 4) : NV8 == 4 ? 2 : 1)
    norm_row_kernel(const int8_t *__restrict__ x, const int8_t *__restrict__ w,
                                                       const int32_t *__restrict__ lut,
                                                       const int8_t *__restrict__ bias, int8_t *__restrict__ out,
                                                       int64_t rows, int n, int m, int s, int c, int e, int center) {
  constexpr int d = 256 * NV8;
  const int lane = threadIdx.x & 31;
  const int ln = 32 - __clz(n);
  uint32_t wp[4 * NV8];                            // weight pairs {w_2j, w_2j, w_2j+1, w_2j+1} for dp2a
  int br[8 * NV8];
#pragma unroll
  for (int v = 0; v < NV8; ++v) {
    const uint2 w2 = reinterpret_cast<const uint2 *>(w)[lane + 32 * v];
    const uint2 b2 = BIAS ? reinterpret_cast<const uint2 *>(bias)[lane + 32 * v] : make_uint2(0, 0);
#pragma unroll
    for (int q = 0; q < 8; ++q) br[8 * v + q] = sbyte_prmt(q < 4 ? b2.x : b2.y, q & 3);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t b0 = (2 * j) & 3, b1 = b0 + 1;
      wp[4 * v + j] = __byte_perm(j < 2 ? w2.x : w2.y, 0u, b0 | b0 << 4 | b1 << 8 | b1 << 12);
    }
  }
  const int rc = c ? 1 << (c - 1) : 0;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  if (warp >= rows) return;
  const int nr = (int)((rows - 1 - warp) / nwarps) + 1;       // rows of this warp: warp, warp + nwarps, ...
  const int64_t step = nwarps * (d / 8);                        // one warp-stride of rows, in 8-byte vectors
  const uint2 *xp = reinterpret_cast<const uint2 *>(x + warp * d) + lane;
  uint2 *op = reinterpret_cast<uint2 *>(out + warp * d) + lane;

  auto row_out = [&](const uint2 (&xv)[NV8], uint2 *orow) {
    int sx = 0, sxx = 0;
#pragma unroll
    for (int v = 0; v < NV8; ++v) {
      sx = __dp4a((int)xv[v].x, 0x01010101, sx);
      sx = __dp4a((int)xv[v].y, 0x01010101, sx);
      sxx = __dp4a((int)xv[v].x, (int)xv[v].x, sxx);
      sxx = __dp4a((int)xv[v].y, (int)xv[v].y, sxx);
    }
    sx = __reduce_add_sync(0xffffffffu, sx);
    int mean = 0;
    // floor((sx + d/2) / d): |sx| <= 128 d, so the offset of 128 d makes the dividend positive
    if (center) mean = (int)((unsigned)(sx + d / 2 + 128 * d) / (unsigned)d) - 128;
    int ss;
    if (c == 0) {
      sxx = __reduce_add_sync(0xffffffffu, sxx);
      ss = sxx - 2 * mean * sx + d * mean * mean;
    } else {
      ss = 0;
#pragma unroll
      for (int v = 0; v < NV8; ++v)
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int xc = sbyte_prmt(q < 4 ? xv[v].x : xv[v].y, q & 3) - mean;
          ss += (xc * xc + rc) >> c;
        }
      ss = __reduce_add_sync(0xffffffffu, ss);
    }
    ss += e;
    int k = 0;
    if (ss >= n) {
      // the smallest k with (ss >> 2k) < n: bit lengths give it to within one step
      const int ka = max(0, (32 - __clz(ss) - ln + 1) >> 1);
      k = ka + ((ss >> (2 * ka)) >= n);
    }
    const int rm = mad_wrap(lut[ss >> (2 * k)], m, 0);
    const int sh = s + k;
    const int rnd = sh ? 1 << (sh - 1) : 0;
    const uint32_t nm = (uint32_t)(-mean) << 16;
#pragma unroll
    for (int v = 0; v < NV8; ++v) {
      int y[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        // {x_q sign-extended, -mean} as two 16-bit halves, so one dp2a gives (x_q - mean) * w_q
        int a;
        asm("prmt.b32 %0, %1, %2, %3;" : "=r"(a) : "r"(q < 4 ? xv[v].x : xv[v].y), "r"(nm),
            "r"((uint32_t)(q & 3) | (uint32_t)((q & 3) | 8) << 4 | 0x7600u));
        const int t = (q & 1) ? __dp2a_hi(a, (int)wp[4 * v + q / 2], 0) : __dp2a_lo(a, (int)wp[4 * v + q / 2], 0);
        y[q] = mad_wrap(t, rm, rnd) >> sh;
        if (BIAS) y[q] += br[8 * v + q];
      }
      orow[32 * v] = make_uint2(pack4_sat_s8(y[0], y[1], y[2], y[3]), pack4_sat_s8(y[4], y[5], y[6], y[7]));
    }
  };

  // three row buffers in turn: the next two rows' vectors are in flight while the current row is computed
  uint2 xa[NV8], xb[NV8], xc[NV8];
#pragma unroll
  for (int v = 0; v < NV8; ++v) xa[v] = xp[32 * v];
  if (nr > 1) {
#pragma unroll
    for (int v = 0; v < NV8; ++v) xb[v] = xp[step + 32 * v];
  }
  for (int i = 0; i < nr; i += 3) {
    if (i + 2 < nr) {
#pragma unroll
      for (int v = 0; v < NV8; ++v) xc[v] = xp[2 * step + 32 * v];
    }
    row_out(xa, op);
    if (i + 1 >= nr) break;
    if (i + 3 < nr) {
#pragma unroll
      for (int v = 0; v < NV8; ++v) xa[v] = xp[3 * step + 32 * v];
    }
    row_out(xb, op + step);
    if (i + 2 >= nr) break;
    if (i + 4 < nr) {
#pragma unroll
      for (int v = 0; v < NV8; ++v) xb[v] = xp[4 * step + 32 * v];
    }
    row_out(xc, op + 2 * step);
    xp += 3 * step;
    op += 3 * step;
  }
}

// ------------------------------------------------------------------------------------------------ softmax
// softmax_lut (anvil/lower/graph_to_tensor.py:352-398): one warp per row of (batch, T1, T2); kept j <= i when
// causal; m = max(-128, x_j); e_j = lut[x_j - m + 255]; S = sum e_j; p_j = (e_j*one + S/2) / S (floor).
template <int OB, bool CHECK>
__global__ void softmax_kernel(const int8_t *__restrict__ x, const int32_t *__restrict__ lut_g, void *__restrict__ o_,
                               int64_t rows, int t1, int t2, long long one, int causal, uint32_t *flags,
                               int op_index) {
  using TO = typename IntOf<OB>::T;
  TO *o = reinterpret_cast<TO *>(o_);
  __shared__ int32_t lut[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) lut[i] = lut_g[i];
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  bool bad = false;
  // row % t1, carried from row to row (the rows of a warp step by nwarps) instead of a division per row
  const int64_t step_i = nwarps % t1;
  int64_t i = warp % t1;
  for (int64_t row = warp; row < rows; row += nwarps, i = i + step_i >= t1 ? i + step_i - t1 : i + step_i) {
    const int kept = causal ? (int)(i + 1 < t2 ? i + 1 : t2) : t2;
    const int8_t *xr = x + row * t2;
    TO *orow = o + row * t2;
    int mx = -128;
    for (int j = lane; j < kept; j += 32) mx = max(mx, (int)xr[j]);
#pragma unroll
    for (int off = 16; off; off >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    long long tot = 0;
    for (int j = lane; j < kept; j += 32) tot += lut[xr[j] - mx + 255];
#pragma unroll
    for (int off = 16; off; off >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
    if (CHECK) bad |= !fits_i32(tot) | (tot <= 0);
    const long long half = tot / 2;
    const long long den = tot > 0 ? tot : 1;
    for (int j = lane; j < t2; j += 32) {
      long long p = 0;
      if (j < kept) {
        long long eo = (long long)lut[xr[j] - mx + 255] * one;
        long long num = eo + half;
        if (CHECK) bad |= !fits_i32(eo) | !fits_i32(num) | (num < 0);
        p = num >= 0 ? num / den : -((-num + den - 1) / den);
      }
      orow[j] = (TO)p;
    }
  }
  if (CHECK && __any_sync(0xffffffffu, bad) && bad) raise_flag(flags, FLAG_OVERFLOW, op_index);
}

// ---------------------------------------------------------------------------------------------- transpose
// Generic strided gather: out[i0..i5] = x[sum i_d * stride_d], rank <= 6 (anvil/interp/graph.py:76-78).
struct TransposeDims {
  int64_t n[6];
  int64_t st[6];
  int rank;
  int small;                           // total and source span < 2^31: 32-bit index decode by tile_div
  uint32_t mg[6];                      // tile_div magics of n[]
  int sh[6];
};

template <int EB>
__global__ void transpose_kernel(const void *__restrict__ x_, void *__restrict__ o_, TransposeDims td, int64_t total) {
  using T = typename IntOf<EB>::T;
  const T *x = reinterpret_cast<const T *>(x_);
  T *o = reinterpret_cast<T *>(o_);
  if (td.small) {
    // dims past the rank have n = 1 and stride 0: their digit is 0 and they leave the quotient unchanged
    const uint32_t stride = gridDim.x * blockDim.x, tot = (uint32_t)total;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < tot; i += stride) {
      uint32_t rem = i, src = 0;
#pragma unroll
      for (int dd = 5; dd >= 0; --dd) {
        const uint32_t nd = (uint32_t)td.n[dd];
        const uint32_t q = tile_div(rem, nd, td.mg[dd], td.sh[dd]);
        src += (rem - q * nd) * (uint32_t)td.st[dd];
        rem = q;
      }
      o[i] = x[src];
    }
    return;
  }
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += stride) {
    int64_t rem = i, src = 0;
    for (int dd = td.rank - 1; dd >= 0; --dd) {
      int64_t q = rem / td.n[dd];
      src += (rem - q * td.n[dd]) * td.st[dd];
      rem = q;
    }
    o[i] = x[src];
  }
}

// ------------------------------------------------------------------------------------------------- embed
// x[b, t] = residual_add(wte[ids[b, t]], wpe[t], Ma, Mb, s), one warp per token (extension a11).
template <bool CHECK>
__global__ void embed_kernel(const int32_t *__restrict__ ids, const int8_t *__restrict__ wte,
                             const int8_t *__restrict__ wpe, int8_t *__restrict__ out, int64_t rows, int t, int d,
                             int64_t vocab, long long ma, long long mb, int s, uint32_t *flags, int op_index) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = (blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const long long rnd = round_term(s);
  bool bad = false, badidx = false;
  // row % t carried from row to row (the rows of a warp step by nwarps) instead of a division per row
  const int64_t step_pos = nwarps % t;
  int64_t pos = warp % t;
  for (int64_t row = warp; row < rows; row += nwarps, pos = pos + step_pos >= t ? pos + step_pos - t : pos + step_pos) {
    const int64_t id = ids[row];
    int8_t *orow = out + row * d;
    if (id < 0 || id >= vocab) {
      badidx = true;
      for (int j = lane; j < d; j += 32) orow[j] = 0;
      continue;
    }
    const int8_t *a = wte + id * d;
    const int8_t *b = wpe + (int64_t)pos * d;
    for (int j = lane; j < d; j += 32) {
      long long pa = (long long)a[j] * ma, pb = (long long)b[j] * mb;
      long long acc = pa + pb, r = acc + rnd;
      if (CHECK) bad |= !fits_i32(pa) | !fits_i32(pb) | !fits_i32(acc) | !fits_i32(r);
      orow[j] = (int8_t)clampi(r >> s, -128, 127);
    }
  }
  if (CHECK && __any_sync(0xffffffffu, bad) && bad) raise_flag(flags, FLAG_OVERFLOW, op_index);
  if (__any_sync(0xffffffffu, badidx) && badidx) raise_flag(flags, FLAG_INDEX, op_index);
}

}  // namespace anvil
