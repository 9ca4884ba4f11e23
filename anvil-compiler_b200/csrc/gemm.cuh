// int8 x int8 -> int32 GEMMs with the exact requant epilogue (qmatmul / qlinear, anvil/semantics.py:95-103):
//   out[b, i, j] = [lut[. + 128] o] clamp_dtype(((sum_k A[b,i,k] * BT[b,j,k] + bias[j]) * M + 2^(s-1)) >> s)
//
// qgemm_tc:   the sm_100a path. Persistent, warp-specialised: warp 0 issues TMA tile loads (128-byte swizzle)
//             into a STAGES-deep shared-memory ring, warp 1 issues tcgen05.mma kind::i8 (M = 128, N = BN, K = 32
//             per instruction) into one of two TMEM accumulators, warps 2-5 drain the other accumulator with
//             tcgen05.ld and run the requant epilogue, so the epilogue of tile i overlaps the MMAs of tile i+1.
// qgemm_simt: CUDA-core fallback for shapes the TMA path cannot address (K or strides not a multiple of 16
//             bytes) and for tiny problems where launch latency dominates.
//
// int32 accumulation wraps mod 2^32, so it is exact whenever the final sum fits int32 (the contract the oracle
// checks); CHECK re-checks acc, acc + bias, acc*M and acc*M + round against int32 on the device.
#pragma once

#include "common.cuh"

namespace anvil {

struct GemmParams {
  int64_t batch, M, N, K;
  int64_t a_bstride, bt_bstride;       // elements between batches (bt 0 = one weight for every batch)
  int64_t o_bstride, o_rstride;        // output elements between batches / rows
  int64_t o_group, o_gstride;          // rows per output group (0: M) and elements between groups
  int64_t o_cstride;                   // output elements between columns (1: row-major)
  const int8_t *A;
  const int8_t *BT;
  void *out;
  const int8_t *lut;                   // nullptr: no LUT epilogue
  const int32_t *bias;                 // nullptr: no bias
  long long mult;
  int shift;
  int out_bytes;                       // 1 (i8) or 2 (i16)
  int check;
  uint32_t *flags;
  int op_index;
  int64_t m_tiles, n_tiles, tiles;     // tc path tiling (tiles < 2^31)
  uint32_t n_magic, m_magic;           // tile_div: x / n_tiles and x / m_tiles for x < 2^31
  int n_shift, m_shift;
  // fused residual add (unchecked only): out = clamp((res*ma + y*mb + 2^(s2-1)) >> s2) where y is the requant
  // result clamped to y_bytes' range and res is (M, N) row-major with res_bytes per element
  const void *res;
  int res_bytes, y_bytes, shift2;
  int ma, mb;
  // tc path, BN = 256, i8 output through shared-memory staging and TMA tile stores: 1 = row-major; 2 = the
  // head-major transposed layout (element (r, c) at (r / o_group) * o_gstride + c * o_group + r % o_group)
  int tma_store;
  // split output (several linears of one input as one GEMM, tc path, BN = 256): the N columns are chunks of split_c
  // columns, chunk c requantised with (smult[c], sshift[c]); columns below split_r leave row-major through the
  // output map, the rest head-major transposed (group o_group2) through the second output map, column - split_r
  int split_c, split_r;
  int64_t o_group2;
  void *out2;
  int smult[8], sshift[8];
};

// Entry e of a lane's LUT copy (entries 128 bytes apart from `base`) where e is unsigned byte k of w: one dp4a
// forms the address base + 128 e (a byte permute and a shift-add otherwise).
__device__ __forceinline__ int lut_ubyte(uint32_t base, uint32_t w, int k) {
  uint32_t a;
  if (k == 0) asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(a) : "r"(w), "n"(128u), "r"(base));
  else if (k == 1) asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(a) : "r"(w), "n"(128u << 8), "r"(base));
  else if (k == 2) asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(a) : "r"(w), "n"(128u << 16), "r"(base));
  else asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(a) : "r"(w), "n"(128u << 24), "r"(base));
  int v;
  asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

// y -> the fused residual add's result (32-bit exact under the static int32 proof)
template <int OB>
__device__ __forceinline__ int residual_add(int y, int rv, const GemmParams &p) {
  constexpr int lo = OB == 1 ? -128 : -32768, hi = OB == 1 ? 127 : 32767;
  const int rnd2 = p.shift2 ? 1 << (p.shift2 - 1) : 0;
  return min(hi, max(lo, mad_wrap(rv, p.ma, mad_wrap(y, p.mb, rnd2)) >> p.shift2));
}

// One output element from its int32 accumulator (shared by both kernels).
template <bool CHECK>
__device__ __forceinline__ int gemm_epi(int32_t acc, int32_t bias, const GemmParams &p, const int8_t *lut_s,
                                        int lo, int hi, bool &bad) {
  long long a = acc;
  if (p.bias) {
    a += bias;
    if (CHECK) bad |= !fits_i32(a);
  }
  int v = requant64<CHECK>(a, p.mult, p.shift, lo, hi, bad);
  if (lut_s) v = lut_s[v + 128];
  return v;
}

// ------------------------------------------------------------------------------------------------------ SIMT
// 64 x 64 output tile per 256-thread block, 4 x 4 per thread, K staged through shared memory 32 at a time.
template <bool CHECK>
__global__ void __launch_bounds__(256) qgemm_simt_kernel(GemmParams p) {
  __shared__ int32_t As[32][65];
  __shared__ int32_t Bs[32][65];
  __shared__ int8_t lut_s[256];
  const int tid = threadIdx.x;
  if (p.lut)
    for (int i = tid; i < 256; i += 256) lut_s[i] = p.lut[i];
  const int64_t b = blockIdx.z;
  const int64_t i0 = blockIdx.y * 64, j0 = blockIdx.x * 64;
  const int8_t *A = p.A + b * p.a_bstride;
  const int8_t *BT = p.BT + b * p.bt_bstride;
  const int tx = tid & 15, ty = tid >> 4;
  int32_t acc[4][4] = {};
  for (int64_t k0 = 0; k0 < p.K; k0 += 32) {
    for (int e = tid; e < 64 * 32; e += 256) {
      int r = e / 32, kk = e % 32;
      int64_t gi = i0 + r, gj = j0 + r, gk = k0 + kk;
      As[kk][r] = (gi < p.M && gk < p.K) ? (int32_t)A[gi * p.K + gk] : 0;
      Bs[kk][r] = (gj < p.N && gk < p.K) ? (int32_t)BT[gj * p.K + gk] : 0;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      int32_t av[4], bv[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        av[q] = As[kk][ty + 16 * q];
        bv[q] = Bs[kk][tx + 16 * q];
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int r = 0; r < 4; ++r) acc[q][r] += av[q] * bv[r];
    }
    __syncthreads();
  }
  int lo, hi;
  if (p.out_bytes == 1) { lo = -128; hi = 127; } else { lo = -32768; hi = 32767; }
  bool bad = false;
  const int8_t *lt = p.lut ? lut_s : nullptr;
  const int64_t R = p.o_group ? p.o_group : p.M;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    int64_t gi = i0 + ty + 16 * q;
    if (gi >= p.M) continue;
    // the output row's offset, once per row (a 32-bit division when row and group fit)
    const int64_t gq = (gi < (1ll << 31) && R < (1ll << 31)) ? (int64_t)((uint32_t)gi / (uint32_t)R) : gi / R;
    const int64_t orow = b * p.o_bstride + gq * p.o_gstride + (gi - gq * R) * p.o_rstride;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      int64_t gj = j0 + tx + 16 * r;
      if (gj >= p.N) continue;
      int v;
      const int ylo = p.res ? (p.y_bytes == 1 ? -128 : -32768) : lo, yhi = p.res ? (p.y_bytes == 1 ? 127 : 32767) : hi;
      if (CHECK || !p.bias) {
        v = gemm_epi<CHECK>(acc[q][r], p.bias ? p.bias[gj] : 0, p, lt, ylo, yhi, bad);
      } else {                  // bias folded as bias*M + 2^(s-1) (ANVIL_F_BIAS_RND)
        v = clampi(((long long)acc[q][r] * p.mult + p.bias[gj]) >> p.shift, ylo, yhi);
        if (lt) v = lt[v + 128];
      }
      if (p.res) {
        const int64_t ri = gi * p.N + gj;
        const int rv = p.res_bytes == 1 ? (int)reinterpret_cast<const int8_t *>(p.res)[ri]
                                        : (int)reinterpret_cast<const int16_t *>(p.res)[ri];
        const int rnd2 = p.shift2 ? 1 << (p.shift2 - 1) : 0;
        v = min(hi, max(lo, (rv * p.ma + v * p.mb + rnd2) >> p.shift2));
      }
      const int64_t o = orow + gj * p.o_cstride;
      if (p.out_bytes == 1) reinterpret_cast<int8_t *>(p.out)[o] = (int8_t)v;
      else reinterpret_cast<int16_t *>(p.out)[o] = (int16_t)v;
    }
  }
  if (CHECK && __any_sync(0xffffffffu, bad) && bad) raise_flag(p.flags, FLAG_OVERFLOW, p.op_index);
}

// ---------------------------------------------------------------------------------------------- tcgen05 (TC)

constexpr int TC_BM = 128;
constexpr int TC_BK = 128;                // bytes of K per stage = one 128-byte swizzle row
constexpr int TC_EPI_WARPS = 16;          // four warps per TMEM lane quarter, each owning a quarter of the columns
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;   // warp 0 TMA, warp 1 MMA, warps 2-17 epilogue
constexpr int TC_SMEM_RING = 192 * 1024;  // bytes of A/B stages

// PAIR: the CTA is one of a cluster pair sharing 256-row tiles (cta_group::2) and stages BN / 2 rows of B.
template <int BN, bool PAIR = false>
struct TcCfg {
  static constexpr int A_BYTES = TC_BM * TC_BK;
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;
  static constexpr int B_BYTES = B_ROWS * TC_BK;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = TC_SMEM_RING / STAGE_BYTES > 8 ? 8 : TC_SMEM_RING / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;     // two accumulators
  // A LUT epilogue keeps the LUT replicated once per lane as int32 words (32 KB: entry e of lane l at word
  // 32 e + l, conflict-free lookups) in the last LUT_STAGES ring stages, and runs with the rest of the ring.
  static constexpr int LUT_STAGES = (32 * 1024 + STAGE_BYTES - 1) / STAGE_BYTES;
  // Each epilogue warp owns 32 accumulator rows (its TMEM lane quarter) x COLS columns, drained 16 at a time.
  static constexpr int COLS = BN / 4;
  static constexpr int NSC = COLS / 16;
  // After the ring: the output staging (one 32-row x COLS-byte tile per epilogue warp), the barriers full[S],
  // empty[S], tmem_full[2], tmem_empty[2], the TMEM base slot and abort word, and a 64-byte bias staging slot per
  // epilogue warp.
  static constexpr int STG_OFF = STAGES * STAGE_BYTES;
  static constexpr int STG_WARP = 32 * COLS;
  static constexpr int STG_BYTES = TC_EPI_WARPS * STG_WARP;
  static constexpr int BAR_OFF = STG_OFF + STG_BYTES;
  static constexpr int MISC_OFF = BAR_OFF + (2 * STAGES + 4) * 8;
  static constexpr int BST_OFF = MISC_OFF + 16;
  static constexpr int SMEM_BYTES = BST_OFF + TC_EPI_WARPS * 64 + 1024;   // + 1 KB slack to align the ring
};

// Load 32 consecutive int8 / int16 values of a row (vector loads when the chunk is whole and aligned).
__device__ __forceinline__ void load_row32(const void *base, int bytes, int64_t elem, int count, int (&rv)[32]) {
  if (bytes == 1) {
    const int8_t *src = reinterpret_cast<const int8_t *>(base) + elem;
    if (count == 32 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      const uint4 a = reinterpret_cast<const uint4 *>(src)[0], b = reinterpret_cast<const uint4 *>(src)[1];
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int q = 0; q < 32; ++q) rv[q] = (int)(int8_t)(w[q >> 2] >> (8 * (q & 3)));
    } else {
#pragma unroll
      for (int q = 0; q < 32; ++q) rv[q] = q < count ? (int)src[q] : 0;
    }
  } else {
    const int16_t *src = reinterpret_cast<const int16_t *>(base) + elem;
    if (count == 32 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      uint32_t w[16];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint4 a = reinterpret_cast<const uint4 *>(src)[q];
        w[4 * q] = a.x; w[4 * q + 1] = a.y; w[4 * q + 2] = a.z; w[4 * q + 3] = a.w;
      }
#pragma unroll
      for (int q = 0; q < 32; ++q) rv[q] = (int)(int16_t)(w[q >> 1] >> (16 * (q & 1)));
    } else {
#pragma unroll
      for (int q = 0; q < 32; ++q) rv[q] = q < count ? (int)src[q] : 0;
    }
  }
}

// Load 16 consecutive int8 / int16 values of a row (vector loads when the chunk is whole and aligned).
__device__ __forceinline__ void load_row16(const void *base, int bytes, int64_t elem, int count, int (&rv)[16]) {
  if (bytes == 1) {
    const int8_t *src = reinterpret_cast<const int8_t *>(base) + elem;
    if (count == 16 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      const uint4 a = reinterpret_cast<const uint4 *>(src)[0];
      const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
      for (int q = 0; q < 16; ++q) rv[q] = (int)(int8_t)(w[q >> 2] >> (8 * (q & 3)));
    } else {
#pragma unroll
      for (int q = 0; q < 16; ++q) rv[q] = q < count ? (int)src[q] : 0;
    }
  } else {
    const int16_t *src = reinterpret_cast<const int16_t *>(base) + elem;
    if (count == 16 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
      const uint4 a = reinterpret_cast<const uint4 *>(src)[0], b = reinterpret_cast<const uint4 *>(src)[1];
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int q = 0; q < 16; ++q) rv[q] = (int)(int16_t)(w[q >> 1] >> (16 * (q & 1)));
    } else {
#pragma unroll
      for (int q = 0; q < 16; ++q) rv[q] = q < count ? (int)src[q] : 0;
    }
  }
}

// Store 16 consecutive results of one output row: 16-byte vector stores when the whole chunk is in range and
// aligned, element stores otherwise.
template <int OB>
__device__ __forceinline__ void store_row16(typename IntOf<OB>::T *dst, const int (&v)[16], int count) {
  if (count == 16 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    if (OB == 1) {                      // saturating pack: values may arrive unclamped
      uint32_t w[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) w[q] = pack4_sat_s8(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      *reinterpret_cast<uint4 *>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
      uint32_t w[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) w[q] = (uint32_t)(uint16_t)v[2 * q] | ((uint32_t)(uint16_t)v[2 * q + 1] << 16);
      uint4 *d4 = reinterpret_cast<uint4 *>(dst);
      d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
      d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 16; ++q)
      if (q < count) dst[q] = (typename IntOf<OB>::T)(OB == 1 ? min(127, max(-128, v[q])) : v[q]);
  }
}

// Store 32 consecutive results of one output row: 16-byte vector stores when the whole chunk is in range and
// aligned, element stores otherwise.
template <int OB>
__device__ __forceinline__ void store_row32(typename IntOf<OB>::T *dst, const int (&v)[32], int count) {
  if (count == 32 && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
    if (OB == 1) {                      // saturating pack: values may arrive unclamped
      uint32_t w[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) w[q] = pack4_sat_s8(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      uint4 *d4 = reinterpret_cast<uint4 *>(dst);
      d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
      d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
    } else {
      uint32_t w[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) w[q] = (uint32_t)(uint16_t)v[2 * q] | ((uint32_t)(uint16_t)v[2 * q + 1] << 16);
      uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
      for (int q = 0; q < 4; ++q) d4[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    }
  } else {
#pragma unroll
    for (int q = 0; q < 32; ++q)
      if (q < count) dst[q] = (typename IntOf<OB>::T)(OB == 1 ? min(127, max(-128, v[q])) : v[q]);
  }
}

// PAIR (launched as clusters of 2): tile t of the pair covers rows [256 mb, 256 mb + 256); CTA rank r loads and
// drains rows 256 mb + 128 r .. + 128 and stages B rows nb*BN + r*BN/2 .. + BN/2. Both CTAs' loads complete on the
// even CTA's full barrier (its producer expects both halves' bytes), the even CTA's MMA warp issues the 256-row
// MMAs and commits to the empty / accumulator-full barriers of both CTAs, and every epilogue warp of either CTA
// releases an accumulator on the even CTA's barrier. Every wait is bounded as in the single-CTA kernel.
template <int BN, int OB, bool RES, bool PAIR = false>
__global__ void __launch_bounds__(TC_THREADS, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmC2,
                    const GemmParams p) {
  using Cfg = TcCfg<BN, PAIR>;
  constexpr int TMR = PAIR ? 2 * TC_BM : TC_BM;       // rows of one tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align_smem_1024(smem_raw);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + Cfg::BAR_OFF);
  uint64_t *empty = full + Cfg::STAGES;
  uint64_t *tfull = empty + Cfg::STAGES;
  uint64_t *tempty = tfull + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Cfg::MISC_OFF);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + Cfg::MISC_OFF + 4);
  const int nst = p.lut ? Cfg::STAGES - Cfg::LUT_STAGES : Cfg::STAGES;   // ring stages in use
  int32_t *lut_r = reinterpret_cast<int32_t *>(smem + nst * Cfg::STAGE_BYTES);   // entry e of lane l: word 32 e + l
  int32_t *bst = reinterpret_cast<int32_t *>(smem + Cfg::BST_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_ctarank() : 0u;
  const int64_t t_first = PAIR ? (blockIdx.x >> 1) : blockIdx.x, t_step = PAIR ? (gridDim.x >> 1) : gridDim.x;
  const uint32_t nt = (uint32_t)p.n_tiles, mt = (uint32_t)p.m_tiles;
  if (threadIdx.x == 0) {
    for (int i = 0; i < Cfg::STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull[i], 1);
      // single CTA: every epilogue thread arrives; pair: one arrival per epilogue warp of both CTAs
      mbar_init(&tempty[i], PAIR ? 2 * TC_EPI_WARPS : 32 * TC_EPI_WARPS);
    }
    *abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (p.tma_store) prefetch_tmap(&tmC);
    if (p.split_c) prefetch_tmap(&tmC2);
  }
  if (p.lut)
    for (int i = threadIdx.x; i < 32 * 256; i += TC_THREADS) lut_r[i] = p.lut[i >> 5];
  if (warp == 1) {
    if constexpr (PAIR) tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
    else tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) {                           // the peer's barriers are initialised before any remote use
    __syncwarp();
    cluster_sync();
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (int)((p.K + TC_BK - 1) / TC_BK);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0, armed = 0, armed_phase = 0;     // per stage: armed at least once, parity of last arm
      bool ok = true;
      for (int64_t t = t_first; t < p.tiles && ok; t += t_step) {
        const uint32_t rest = tile_div((uint32_t)t, nt, p.n_magic, p.n_shift), nb = (uint32_t)t - rest * nt;
        const uint32_t bb = tile_div(rest, mt, p.m_magic, p.m_shift), mb = rest - bb * mt;
        const int row0 = (int)(mb * TMR + rank * TC_BM);
        const int bz = p.bt_bstride ? (int)bb : 0;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort, p.flags, p.op_index)) { ok = false; break; }
          armed |= 1u << stage;
          armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
          uint8_t *sa = smem + stage * Cfg::STAGE_BYTES;
          uint8_t *sb = sa + Cfg::A_BYTES;
          if constexpr (PAIR) {
            if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::STAGE_BYTES);
            const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
            tma_load_3d_pair(sa, &tmA, kb * TC_BK, row0, (int)bb, fb);
            tma_load_3d_pair(sb, &tmB, kb * TC_BK, (int)(nb * BN + rank * Cfg::B_ROWS), bz, fb);
          } else {
            mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
            tma_load_3d(sa, &tmA, kb * TC_BK, row0, (int)bb, &full[stage]);
            tma_load_3d(sb, &tmB, kb * TC_BK, (int)(nb * BN), bz, &full[stage]);
          }
          if (++stage == nst) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {      // aborted: let every tile load already issued land before the CTA's smem is released
        if constexpr (PAIR) {
          // this CTA's loads complete on the even CTA's barrier: give them a fixed 2 ms to land
          const uint64_t t0 = globaltimer();
          while (globaltimer() - t0 < 2000000ull) {}
        } else {
          for (int s = 0; s < nst; ++s)
            if (armed & (1u << s)) mbar_wait_ns(&full[s], (armed_phase >> s) & 1u, 10000000ull);
        }
      } else if (PAIR) {
        // the MMA commits of the last fills arrive on this CTA's empty barriers: take every stage once more so
        // that none is still in flight when the pair exits
        for (int i = 0; i < nst; ++i) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort, p.flags, p.op_index)) break;
          if (++stage == nst) { stage = 0; phase ^= 1u; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (the even CTA of a pair)
    if ((!PAIR || rank == 0) && elect_one()) {
      constexpr uint32_t idesc = idesc_i8(TMR, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t aphase = 0;
      bool ok = true;
      for (int64_t t = t_first; t < p.tiles && ok; t += t_step) {
        if (!mbar_wait(&tempty[acc], aphase ^ 1u, abort, p.flags, p.op_index)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort, p.flags, p.op_index)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t sb = sa + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < TC_BK / 32; ++k) {
            if constexpr (PAIR)
              mma_i8_pair(d_tmem, sw128_kmajor_desc(sa + 32 * k), sw128_kmajor_desc(sb + 32 * k), idesc,
                          (kb > 0 || k > 0) ? 1u : 0u);
            else
              mma_i8(d_tmem, sw128_kmajor_desc(sa + 32 * k), sw128_kmajor_desc(sb + 32 * k), idesc,
                     (kb > 0 || k > 0) ? 1u : 0u);
          }
          if constexpr (PAIR) mma_commit_pair(&empty[stage]);
          else mma_commit(&empty[stage]);
          if (++stage == nst) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        if constexpr (PAIR) mma_commit_pair(&tfull[acc]);
        else mma_commit(&tfull[acc]);
        if (++acc == 2) { acc = 0; aphase ^= 1u; }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..17)
    // warp w reads TMEM lane quarter (w % 4) and columns [cq*COLS, cq*COLS + COLS), cq = (w - 2) / 4, 16 at a time
    constexpr int NSC = Cfg::NSC;
    const int lane_base = 32 * (warp & 3);
    const int cq = (warp - 2) >> 2;
    int32_t *bslot = bst + (warp - 2) * 16;
    int acc = 0;
    uint32_t aphase = 0;
    constexpr int lo = OB == 1 ? -128 : -32768, hi = OB == 1 ? 127 : 32767;
    const int32_t *lt = p.lut ? lut_r + lane : nullptr;       // this lane's copy: lt[32 e] = lut[e]
    const uint32_t lt_addr = smem_u32(lut_r + lane);            // its shared address: entry e at + 128 e
    // the requant constants (per tile for a split output, whose chunks have their own)
    int m32 = 0, sh = 0, rnd = 0;
    auto set_requant = [&](long long mult, int shift) {
      m32 = (int)mult;
      sh = shift;
      rnd = sh ? 1 << (sh - 1) : 0;
    };
    set_requant(p.mult, p.shift);
    // fused residual with i8 y and i8 residual: both enter biased by 128 (u = x + 128, one byte extract each),
    // and -128 (Ma + Mb) folds into the rounding constant; the sum is formed mod 2^32 and is exact because the
    // static int32 proof bounds the true value
    const bool res_fast = RES && p.res_bytes == 1 && p.y_bytes == 1;
    const int s2 = p.shift2;
    const uint32_t c2 = (uint32_t)(s2 ? 1 << (s2 - 1) : 0) - 128u * ((uint32_t)p.ma + (uint32_t)p.mb);
    // TMA-store epilogue (BN = 256): this warp's 32 rows x 64 columns are packed into its 2 KB staging tile and
    // leave as one tile store, edges clipped by the tensor map. Row-major mode: row r at r*64 bytes, 16-byte chunk
    // c at position c ^ ((r >> 1) & 3) (the 64-byte swizzle of the output map). Transposed mode: 64 column-rows of
    // 32 bytes, lane = byte.
    int tmode = p.tma_store;
    const bool tma_st = tmode != 0;
    uint8_t *stg_w = smem + Cfg::STG_OFF + (warp - 2) * Cfg::STG_WARP;
    uint8_t *stg = stg_w + lane * Cfg::COLS;
    // the folded bias of a sub-chunk's 16 columns (lanes 0-15), loaded one sub-chunk ahead like the residual
    const bool bias_pre = p.bias && !p.check;
    bool bad = false;
    const uint32_t tempty0 = PAIR ? mapa_shared(smem_u32(&tempty[0]), 0) : 0u;
    for (int64_t t = t_first; t < p.tiles; t += t_step) {
      const uint32_t rest = tile_div((uint32_t)t, nt, p.n_magic, p.n_shift), nb = (uint32_t)t - rest * nt;
      const uint32_t bb = tile_div(rest, mt, p.m_magic, p.m_shift), mb = rest - bb * mt;
      const int64_t row0 = (int64_t)mb * TMR + rank * TC_BM;
      const int64_t row = row0 + lane_base + lane;
      const bool row_ok = row < p.M;
      const int64_t cbase = nb * BN + cq * Cfg::COLS;
      const CUtensorMap *omap = &tmC;                 // this tile's output map, column offset and row group
      int64_t ocol = cbase, ogrp = p.o_group;
      if (p.split_c) {
        const int64_t c0t = (int64_t)nb * BN;
        const int ch = (int)(c0t / p.split_c);
        set_requant(p.smult[ch], p.sshift[ch]);
        if (c0t >= p.split_r) {
          tmode = 2;
          omap = &tmC2;
          ocol = cbase - p.split_r;
          ogrp = p.o_group2;
        } else {
          tmode = 1;
        }
      }
      uint4 rcur = make_uint4(0, 0, 0, 0), rnxt = make_uint4(0, 0, 0, 0);
      bool rcur_ok = false, rnxt_ok = false;
      auto prefetch = [&](int sc, uint4 &dst, bool &ok) {
        const int64_t col0 = cbase + sc * 16;
        const int8_t *src = reinterpret_cast<const int8_t *>(p.res) + row * p.N + col0;
        ok = res_fast && row_ok && col0 + 16 <= p.N && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
        if (ok) dst = *reinterpret_cast<const uint4 *>(src);
      };
      auto bias_at = [&](int sc) -> int {
        const int64_t c = cbase + sc * 16 + (lane & 15);
        return c < p.N ? __ldg(p.bias + c) : 0;
      };
      if (RES) prefetch(0, rcur, rcur_ok);
      int bcur = bias_pre ? bias_at(0) : 0, bnxt = 0;
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull[acc], aphase, abort, p.flags, p.op_index))) break;
      tc_fence_after();
      if (tma_st) {                                    // the previous tile's store has read the staging tile
        if (lane == 0) bulk_wait_read();
        __syncwarp();
      }
      using TO = typename IntOf<OB>::T;
      TO *orow = nullptr;                              // direct stores only (the TMA store path needs no row pointer)
      if (!tma_st) {
        const int64_t R = p.o_group ? p.o_group : p.M;
        orow = reinterpret_cast<TO *>(p.out) + (int64_t)bb * p.o_bstride + (row / R) * p.o_gstride +
               (row % R) * p.o_rstride;
      }
#pragma unroll 1
      for (int sc = 0; sc < NSC; ++sc) {
        const int c0 = cq * Cfg::COLS + sc * 16;
        if (RES && sc + 1 < NSC) prefetch(sc + 1, rnxt, rnxt_ok);
        if (bias_pre && sc + 1 < NSC) bnxt = bias_at(sc + 1);
        int32_t r[16];
        tmem_ld16(tmem_base + ((uint32_t)lane_base << 16) + (uint32_t)(acc * BN + c0), r);
        const int64_t col0 = nb * BN + c0;
        if (col0 >= p.N) continue;                     // warp-uniform
        int v[16];
        if (p.check) {
#pragma unroll
          for (int q = 0; q < 16; ++q)
            v[q] = gemm_epi<true>(r[q], (p.bias && col0 + q < p.N) ? p.bias[col0 + q] : 0, p, p.lut, lo, hi, bad);
        } else {
          // the static int32 proof holds: (acc [+ bias]) * M + 2^(s-1) fits int32, so 32-bit wrap-free math is
          // exact; a bias arrives pre-folded as bias*M + 2^(s-1) (ANVIL_F_BIAS_RND)
          int br[16];
          if (p.bias) {
            __syncwarp();
            if (lane < 16) bslot[lane] = bcur;
            __syncwarp();
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int4 b4 = reinterpret_cast<const int4 *>(bslot)[q];
              br[4 * q] = b4.x; br[4 * q + 1] = b4.y; br[4 * q + 2] = b4.z; br[4 * q + 3] = b4.w;
            }
          } else {
#pragma unroll
            for (int q = 0; q < 16; ++q) br[q] = rnd;
          }
          int y[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) y[q] = mad_wrap(r[q], m32, br[q]) >> sh;
          if (!RES) {
            if (OB == 1 && lt) {
              // saturate four at a time, bias the bytes by 128 and look each up in this lane's LUT copy
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t w = pack4_sat_s8(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]) ^ 0x80808080u;
#pragma unroll
                for (int k = 0; k < 4; ++k) v[4 * q + k] = lut_ubyte(lt_addr, w, k);
              }
            } else {
#pragma unroll
              for (int q = 0; q < 16; ++q) v[q] = OB == 1 ? y[q] : min(hi, max(lo, y[q]));   // i8 saturates in the pack
            }
          } else if (rcur_ok) {
            const uint32_t rwv[4] = {rcur.x ^ 0x80808080u, rcur.y ^ 0x80808080u, rcur.z ^ 0x80808080u,
                                     rcur.w ^ 0x80808080u};
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const uint32_t yw = pack4_sat_s8(y[4 * q], y[4 * q + 1], y[4 * q + 2], y[4 * q + 3]) ^ 0x80808080u;
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const int x = (int)(ubyte(rwv[q], k) * (uint32_t)p.ma + ubyte(yw, k) * (uint32_t)p.mb + c2);
                const int o = x >> s2;
                v[4 * q + k] = OB == 1 ? o : min(hi, max(lo, o));
              }
            }
          } else {          // fused residual add: y clamped to its own dtype, then res*Ma + y*Mb requantised
            const int ylo = p.y_bytes == 1 ? -128 : -32768, yhi = p.y_bytes == 1 ? 127 : 32767;
            int rv[16];
            const int cnt = (int)(p.N - col0 < 16 ? p.N - col0 : 16);
            if (row_ok) load_row16(p.res, p.res_bytes, row * p.N + col0, cnt, rv);
#pragma unroll
            for (int q = 0; q < 16; ++q) v[q] = residual_add<OB>(min(yhi, max(ylo, y[q])), row_ok ? rv[q] : 0, p);
          }
        }
        if (tmode == 1) {
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) w[q] = pack4_sat_s8(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
          st_shared_v4(stg + ((sc ^ ((lane >> 1) & 3)) << 4), w[0], w[1], w[2], w[3]);
        } else if (tmode == 2) {
          // column c of the sub-chunk -> staging row sc*16 + c, byte = this lane's row. A 4 x 4 byte transpose
          // inside each quad of lanes (rows 4g..4g+3) gives lane 4g+i, for each word q, column 4q+i of the quad's
          // four rows as one word, stored at offset 4g (the banks 8i + g are all different)
          const int qi = lane & 3;
          const uint32_t sel1 = (qi & 1) ? 0x3715u : 0x6240u, sel2 = qi < 2 ? 0x5410u : 0x3276u;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint32_t w = pack4_sat_s8(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            const uint32_t u = __byte_perm(w, __shfl_xor_sync(0xffffffffu, w, 1), sel1);
            const uint32_t t = __byte_perm(u, __shfl_xor_sync(0xffffffffu, u, 2), sel2);
            st_shared_u32(stg_w + (sc * 16 + 4 * q + qi) * 32 + 4 * (lane >> 2), t);
          }
        } else if (row_ok) {
          const int cnt = (int)(p.N - col0 < 16 ? p.N - col0 : 16);
          if (p.o_cstride == 1) {
            store_row16<OB>(orow + col0, v, cnt);
          } else {            // strided columns (head-major transposed output): lanes = consecutive rows
            TO *dst = orow + col0 * p.o_cstride;
#pragma unroll
            for (int q = 0; q < 16; ++q)
              if (q < cnt) dst[q * p.o_cstride] = (TO)min(hi, max(lo, v[q]));
          }
        }
        rcur = rnxt;
        rcur_ok = rnxt_ok;
        bcur = bnxt;
      }
      tc_fence_before();
      if constexpr (PAIR) {                            // every lane's TMEM loads have completed (wait::ld)
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty0 + 8u * (uint32_t)acc);
      } else {
        mbar_arrive(&tempty[acc]);
      }
      if (++acc == 2) { acc = 0; aphase ^= 1u; }
      if (tma_st) {
        fence_proxy_async();
        __syncwarp();
        if (lane == 0 && row0 + lane_base < p.M) {    // a pair's odd CTA may have no rows left in the last tile
          const int64_t r0 = row0 + lane_base;
          const int c0 = (int)ocol;
          if (tmode == 2) {                            // r0 and the group (T) are below 2^31
            const uint32_t grp = (uint32_t)ogrp, gq = (uint32_t)r0 / grp;
            tma_store_3d(omap, stg_w, (int)((uint32_t)r0 - gq * grp), c0, (int)gq);
          }
          else if (p.batch > 1) tma_store_3d(omap, stg_w, c0, (int)r0, (int)bb);
          else tma_store_2d(omap, stg_w, c0, (int)r0);
          bulk_commit();
        }
      }
    }
    if (tma_st && lane == 0) bulk_wait_all();
    if (p.check && __any_sync(0xffffffffu, bad) && bad) raise_flag(p.flags, FLAG_OVERFLOW, p.op_index);
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (PAIR) {                           // neither CTA's shared memory or barriers are used any more
    __syncwarp();
    cluster_sync();
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
    else tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace anvil
