// Fused causal attention with Anvil's integer softmax, scores kept on chip:
//   scores = requant(q . k^T, M1, s1)                                  (qmatmul, anvil/semantics.py:95-103)
//   p      = softmax_lut(scores, exp_lut, one, causal)                  (anvil/lower/graph_to_tensor.py:352-398)
//   o      = requant(p @ v, M2, s2), written straight into the merged-heads layout (b, t, h*hd + d)
//
// Persistent: one CTA per SM walks the (batch, head, 128-query tile) work items, heaviest causal tiles first, in a
// boustrophedon order over the CTAs. The exp LUT, the TMEM allocation and the barriers are set up once per CTA.
// Warp roles:
//   warp 0     TMA: per tile the Q tile (one buffer, reloaded once the tile's score MMAs are done) and the K tiles
//              (128 keys x hd) through a KS-deep ring
//   warp 18    TMA: the V^T slabs (hd x 128 keys, from the head-major transposed V the v-projection GEMM writes)
//              through a VS-deep ring
//   warp 1     tcgen05.mma kind::i8: S_j = Q K_j^T into one of NSB TMEM score buffers (128 x 128 int32 each); the
//              next tile's first NSB score MMAs are issued before this tile's P V MMAs; O = sum_j P_j V_j slab by
//              slab as the softmax warps finish each slab's probabilities, into a separate TMEM region (128 x hd)
//   warps 2-17 four threads per query row, each owning a 32-column part of every 128-key slab: drain S_j from
//              TMEM, requant to int8, track the partial row max, store into the P slab j in shared memory (the
//              128-byte-swizzled K-major layout the P @ V MMA reads) once the previous tile's P V MMA has read it;
//              then the previous tile's O epilogue (TMEM -> requant -> global, off the tile boundary); combine the
//              row max across the four parts, then the two exact softmax passes (partial sums of exp_lut combined
//              the same way, then (e*one + S/2) / S as a multiply by a per-row invariant-divisor magic number)
// The whole score row (up to 1024 keys, int8) stays in shared memory, so the row max and row sum are exact before
// any probability is formed, as the reference's three-stage loop nest requires; an online (rescaled) softmax
// would not be bit-exact.
#pragma once

#include "common.cuh"

namespace anvil {

struct AttnParams {
  int B, H, T1, T2, nqt;
  int64_t o_bs, o_rs;                  // out element (b, t, h*hd + d) = b*o_bs + t*o_rs + h*hd + d
  int8_t *out;
  const int32_t *lut;                  // 256 x i32 exp LUT
  long long m1, m2;
  int s1, s2, one, causal;
  uint32_t *flags;
  int op_index;
  uint32_t bh_magic, h_magic;          // tile_div by B*H and by H (work-item decode)
  int bh_shift, h_shift;
  // work items come in blocks of hb (batch, head) pairs x nqt query tiles: tile_div by hb * nqt, by hb and by the
  // head count of the last, partial block (hb_last)
  int hb, hb_last;
  uint32_t blk_magic, hb_magic, last_magic;
  int blk_shift, hb_shift, last_shift;
};

template <int HD>
struct AttnCfg {
  static constexpr int KS = HD == 64 ? 3 : 2;            // K-tile ring slots
  static constexpr int VS = HD == 64 ? 3 : 2;            // V^T-slab ring slots
  static constexpr int LUT_COPIES = HD == 64 ? 32 : 8;  // exp LUT replicated per lane: conflict-free lookups
  static constexpr int Q_BYTES = 128 * HD;
  static constexpr int T_BYTES = 128 * HD;              // a K tile (128 keys x hd) or a V^T slab (hd x 128 keys)
  static constexpr int MAX_SLABS = 8;                   // T2 <= 1024
  static constexpr int P_SLAB = 128 * 128;
  static constexpr int NSB = 3;                         // score buffers in TMEM (128 columns each)
  static constexpr int O_COL = NSB * 128;               // the O accumulator (hd columns) after them
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + KS * T_BYTES;
  static constexpr int OFF_P = OFF_V + VS * T_BYTES;
  static constexpr int OFF_LUT = OFF_P + MAX_SLABS * P_SLAB;
  static constexpr int OFF_RED = OFF_LUT + 1024 * LUT_COPIES;       // [2][4][128] int32: row max, row sum partials
  static constexpr int OFF_BAR = OFF_RED + 4096;
  static constexpr int NBAR = 2 + 2 * KS + 2 * VS + 2 * NSB + 2 * MAX_SLABS + 1;
  static constexpr int OFF_MISC = OFF_BAR + NBAR * 8;
  static constexpr int SMEM_BYTES = OFF_MISC + 16 + 1024;
  // Q / K tiles: rows of HD bytes. 64-byte rows use the 64-byte swizzle (8-row atoms of 512 B), 128-byte rows
  // the 128-byte swizzle (1024 B atoms); the descriptor layout types are 4 and 2.
  static constexpr uint32_t QK_LAYOUT = HD == 64 ? 4u : 2u;
  static constexpr uint32_t QK_SBO = HD == 64 ? 512u : 1024u;
};

__device__ __forceinline__ uint64_t kmajor_desc(uint32_t smem_addr, uint32_t layout, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)(sbo >> 4) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

__device__ __forceinline__ void tma_load_4d(void *smem_dst, const CUtensorMap *map, int x, int y, int z, int w,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(void *smem_dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}


// Entry x of this lane's copy of the replicated exp LUT, whose entry 0 sits at shared address `base` (entries
// COPIES words apart): one shift-add and one 32-bit shared load. The table does not change while the softmax passes
// read it (it is written once, before the block-wide barrier that starts the kernel), so the load needs no ordering.
template <int COPIES>
__device__ __forceinline__ int lut_at(uint32_t base, int x) {
  int v;
  asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(base + (uint32_t)(x * (4 * COPIES))));
  return v;
}

// Entry x of that copy where x is signed byte Q of the word w: one dp4a forms the address base + x * 4 * COPIES
// (w's bytes signed, the selector's unsigned, only byte Q of it non-zero), replacing a byte permute and a
// shift-add on the ALU pipe, the softmax passes' busiest.
template <int COPIES, int Q>
__device__ __forceinline__ int lut_byte(uint32_t base, uint32_t w) {
  static_assert(4 * COPIES <= 255, "the entry stride must fit the selector byte");
  uint32_t a;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(a) : "r"(w), "n"((4u * COPIES) << (8 * Q)), "r"(base));
  int v;
  asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}

template <int COPIES>
__device__ __forceinline__ int lut_byte_q(uint32_t base, uint32_t w, int q) {
  return q == 0 ? lut_byte<COPIES, 0>(base, w) : q == 1 ? lut_byte<COPIES, 1>(base, w)
       : q == 2 ? lut_byte<COPIES, 2>(base, w) : lut_byte<COPIES, 3>(base, w);
}

// byte offset of 16-byte chunk `ch` (0..7) of row `r` (0..127) inside one 128 x 128 P slab (SW128 K-major)
__device__ __forceinline__ int pslab_off(int r, int ch) { return (r >> 3) * 1024 + (r & 7) * 128 + ((ch ^ (r & 7)) << 4); }

constexpr int ATTN_SOFTMAX_THREADS = 512;                 // 16 warps: 4 threads per query row
constexpr int ATTN_THREADS = 64 + ATTN_SOFTMAX_THREADS + 32;   // + warp 18, the V^T producer

// One work item: (batch, head) and a 128-query tile. Items come in blocks of hb (batch, head) pairs (the last
// block may hold fewer); inside a block the query tiles go heaviest causal tile first, the pairs fastest. A
// block's items run within a few rounds of the persistent CTAs, so the K tiles and V^T slabs its pairs share are
// read from HBM once and then from L2, while the CTAs of one round still see tiles of equal or neighbouring weight.
struct AttnTile {
  int b, h, bh, q0, nkv;
};

__device__ __forceinline__ AttnTile attn_tile(const AttnParams &p, int t) {
  AttnTile w;
  const uint32_t per_blk = (uint32_t)(p.hb * p.nqt);
  const uint32_t blk = tile_div((uint32_t)t, per_blk, p.blk_magic, p.blk_shift);
  const uint32_t wi = (uint32_t)t - blk * per_blk;
  const int base = (int)blk * p.hb;
  const bool last = base + p.hb > p.B * p.H;
  const uint32_t heads = last ? (uint32_t)p.hb_last : (uint32_t)p.hb;
  const uint32_t r = last ? tile_div(wi, heads, p.last_magic, p.last_shift) : tile_div(wi, heads, p.hb_magic, p.hb_shift);
  const int qt = p.nqt - 1 - (int)r;
  w.bh = base + (int)(wi - r * heads);
  w.b = (int)tile_div((uint32_t)w.bh, (uint32_t)p.H, p.h_magic, p.h_shift);
  w.h = w.bh - w.b * p.H;
  w.q0 = qt * 128;
  const int kv_end = p.causal ? min(p.T2, w.q0 + 128) : p.T2;
  w.nkv = (kv_end + 127) / 128;
  return w;
}

// The k-th work item of this CTA: rounds of gridDim.x items, alternating direction (boustrophedon), so the CTAs
// that take the heavier end of one round take the lighter end of the next. -1 past the end.
__device__ __forceinline__ int attn_item(int k, int ntiles) {
  const int g = (int)gridDim.x, c = (int)blockIdx.x;
  const int t = k * g + ((k & 1) ? g - 1 - c : c);
  return t < ntiles ? t : -1;
}

// ceil(2^(31 + lg) / S) for 2 <= S < 2^31 and lg = ceil(log2 S) (below 2^32): the correctly rounded double quotient
// is within 2^-21 of the true one, so its truncation + 1 is the ceiling or one off it, and the two exact 64-bit
// checks below settle which. Cheaper, once per row and tile, than a 64-bit integer division.
__device__ __forceinline__ unsigned ceil_pow2_div(int S, int lg) {
  const unsigned long long N = 1ull << (31 + lg), s = (unsigned long long)S;
  unsigned long long m = (unsigned long long)((double)N / (double)S) + 1ull;
  if ((m - 1ull) * s >= N) --m;
  if (m * s < N) ++m;
  return (unsigned)m;
}

template <int HD>
__global__ void __launch_bounds__(ATTN_THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                const __grid_constant__ CUtensorMap mapV, const AttnParams p) {
  using Cfg = AttnCfg<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align_smem_1024(smem_raw);
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Cfg::OFF_BAR);
  uint64_t *qfull = bars, *qempty = bars + 1;
  uint64_t *kfull = bars + 2, *kempty = kfull + Cfg::KS;
  uint64_t *vfull = kempty + Cfg::KS, *vempty = vfull + Cfg::VS;
  uint64_t *sfull = vempty + Cfg::VS, *sempty = sfull + Cfg::NSB;
  uint64_t *pslab = sempty + Cfg::NSB;     // pslab[j]: P slab j holds probabilities (512 softmax arrivals)
  uint64_t *pfree = pslab + Cfg::MAX_SLABS;  // pfree[j]: the P V MMA has read P slab j (committed by the MMA)
  uint64_t *ofull = pfree + Cfg::MAX_SLABS;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + Cfg::OFF_MISC);
  volatile int *abort = reinterpret_cast<volatile int *>(smem + Cfg::OFF_MISC + 4);
  int32_t *lut = reinterpret_cast<int32_t *>(smem + Cfg::OFF_LUT);   // entry i of copy c at word i*COPIES + c
  uint8_t *pbuf = smem + Cfg::OFF_P;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = p.B * p.H * p.nqt;

  if (threadIdx.x == 0) {
    mbar_init(qfull, 1);
    mbar_init(qempty, 1);
    for (int i = 0; i < Cfg::KS; ++i) { mbar_init(&kfull[i], 1); mbar_init(&kempty[i], 1); }
    for (int i = 0; i < Cfg::VS; ++i) { mbar_init(&vfull[i], 1); mbar_init(&vempty[i], 1); }
    for (int i = 0; i < Cfg::NSB; ++i) { mbar_init(&sfull[i], 1); mbar_init(&sempty[i], ATTN_SOFTMAX_THREADS); }
    for (int i = 0; i < Cfg::MAX_SLABS; ++i) { mbar_init(&pslab[i], ATTN_SOFTMAX_THREADS); mbar_init(&pfree[i], 1); }
    mbar_init(ofull, 1);
    *abort = 0;
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 64 * Cfg::LUT_COPIES; i += blockDim.x) {
    const int32_t e = __ldg(p.lut + (4 * i) / Cfg::LUT_COPIES);
    reinterpret_cast<int4 *>(lut)[i] = make_int4(e, e, e, e);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA: Q and the K tiles
    if (elect_one()) {
      prefetch_tmap(&mapQ);
      prefetch_tmap(&mapK);
      bool ok = true;
      uint32_t gk = 0;
      for (int k = 0, t; ok && (t = attn_item(k, ntiles)) >= 0; ++k) {
        const AttnTile w = attn_tile(p, t);
        if (!mbar_wait_idle(qempty, (k & 1) ^ 1, abort, p.flags, p.op_index)) { ok = false; break; }
        mbar_arrive_expect_tx(qfull, Cfg::Q_BYTES);
        // query rows q0 + 32 b + i go to TMEM lane 32 (b ^ flip) + i (flip = 3 on odd items of this CTA)
        const int flip = (k & 1) * 3;
#pragma unroll
        for (int b = 0; b < 4; ++b)
          tma_load_4d(smem + Cfg::OFF_Q + (b ^ flip) * (Cfg::Q_BYTES / 4), &mapQ, 0, w.h, w.q0 + 32 * b, w.b, qfull);
        for (int j = 0; j < w.nkv; ++j, ++gk) {
          const int st = gk % Cfg::KS;
          if (!mbar_wait_idle(&kempty[st], ((gk / Cfg::KS) & 1) ^ 1, abort, p.flags, p.op_index)) { ok = false; break; }
          mbar_arrive_expect_tx(&kfull[st], Cfg::T_BYTES);
          tma_load_4d(smem + Cfg::OFF_K + st * Cfg::T_BYTES, &mapK, 0, w.h, j * 128, w.b, &kfull[st]);
        }
      }
      if (!ok) {              // aborted: let the copies already issued land before the CTA exits
        mbar_wait_ns(qfull, 0, 10000000ull);
        mbar_wait_ns(qfull, 1, 10000000ull);
        for (int s2 = 0; s2 < Cfg::KS; ++s2) {
          mbar_wait_ns(&kfull[s2], 0, 10000000ull);
          mbar_wait_ns(&kfull[s2], 1, 10000000ull);
        }
      }
    }
  } else if (warp == 2 + ATTN_SOFTMAX_THREADS / 32) {
    // ------------------------------------------------------------------ TMA: the V^T slabs
    if (elect_one()) {
      prefetch_tmap(&mapV);
      bool ok = true;
      uint32_t gv = 0;
      for (int k = 0, t; ok && (t = attn_item(k, ntiles)) >= 0; ++k) {
        const AttnTile w = attn_tile(p, t);
        for (int j = 0; j < w.nkv; ++j, ++gv) {
          const int st = gv % Cfg::VS;
          if (!mbar_wait_idle(&vempty[st], ((gv / Cfg::VS) & 1) ^ 1, abort, p.flags, p.op_index)) { ok = false; break; }
          mbar_arrive_expect_tx(&vfull[st], Cfg::T_BYTES);
          tma_load_2d(smem + Cfg::OFF_V + st * Cfg::T_BYTES, &mapV, j * 128, w.bh * HD, &vfull[st]);
        }
      }
      if (!ok) {
        for (int s2 = 0; s2 < Cfg::VS; ++s2) {
          mbar_wait_ns(&vfull[s2], 0, 10000000ull);
          mbar_wait_ns(&vfull[s2], 1, 10000000ull);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idesc_qk = idesc_i8(128, 128);
      constexpr uint32_t idesc_pv = idesc_i8(128, HD);
      const uint32_t sq = smem_u32(smem + Cfg::OFF_Q);
      uint32_t gk = 0, gv = 0, gs = 0;
      uint32_t pph = 0;                 // bit j: parity of pslab[j]'s next phase (a tile completes slabs 0..nkv-1)
      // S = Q K_j^T for the next K tile into the next S buffer (the tile's Q is resident)
      auto issue_s = [&]() -> bool {
        const int sb = gs % Cfg::NSB, st = gk % Cfg::KS;
        if (!mbar_wait_idle(&sempty[sb], ((gs / Cfg::NSB) & 1) ^ 1, abort, p.flags, p.op_index)) return false;
        if (!mbar_wait_idle(&kfull[st], (gk / Cfg::KS) & 1, abort, p.flags, p.op_index)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + Cfg::OFF_K + st * Cfg::T_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 32; ++kk)
          mma_i8(tmem + sb * 128, kmajor_desc(sq + 32 * kk, Cfg::QK_LAYOUT, Cfg::QK_SBO),
                 kmajor_desc(sk + 32 * kk, Cfg::QK_LAYOUT, Cfg::QK_SBO), idesc_qk, kk > 0 ? 1u : 0u);
        mma_commit(&kempty[st]);
        mma_commit(&sfull[sb]);
        ++gk;
        ++gs;
        return true;
      };
      bool ok = true;
      int t = attn_item(0, ntiles);
      if (t >= 0) {                     // the first tile's first NSB score MMAs
        const AttnTile w = attn_tile(p, t);
        ok = mbar_wait_idle(qfull, 0, abort, p.flags, p.op_index);
        tc_fence_after();
        for (int j = 0; ok && j < min(Cfg::NSB, w.nkv); ++j) ok = issue_s();
      }
      for (int k = 0; ok && t >= 0; ++k) {
        const AttnTile w = attn_tile(p, t);
        for (int j = Cfg::NSB; ok && j < w.nkv; ++j) ok = issue_s();
        if (!ok) break;
        mma_commit(qempty);             // the Q buffer is free once this tile's score MMAs are done
        // the next tile's first NSB score MMAs overlap this tile's softmax passes
        const int tn = attn_item(k + 1, ntiles);
        if (tn >= 0) {
          const AttnTile wn = attn_tile(p, tn);
          if (!mbar_wait_idle(qfull, (k + 1) & 1, abort, p.flags, p.op_index)) break;
          tc_fence_after();
          for (int j = 0; ok && j < min(Cfg::NSB, wn.nkv); ++j) ok = issue_s();
          if (!ok) break;
        }
        // O = sum_j P_j V_j, slab by slab as the softmax warps finish each slab's probabilities, so the MMAs and
        // the V^T loads they free ring slots for run under the rest of the probability pass
        for (int j = 0; ok && j < w.nkv; ++j, ++gv) {
          const int st = gv % Cfg::VS;
          if (!mbar_wait_idle(&pslab[j], (pph >> j) & 1u, abort, p.flags, p.op_index)) { ok = false; break; }
          pph ^= 1u << j;
          if (!mbar_wait_idle(&vfull[st], (gv / Cfg::VS) & 1, abort, p.flags, p.op_index)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sp = smem_u32(pbuf + j * Cfg::P_SLAB);
          const uint32_t sv = smem_u32(smem + Cfg::OFF_V + st * Cfg::T_BYTES);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_i8(tmem + Cfg::O_COL, kmajor_desc(sp + 32 * kk, 2u, 1024u), kmajor_desc(sv + 32 * kk, 2u, 1024u),
                   idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&vempty[st]);
          mma_commit(&pfree[j]);
        }
        if (!ok) break;
        mma_commit(ofull);
        t = tn;
      }
    }
  } else {
    // -------------------------------------------- softmax warps: 4 threads per query row, one 32-column part each
    const int lane_base = 32 * (warp & 3);           // TMEM lanes this warp may read
    const int part = (warp - 2) >> 2;                // 0..3: columns [32*part, 32*part + 32) of every slab
    const int r = lane_base + lane;
    const int m1 = (int)p.m1;
    const int rnd1 = (int)round_term(p.s1);
    int32_t *red_max = reinterpret_cast<int32_t *>(smem + Cfg::OFF_RED);   // [4][128] partial row max
    int32_t *red_sum = red_max + 512;                                          // [4][128] partial row sum
    const int lcopy = lane % Cfg::LUT_COPIES;
    const long long rnd2 = round_term(p.s2);
    const bool m2_32 = p.m2 >= 0 && p.m2 <= 0x7fffffffll && rnd2 <= 0x7fffffffll;
    uint32_t gs = 0;
    uint32_t fph = 0;                                // bit j: parity of P slab j's uses so far
    // O = P V of a finished tile: TMEM -> requant -> merged-heads output row. The last HD/32 parts take 32
    // columns each: their columns of a causal tile's diagonal slab are the ones with the fewest kept scores, so
    // these are the warps with the least probability work. It runs after the next tile's score pass, by which
    // time the tile's P V MMAs are long done, so no warp waits on them at a tile boundary.
    const int opart = part - (4 - HD / 32);
    // query row (within the tile) of this thread's TMEM lane on the CTA's k-th item: the Q producer reverses the
    // order of the four 32-row blocks on odd items, so the row group holding the heaviest causal rows alternates
    // between the SMSPs (a warp reads TMEM lanes 32 (warp % 4) + i only, and runs on SMSP warp % 4)
    const auto qrow = [&](int k) { return 32 * ((warp & 3) ^ ((k & 1) * 3)) + lane; };
    // the four warps of one row group (one per part) meet at named barrier 1 + (warp & 3); the row groups do not
    // wait for one another
    const int gbar = 1 + (warp & 3);
    auto o_epilogue = [&](const AttnTile &w, int k) {
      const int row = w.q0 + qrow(k);
      if (opart >= 0 && __all_sync(0xffffffffu, mbar_wait_idle(ofull, k & 1, abort, p.flags, p.op_index))) {
        tc_fence_after();
        int32_t acc[32];
        tmem_ld32(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(Cfg::O_COL + opart * 32), acc);
        uint32_t wq[8];
        int v[32];
        if (m2_32) {                       // the static int32 proof bounds acc*M2 + 2^(s2-1): 32-bit, clamp in the pack
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = mad_wrap(acc[q], (int)p.m2, (int)rnd2) >> p.s2;
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) v[q] = (int)clampi(((long long)acc[q] * p.m2 + rnd2) >> p.s2, -128, 127);
        }
#pragma unroll
        for (int q = 0; q < 8; ++q) wq[q] = pack4_sat_s8(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        if (row < p.T1) {
          int8_t *orow = p.out + (int64_t)w.b * p.o_bs + (int64_t)row * p.o_rs + (int64_t)w.h * HD + opart * 32;
          uint4 *d4 = reinterpret_cast<uint4 *>(orow);
          d4[0] = make_uint4(wq[0], wq[1], wq[2], wq[3]);
          d4[1] = make_uint4(wq[4], wq[5], wq[6], wq[7]);
        }
        tc_fence_before();
      }
    };
    AttnTile prev;
    int k = 0;
    bool stopped = false;
    // this thread's two 16-byte chunks of every P slab (the swizzle depends on the row only)
    const int off0 = pslab_off(r, 2 * part), off1 = pslab_off(r, 2 * part + 1);
    for (int t; (t = attn_item(k, ntiles)) >= 0; ++k) {
      const AttnTile w = attn_tile(p, t);
      const int row = w.q0 + qrow(k);
      const int kept = p.causal ? min(row + 1, p.T2) : p.T2;
      // Every pass classifies this thread's 32 columns of slab j for the warp as a whole (votes, so the branches
      // are warp-uniform): all kept for every row of the warp (no mask), none kept (nothing to read), or the
      // causal diagonal / the ragged end of T2 (a per-lane mask, by selects).
      int mx = -128;
      bool ok = true;
      for (int j = 0; j < w.nkv; ++j, ++gs) {
        const int sb = gs % Cfg::NSB;
        ok = __all_sync(0xffffffffu, mbar_wait_idle(&sfull[sb], (gs / Cfg::NSB) & 1, abort, p.flags, p.op_index));
        if (!ok) break;                     // warp-uniform: the TMEM load below is .sync.aligned
        tc_fence_after();
        int32_t acc[32];
        tmem_ld32(tmem + ((uint32_t)lane_base << 16) + (uint32_t)(sb * 128 + part * 32), acc);
        const int cb = j * 128 + part * 32;
        // the static int32 proof holds on this path: acc*M1 + 2^(s1-1) fits int32. The row max is taken over the
        // unclamped values (clamping is monotone, so max of clamped = clamp of max) and the clamp happens in the
        // saturating pack.
        int v[32];
#pragma unroll
        for (int q = 0; q < 32; ++q) v[q] = mad_wrap(acc[q], m1, rnd1) >> p.s1;
        if (__all_sync(0xffffffffu, cb + 32 <= kept)) {
#pragma unroll
          for (int q = 0; q < 32; ++q) mx = max(mx, v[q]);
        } else {
          // masked columns are stored as -128: a value no kept score exceeds the row max with, so every LUT index
          // below stays in [0, 255] without a clamp
#pragma unroll
          for (int q = 0; q < 32; ++q) {
            v[q] = cb + q < kept ? v[q] : -128;
            mx = max(mx, v[q]);
          }
        }
        uint32_t wq[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) wq[q] = pack4_sat_s8(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        // P slab j still feeds the previous tile's P V MMA until pfree[j] completes
        ok = __all_sync(0xffffffffu, mbar_wait_idle(&pfree[j], ((fph >> j) & 1u) ^ 1u, abort, p.flags, p.op_index));
        fph ^= 1u << j;
        if (!ok) break;
        uint8_t *slab = pbuf + j * Cfg::P_SLAB;
        *reinterpret_cast<uint4 *>(slab + off0) = make_uint4(wq[0], wq[1], wq[2], wq[3]);
        *reinterpret_cast<uint4 *>(slab + off1) = make_uint4(wq[4], wq[5], wq[6], wq[7]);
        tc_fence_before();
        mbar_arrive(&sempty[sb]);
      }
      // row max over the 4 parts (clamped: the raw scores were tracked). The max and the sum have their own
      // partial arrays, so a warp that runs ahead into the next tile cannot overwrite what a slower one still reads.
      if (k > 0 && ok) o_epilogue(prev, k - 1);
      prev = w;
      red_max[part * 128 + r] = min(127, mx);
      // the four warps of the row group take the same decision to stop (their named barrier needs all four): the
      // abort word is OR-reduced across the group's 128 threads by this barrier itself. Other groups see the abort
      // word at their next barrier or bounded wait.
      int stop;
      asm volatile(
          "{\n\t.reg .pred P;\n\t"
          "setp.ne.s32 P, %1, 0;\n\t"
          "bar.red.or.pred P, %2, 128, P;\n\t"
          "selp.s32 %0, 1, 0, P;\n\t}"
          : "=r"(stop)
          : "r"(*abort), "r"(gbar)
          : "memory");
      if (stop) { stopped = true; break; }
      mx = max(max(red_max[r], red_max[128 + r]), max(red_max[256 + r], red_max[384 + r]));
      // a kept score x <= mx (a signed byte of the slab) has lut[x - mx + 255] at lut_at(lutc, x) in this lane's
      // copy; a masked column holds -128 (stored so by the drain), so every index is in [0, 255]
      const uint32_t lutc = smem_u32(lut + (255 - mx) * Cfg::LUT_COPIES + lcopy);
      // pass A: partial S = sum over this part's kept columns of lut[x - max + 255]
      int tot0 = 0, tot1 = 0;
      for (int j = 0; j < w.nkv && ok; ++j) {
        const int cb = j * 128 + part * 32;
        if (__all_sync(0xffffffffu, cb >= kept)) continue;
        const uint8_t *slab = pbuf + j * Cfg::P_SLAB;
        const uint4 a4 = *reinterpret_cast<const uint4 *>(slab + off0);
        const uint4 b4 = *reinterpret_cast<const uint4 *>(slab + off1);
        const uint32_t wv[8] = {a4.x, a4.y, a4.z, a4.w, b4.x, b4.y, b4.z, b4.w};
        if (__all_sync(0xffffffffu, cb + 32 <= kept)) {
          // two independent three-input adds per word (each folds two entries into one accumulator)
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            tot0 += lut_byte<Cfg::LUT_COPIES, 0>(lutc, wv[q]) + lut_byte<Cfg::LUT_COPIES, 1>(lutc, wv[q]);
            tot1 += lut_byte<Cfg::LUT_COPIES, 2>(lutc, wv[q]) + lut_byte<Cfg::LUT_COPIES, 3>(lutc, wv[q]);
          }
        } else {
          // all 32 looked up as in the full case; the masked ones (stored as -128) are taken out again as a count
          // times lut[-128 - max + 255]
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            tot0 += lut_byte<Cfg::LUT_COPIES, 0>(lutc, wv[q]) + lut_byte<Cfg::LUT_COPIES, 1>(lutc, wv[q]);
            tot1 += lut_byte<Cfg::LUT_COPIES, 2>(lutc, wv[q]) + lut_byte<Cfg::LUT_COPIES, 3>(lutc, wv[q]);
          }
          const int nmask = 32 - min(32, max(0, kept - cb));
          tot0 -= nmask * lut_at<Cfg::LUT_COPIES>(lutc, -128);
        }
      }
      red_sum[part * 128 + r] = tot0 + tot1;
      asm volatile("bar.sync %0, 128;" ::"r"(gbar) : "memory");
      const int tot = red_sum[r] + red_sum[128 + r] + red_sum[256 + r] + red_sum[384 + r];
      // pass B: p = floor((e*one + S/2) / S), masked entries 0. The division is a multiply by a per-row magic
      // number (Granlund & Montgomery, "Division by invariant integers using multiplication", 1994): with
      // l = ceil(log2 S), k = 31 + l and m = ceil(2^k / S) (m <= 2^32), floor(n m / 2^k) = floor(n / S) for every
      // 0 <= n < 2^31, because m S - 2^k < S <= 2^l makes the error term n (m S - 2^k) / (S 2^k) < 1 / S.
      // With m < 2^32 this is a 32 x 32 -> high 32 multiply and a shift by l - 1. S = 1 takes the same form with
      // n doubled (one2 = 2*one, m = 2^31, shift 0): the high word of 2n * 2^31 is n (2n < 2^32 as e*one < 2^31).
      const int S = tot > 0 ? tot : 1;
      const int lg = S > 1 ? 32 - __clz(S - 1) : 0;
      const unsigned magic = S > 1 ? ceil_pow2_div(S, lg) : 0x80000000u;
      const int msh = lg > 0 ? lg - 1 : 0;
      const unsigned one2 = S > 1 ? (unsigned)p.one : 2u * (unsigned)p.one;
      const unsigned half2 = S > 1 ? (unsigned)(tot >> 1) : 2u * (unsigned)(tot >> 1);
      for (int j = 0; j < w.nkv && ok; ++j) {
        uint8_t *slab = pbuf + j * Cfg::P_SLAB;
        const int cb = j * 128 + part * 32;
        uint32_t ov[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        if (!__all_sync(0xffffffffu, cb >= kept)) {
          const uint4 a4 = *reinterpret_cast<const uint4 *>(slab + off0);
          const uint4 b4 = *reinterpret_cast<const uint4 *>(slab + off1);
          const uint32_t wv[8] = {a4.x, a4.y, a4.z, a4.w, b4.x, b4.y, b4.z, b4.w};
          int pv[32];
          if (__all_sync(0xffffffffu, cb + 32 <= kept)) {
#pragma unroll
            for (int q = 0; q < 32; ++q) {
              const unsigned num = (unsigned)lut_byte_q<Cfg::LUT_COPIES>(lutc, wv[q >> 2], q & 3) * one2 + half2;
              pv[q] = (int)(__umulhi(num, magic) >> msh);
            }
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q) {
              const unsigned num = (unsigned)lut_byte_q<Cfg::LUT_COPIES>(lutc, wv[q >> 2], q & 3) * one2 + half2;
              pv[q] = cb + q < kept ? (int)(__umulhi(num, magic) >> msh) : 0;
            }
          }
#pragma unroll
          for (int q = 0; q < 8; ++q) ov[q] = pack4_sat_s8(pv[4 * q], pv[4 * q + 1], pv[4 * q + 2], pv[4 * q + 3]);
        }
        *reinterpret_cast<uint4 *>(slab + off0) = make_uint4(ov[0], ov[1], ov[2], ov[3]);
        *reinterpret_cast<uint4 *>(slab + off1) = make_uint4(ov[4], ov[5], ov[6], ov[7]);
        fence_proxy_async();                // this thread's part of slab j is final: the P V MMA may read it
        mbar_arrive(&pslab[j]);
      }
    }
    if (!stopped && k > 0) o_epilogue(prev, k - 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace anvil
