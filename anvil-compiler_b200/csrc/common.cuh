// Shared device helpers for libanvil_cuda: checked-int32 requant arithmetic, error flags, and thin inline-PTX
// wrappers for the sm_100a features the kernels use (mbarrier, TMA tile loads, tcgen05 MMA / TMEM).
//
// Every wait on an mbarrier is bounded by wall time (%globaltimer): a wait that gives up records
// ANVIL_DEV_TIMEOUT in the model's flag words and sets the CTA's abort word, so the kernel winds down and
// returns instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/anvil_cuda.h"

#define ANVIL_DEV_WAIT_NS 2000000000ull   // a bounded mbarrier wait gives up after 2 s of wall time

// Device flag words, one array per model: [0] overflow (op index + 1), [1] index error (op index + 1),
// [2] device wait timeout (op index + 1). The first failing op wins (atomicCAS from 0).
enum { FLAG_OVERFLOW = 0, FLAG_INDEX = 1, FLAG_TIMEOUT = 2, FLAG_WORDS = 4 };

__device__ __forceinline__ void raise_flag(uint32_t *flags, int which, int op_index) {
  if (flags) atomicCAS(flags + which, 0u, (uint32_t)(op_index + 1));
}

__device__ __forceinline__ bool fits_i32(long long v) { return v >= -2147483648LL && v <= 2147483647LL; }

__device__ __forceinline__ long long round_term(int s) { return s ? (1LL << (s - 1)) : 0LL; }

// a * b + c in 32-bit two's-complement arithmetic (wrap-around, defined for every operand): the unchecked
// epilogues' form, exact whenever the mathematical value fits int32, which the static int32 proof guarantees for
// every intermediate it admits. The instruction is the same multiply-add a signed form would compile to.
__device__ __forceinline__ int mad_wrap(int a, int b, int c) {
  return (int)((uint32_t)a * (uint32_t)b + (uint32_t)c);
}

__device__ __forceinline__ int clampi(long long v, int lo, int hi) {
  return (int)(v < lo ? lo : (v > hi ? hi : v));
}

// requant_dtype (anvil/semantics.py:146-155): clamp((acc*M + 2^(s-1)) >> s) with acc, acc*M and the rounded
// numerator each required to fit int32 (`bad` collects violations when CHECK). The arithmetic itself is done in
// 64 bits, so the value equals the exact mathematical one whenever the checked contract holds.
template <bool CHECK>
__device__ __forceinline__ int requant64(long long acc, long long m, int s, int lo, int hi, bool &bad) {
  long long p = acc * m;
  long long r = p + round_term(s);
  if (CHECK) bad |= !fits_i32(acc) | !fits_i32(p) | !fits_i32(r);
  return clampi(r >> s, lo, hi);
}

namespace anvil {
template <int B>
struct IntOf;
template <>
struct IntOf<1> { using T = int8_t; };
template <>
struct IntOf<2> { using T = int16_t; };
template <>
struct IntOf<4> { using T = int32_t; };

}  // namespace anvil

// Saturate four int32 values to int8 and pack them little-endian (a0 in byte 0) with two cvt.pack.sat ops:
// cvt.pack.sat.s8.s32.b32 d, a, b, c puts sat8(b) in d[7:0], sat8(a) in d[15:8] and c[15:0] in d[31:16].
__device__ __forceinline__ uint32_t pack4_sat_s8(int a0, int a1, int a2, int a3) {
  uint32_t hi, d;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(a3), "r"(a2));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a1), "r"(a0), "r"(hi));
  return d;
}

// Signed byte q (0..3) of w, sign-extended: always in [-128, 127].
__device__ __forceinline__ int sbyte(uint32_t w, int q) { return (int)(int8_t)(w >> (8 * q)); }

// Sign-extended byte q (0..3) of w in one byte permute: prmt's default mode replicates the sign bit of the
// selected byte when the selector nibble's msb is set, so bytes 1-3 of the result copy the sign of byte q.
__device__ __forceinline__ int sbyte_prmt(uint32_t w, int q) {
  int r;
  const uint32_t sel = (uint32_t)q | ((uint32_t)(q | 8) * 0x1110u);
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
  return r;
}

// Unsigned byte q (0..3) of w, zero-extended (one byte permute): always in [0, 255].
__device__ __forceinline__ uint32_t ubyte(uint32_t w, int q) { return __byte_perm(w, 0u, 0x4440u | (uint32_t)q); }

// ------------------------------------------------------------------------------------------------- PTX: misc

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The dynamic shared-memory base rounded up to 1024 bytes by pointer arithmetic on the __shared__ array itself:
// the compiler then keeps every pointer derived from it in the shared state space (ld/st.shared), where an
// integer round trip would leave it generic (slower generic loads and stores, long-scoreboard waits).
__device__ __forceinline__ uint8_t *align_smem_1024(uint8_t *raw) {
  return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "elect.sync _|P, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// x / d for 0 <= x < 2^31 and d >= 1, from the host's div_magic(d) = (m, s): with l = ceil(log2 d) and
// m = ceil(2^(31 + l) / d) (< 2^32), floor(x m / 2^(31 + l)) = floor(x / d) for every x < 2^31 (Granlund &
// Montgomery, "Division by invariant integers using multiplication", 1994); s = l - 1. d = 1 is taken apart.
__device__ __forceinline__ uint32_t tile_div(uint32_t x, uint32_t d, uint32_t m, int s) {
  return d == 1 ? x : (__umulhi(x, m) >> s);
}

// ------------------------------------------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with `parity` to complete. Returns false (after setting *abort and the timeout flag)
// if the wait gives up, or immediately if another role of the CTA already aborted.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *flags,
                                              int op_index, uint64_t limit_ns) {
  uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(a, parity)) return true;
    if ((it & 255u) == 0) {
      if (*abort) return false;
      if (globaltimer() - t0 > limit_ns) {
        *abort = 1;
        raise_flag(flags, FLAG_TIMEOUT, op_index);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *flags,
                                          int op_index) {
  return mbar_wait_for(bar, parity, abort, flags, op_index, ANVIL_DEV_WAIT_NS);
}

// mbarrier.try_wait with a suspend-time hint: the thread sleeps until the phase completes or `hint_ns` passes.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred P;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, P;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// mbar_wait for long waits of a single elected thread (a producer or MMA issuer idle while other warps compute):
// each try suspends the thread for up to 20 us instead of spinning, so it takes no issue slots from the warps
// doing the work. Bounded like mbar_wait.
__device__ __forceinline__ bool mbar_wait_idle(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *flags,
                                               int op_index) {
  uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  uint64_t t0 = globaltimer();
  for (;;) {
    if (mbar_try_wait_hint(a, parity, 20000u)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > ANVIL_DEV_WAIT_NS) {
      *abort = 1;
      raise_flag(flags, FLAG_TIMEOUT, op_index);
      return false;
    }
  }
}

// Wait up to `ns` nanoseconds, ignoring the abort word (drains copies still in flight after an abort).
__device__ __forceinline__ bool mbar_wait_ns(uint64_t *bar, uint32_t parity, uint64_t ns) {
  uint32_t a = smem_u32(bar);
  uint64_t t0 = globaltimer();
  while (!mbar_try_wait(a, parity)) {
    if (globaltimer() - t0 > ns) return false;
  }
  return true;
}

// ------------------------------------------------------------------------------------------------------ TMA

__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Shared -> global tile stores (bulk-group completion). The writer threads make their shared-memory stores
// visible to the async proxy (fence_proxy_async) before one thread issues the copy; the issuer waits with
// bulk_wait_read before the staging buffer is written again and with bulk_wait_all before the CTA exits.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *smem_src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's generic shared-memory writes before later async-proxy reads (TMA stores, tcgen05.mma).
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void st_shared_v4(void *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(smem_u32(p)), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

__device__ __forceinline__ void st_shared_u32(void *p, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

__device__ __forceinline__ void st_shared_u8(void *p, uint32_t v) {
  asm volatile("st.shared.u8 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------------------------------------------- tcgen05

__device__ __forceinline__ void tmem_alloc(uint32_t *smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], int8 x int8 -> int32 (kind::i8), one CTA.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 op this thread issued before has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ------------------------------------------------------------------------------------------- CTA pairs
// A cluster of two CTAs on neighbouring SMs computes one 256-row MMA tile (tcgen05 cta_group::2): each CTA stages
// its 128 rows of A and half of B's rows in its own shared memory, the even CTA (rank 0) issues the MMAs, and each
// CTA's TMEM receives its own 128 accumulator rows.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of the variable at shared::cta address `addr` in the cluster's CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// Every thread of both CTAs: prior shared-memory writes (barrier inits included) are visible cluster-wide after.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's), with the default
// (CTA-scope release) semantics: a cluster-scope release would fence all of the thread's outstanding memory
// operations first. The accumulator hand-off it signals is ordered by the tcgen05 fences around it.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// TMA tile load into this CTA's shared memory whose completion (bytes) is counted on an mbarrier that may sit in
// the peer CTA (shared::cluster address), as the pair's loads all complete on the even CTA's barrier.
__device__ __forceinline__ void tma_load_3d_pair(void *smem_dst, const CUtensorMap *map, int x, int y, int z,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], "
      "[%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(bar)
      : "memory");
}

// TMEM allocation of both CTAs of the pair: one warp of each CTA (the same warp index, the same slot offset).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D (+)= A * B over the pair, int8 x int8 -> int32: issued by the even CTA with descriptors of its own shared
// memory; the peer's operand halves sit at the same offsets in the peer CTA.
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at this offset in both CTAs of the pair once the pair MMAs issued before have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

// 32 lanes x 32 consecutive columns of 32-bit TMEM cells: thread i of the warp gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored in the 128-byte swizzle layout that a TMA
// load with CU_TENSOR_MAP_SWIZZLE_128B writes: rows of 128 bytes, 8-row groups 1024 bytes apart (SBO = 1024),
// LBO unused for swizzled K-major (1), descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                 // leading byte offset (16 B units)
  d |= (uint64_t)(1024u >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;                 // version
  d |= (uint64_t)2u << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::i8: s32 accumulators, signed int8 A and B, both K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4)            // D format: s32
         | (1u << 7)          // A format: signed 8-bit
         | (1u << 10)         // B format: signed 8-bit
         | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
