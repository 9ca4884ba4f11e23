// libanvil_cuda.so: the C-ABI declared in include/anvil_cuda.h and the runtime behind it.
//
// A model owns, on one device: the const region (weights, LUTs, biases in device layout, uploaded once), an
// activation arena laid out by the host's liveness plan (anvil/memplan.py:190-198, in bytes), a small flag array
// the checked kernels write, and one non-blocking stream. anvil_model_prepare turns the host's anvil_op list into
// resolved launches (device pointers, grid sizes, TMA tensor maps) after checking every byte range each op
// touches against the region it lives in; anvil_model_run then only copies and launches.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/anvil_cuda.h"
#include "common.cuh"
#include "attention.cuh"
#include "gemm.cuh"
#include "rowops.cuh"

using namespace anvil;

// --------------------------------------------------------------------------------------------- error state

static thread_local std::string g_err = "";

static int fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

#define CK(call)                                                                                          \
  do {                                                                                                    \
    cudaError_t e_ = (call);                                                                              \
    if (e_ != cudaSuccess) return fail(e_ == cudaErrorMemoryAllocation ? ANVIL_E_OOM : ANVIL_E_CUDA,      \
                                       "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, \
                                       __LINE__);                                                         \
  } while (0)

extern "C" int anvil_abi_version(void) { return ANVIL_ABI_VERSION; }
extern "C" const char *anvil_last_error(void) { return g_err.c_str(); }

// ------------------------------------------------------------------------------------ driver entry points

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// int8 tensor map over a (z, y, x) array with x contiguous: box = (1, box_y, 128 bytes), 128-byte swizzle.
static int make_map_i8(CUtensorMap *map, const void *base, uint64_t x, uint64_t y, uint64_t z, uint64_t ystride,
                       uint64_t zstride, uint32_t box_y) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(ANVIL_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {x, y, z};
  cuuint64_t strides[2] = {ystride, zstride};
  cuuint32_t box[3] = {128, box_y, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ANVIL_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return ANVIL_OK;
}

// General int8 tiled map: rank 2..4, dims/strides in elements = bytes, given box and swizzle.
static int make_map(CUtensorMap *map, const void *base, int rank, const uint64_t *dims, const uint64_t *strides,
                    const uint32_t *box, CUtensorMapSwizzle swz) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(ANVIL_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
    if (i) st[i - 1] = strides[i - 1];
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank, const_cast<void *>(base), d, st, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ANVIL_E_CUDA, "cuTensorMapEncodeTiled (rank %d) failed (%d)", rank, (int)r);
  return ANVIL_OK;
}

// ------------------------------------------------------------------------------------------------- model

struct Launch {
  anvil_op op;
  // resolved device pointers, one per op.off slot
  void *ptr[8];
  // GEMM tensor-core path; pair: 256-row tiles over CTA pairs (BN = 256)
  bool tc = false;
  bool pair = false;
  int bn = 0;
  CUtensorMap mapA, mapB, mapC, mapC2;   // mapC2: the transposed part of a split output
  GemmParams gp;
  AttnParams ap;
  int hd = 0;
};

struct anvil_model {
  int device = 0;
  int sms = 148;
  cudaStream_t stream = nullptr;
  void *consts = nullptr;
  uint64_t const_bytes = 0;
  void *arena = nullptr;
  uint64_t arena_bytes = 0;
  uint32_t *flags = nullptr;         // FLAG_WORDS device words
  std::vector<Launch> launches;
  cudaGraphExec_t graph = nullptr;
  std::vector<cudaEvent_t> events;
  // pipelined enqueues: recorded after this model's last input copies and after its last launch chain
  cudaEvent_t ev_in = nullptr, ev_run = nullptr;
  int pair_clusters = -1;            // co-resident CTA pairs of the pair GEMM (0: the pair path is off)
  // completion tickets (anvil_model_record / anvil_model_wait_ticket): ticket t owns ring slot t % TICKETS, which
  // holds the event recorded after the work it covers and a device snapshot of the check words at that point
  static constexpr int TICKETS = 64;
  uint32_t *ticket_flags = nullptr;  // TICKETS x FLAG_WORDS device words
  cudaEvent_t ticket_ev[TICKETS] = {};
  bool ticket_pending[TICKETS] = {};
  uint64_t ticket_next = 0;
  cudaStream_t status_stream = nullptr;   // reads the snapshots without queueing behind the model's stream
  cudaEvent_t ticket_snap[TICKETS] = {};  // after the snapshot, on the model's stream
  // pipelined enqueues move their copies to the device's shared copy streams: recorded after this model's last
  // copies out (the arena is free again once it completes)
  cudaEvent_t ev_free = nullptr;
  bool free_pending = false;
};

// The device's two copy streams for pipelined enqueues (one for copies in, one for copies out), shared by every
// model on the device and kept until the process exits: chunks queued from several models reach the bus back to
// back in enqueue order, with no cross-stream wait between consecutive copies of one direction.
struct CopyStreams {
  std::once_flag once;
  cudaStream_t in = nullptr, out = nullptr;
  cudaError_t err = cudaSuccess;
};
static CopyStreams g_copy_streams[64];

static int copy_streams(int dev, cudaStream_t *in, cudaStream_t *out) {
  if (dev < 0 || dev >= 64) return fail(ANVIL_E_BAD_ARG, "device %d out of range", dev);
  CopyStreams &c = g_copy_streams[dev];
  std::call_once(c.once, [&]() {
    c.err = cudaStreamCreateWithFlags(&c.in, cudaStreamNonBlocking);
    if (c.err == cudaSuccess) c.err = cudaStreamCreateWithFlags(&c.out, cudaStreamNonBlocking);
  });
  if (c.err != cudaSuccess) return fail(ANVIL_E_CUDA, "copy stream creation failed: %s", cudaGetErrorString(c.err));
  *in = c.in;
  *out = c.out;
  return ANVIL_OK;
}

// Orders the model's own stream after its last pipelined copies out (which run on the device's copy-out stream):
// every path that touches the arena from the model's stream goes through here first.
static int join_copies(anvil_model *m) {
  if (m->free_pending) CK(cudaStreamWaitEvent(m->stream, m->ev_free, 0));
  return ANVIL_OK;
}

extern "C" int anvil_device_count(int *count) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  if (count) *count = n;
  return ANVIL_OK;
}

extern "C" int anvil_cuda_init(int device) {
  int n = 0;
  anvil_device_count(&n);
  if (device < 0 || device >= n) return fail(ANVIL_E_UNSUPPORTED, "device %d not available (%d visible)", device, n);
  cudaDeviceProp prop;
  CK(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(ANVIL_E_UNSUPPORTED, "device %d is sm_%d%d; libanvil_cuda is built for sm_100a (B200)", device,
                prop.major, prop.minor);
  CK(cudaSetDevice(device));
  return ANVIL_OK;
}

template <typename K>
static int set_smem(K kernel, int bytes) {
  CK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return ANVIL_OK;
}

static int kernel_attrs(int device);

extern "C" int anvil_model_create(int device, const void *consts, uint64_t const_bytes, anvil_model **out) {
  if (!out) return fail(ANVIL_E_BAD_ARG, "out is NULL");
  *out = nullptr;
  int rc = anvil_cuda_init(device);
  if (rc) return rc;
  anvil_model *m = new anvil_model();
  m->device = device;
  cudaDeviceGetAttribute(&m->sms, cudaDevAttrMultiProcessorCount, device);
  auto cleanup = [&](int code) {
    anvil_model_free(m);
    return code;
  };
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess)
    return cleanup(fail(ANVIL_E_CUDA, "cudaStreamCreate failed"));
  if (cudaMalloc(&m->flags, FLAG_WORDS * sizeof(uint32_t)) != cudaSuccess)
    return cleanup(fail(ANVIL_E_OOM, "cannot allocate the flag words"));
  if (const_bytes) {
    if (!consts) return cleanup(fail(ANVIL_E_BAD_ARG, "consts is NULL with const_bytes = %llu",
                                     (unsigned long long)const_bytes));
    if (cudaMalloc(&m->consts, const_bytes) != cudaSuccess)
      return cleanup(fail(ANVIL_E_OOM, "cannot allocate %llu const bytes", (unsigned long long)const_bytes));
    if (cudaMemcpy(m->consts, consts, const_bytes, cudaMemcpyHostToDevice) != cudaSuccess)
      return cleanup(fail(ANVIL_E_CUDA, "const upload failed"));
  }
  m->const_bytes = const_bytes;
  if ((rc = kernel_attrs(device))) return cleanup(rc);
  *out = m;
  return ANVIL_OK;
}

// Per-device facts every entry point needs, set up once per device (std::call_once: host threads that make
// their first call on one device at the same time wait for a single set-up): the kernels' shared-memory opt-in
// (a per-function, per-device attribute), the SM count and how many CTA pairs of the pair GEMM fit at once.
struct DeviceInfo {
  std::once_flag once;
  int rc = ANVIL_OK;
  std::string err;
  int sms = 0;
  int pair_capacity = 0;
};
static DeviceInfo g_dev_info[64];

static int set_kernel_attrs();

// The set-up of `device`, which must be the current device. Returns its status (the first failure is kept).
static int device_info(int device, DeviceInfo **out) {
  if (device < 0 || device >= 64) return fail(ANVIL_E_BAD_ARG, "device %d out of range", device);
  DeviceInfo &d = g_dev_info[device];
  std::call_once(d.once, [&]() {
    int rc = set_kernel_attrs();
    if (!rc && cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess)
      rc = fail(ANVIL_E_CUDA, "cannot read the SM count of device %d", device);
    if (!rc) {
      cudaLaunchConfig_t cfg = {};
      cudaLaunchAttribute attr[1];
      cfg.gridDim = dim3((unsigned)(d.sms & ~1));
      cfg.blockDim = dim3(TC_THREADS);
      cfg.dynamicSmemBytes = TcCfg<256, true>::SMEM_BYTES;
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 2;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&d.pair_capacity, qgemm_tc_kernel<256, 1, false, true>, &cfg) !=
          cudaSuccess) {
        cudaGetLastError();
        d.pair_capacity = 0;
      }
    }
    d.rc = rc;
    if (rc) d.err = g_err;
  });
  if (d.rc) {
    g_err = d.err;
    return d.rc;
  }
  if (out) *out = &d;
  return ANVIL_OK;
}

static int kernel_attrs(int device) { return device_info(device, nullptr); }

// Opt every large-shared-memory kernel in to its dynamic shared memory size on the current device.
static int set_kernel_attrs() {
  {
    int r = 0;
    r |= set_smem(attn_kernel<64>, AttnCfg<64>::SMEM_BYTES);
    r |= set_smem(attn_kernel<128>, AttnCfg<128>::SMEM_BYTES);
#define TC_ATTR(BN, OB)                                                        \
  r |= set_smem(qgemm_tc_kernel<BN, OB, false>, TcCfg<BN>::SMEM_BYTES);      \
  r |= set_smem(qgemm_tc_kernel<BN, OB, true>, TcCfg<BN>::SMEM_BYTES);
    TC_ATTR(64, 1) TC_ATTR(64, 2) TC_ATTR(128, 1) TC_ATTR(128, 2) TC_ATTR(256, 1) TC_ATTR(256, 2)
#undef TC_ATTR
#define TC_PAIR_ATTR(OB)                                                                   \
  r |= set_smem(qgemm_tc_kernel<256, OB, false, true>, TcCfg<256, true>::SMEM_BYTES);    \
  r |= set_smem(qgemm_tc_kernel<256, OB, true, true>, TcCfg<256, true>::SMEM_BYTES);
    TC_PAIR_ATTR(1) TC_PAIR_ATTR(2)
#undef TC_PAIR_ATTR
    if (r) return ANVIL_E_CUDA;
  }
  return ANVIL_OK;
}

extern "C" void anvil_model_free(anvil_model *m) {
  if (!m) return;
  cudaSetDevice(m->device);
  if (m->free_pending) cudaEventSynchronize(m->ev_free);
  for (auto e : m->ticket_snap)
    if (e) cudaEventDestroy(e);
  if (m->ev_free) cudaEventDestroy(m->ev_free);
  if (m->stream) cudaStreamSynchronize(m->stream);
  if (m->graph) cudaGraphExecDestroy(m->graph);
  for (auto e : m->events) cudaEventDestroy(e);
  if (m->ev_in) cudaEventDestroy(m->ev_in);
  if (m->ev_run) cudaEventDestroy(m->ev_run);
  for (auto e : m->ticket_ev)
    if (e) cudaEventDestroy(e);
  if (m->ticket_flags) cudaFree(m->ticket_flags);
  if (m->status_stream) cudaStreamDestroy(m->status_stream);
  if (m->arena) cudaFree(m->arena);
  if (m->consts) cudaFree(m->consts);
  if (m->flags) cudaFree(m->flags);
  if (m->stream) cudaStreamDestroy(m->stream);
  delete m;
}

// Resolve a location to a device pointer, checking [off, off + bytes) against its region.
static int resolve(anvil_model *m, const anvil_op &op, int slot, uint64_t bytes, void **ptr, bool required = true) {
  uint64_t loc = op.off[slot];
  if (loc == ANVIL_LOC_NONE) {
    *ptr = nullptr;
    if (required) return fail(ANVIL_E_BAD_ARG, "op %d (kind %d): operand slot %d is missing", op.op_index, op.kind, slot);
    return ANVIL_OK;
  }
  bool is_const = (loc & ANVIL_LOC_CONST) != 0;
  uint64_t off = loc & ~ANVIL_LOC_CONST;
  uint64_t size = is_const ? m->const_bytes : m->arena_bytes;
  if (off > size || bytes > size - off)
    return fail(ANVIL_E_BAD_ARG, "op %d (kind %d): slot %d range [%llu, %llu) outside the %s region (%llu bytes)",
                op.op_index, op.kind, slot, (unsigned long long)off, (unsigned long long)(off + bytes),
                is_const ? "const" : "arena", (unsigned long long)size);
  *ptr = static_cast<uint8_t *>(is_const ? m->consts : m->arena) + off;
  return ANVIL_OK;
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Launch configuration of the pair GEMM: clusters of two CTAs (one per SM of a neighbouring pair).
static cudaLaunchConfig_t pair_config(dim3 grid, cudaStream_t st, cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TcCfg<256, true>::SMEM_BYTES;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// How many CTA pairs of the pair GEMM fit on the device at once (0 turns the pair path off; so does
// ANVIL_GEMM_PAIR=0 in the environment, read once per model).
static int pair_clusters(anvil_model *m) {
  if (m->pair_clusters < 0) {
    const char *env = getenv("ANVIL_GEMM_PAIR");
    DeviceInfo *di = nullptr;
    m->pair_clusters = (env && atoi(env) == 0) || device_info(m->device, &di) ? 0 : di->pair_capacity;
  }
  return m->pair_clusters;
}

// The tile shape of a tcgen05 GEMM launch: BN (64, 128 or 256 output columns per tile) and single-CTA 128-row
// tiles or 256-row tiles on CTA pairs (BN = 256 only). A persistent launch runs ceil(tiles / resident tiles)
// rounds, and every SM of a round does 128 x BN x K MACs, so the time is about rounds x BN x K, weighted by how
// efficiently each shape keeps the tensor pipe busy (measured on the c3 GEMMs: a single-CTA 256-column tile takes
// about 1.1 x the pair's time per MAC; narrower tiles re-read A for fewer columns per MMA). The cheapest shape
// wins, ties going to wider tiles. A fused residual epilogue over a short K is bound by its residual reads and
// keeps single-CTA tiles (measured: 768 x 768 residual GEMM 58 us single, 60 us paired).
struct TileChoice {
  int bn;
  bool pair;
};

static TileChoice choose_tiles(int64_t batch, int64_t M, int64_t N, int64_t K, int sms, int pair_cap, bool res,
                               bool bn256_only = false) {
  struct Cand { int bn; bool pair; double weight; };
  const Cand cands[4] = {{256, true, 1.0}, {256, false, 1.1}, {128, false, 1.2}, {64, false, 1.45}};
  TileChoice best = {256, false};
  double best_cost = -1;
  for (const Cand &c : cands) {
    if (c.pair && (pair_cap <= 0 || M < 4 * TC_BM || (res && K < 2048) || N <= 128)) continue;
    if (!c.pair && c.bn > 64 && N <= c.bn / 2 && !bn256_only) continue;   // a narrower tile holds every column
    if (bn256_only && c.bn != 256) continue;
    const int64_t rows = c.pair ? 2 * TC_BM : TC_BM;
    const int64_t tiles = batch * ((M + rows - 1) / rows) * ((N + c.bn - 1) / c.bn);
    const int64_t cap = c.pair ? pair_cap : sms;
    const double rounds = (double)((tiles + cap - 1) / cap);
    const double cost = rounds * c.bn * (double)K * c.weight;
    if (best_cost < 0 || cost < best_cost * 0.999) {
      best_cost = cost;
      best = {c.bn, c.pair};
    }
  }
  return best;
}


// tc GEMMs with i8 row-major outputs of 256-column tiles store through TMA (32 rows x 64 bytes per epilogue warp);
// the tensor map goes in L.mapC and sets gp.tma_store. Other outputs keep the per-lane global stores.
static int gemm_out_map(Launch &L) {
  GemmParams &p = L.gp;
  memset(&L.mapC, 0, sizeof L.mapC);
  memset(&L.mapC2, 0, sizeof L.mapC2);
  p.tma_store = 0;
  if (p.split_c) {
    // split output: columns [0, split_r) row-major in OUT (row stride o_rstride), the rest head-major transposed
    // in OUT2 (group o_group2); the caller checked the shapes and alignments
    if (!L.tc || L.bn != 256) return fail(ANVIL_E_BAD_ARG, "op %d: a split gemm needs 256-column tcgen05 tiles",
                                          p.op_index);
    const uint64_t cdims[2] = {(uint64_t)p.split_r, (uint64_t)p.M};
    const uint64_t cstr[1] = {(uint64_t)p.o_rstride};
    const uint32_t cbox[2] = {64, 32};
    int rc;
    if (p.split_r > 0 && (rc = make_map(&L.mapC, p.out, 2, cdims, cstr, cbox, CU_TENSOR_MAP_SWIZZLE_64B))) return rc;
    const int64_t T = p.o_group2, N2 = p.N - p.split_r;
    if (N2 > 0) {
      const uint64_t tdims[3] = {(uint64_t)T, (uint64_t)N2, (uint64_t)(p.M / T)};
      const uint64_t tstr[2] = {(uint64_t)T, (uint64_t)(N2 * T)};
      const uint32_t tbox[3] = {32, 64, 1};
      if ((rc = make_map(&L.mapC2, p.out2, 3, tdims, tstr, tbox, CU_TENSOR_MAP_SWIZZLE_NONE))) return rc;
    }
    p.tma_store = 1;
    return ANVIL_OK;
  }
  if (!L.tc || L.bn != 256 || p.out_bytes != 1 || !aligned16(p.out) || p.M > (1ll << 31) - 1 ||
      p.N > (1ll << 31) - 1)
    return ANVIL_OK;
  // head-major transposed output (the V^T layout the fused attention reads): element (r, c) at
  // (r / T) * N * T + c * T + r % T with T = o_group; each warp's 32 rows stay inside one group
  const int64_t T = p.o_group;
  if (p.batch == 1 && T > 0 && T % 32 == 0 && p.M % T == 0 && p.o_rstride == 1 && p.o_cstride == T &&
      p.o_gstride == p.N * T && T <= (1ll << 31) - 1) {
    const uint64_t cdims[3] = {(uint64_t)T, (uint64_t)p.N, (uint64_t)(p.M / T)};
    const uint64_t cstr[2] = {(uint64_t)T, (uint64_t)(p.N * T)};
    const uint32_t cbox[3] = {32, 64, 1};               // one epilogue warp's 32 rows x 64 columns, transposed
    int rc = make_map(&L.mapC, p.out, 3, cdims, cstr, cbox, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    p.tma_store = 2;
    return ANVIL_OK;
  }
  if (p.o_cstride != 1 || p.o_group != 0 || p.o_rstride % 16 != 0 || (p.batch > 1 && p.o_bstride % 16 != 0))
    return ANVIL_OK;
  const uint64_t cdims[3] = {(uint64_t)p.N, (uint64_t)p.M, (uint64_t)p.batch};
  const uint64_t cstr[2] = {(uint64_t)p.o_rstride, (uint64_t)p.o_bstride};
  const uint32_t cbox[3] = {64, 32, 1};                  // one epilogue warp's 32 rows x 64 columns
  int rc = make_map(&L.mapC, p.out, p.batch > 1 ? 3 : 2, cdims, cstr, cbox, CU_TENSOR_MAP_SWIZZLE_64B);
  if (rc) return rc;
  p.tma_store = 1;
  return ANVIL_OK;
}

// (m, s) of tile_div (common.cuh) for the divisor d >= 1: m = ceil(2^(31 + l) / d), s = l - 1, l = ceil(log2 d).
static void div_magic(int64_t d, uint32_t *m, int *s) {
  if (d <= 1) {
    *m = 0;
    *s = 0;
    return;
  }
  int l = 0;
  while ((1ll << l) < d) ++l;
  *m = (uint32_t)(((1ull << (31 + l)) + (uint64_t)d - 1) / (uint64_t)d);
  *s = l - 1;
}

// The tile decode's divisors n_tiles and m_tiles; tiles must stay < 2^31.
static int tile_magics(GemmParams &p, int op_index) {
  if (p.tiles >= (1ll << 31)) return fail(ANVIL_E_BAD_ARG, "op %d: %lld gemm tiles (at most 2^31 - 1)", op_index,
                                          (long long)p.tiles);
  div_magic(p.n_tiles, &p.n_magic, &p.n_shift);
  div_magic(p.m_tiles, &p.m_magic, &p.m_shift);
  return ANVIL_OK;
}

// Tile shape, tile count, tile-decode magics and tensor maps of a tcgen05 GEMM whose GemmParams are filled in.
static int tc_tiles(anvil_model *m, Launch &L) {
  GemmParams &p = L.gp;
  const TileChoice tc = choose_tiles(p.batch, p.M, p.N, p.K, m->sms, pair_clusters(m), p.res != nullptr,
                                     p.split_c != 0);
  L.bn = tc.bn;
  L.pair = tc.pair;
  const int64_t tile_rows = L.pair ? 2 * TC_BM : TC_BM;
  p.m_tiles = (p.M + tile_rows - 1) / tile_rows;
  p.n_tiles = (p.N + L.bn - 1) / L.bn;
  p.tiles = p.batch * p.m_tiles * p.n_tiles;
  int rc;
  if ((rc = tile_magics(p, p.op_index))) return rc;
  const int64_t M = p.M, N = p.N, K = p.K;
  const uint64_t a_z = p.batch, a_zs = p.a_bstride ? p.a_bstride : M * K;
  const uint64_t b_z = p.bt_bstride ? p.batch : 1, b_zs = p.bt_bstride ? p.bt_bstride : N * K;
  if ((rc = make_map_i8(&L.mapA, p.A, K, M, a_z, K, a_zs, TC_BM))) return rc;
  if ((rc = make_map_i8(&L.mapB, p.BT, K, N, b_z, K, b_zs, L.pair ? L.bn / 2 : L.bn))) return rc;
  return gemm_out_map(L);
}

static int prepare_gemm(anvil_model *m, Launch &L) {
  const anvil_op &op = L.op;
  const int64_t batch = op.dims[0], M = op.dims[1], N = op.dims[2], K = op.dims[3];
  const int64_t a_bs = op.strides[0], bt_bs = op.strides[1], o_bs = op.strides[2], o_rs = op.strides[3];
  if (batch < 1 || M < 1 || N < 1 || K < 1) return fail(ANVIL_E_BAD_ARG, "op %d: bad gemm dims", op.op_index);
  if (op.out_bytes != 1 && op.out_bytes != 2) return fail(ANVIL_E_BAD_ARG, "op %d: gemm output must be i8 or i16", op.op_index);
  if (op.shift < 0 || op.shift > 31) return fail(ANVIL_E_BAD_ARG, "op %d: shift %lld outside [0, 31]", op.op_index, (long long)op.shift);
  if ((op.flags & ANVIL_F_LUT) && op.out_bytes != 1)
    return fail(ANVIL_E_BAD_ARG, "op %d: a LUT epilogue needs an i8 result", op.op_index);
  const int64_t o_grp = op.strides[4], o_gs = op.strides[5], o_cs = op.strides[6] ? op.strides[6] : 1;
  const bool split = (op.flags & ANVIL_F_SPLIT) != 0;
  const int64_t ncols = split ? op.dims[5] : N;        // columns that go to OUT (the rest of a split to off[6])
  if (a_bs < 0 || bt_bs < 0 || o_bs < 0 || o_rs < 0 || o_grp < 0 || o_gs < 0 || o_cs < 1 || ncols < 0 ||
      ncols > N || (o_cs == 1 && o_rs < ncols))
    return fail(ANVIL_E_BAD_ARG, "op %d: bad gemm strides", op.op_index);
  int rc;
  const uint64_t a_bytes = (uint64_t)((batch - 1) * a_bs + M * K);
  const uint64_t b_bytes = (uint64_t)((bt_bs ? (batch - 1) * bt_bs : 0) + N * K);
  const int64_t R = o_grp ? o_grp : M;
  const int64_t last_row = M - 1;
  const uint64_t o_bytes = ncols == 0 ? 0 : (uint64_t)(((batch - 1) * o_bs + (last_row / R) * o_gs +
                                                        std::min<int64_t>(R - 1, last_row) * o_rs +
                                                        (ncols - 1) * o_cs + 1) * op.out_bytes);
  if ((rc = resolve(m, op, 0, a_bytes, &L.ptr[0]))) return rc;
  if ((rc = resolve(m, op, 1, b_bytes, &L.ptr[1]))) return rc;
  if ((rc = resolve(m, op, 2, o_bytes, &L.ptr[2]))) return rc;
  if ((rc = resolve(m, op, 3, 256, &L.ptr[3], (op.flags & ANVIL_F_LUT) != 0))) return rc;
  if ((rc = resolve(m, op, 4, (uint64_t)N * 4, &L.ptr[4], (op.flags & ANVIL_F_BIAS) != 0))) return rc;
  GemmParams &p = L.gp;
  memset(&p, 0, sizeof p);
  p.batch = batch; p.M = M; p.N = N; p.K = K;
  p.a_bstride = a_bs; p.bt_bstride = bt_bs; p.o_bstride = o_bs; p.o_rstride = o_rs;
  if (op.flags & ANVIL_F_RESIDUAL) {
    if ((op.flags & ANVIL_F_CHECKED) || (op.flags & ANVIL_F_LUT) || batch != 1 || o_rs != N || o_cs != 1 ||
        op.strides[4] != 0 || (op.in_bytes != 1 && op.in_bytes != 2) || (op.in2_bytes != 1 && op.in2_bytes != 2) ||
        op.shift2 < 0 || op.shift2 > 31)
      return fail(ANVIL_E_BAD_ARG, "op %d: bad fused residual gemm", op.op_index);
    if ((rc = resolve(m, op, 5, (uint64_t)M * N * op.in2_bytes, &L.ptr[5]))) return rc;
    p.res = L.ptr[5];
    p.res_bytes = op.in2_bytes;
    p.y_bytes = op.in_bytes;
    p.shift2 = (int)op.shift2;
    p.ma = (int)op.ma;
    p.mb = (int)op.mb;
  }
  p.o_group = op.strides[4];
  p.o_gstride = op.strides[5];
  p.o_cstride = op.strides[6] ? op.strides[6] : 1;
  p.A = (const int8_t *)L.ptr[0];
  p.BT = (const int8_t *)L.ptr[1];
  p.out = L.ptr[2];
  p.lut = (op.flags & ANVIL_F_LUT) ? (const int8_t *)L.ptr[3] : nullptr;
  p.bias = (op.flags & ANVIL_F_BIAS) ? (const int32_t *)L.ptr[4] : nullptr;
  if (p.bias && (((op.flags & ANVIL_F_BIAS_RND) != 0) == ((op.flags & ANVIL_F_CHECKED) != 0)))
    return fail(ANVIL_E_BAD_ARG, "op %d: a checked gemm takes a raw bias, an unchecked one a folded bias*M + round",
                op.op_index);
  p.mult = op.mult;
  p.shift = (int)op.shift;
  p.out_bytes = op.out_bytes;
  p.check = (op.flags & ANVIL_F_CHECKED) ? 1 : 0;
  p.flags = m->flags;
  p.op_index = op.op_index;
  if (op.flags & ANVIL_F_SPLIT) {
    // several linears of one input as one GEMM: dims[4] = chunk columns C, dims[5] = row-major columns R,
    // dims[6] = the transposed part's row group T; aux[c] = (M_c << 8) | s_c; off[6] = the transposed part
    const int64_t C = op.dims[4], Rr = op.dims[5], T = op.dims[6];
    const int64_t nch = C > 0 ? N / C : 0;
    if ((op.flags & (ANVIL_F_CHECKED | ANVIL_F_LUT | ANVIL_F_RESIDUAL | ANVIL_F_SIMT)) || batch != 1 ||
        op.out_bytes != 1 || C <= 0 || C % 256 || N % C || nch > 8 || Rr < 0 || Rr > N || Rr % C ||
        o_rs < Rr || o_rs % 16 || o_cs != 1 || op.strides[4] != 0 ||
        (Rr < N && (T <= 0 || T % 32 || M % T || T > (1ll << 31) - 1)))
      return fail(ANVIL_E_BAD_ARG, "op %d: bad split gemm", op.op_index);
    for (int64_t c = 0; c < nch; ++c) {
      const int64_t mc = op.aux[c] >> 8, sc = op.aux[c] & 255;
      if (mc < 0 || mc > 0x7fffffffll || sc > 31) return fail(ANVIL_E_BAD_ARG, "op %d: bad split chunk %lld",
                                                              op.op_index, (long long)c);
      p.smult[c] = (int)mc;
      p.sshift[c] = (int)sc;
    }
    if (Rr < N && (rc = resolve(m, op, 6, (uint64_t)M * (N - Rr), &L.ptr[6]))) return rc;
    p.split_c = (int)C;
    p.split_r = (int)Rr;
    p.o_group2 = T;
    p.out2 = L.ptr[6];
    if (!aligned16(p.out) || (p.out2 && !aligned16(p.out2)))
      return fail(ANVIL_E_BAD_ARG, "op %d: split gemm outputs must be 16-byte aligned", op.op_index);
  }
  const bool tc_ok = !(op.flags & ANVIL_F_SIMT) && K % 16 == 0 && a_bs % 16 == 0 && bt_bs % 16 == 0 &&
                     aligned16(p.A) && aligned16(p.BT) && M <= (1ll << 31) - 256 && N <= (1ll << 31) - 256 &&
                     batch <= (1ll << 31) - 1;
  L.tc = tc_ok;
  if (!tc_ok) {
    if (p.split_c) return fail(ANVIL_E_BAD_ARG, "op %d: a split gemm needs the tcgen05 path", op.op_index);
    return ANVIL_OK;
  }
  return tc_tiles(m, L);
}

// ATTENTION: dims = {B, H, T1, T2, hd}; strides = {q_b, q_h, q_t, k_b, k_h, k_t, o_b, o_t};
// off = {Q, K, VT (dense (B, H, hd, T2)), OUT, EXP_LUT}
static int prepare_attention(anvil_model *m, Launch &L) {
  const anvil_op &op = L.op;
  const int64_t B = op.dims[0], H = op.dims[1], T1 = op.dims[2], T2 = op.dims[3], HD = op.dims[4];
  const int64_t *st = op.strides;
  if (B < 1 || H < 1 || T1 < 1 || T2 < 1 || (HD != 64 && HD != 128))
    return fail(ANVIL_E_BAD_ARG, "op %d: attention needs hd 64 or 128 (got %lld)", op.op_index, (long long)HD);
  if (T2 > 1024 || T2 % 16) return fail(ANVIL_E_BAD_ARG, "op %d: attention needs T2 <= 1024, T2 % 16 == 0", op.op_index);
  for (int i = 0; i < 8; ++i)
    if (st[i] < 0 || st[i] % 16) return fail(ANVIL_E_BAD_ARG, "op %d: attention strides must be multiples of 16", op.op_index);
  if (op.one < 1 || op.one > 127 || op.shift < 0 || op.shift > 31 || op.shift2 < 0 || op.shift2 > 31)
    return fail(ANVIL_E_BAD_ARG, "op %d: bad attention constants", op.op_index);
  int rc;
  const uint64_t qb = (B - 1) * st[0] + (H - 1) * st[1] + (T1 - 1) * st[2] + HD;
  const uint64_t kb = (B - 1) * st[3] + (H - 1) * st[4] + (T2 - 1) * st[5] + HD;
  const uint64_t vb = B * H * HD * T2;
  const uint64_t ob = (B - 1) * st[6] + (T1 - 1) * st[7] + H * HD;
  if ((rc = resolve(m, op, 0, qb, &L.ptr[0]))) return rc;
  if ((rc = resolve(m, op, 1, kb, &L.ptr[1]))) return rc;
  if ((rc = resolve(m, op, 2, vb, &L.ptr[2]))) return rc;
  if ((rc = resolve(m, op, 3, ob, &L.ptr[3]))) return rc;
  if ((rc = resolve(m, op, 4, 1024, &L.ptr[4]))) return rc;
  for (int i = 0; i < 3; ++i)
    if (!aligned16(L.ptr[i])) return fail(ANVIL_E_BAD_ARG, "op %d: attention operand %d not 16-byte aligned", op.op_index, i);
  const CUtensorMapSwizzle qk_swz = HD == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  const uint64_t qdims[4] = {(uint64_t)HD, (uint64_t)H, (uint64_t)T1, (uint64_t)B};
  const uint64_t qstr[3] = {(uint64_t)st[1], (uint64_t)st[2], (uint64_t)(B > 1 ? st[0] : st[2] * T1)};
  // Q tiles arrive as four 32-row blocks (the kernel places them in either order), K tiles as 128 keys
  const uint32_t qbox[4] = {(uint32_t)HD, 1, 32, 1};
  if ((rc = make_map(&L.mapA, L.ptr[0], 4, qdims, qstr, qbox, qk_swz))) return rc;
  const uint64_t kdims[4] = {(uint64_t)HD, (uint64_t)H, (uint64_t)T2, (uint64_t)B};
  const uint64_t kstr[3] = {(uint64_t)st[4], (uint64_t)st[5], (uint64_t)(B > 1 ? st[3] : st[5] * T2)};
  const uint32_t kbox[4] = {(uint32_t)HD, 1, 128, 1};
  if ((rc = make_map(&L.mapB, L.ptr[1], 4, kdims, kstr, kbox, qk_swz))) return rc;
  const uint64_t vdims[2] = {(uint64_t)T2, (uint64_t)(B * H * HD)};
  const uint64_t vstr[1] = {(uint64_t)T2};
  const uint32_t vbox[2] = {128, (uint32_t)HD};
  if ((rc = make_map(&L.mapC, L.ptr[2], 2, vdims, vstr, vbox, CU_TENSOR_MAP_SWIZZLE_128B))) return rc;
  AttnParams &a = L.ap;
  memset(&a, 0, sizeof a);
  a.B = (int)B; a.H = (int)H; a.T1 = (int)T1; a.T2 = (int)T2;
  a.nqt = (int)((T1 + 127) / 128);
  a.o_bs = st[6]; a.o_rs = st[7];
  a.out = (int8_t *)L.ptr[3];
  a.lut = (const int32_t *)L.ptr[4];
  a.m1 = op.mult; a.s1 = (int)op.shift; a.m2 = op.mult2; a.s2 = (int)op.shift2;
  a.one = (int)op.one;
  a.causal = (op.flags & ANVIL_F_CAUSAL) ? 1 : 0;
  a.flags = m->flags;
  a.op_index = op.op_index;
  div_magic((int64_t)B * H, &a.bh_magic, &a.bh_shift);
  div_magic(H, &a.h_magic, &a.h_shift);
  // blocks of about two rounds of items: hb * nqt close to 2 x the CTAs, at most every (batch, head) pair
  {
    const int64_t grid = std::min<int64_t>((int64_t)B * H * a.nqt, m->sms);
    int64_t hb = std::max<int64_t>(1, (2 * grid + a.nqt / 2) / a.nqt);
    hb = std::min<int64_t>(hb, (int64_t)B * H);
    const int64_t last = (int64_t)B * H - ((int64_t)B * H - 1) / hb * hb;
    a.hb = (int)hb;
    a.hb_last = (int)last;
    div_magic(hb * a.nqt, &a.blk_magic, &a.blk_shift);
    div_magic(hb, &a.hb_magic, &a.hb_shift);
    div_magic(last, &a.last_magic, &a.last_shift);
  }
  L.hd = (int)HD;
  return ANVIL_OK;
}

static int prepare_op(anvil_model *m, Launch &L) {
  const anvil_op &op = L.op;
  int rc;
  const int64_t *d = op.dims;
  switch (op.kind) {
    case ANVIL_OP_GEMM:
      return prepare_gemm(m, L);
    case ANVIL_OP_LUT:
      if ((rc = resolve(m, op, 0, d[0], &L.ptr[0]))) return rc;
      if ((rc = resolve(m, op, 1, 256, &L.ptr[1]))) return rc;
      return resolve(m, op, 2, d[0], &L.ptr[2]);
    case ANVIL_OP_LUT_MUL:
      if ((rc = resolve(m, op, 0, d[0], &L.ptr[0]))) return rc;
      if ((rc = resolve(m, op, 1, d[0], &L.ptr[1]))) return rc;
      if ((rc = resolve(m, op, 2, 256, &L.ptr[2]))) return rc;
      return resolve(m, op, 3, d[0], &L.ptr[3]);
    case ANVIL_OP_ADD_REQUANT:
      if ((op.in_bytes != 1 && op.in_bytes != 2) || (op.in2_bytes != 1 && op.in2_bytes != 2) ||
          (op.out_bytes != 1 && op.out_bytes != 2))
        return fail(ANVIL_E_BAD_ARG, "op %d: add_requant operands must be i8 or i16", op.op_index);
      if ((rc = resolve(m, op, 0, d[0] * op.in_bytes, &L.ptr[0]))) return rc;
      if ((rc = resolve(m, op, 1, d[0] * op.in2_bytes, &L.ptr[1]))) return rc;
      return resolve(m, op, 2, d[0] * op.out_bytes, &L.ptr[2]);
    case ANVIL_OP_NORM:
      if (op.in_bytes != 1 && op.in_bytes != 2) return fail(ANVIL_E_BAD_ARG, "op %d: norm input must be i8 or i16", op.op_index);
      if (d[1] < 1 || d[2] < 1) return fail(ANVIL_E_BAD_ARG, "op %d: bad norm dims", op.op_index);
      if ((rc = resolve(m, op, 0, d[0] * d[1] * op.in_bytes, &L.ptr[0]))) return rc;
      if ((rc = resolve(m, op, 1, d[1], &L.ptr[1]))) return rc;
      if ((rc = resolve(m, op, 2, d[2] * 4, &L.ptr[2]))) return rc;
      if ((rc = resolve(m, op, 3, d[0] * d[1], &L.ptr[3]))) return rc;
      return resolve(m, op, 4, d[1], &L.ptr[4], (op.flags & ANVIL_F_BIAS) != 0);
    case ANVIL_OP_SOFTMAX:
      if (op.out_bytes != 1 && op.out_bytes != 4) return fail(ANVIL_E_BAD_ARG, "op %d: softmax output must be i8 or i32", op.op_index);
      if ((rc = resolve(m, op, 0, d[0] * d[1] * d[2], &L.ptr[0]))) return rc;
      if ((rc = resolve(m, op, 1, 256 * 4, &L.ptr[1]))) return rc;
      return resolve(m, op, 2, d[0] * d[1] * d[2] * op.out_bytes, &L.ptr[2]);
    case ANVIL_OP_TRANSPOSE: {
      const int rank = (int)d[0];
      if (rank < 1 || rank > 6 || (op.in_bytes != 1 && op.in_bytes != 2 && op.in_bytes != 4))
        return fail(ANVIL_E_BAD_ARG, "op %d: bad transpose rank/element size", op.op_index);
      int64_t total = 1, span = 0;
      for (int i = 0; i < rank; ++i) {
        if (d[1 + i] < 1 || op.strides[i] < 0) return fail(ANVIL_E_BAD_ARG, "op %d: bad transpose dims", op.op_index);
        total *= d[1 + i];
        span += (d[1 + i] - 1) * op.strides[i];
      }
      if ((rc = resolve(m, op, 0, (span + 1) * op.in_bytes, &L.ptr[0]))) return rc;
      return resolve(m, op, 1, total * op.in_bytes, &L.ptr[1]);
    }
    case ANVIL_OP_EMBED:
      if ((rc = resolve(m, op, 0, d[0] * d[1] * 4, &L.ptr[0]))) return rc;
      if ((rc = resolve(m, op, 1, d[3] * d[2], &L.ptr[1]))) return rc;
      if ((rc = resolve(m, op, 2, d[1] * d[2], &L.ptr[2]))) return rc;
      return resolve(m, op, 3, d[0] * d[1] * d[2], &L.ptr[3]);
    case ANVIL_OP_COPY:
      if ((rc = resolve(m, op, 0, d[0], &L.ptr[0]))) return rc;
      return resolve(m, op, 1, d[0], &L.ptr[1]);
    case ANVIL_OP_ATTENTION:
      return prepare_attention(m, L);
    default:
      return fail(ANVIL_E_UNSUPPORTED, "op %d: unknown kind %d", op.op_index, op.kind);
  }
}

extern "C" int anvil_model_prepare(anvil_model *m, const anvil_op *ops, int n_ops, uint64_t arena_bytes) {
  if (!m || (n_ops && !ops) || n_ops < 0) return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_prepare");
  CK(cudaSetDevice(m->device));
  if (m->free_pending) CK(cudaEventSynchronize(m->ev_free));
  CK(cudaStreamSynchronize(m->stream));
  if (m->graph) {
    cudaGraphExecDestroy(m->graph);
    m->graph = nullptr;
  }
  if (arena_bytes > m->arena_bytes) {
    if (m->arena) cudaFree(m->arena);
    m->arena = nullptr;
    m->arena_bytes = 0;
    if (cudaMalloc(&m->arena, arena_bytes) != cudaSuccess) {
      cudaGetLastError();
      return fail(ANVIL_E_OOM, "cannot allocate a %llu-byte activation arena", (unsigned long long)arena_bytes);
    }
    m->arena_bytes = arena_bytes;
  }
  std::vector<Launch> ls(n_ops);
  for (int i = 0; i < n_ops; ++i) {
    ls[i].op = ops[i];
    for (int s = 0; s < 8; ++s) ls[i].ptr[s] = nullptr;
    int rc = prepare_op(m, ls[i]);
    if (rc) return rc;
  }
  m->launches.swap(ls);
  for (auto e : m->events) cudaEventDestroy(e);
  m->events.clear();
  return ANVIL_OK;
}

static int grid_for(anvil_model *m, int64_t work, int per_block, int max_waves = 8) {
  int64_t g = (work + per_block - 1) / per_block;
  int64_t cap = (int64_t)m->sms * max_waves;
  if (g > cap) g = cap;
  return (int)std::max<int64_t>(1, g);
}

static int launch_op(anvil_model *m, Launch &L) {
  const anvil_op &op = L.op;
  const int64_t *d = op.dims;
  cudaStream_t st = m->stream;
  const bool chk = (op.flags & ANVIL_F_CHECKED) != 0;
  uint32_t *fl = m->flags;
  const int oi = op.op_index;
  switch (op.kind) {
    case ANVIL_OP_GEMM: {
      GemmParams &p = L.gp;
      if (L.tc && L.pair) {
        const int ncl = (int)std::min<int64_t>(p.tiles, pair_clusters(m));
        cudaLaunchAttribute attr[1];
        const cudaLaunchConfig_t cfg = pair_config(dim3((unsigned)(2 * ncl)), st, attr);
        cudaError_t e;
        if (op.out_bytes == 1)
          e = cudaLaunchKernelEx(&cfg, p.res ? qgemm_tc_kernel<256, 1, true, true> : qgemm_tc_kernel<256, 1, false, true>,
                                 L.mapA, L.mapB, L.mapC, L.mapC2, p);
        else
          e = cudaLaunchKernelEx(&cfg, p.res ? qgemm_tc_kernel<256, 2, true, true> : qgemm_tc_kernel<256, 2, false, true>,
                                 L.mapA, L.mapB, L.mapC, L.mapC2, p);
        if (e != cudaSuccess) return fail(ANVIL_E_CUDA, "op %d: pair gemm launch failed: %s", oi, cudaGetErrorString(e));
      } else if (L.tc) {
        const int grid = (int)std::min<int64_t>(p.tiles, m->sms);
#define TC_LAUNCH(BN, OB)                                                                                       \
  do {                                                                                                          \
    if (p.res)                                                                                                  \
      qgemm_tc_kernel<BN, OB, true><<<grid, TC_THREADS, TcCfg<BN>::SMEM_BYTES, st>>>(L.mapA, L.mapB, L.mapC, L.mapC2, p); \
    else                                                                                                        \
      qgemm_tc_kernel<BN, OB, false><<<grid, TC_THREADS, TcCfg<BN>::SMEM_BYTES, st>>>(L.mapA, L.mapB, L.mapC, L.mapC2, p);\
  } while (0)
        if (L.bn == 64) { if (op.out_bytes == 1) TC_LAUNCH(64, 1); else TC_LAUNCH(64, 2); }
        else if (L.bn == 128) { if (op.out_bytes == 1) TC_LAUNCH(128, 1); else TC_LAUNCH(128, 2); }
        else { if (op.out_bytes == 1) TC_LAUNCH(256, 1); else TC_LAUNCH(256, 2); }
#undef TC_LAUNCH
      } else {
        dim3 grid((unsigned)((p.N + 63) / 64), (unsigned)((p.M + 63) / 64), (unsigned)p.batch);
        if (grid.y > 65535 || grid.z > 65535) return fail(ANVIL_E_BAD_ARG, "op %d: gemm too large for the SIMT path", oi);
        if (chk) qgemm_simt_kernel<true><<<grid, 256, 0, st>>>(p);
        else qgemm_simt_kernel<false><<<grid, 256, 0, st>>>(p);
      }
      break;
    }
    case ANVIL_OP_LUT:
      lut_kernel<<<grid_for(m, d[0], 256 * 16), 256, 0, st>>>((const int8_t *)L.ptr[0], (const int8_t *)L.ptr[1],
                                                            (int8_t *)L.ptr[2], d[0]);
      break;
    case ANVIL_OP_LUT_MUL: {
      auto k = chk ? lut_mul_kernel<true> : lut_mul_kernel<false>;
      k<<<grid_for(m, d[0], 256 * 4), 256, 0, st>>>((const int8_t *)L.ptr[0], (const int8_t *)L.ptr[1],
                                                   (const int8_t *)L.ptr[2], (int8_t *)L.ptr[3], d[0], op.mult,
                                                   (int)op.shift, fl, oi);
      break;
    }
    case ANVIL_OP_ADD_REQUANT: {
      const int code = (op.in_bytes - 1) * 4 + (op.in2_bytes - 1) * 2 + (op.out_bytes - 1) + (chk ? 8 : 0);
      void (*k)(const void *, const void *, void *, int64_t, long long, long long, int, uint32_t *, int) = nullptr;
      switch (code) {
#define AR(C, A, B, O, CH) case C: k = add_requant_kernel<A, B, O, CH>; break;
        AR(0, 1, 1, 1, false) AR(1, 1, 1, 2, false) AR(2, 1, 2, 1, false) AR(3, 1, 2, 2, false)
        AR(4, 2, 1, 1, false) AR(5, 2, 1, 2, false) AR(6, 2, 2, 1, false) AR(7, 2, 2, 2, false)
        AR(8, 1, 1, 1, true) AR(9, 1, 1, 2, true) AR(10, 1, 2, 1, true) AR(11, 1, 2, 2, true)
        AR(12, 2, 1, 1, true) AR(13, 2, 1, 2, true) AR(14, 2, 2, 1, true) AR(15, 2, 2, 2, true)
#undef AR
      }
      k<<<grid_for(m, d[0], 256 * 8), 256, 0, st>>>(L.ptr[0], L.ptr[1], L.ptr[2], d[0], op.ma, op.mb, (int)op.shift,
                                                   fl, oi);
      break;
    }
    case ANVIL_OP_NORM: {
      const int dd = (int)op.dims[1];
      if (!chk && op.in_bytes == 1 && dd % 16 == 0 && dd <= 2048 && aligned16(L.ptr[0]) &&
          aligned16(L.ptr[1]) && aligned16(L.ptr[3]) && (!L.ptr[4] || aligned16(L.ptr[4]))) {
        const int8_t *bias = (op.flags & ANVIL_F_BIAS) ? (const int8_t *)L.ptr[4] : nullptr;
        if (dd % 256 == 0) {          // whole 8-byte vectors on every lane: the register-resident row kernel
          // one resident wave: every warp then walks several rows with the next row's load in flight
#define NR_LAUNCH(NV8)                                                                                            \
  do {                                                                                                            \
    auto kern = bias ? norm_row_kernel<NV8, true> : norm_row_kernel<NV8, false>;                                  \
    int per_sm = 0;                                                                                               \
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, 0) != cudaSuccess) {                    \
      cudaGetLastError();                                                                                         \
      per_sm = 1;                                                                                                 \
    }                                                                                                             \
    const int g = grid_for(m, op.dims[0], 8, std::max(1, per_sm));                                                \
    kern<<<g, 256, 0, st>>>((const int8_t *)L.ptr[0], (const int8_t *)L.ptr[1], (const int32_t *)L.ptr[2], bias,  \
                            (int8_t *)L.ptr[3], op.dims[0], (int)op.dims[2], (int)op.mult, (int)op.shift,         \
                            (int)op.ss_shift, (int)op.ss_init, (op.flags & ANVIL_F_CENTER) ? 1 : 0);              \
  } while (0)
          switch (dd / 256) {
            case 1: NR_LAUNCH(1); break;
            case 2: NR_LAUNCH(2); break;
            case 3: NR_LAUNCH(3); break;
            case 4: NR_LAUNCH(4); break;
            case 5: NR_LAUNCH(5); break;
            case 6: NR_LAUNCH(6); break;
            case 7: NR_LAUNCH(7); break;
            default: NR_LAUNCH(8); break;
          }
#undef NR_LAUNCH
          break;
        }
        const int nv = (dd / 16 + 31) / 32;
        const int g = grid_for(m, op.dims[0], 8, 16);
#define NV_LAUNCH(NV)                                                                                             \
  norm_vec_kernel<NV><<<g, 256, 0, st>>>((const int8_t *)L.ptr[0], (const int8_t *)L.ptr[1],                      \
                                         (const int32_t *)L.ptr[2], bias, (int8_t *)L.ptr[3], op.dims[0], dd,      \
                                         (int)op.dims[2], (int)op.mult, (int)op.shift, (int)op.ss_shift,          \
                                         (int)op.ss_init, (op.flags & ANVIL_F_CENTER) ? 1 : 0)
        if (nv <= 1) NV_LAUNCH(1);
        else if (nv == 2) NV_LAUNCH(2);
        else NV_LAUNCH(4);
#undef NV_LAUNCH
        break;
      }
      auto k = op.in_bytes == 1 ? (chk ? norm_kernel<1, true> : norm_kernel<1, false>)
                                : (chk ? norm_kernel<2, true> : norm_kernel<2, false>);
      k<<<grid_for(m, d[0], 8), 256, 0, st>>>(L.ptr[0], (const int8_t *)L.ptr[1], (const int32_t *)L.ptr[2],
                                             (const int8_t *)L.ptr[4], (int8_t *)L.ptr[3], d[0], (int)d[1], (int)d[2],
                                             op.mult, (int)op.shift, (int)op.ss_shift, op.ss_init,
                                             (op.flags & ANVIL_F_CENTER) ? 1 : 0, fl, oi);
      break;
    }
    case ANVIL_OP_SOFTMAX: {
      const int64_t rows = d[0] * d[1];
      auto k = op.out_bytes == 1 ? (chk ? softmax_kernel<1, true> : softmax_kernel<1, false>)
                                 : (chk ? softmax_kernel<4, true> : softmax_kernel<4, false>);
      k<<<grid_for(m, rows, 8), 256, 0, st>>>((const int8_t *)L.ptr[0], (const int32_t *)L.ptr[1], L.ptr[2], rows,
                                             (int)d[1], (int)d[2], op.one, (op.flags & ANVIL_F_CAUSAL) ? 1 : 0, fl,
                                             oi);
      break;
    }
    case ANVIL_OP_TRANSPOSE: {
      TransposeDims td;
      td.rank = (int)d[0];
      int64_t total = 1, span = 0;
      for (int i = 0; i < 6; ++i) {
        td.n[i] = i < td.rank ? d[1 + i] : 1;
        td.st[i] = i < td.rank ? op.strides[i] : 0;
        total *= td.n[i];
        span += (td.n[i] - 1) * td.st[i];
        div_magic(td.n[i], &td.mg[i], &td.sh[i]);
      }
      td.small = total < (1ll << 31) && span < (1ll << 31);
      const int g = grid_for(m, total, 256);
      if (op.in_bytes == 1) transpose_kernel<1><<<g, 256, 0, st>>>(L.ptr[0], L.ptr[1], td, total);
      else if (op.in_bytes == 2) transpose_kernel<2><<<g, 256, 0, st>>>(L.ptr[0], L.ptr[1], td, total);
      else transpose_kernel<4><<<g, 256, 0, st>>>(L.ptr[0], L.ptr[1], td, total);
      break;
    }
    case ANVIL_OP_EMBED: {
      auto k = chk ? embed_kernel<true> : embed_kernel<false>;
      const int64_t rows = d[0] * d[1];
      k<<<grid_for(m, rows, 8), 256, 0, st>>>((const int32_t *)L.ptr[0], (const int8_t *)L.ptr[1],
                                             (const int8_t *)L.ptr[2], (int8_t *)L.ptr[3], rows, (int)d[1], (int)d[2],
                                             d[3], op.ma, op.mb, (int)op.shift, fl, oi);
      break;
    }
    case ANVIL_OP_COPY:
      CK(cudaMemcpyAsync(L.ptr[1], L.ptr[0], d[0], cudaMemcpyDeviceToDevice, st));
      break;
    case ANVIL_OP_ATTENTION: {
      const AttnParams &a = L.ap;
      const int64_t tiles = (int64_t)a.B * a.H * a.nqt;      // persistent: one CTA per SM walks the tiles
      if (tiles > 0x7fffffff) return fail(ANVIL_E_BAD_ARG, "op %d: attention has too many tiles", oi);
      const int64_t grid = std::min<int64_t>(tiles, m->sms);
      if (L.hd == 64)
        attn_kernel<64><<<(unsigned)grid, ATTN_THREADS, AttnCfg<64>::SMEM_BYTES, st>>>(L.mapA, L.mapB, L.mapC, a);
      else
        attn_kernel<128><<<(unsigned)grid, ATTN_THREADS, AttnCfg<128>::SMEM_BYTES, st>>>(L.mapA, L.mapB, L.mapC, a);
      break;
    }
    default:
      return fail(ANVIL_E_UNSUPPORTED, "op %d: unknown kind %d", oi, op.kind);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(ANVIL_E_CUDA, "op %d (kind %d) launch failed: %s", oi, op.kind, cudaGetErrorString(e));
  return ANVIL_OK;
}

static int check_flags(anvil_model *m, const uint32_t *h) {
  if (h[FLAG_TIMEOUT])
    return fail(ANVIL_E_TIMEOUT, "op %u: a device wait timed out", h[FLAG_TIMEOUT] - 1);
  if (h[FLAG_OVERFLOW])
    return fail(ANVIL_E_OVERFLOW, "op %u: an int32 intermediate left int32", h[FLAG_OVERFLOW] - 1);
  if (h[FLAG_INDEX])
    return fail(ANVIL_E_INDEX, "op %u: an index left its table", h[FLAG_INDEX] - 1);
  return ANVIL_OK;
}

// Self-test of the device wait bound: two warps wait on an mbarrier that nothing arrives on, through the same
// bounded wait the kernels use (here with the caller's limit); the wait gives up, raises the timeout flag and sets
// the block's abort word, so the other warp gives up too, and the kernel returns.
__global__ void __launch_bounds__(64) selftest_wait_kernel(uint32_t *flags, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_word;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_word = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0)
    mbar_wait_for(&bar, 0, reinterpret_cast<volatile int *>(&abort_word), flags, 0, limit_ns);
  __syncwarp();
}

extern "C" int anvil_model_selftest_timeout(anvil_model *m, uint64_t wait_ns) {
  if (!m || wait_ns == 0 || wait_ns > ANVIL_DEV_WAIT_NS)
    return fail(ANVIL_E_BAD_ARG, "anvil_model_selftest_timeout: wait_ns must be in (0, %llu]",
                (unsigned long long)ANVIL_DEV_WAIT_NS);
  CK(cudaSetDevice(m->device));
  CK(cudaMemsetAsync(m->flags, 0, FLAG_WORDS * sizeof(uint32_t), m->stream));
  selftest_wait_kernel<<<1, 64, 0, m->stream>>>(m->flags, wait_ns);
  CK(cudaGetLastError());
  uint32_t hflags[FLAG_WORDS];
  CK(cudaMemcpyAsync(hflags, m->flags, sizeof hflags, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  return check_flags(m, hflags);
}

extern "C" int anvil_model_run(anvil_model *m, const anvil_io *inputs, int n_inputs, const anvil_io *outputs,
                               int n_outputs, float *kernel_us) {
  if (!m) return fail(ANVIL_E_BAD_ARG, "model is NULL");
  CK(cudaSetDevice(m->device));
  cudaStream_t st = m->stream;
  if (int rc = join_copies(m)) return rc;
  for (int i = 0; i < n_inputs; ++i) {
    const anvil_io &io = inputs[i];
    if (io.offset > m->arena_bytes || io.bytes > m->arena_bytes - io.offset)
      return fail(ANVIL_E_BAD_ARG, "input %d: [%llu, +%llu) outside the arena", i, (unsigned long long)io.offset,
                  (unsigned long long)io.bytes);
    CK(cudaMemcpyAsync(static_cast<uint8_t *>(m->arena) + io.offset, io.host, io.bytes, cudaMemcpyHostToDevice, st));
  }
  CK(cudaMemsetAsync(m->flags, 0, FLAG_WORDS * sizeof(uint32_t), st));
  const int n = (int)m->launches.size();
  if (kernel_us && (int)m->events.size() < n + 1) {
    for (auto e : m->events) cudaEventDestroy(e);
    m->events.assign(n + 1, nullptr);
    for (auto &e : m->events) CK(cudaEventCreate(&e));
  }
  if (kernel_us) CK(cudaEventRecord(m->events[0], st));
  for (int i = 0; i < n; ++i) {
    int rc = launch_op(m, m->launches[i]);
    if (rc) return rc;
    if (kernel_us) CK(cudaEventRecord(m->events[i + 1], st));
  }
  uint32_t hflags[FLAG_WORDS];
  CK(cudaMemcpyAsync(hflags, m->flags, sizeof hflags, cudaMemcpyDeviceToHost, st));
  for (int i = 0; i < n_outputs; ++i) {
    const anvil_io &io = outputs[i];
    if (io.offset > m->arena_bytes || io.bytes > m->arena_bytes - io.offset)
      return fail(ANVIL_E_BAD_ARG, "output %d: [%llu, +%llu) outside the arena", i, (unsigned long long)io.offset,
                  (unsigned long long)io.bytes);
    CK(cudaMemcpyAsync(io.host, static_cast<uint8_t *>(m->arena) + io.offset, io.bytes, cudaMemcpyDeviceToHost, st));
  }
  CK(cudaStreamSynchronize(st));
  if (kernel_us)
    for (int i = 0; i < n; ++i) {
      float ms = 0;
      CK(cudaEventElapsedTime(&ms, m->events[i], m->events[i + 1]));
      kernel_us[i] = ms * 1000.0f;
    }
  return check_flags(m, hflags);
}

// Capture the launch list once as a CUDA graph (re-captured after every anvil_model_prepare).
static int ensure_graph(anvil_model *m) {
  if (m->graph) return ANVIL_OK;
  cudaGraph_t g;
  CK(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal));
  int rc = ANVIL_OK;
  for (auto &L : m->launches)
    if ((rc = launch_op(m, L))) break;
  cudaError_t e = cudaStreamEndCapture(m->stream, &g);
  if (rc) return rc;
  if (e != cudaSuccess) return fail(ANVIL_E_CUDA, "graph capture failed: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(&m->graph, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) return fail(ANVIL_E_CUDA, "graph instantiate failed: %s", cudaGetErrorString(e));
  return ANVIL_OK;
}

static int check_io(const anvil_model *m, const anvil_io *io, int n, const char *what) {
  for (int i = 0; i < n; ++i)
    if (io[i].offset > m->arena_bytes || io[i].bytes > m->arena_bytes - io[i].offset)
      return fail(ANVIL_E_BAD_ARG, "%s %d: [%llu, +%llu) outside the arena", what, i,
                  (unsigned long long)io[i].offset, (unsigned long long)io[i].bytes);
  return ANVIL_OK;
}

extern "C" int anvil_model_enqueue(anvil_model *m, const anvil_io *inputs, int n_inputs, const anvil_io *outputs,
                                   int n_outputs, anvil_model *after) {
  if (!m || n_inputs < 0 || n_outputs < 0 || (n_inputs && !inputs) || (n_outputs && !outputs))
    return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_enqueue");
  if (after && (after == m || after->device != m->device))
    return fail(ANVIL_E_BAD_ARG, "anvil_model_enqueue: `after` must be another model on the same device");
  int rc;
  if ((rc = check_io(m, inputs, n_inputs, "input")) || (rc = check_io(m, outputs, n_outputs, "output"))) return rc;
  CK(cudaSetDevice(m->device));
  cudaStream_t st = m->stream;
  if ((rc = ensure_graph(m))) return rc;
  if (!m->ev_in) CK(cudaEventCreateWithFlags(&m->ev_in, cudaEventDisableTiming));
  if (!m->ev_run) CK(cudaEventCreateWithFlags(&m->ev_run, cudaEventDisableTiming));
  if (!m->ev_free) CK(cudaEventCreateWithFlags(&m->ev_free, cudaEventDisableTiming));
  cudaStream_t sin, sout;
  if ((rc = copy_streams(m->device, &sin, &sout))) return rc;
  // copies in on the device's copy-in stream, once this arena's previous chunk has been copied out (and after
  // whatever ran on the model's own stream); copies of consecutive chunks follow each other in that one stream
  if (m->free_pending) CK(cudaStreamWaitEvent(sin, m->ev_free, 0));
  CK(cudaEventRecord(m->ev_in, st));
  CK(cudaStreamWaitEvent(sin, m->ev_in, 0));
  for (int i = 0; i < n_inputs; ++i)
    CK(cudaMemcpyAsync(static_cast<uint8_t *>(m->arena) + inputs[i].offset, inputs[i].host, inputs[i].bytes,
                       cudaMemcpyHostToDevice, sin));
  CK(cudaEventRecord(m->ev_in, sin));
  // the launch chain on the model's stream once its inputs are in and `after`'s chain is done (one chunk's
  // kernels on the SMs at a time)
  CK(cudaStreamWaitEvent(st, m->ev_in, 0));
  if (after && after->ev_run) CK(cudaStreamWaitEvent(st, after->ev_run, 0));
  CK(cudaGraphLaunch(m->graph, st));
  CK(cudaEventRecord(m->ev_run, st));
  // copies out on the device's copy-out stream once the chain is done
  CK(cudaStreamWaitEvent(sout, m->ev_run, 0));
  for (int i = 0; i < n_outputs; ++i)
    CK(cudaMemcpyAsync(outputs[i].host, static_cast<uint8_t *>(m->arena) + outputs[i].offset, outputs[i].bytes,
                       cudaMemcpyDeviceToHost, sout));
  CK(cudaEventRecord(m->ev_free, sout));
  m->free_pending = true;
  return ANVIL_OK;
}

extern "C" int anvil_model_clear_flags(anvil_model *m) {
  if (!m) return fail(ANVIL_E_BAD_ARG, "model is NULL");
  CK(cudaSetDevice(m->device));
  CK(cudaMemsetAsync(m->flags, 0, FLAG_WORDS * sizeof(uint32_t), m->stream));
  return ANVIL_OK;
}

extern "C" int anvil_model_wait(anvil_model *m) {
  if (!m) return fail(ANVIL_E_BAD_ARG, "model is NULL");
  CK(cudaSetDevice(m->device));
  uint32_t hflags[FLAG_WORDS];
  CK(cudaMemcpyAsync(hflags, m->flags, sizeof hflags, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  if (m->free_pending) CK(cudaEventSynchronize(m->ev_free));
  return check_flags(m, hflags);
}

// Completion tickets: the asynchronous form of anvil_model_wait. A ticket marks everything enqueued on the model's
// stream so far; the check words that work raised are snapshotted into the ticket's slot and then cleared in stream
// order, so each ticket reports exactly the checks of the work between the previous ticket (or clear_flags) and
// itself, however much later work has been enqueued behind it by the time it is waited on.
extern "C" int anvil_model_record(anvil_model *m, uint64_t *ticket) {
  if (!m || !ticket) return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_record");
  CK(cudaSetDevice(m->device));
  const int slot = (int)(m->ticket_next % anvil_model::TICKETS);
  if (m->ticket_pending[slot])
    return fail(ANVIL_E_BAD_ARG, "anvil_model_record: %d tickets are outstanding on this model; wait on the oldest "
                "first", anvil_model::TICKETS);
  if (!m->ticket_flags) CK(cudaMalloc(&m->ticket_flags, anvil_model::TICKETS * FLAG_WORDS * sizeof(uint32_t)));
  if (!m->status_stream) CK(cudaStreamCreateWithFlags(&m->status_stream, cudaStreamNonBlocking));
  if (!m->ticket_ev[slot]) CK(cudaEventCreateWithFlags(&m->ticket_ev[slot], cudaEventDisableTiming));
  uint32_t *snap = m->ticket_flags + slot * FLAG_WORDS;
  CK(cudaMemcpyAsync(snap, m->flags, FLAG_WORDS * sizeof(uint32_t), cudaMemcpyDeviceToDevice, m->stream));
  CK(cudaMemsetAsync(m->flags, 0, FLAG_WORDS * sizeof(uint32_t), m->stream));
  if (m->free_pending) {
    // the ticket also covers this model's copies out, queued on the device's copy-out stream
    cudaStream_t sin, sout;
    if (int rc = copy_streams(m->device, &sin, &sout)) return rc;
    if (!m->ticket_snap[slot]) CK(cudaEventCreateWithFlags(&m->ticket_snap[slot], cudaEventDisableTiming));
    CK(cudaEventRecord(m->ticket_snap[slot], m->stream));
    CK(cudaStreamWaitEvent(sout, m->ticket_snap[slot], 0));
    CK(cudaEventRecord(m->ticket_ev[slot], sout));
  } else {
    CK(cudaEventRecord(m->ticket_ev[slot], m->stream));
  }
  m->ticket_pending[slot] = true;
  *ticket = m->ticket_next++;
  return ANVIL_OK;
}

extern "C" int anvil_model_wait_ticket(anvil_model *m, uint64_t ticket) {
  if (!m) return fail(ANVIL_E_BAD_ARG, "model is NULL");
  const int slot = (int)(ticket % anvil_model::TICKETS);
  if (ticket >= m->ticket_next || m->ticket_next - ticket > (uint64_t)anvil_model::TICKETS ||
      !m->ticket_pending[slot])
    return fail(ANVIL_E_BAD_ARG, "anvil_model_wait_ticket: ticket %llu is not outstanding on this model",
                (unsigned long long)ticket);
  CK(cudaSetDevice(m->device));
  CK(cudaEventSynchronize(m->ticket_ev[slot]));
  uint32_t hflags[FLAG_WORDS];
  CK(cudaMemcpyAsync(hflags, m->ticket_flags + slot * FLAG_WORDS, sizeof hflags, cudaMemcpyDeviceToHost,
                     m->status_stream));
  CK(cudaStreamSynchronize(m->status_stream));
  m->ticket_pending[slot] = false;
  return check_flags(m, hflags);
}

// Per-launch device time inside a CUDA-graph replay of the chain: a second graph is captured with a timing event
// recorded (as an external event node) before the first launch and after every launch, replayed `iters` times on
// the model's stream, and the shortest time between consecutive events over the replays kept per launch. The launches follow each
// other as in the chain's own graph, so a launch's figure excludes the host-side launch cost that events around
// separately issued launches include. The production graph is untouched; the timing graph is freed before return.
extern "C" int anvil_model_time_launches(anvil_model *m, int iters, float *op_us) {
  if (!m || iters < 1 || !op_us) return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_time_launches");
  CK(cudaSetDevice(m->device));
  cudaStream_t st = m->stream;
  if (int rc = join_copies(m)) return rc;
  const int n = (int)m->launches.size();
  if (n == 0) return ANVIL_OK;
  std::vector<cudaEvent_t> ev(n + 1, nullptr);
  for (auto &e : ev) CK(cudaEventCreate(&e));
  auto release = [&](cudaGraphExec_t gx) {
    if (gx) cudaGraphExecDestroy(gx);
    for (auto e : ev) cudaEventDestroy(e);
  };
  cudaGraph_t g;
  CK(cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal));
  int rc = ANVIL_OK;
  cudaError_t e = cudaEventRecordWithFlags(ev[0], st, cudaEventRecordExternal);
  for (int i = 0; i < n && !rc && e == cudaSuccess; ++i) {
    rc = launch_op(m, m->launches[i]);
    if (!rc) e = cudaEventRecordWithFlags(ev[i + 1], st, cudaEventRecordExternal);
  }
  cudaError_t e2 = cudaStreamEndCapture(st, &g);
  if (rc || e != cudaSuccess || e2 != cudaSuccess) {
    if (e2 == cudaSuccess) cudaGraphDestroy(g);
    release(nullptr);
    if (rc) return rc;
    return fail(ANVIL_E_CUDA, "timing graph capture failed: %s",
                cudaGetErrorString(e != cudaSuccess ? e : e2));
  }
  cudaGraphExec_t gx = nullptr;
  e = cudaGraphInstantiate(&gx, g, 0);
  cudaGraphDestroy(g);
  if (e != cudaSuccess) {
    release(nullptr);
    return fail(ANVIL_E_CUDA, "timing graph instantiate failed: %s", cudaGetErrorString(e));
  }
  std::vector<float> best(n, 3.0e38f);
  CK(cudaMemsetAsync(m->flags, 0, FLAG_WORDS * sizeof(uint32_t), st));
  for (int it = 0; it < iters; ++it) {
    if ((e = cudaGraphLaunch(gx, st)) == cudaSuccess) e = cudaStreamSynchronize(st);
    for (int i = 0; i < n && e == cudaSuccess; ++i) {
      float t = 0;
      e = cudaEventElapsedTime(&t, ev[i], ev[i + 1]);
      best[i] = std::min(best[i], 1000.0f * t);
    }
    if (e != cudaSuccess) {
      release(gx);
      return fail(ANVIL_E_CUDA, "timing replay failed: %s", cudaGetErrorString(e));
    }
  }
  release(gx);
  for (int i = 0; i < n; ++i) op_us[i] = best[i];
  uint32_t hflags[FLAG_WORDS];
  CK(cudaMemcpyAsync(hflags, m->flags, sizeof hflags, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  return check_flags(m, hflags);
}

extern "C" int anvil_model_run_device(anvil_model *m, int iters, int use_graph, float *ms) {
  if (!m || iters < 1) return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_run_device");
  CK(cudaSetDevice(m->device));
  cudaStream_t st = m->stream;
  if (int rc = join_copies(m)) return rc;
  if (use_graph) {
    int rc = ensure_graph(m);
    if (rc) return rc;
  }
  cudaEvent_t e0, e1;
  CK(cudaEventCreate(&e0));
  CK(cudaEventCreate(&e1));
  CK(cudaMemsetAsync(m->flags, 0, FLAG_WORDS * sizeof(uint32_t), st));
  CK(cudaEventRecord(e0, st));
  for (int it = 0; it < iters; ++it) {
    if (use_graph) {
      CK(cudaGraphLaunch(m->graph, st));
    } else {
      for (auto &L : m->launches) {
        int rc = launch_op(m, L);
        if (rc) return rc;
      }
    }
  }
  CK(cudaEventRecord(e1, st));
  uint32_t hflags[FLAG_WORDS];
  CK(cudaMemcpyAsync(hflags, m->flags, sizeof hflags, cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  float t = 0;
  CK(cudaEventElapsedTime(&t, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (ms) *ms = t;
  return check_flags(m, hflags);
}

extern "C" int anvil_model_read(anvil_model *m, uint64_t offset, void *host, uint64_t bytes) {
  if (!m || !host) return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_read");
  if (offset > m->arena_bytes || bytes > m->arena_bytes - offset) return fail(ANVIL_E_BAD_ARG, "read outside the arena");
  CK(cudaSetDevice(m->device));
  if (int rc = join_copies(m)) return rc;
  CK(cudaMemcpyAsync(host, static_cast<uint8_t *>(m->arena) + offset, bytes, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  return ANVIL_OK;
}

extern "C" int anvil_model_write(anvil_model *m, uint64_t offset, const void *host, uint64_t bytes) {
  if (!m || !host) return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_write");
  if (offset > m->arena_bytes || bytes > m->arena_bytes - offset) return fail(ANVIL_E_BAD_ARG, "write outside the arena");
  CK(cudaSetDevice(m->device));
  if (int rc = join_copies(m)) return rc;
  CK(cudaMemcpyAsync(static_cast<uint8_t *>(m->arena) + offset, host, bytes, cudaMemcpyHostToDevice, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  return ANVIL_OK;
}

extern "C" int anvil_model_read_const(anvil_model *m, uint64_t offset, void *host, uint64_t bytes) {
  if (!m || !host) return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_read_const");
  if (offset > m->const_bytes || bytes > m->const_bytes - offset)
    return fail(ANVIL_E_BAD_ARG, "read outside the const region");
  CK(cudaSetDevice(m->device));
  CK(cudaMemcpyAsync(host, static_cast<uint8_t *>(m->consts) + offset, bytes, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  return ANVIL_OK;
}

extern "C" int anvil_model_describe(anvil_model *m, int op, int64_t *info) {
  if (!m || !info || op < 0 || op >= (int)m->launches.size())
    return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_model_describe");
  const Launch &L = m->launches[op];
  for (int i = 0; i < 4; ++i) info[i] = 0;
  if (L.op.kind == ANVIL_OP_GEMM) {
    const GemmParams &p = L.gp;
    if (L.tc) {
      info[0] = L.bn;
      info[1] = L.pair ? 2 : 1;
      info[2] = p.tiles;
      info[3] = L.pair ? 2 * std::min<int64_t>(p.tiles, pair_clusters(m)) : std::min<int64_t>(p.tiles, m->sms);
    } else {
      info[2] = ((p.N + 63) / 64) * ((p.M + 63) / 64) * p.batch;
      info[3] = info[2];
    }
  } else if (L.op.kind == ANVIL_OP_ATTENTION) {
    const int64_t items = (int64_t)L.ap.B * L.ap.H * L.ap.nqt;
    info[0] = L.hd;
    info[2] = items;
    info[3] = std::min<int64_t>(items, m->sms);
  }
  return ANVIL_OK;
}

extern "C" int anvil_model_arena(anvil_model *m, uint64_t *arena_ptr, uint64_t *const_ptr) {
  if (!m) return fail(ANVIL_E_BAD_ARG, "model is NULL");
  if (arena_ptr) *arena_ptr = reinterpret_cast<uint64_t>(m->arena);
  if (const_ptr) *const_ptr = reinterpret_cast<uint64_t>(m->consts);
  return ANVIL_OK;
}

// ------------------------------------------------------------------------------------- standalone GEMM

// One GEMM + requant on caller-owned device operands (the body of both standalone entry points): launched on
// m->stream with m->flags as its status words, which are cleared before the launch and read back after it, so a
// device-side failure (an overflow in checked mode, a device wait that gave up in either mode) is reported by
// this call whatever the flags. The call synchronises the stream.
static int standalone_gemm(anvil_model *m, const int8_t *A, const int8_t *BT, int8_t *out, int64_t M, int64_t N,
                           int64_t K, int32_t mult, int32_t shift, uint32_t flags) {
  Launch L;
  memset(&L.op, 0, sizeof L.op);
  L.op.kind = ANVIL_OP_GEMM;
  L.op.flags = flags & (ANVIL_F_CHECKED | ANVIL_F_SIMT);
  L.op.out_bytes = 1;
  L.op.op_index = 0;                               // status words record op index + 1: this call is op 0
  L.op.dims[0] = 1; L.op.dims[1] = M; L.op.dims[2] = N; L.op.dims[3] = K;
  L.op.strides[3] = N;
  L.op.mult = mult;
  L.op.shift = shift;
  for (int s = 0; s < 8; ++s) L.op.off[s] = ANVIL_LOC_NONE;
  // caller-owned device pointers: no region resolution
  GemmParams &p = L.gp;
  memset(&p, 0, sizeof p);
  p.batch = 1; p.M = M; p.N = N; p.K = K;
  p.o_rstride = N;
  p.o_cstride = 1;
  p.A = A; p.BT = BT; p.out = out;
  p.mult = mult; p.shift = shift; p.out_bytes = 1;
  p.check = (flags & ANVIL_F_CHECKED) ? 1 : 0;
  p.flags = m->flags;
  p.op_index = 0;
  L.tc = !(flags & ANVIL_F_SIMT) && K % 16 == 0 && aligned16(A) && aligned16(BT) && M <= (1ll << 31) - 256 &&
         N <= (1ll << 31) - 256;
  int rc;
  if (L.tc && (rc = tc_tiles(m, L))) return rc;
  CK(cudaMemsetAsync(m->flags, 0, FLAG_WORDS * sizeof(uint32_t), m->stream));
  if ((rc = launch_op(m, L))) return rc;
  uint32_t h[FLAG_WORDS];
  CK(cudaMemcpyAsync(h, m->flags, sizeof h, cudaMemcpyDeviceToHost, m->stream));
  CK(cudaStreamSynchronize(m->stream));
  return check_flags(m, h);
}

extern "C" int anvil_gemm_requant(const int8_t *A, const int8_t *BT, int8_t *out, int64_t M, int64_t N, int64_t K,
                                  int32_t mult, int32_t shift, uint32_t flags, void *stream) {
  if (!A || !BT || !out || M < 1 || N < 1 || K < 1 || shift < 0 || shift > 31)
    return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_gemm_requant");
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev >= 64) return fail(ANVIL_E_BAD_ARG, "device %d out of range", dev);
  // one scratch model per device and host thread: its flag words (the only device memory this call uses besides
  // the caller's operands) are private to the thread, so calls from several threads do not share them
  static thread_local anvil_model *scratch[64] = {};
  if (!scratch[dev]) {
    int rc = anvil_model_create(dev, nullptr, 0, &scratch[dev]);
    if (rc) return rc;
  }
  anvil_model *m = scratch[dev];
  cudaStream_t saved = m->stream;
  m->stream = static_cast<cudaStream_t>(stream);
  int rc = standalone_gemm(m, A, BT, out, M, N, K, mult, shift, flags);
  m->stream = saved;
  return rc;
}

// ------------------------------------------------------------------- standalone GEMM without allocation
//
// For callers that must not allocate device memory (an embedding whose host owns every allocation, code running
// where cudaMalloc is unavailable or forbidden): the same GEMM + requant as anvil_gemm_requant, but the only device
// memory beyond the caller's A, BT and out is this file-scope array, which holds the kernel's status words
// (overflow / index / device-wait timeout). Every GPU that loads the library keeps one copy until the process
// exits. The host reaches the copy of the current device through cudaGetSymbolAddress, once per device.

#define ANVIL_NOALLOC_SCRATCH_WORDS 16            // 64 bytes; the GEMM needs FLAG_WORDS of them
static __device__ __align__(256) uint32_t g_noalloc_scratch[ANVIL_NOALLOC_SCRATCH_WORDS];

extern "C" int anvil_gemm_requant_noalloc(const int8_t *A, const int8_t *BT, int8_t *out, int64_t M, int64_t N,
                                          int64_t K, int32_t mult, int32_t shift, uint32_t flags, void *stream) {
  if (!A || !BT || !out || M < 1 || N < 1 || K < 1 || shift < 0 || shift > 31)
    return fail(ANVIL_E_BAD_ARG, "bad arguments to anvil_gemm_requant_noalloc");
  if (FLAG_WORDS > ANVIL_NOALLOC_SCRATCH_WORDS)
    return fail(ANVIL_E_BAD_ARG, "anvil_gemm_requant_noalloc needs %d scratch words, the static array holds %d",
                (int)FLAG_WORDS, ANVIL_NOALLOC_SCRATCH_WORDS);
  int dev = 0;
  CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(ANVIL_E_BAD_ARG, "device %d out of range", dev);
  // set-up, once per device, with that device current (std::call_once: concurrent first calls on one device wait
  // for a single set-up): the kernels' shared-memory opt-in and the SM count (device_info), then the array's
  // device address. None of it allocates.
  static std::once_flag once[64];
  static uint32_t *scratch_ptr[64] = {};
  static int setup_rc[64] = {};
  static std::string setup_err[64];
  std::call_once(once[dev], [&]() {
    cudaDeviceProp prop;
    int rc = ANVIL_OK;
    uint32_t *ptr = nullptr;
    cudaError_t e;
    if ((e = cudaGetDeviceProperties(&prop, dev)) != cudaSuccess)
      rc = fail(ANVIL_E_CUDA, "cudaGetDeviceProperties failed: %s", cudaGetErrorString(e));
    else if (prop.major != 10)
      rc = fail(ANVIL_E_UNSUPPORTED, "device %d is sm_%d%d; libanvil_cuda is built for sm_100a (B200)", dev,
                prop.major, prop.minor);
    else if (!(rc = kernel_attrs(dev)) &&
             (e = cudaGetSymbolAddress((void **)&ptr, g_noalloc_scratch)) != cudaSuccess)
      rc = fail(ANVIL_E_CUDA, "cudaGetSymbolAddress of the scratch array failed: %s", cudaGetErrorString(e));
    setup_rc[dev] = rc;
    if (rc) setup_err[dev] = g_err;
    else scratch_ptr[dev] = ptr;
  });
  if (setup_rc[dev]) {
    g_err = setup_err[dev];
    return setup_rc[dev];
  }
  DeviceInfo *di = nullptr;
  int rc = device_info(dev, &di);
  if (rc) return rc;
  anvil_model m;                                   // a host-side view only: no stream, arena or consts are created
  m.device = dev;
  m.sms = di->sms;
  m.stream = static_cast<cudaStream_t>(stream);
  m.flags = scratch_ptr[dev];                      // cleared by standalone_gemm before its kernel can raise any
  return standalone_gemm(&m, A, BT, out, M, N, K, mult, shift, flags);
}
