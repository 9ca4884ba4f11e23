/* libanvil_cuda.so: the C-ABI of Anvil's B200 (sm_100a) execution target.
 *
 * The reference runs a compiled graph through one backend call, anvil/runtime/api.py:127-141
 * (run(job, backend) -> RunResult, ValueError on an unknown backend, TimeoutError on a hung launch), reached from
 * CompiledModel.run (anvil/driver.py:305-322). The `cuda` target replaces the tiny-gpu Job/word-image pair with
 * this library: the host (Python, over ctypes) lowers the graph to a list of anvil_op records with byte offsets
 * into two device regions, and the library owns the device memory, launches the kernels on one stream per model
 * and copies inputs/outputs. No torch types cross this boundary: plain pointers, sizes and POD structs.
 *
 * Every call returns ANVIL_OK (0) or a negative ANVIL_E_* code; anvil_last_error() gives the message of the
 * last failure on the calling thread. A model handle is not re-entrant: one host thread at a time.
 */
#ifndef ANVIL_CUDA_H
#define ANVIL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define ANVIL_API __attribute__((visibility("default")))
#else
#define ANVIL_API
#endif

#define ANVIL_ABI_VERSION 2

/* status codes (mapped to the reference's exception types by anvil/runtime/cuda.py) */
#define ANVIL_OK 0
#define ANVIL_E_BAD_ARG -1        /* ValueError    (anvil/runtime/api.py:104-124 validation)          */
#define ANVIL_E_OOM -2            /* MemoryError   (anvil/memplan.py:27-28 MemoryPlanError analogue)  */
#define ANVIL_E_CUDA -3           /* RuntimeError  (a CUDA API call failed)                            */
#define ANVIL_E_TIMEOUT -4        /* TimeoutError  (a bounded device wait gave up, api.py:127-130)     */
#define ANVIL_E_OVERFLOW -5       /* OverflowError (a checked int32 intermediate left int32,
                                     anvil/semantics.py:47-49)                                        */
#define ANVIL_E_INDEX -6          /* IndexError    (a LUT / token index outside its table,
                                     anvil/semantics.py:76-84)                                        */
#define ANVIL_E_UNSUPPORTED -7    /* NotImplementedError (no sm_100 device, op kind unknown)          */

/* device buffer locations inside anvil_op.off[]: bit 63 set = the read-only const region, else the arena */
#define ANVIL_LOC_CONST (1ull << 63)
#define ANVIL_LOC_NONE (~0ull)

/* op kinds: one per device kernel family (the graph ops of anvil/ir/graph.py:1-25 after lowering) */
enum anvil_op_kind {
  ANVIL_OP_GEMM = 1,        /* qmatmul / qlinear: requant(A @ B + bias, M, s) [-> lut]          (a1, a2, a10) */
  ANVIL_OP_LUT = 2,         /* table[x + 128]                                                     (a3)      */
  ANVIL_OP_LUT_MUL = 3,     /* requant(table[x + 128] * y, M, s)                                  (a4)      */
  ANVIL_OP_ADD_REQUANT = 4, /* clamp((a*Ma + b*Mb + 2^(s-1)) >> s)                                (a7)      */
  ANVIL_OP_NORM = 5,        /* rmsnorm_int / layernorm_int over the last axis                     (a5, a5x) */
  ANVIL_OP_SOFTMAX = 6,     /* softmax_lut over the last axis                                     (a6)      */
  ANVIL_OP_TRANSPOSE = 7,   /* strided copy (materialises a transpose)                           (a8)      */
  ANVIL_OP_EMBED = 8,       /* add_requant(wte[ids], wpe[pos])                                    (a11)     */
  ANVIL_OP_ATTENTION = 9,   /* fused causal qk^T -> softmax_lut -> p@v, scores kept on chip      (a1, a6)  */
  ANVIL_OP_COPY = 10        /* contiguous byte copy (graph outputs that alias another buffer)              */
};

/* op flags */
#define ANVIL_F_CAUSAL 1u     /* softmax / attention: row i keeps j <= i                          */
#define ANVIL_F_CHECKED 2u    /* check every int32 intermediate on the device (sets the overflow flag) */
#define ANVIL_F_LUT 4u        /* gemm: fused lut[. + 128] epilogue                                 */
#define ANVIL_F_BIAS 8u       /* gemm: int32 bias per column; norm: int8 bias per channel          */
#define ANVIL_F_CENTER 16u    /* norm: layernorm (mean-centre the row first)                        */
#define ANVIL_F_SIMT 32u      /* gemm: force the CUDA-core kernel (shapes the TMA path cannot take) */
#define ANVIL_F_BIAS_RND 64u  /* gemm: the BIAS slot holds bias*M + 2^(s-1) per column (int32); only without
                                 ANVIL_F_CHECKED, where the int32 proof makes the 32-bit epilogue exact  */
#define ANVIL_F_RESIDUAL 128u /* gemm: fused add_requant with off[5] = RES ((M, N) row-major, in2_bytes):
                                 out = clamp((res*ma + y*mb + 2^(shift2-1)) >> shift2), y the requant result
                                 clamped to in_bytes' range; unchecked, unbatched, row-major output only     */
#define ANVIL_F_SPLIT 256u    /* gemm: several linears of one input as one GEMM (the q, k, v projections):
                                 dims[4] = C columns per chunk (a multiple of 256), chunk c requantised with
                                 aux[c] = (M_c << 8) | s_c; columns below dims[5] = R go row-major to OUT (row
                                 stride strides[3]), the rest head-major transposed (the ATTENTION VT layout,
                                 row group dims[6] = T) to off[6]; unchecked, unbatched, i8, no LUT / residual  */

/* One lowered kernel launch. Field meaning per kind (all sizes in elements, offsets in bytes):
 *   GEMM        dims  = {batch, M, N, K}; strides = {a_batch, bt_batch (0: shared weight), out_batch,
 *                       out_row, out_group_rows (0: M), out_group, out_col (0: 1)}: element (b, row, col) goes to
 *                       b*out_batch + (row / R)*out_group + (row % R)*out_row + col*out_col;
 *                       off = {A (batch, M, K) int8, BT (batch|1, N, K) int8, OUT, LUT (256 i8), BIAS (N i32)};
 *                       mult = M, shift = s; out_bytes = 1 (i8) or 2 (i16); ANVIL_F_RESIDUAL adds off[5]
 *   LUT         dims  = {n}; off = {X, TABLE, OUT}
 *   LUT_MUL     dims  = {n}; off = {X, Y, TABLE, OUT}; mult, shift
 *   ADD_REQUANT dims  = {n}; off = {A, B, OUT}; in_bytes = a bytes, in2_bytes = b bytes, out_bytes;
 *               ma, mb, shift
 *   NORM        dims  = {rows, d, lut_len}; off = {X, W, LUT, OUT, BIAS}; in_bytes; mult, shift,
 *               ss_shift, ss_init; flags CENTER / BIAS
 *   SOFTMAX     dims  = {batch, T1, T2}; off = {X, LUT (256 i32), OUT}; one; out_bytes 1 or 4; flags CAUSAL
 *   TRANSPOSE   dims  = {rank, n0, n1, n2, n3, n4, n5} (output dims); strides = input element strides per
 *               output dim; off = {X, OUT}; in_bytes = element bytes
 *   EMBED       dims  = {batch, T, d, vocab}; off = {IDS (i32), WTE, WPE, OUT}; ma, mb, shift
 *   ATTENTION   dims  = {B, H, T1, T2, hd (64 | 128)}; strides = {q_b, q_h, q_t, k_b, k_h, k_t, o_b, o_t}
 *               (bytes; q element (b, h, t, d) at b*q_b + h*q_h + t*q_t + d, likewise k; the output element
 *               (b, h, t, d) goes to b*o_b + t*o_t + h*hd + d, i.e. heads merged); off = {Q, K, VT, OUT, EXP_LUT}
 *               with VT dense (B, H, hd, T2) (V transposed per head); mult/shift = scores (M, s),
 *               mult2/shift2 = p@v (M, s); one (<= 127, i8 p); flags CAUSAL. T2 <= 1024, T2 % 16 == 0.
 *   COPY        dims  = {bytes}; off = {X, OUT}
 */
typedef struct anvil_op {
  int32_t kind;
  uint32_t flags;
  int32_t in_bytes;
  int32_t in2_bytes;
  int32_t out_bytes;
  int32_t op_index;        /* graph op index, for error messages */
  int64_t dims[8];
  int64_t strides[8];
  uint64_t off[8];
  int64_t mult, shift, ma, mb, one, ss_shift, ss_init, mult2, shift2;
  int64_t aux[8];          /* GEMM with ANVIL_F_SPLIT: (M_c << 8) | s_c of output chunk c */
} anvil_op;

/* A host buffer bound to an arena range for one run (graph inputs and outputs). */
typedef struct anvil_io {
  uint64_t offset;         /* arena byte offset */
  void *host;              /* host pointer (pinned or pageable) */
  uint64_t bytes;
} anvil_io;

typedef struct anvil_model anvil_model;

/* Library version and the message of the last failure on this thread (never NULL). */
ANVIL_API int anvil_abi_version(void);
ANVIL_API const char *anvil_last_error(void);

/* Number of visible CUDA devices (0 without a driver); ANVIL_E_UNSUPPORTED if `device` is not sm_100. */
ANVIL_API int anvil_device_count(int *count);
ANVIL_API int anvil_cuda_init(int device);

/* Create a model on `device`: uploads `const_bytes` of constants (weights, LUTs, biases, in device layout).
 * Replaces the tiny-gpu image build of anvil/codegen/__init__.py:214 (program_job) for the cuda target. */
ANVIL_API int anvil_model_create(int device, const void *consts, uint64_t const_bytes, anvil_model **out);

/* Install the launch list for one batch size: validates every op against the region sizes, grows the device
 * arena to `arena_bytes` (the liveness plan of anvil/memplan.py:190-198, in bytes) and builds the tensor maps. */
ANVIL_API int anvil_model_prepare(anvil_model *m, const anvil_op *ops, int n_ops, uint64_t arena_bytes);

/* One run: H2D copies of `inputs`, every op in order on the model's stream, D2H copies of `outputs`, then a
 * stream synchronise. kernel_us (optional, n_ops floats) receives per-op device microseconds measured with CUDA
 * events (adds one event pair per op). Overflow/index flags raised by checked kernels map to
 * ANVIL_E_OVERFLOW / ANVIL_E_INDEX with the op index in the message. */
ANVIL_API int anvil_model_run(anvil_model *m, const anvil_io *inputs, int n_inputs, const anvil_io *outputs, int n_outputs,
                    float *kernel_us);

/* The same launch chain on device-resident data (no host copies): `iters` back-to-back runs of every op,
 * optionally captured once in a CUDA graph and replayed. Returns the device milliseconds of the whole loop
 * (CUDA events on the model's stream) in *ms. Used by benchmarks to time kernels with inputs already in HBM. */
ANVIL_API int anvil_model_run_device(anvil_model *m, int iters, int use_graph, float *ms);

/* Benchmark-only: each launch's device time inside a CUDA-graph replay of the prepared chain on the arena as it is
 * (a timing graph with an event recorded before the first launch and after each one, replayed `iters` times,
 * synchronised after each replay); op_us[i] = the shortest time of launch i over the replays, in microseconds
 * (n_ops floats, as prepared).
 * Device checks are reported as by anvil_model_run. The per-launch timing of the reference's RunOutput.cycles
 * (anvil/driver.py:56-76) at graph-replay launch cost; no separate reference entry point. */
ANVIL_API int anvil_model_time_launches(anvil_model *m, int iters, float *op_us);

/* The run of anvil_model_run split for pipelines over several models (each its own arena and stream): the H2D
 * copies of `inputs`, the launch chain (one CUDA graph launch, captured on first use) and the D2H copies of
 * `outputs`, returning without waiting. The copies go to the device's two shared copy streams (one per direction,
 * created on first use and kept until exit), in enqueue order, so the copies of consecutive enqueues, from
 * whichever models, follow each other on the bus with no wait in between; a model's copies in start once its
 * previous enqueue's copies out are done, its launch chain (on the model's stream) once its copies in are done,
 * and with `after` (another model on the same device, or NULL) once `after`'s latest launch chain is done too. A
 * batch enqueued chunk by chunk round-robin over two or more models, each chunk after the previous one's model,
 * runs as a copy-in / compute / copy-out pipeline: one chunk's kernels at a time, with the next chunk's input and
 * the previous chunk's output crossing the bus meanwhile (the host buffers should be pinned, and must stay valid
 * until anvil_model_wait returns). Every other call that touches the arena first waits for the model's pending
 * copies out. Device flags persist across enqueues: anvil_model_clear_flags resets them (stream-ordered) and
 * anvil_model_wait synchronises the model (its stream and its copies out) and maps any raised flag to its status,
 * as anvil_model_run does. The pipelined form of the reference's CompiledModel.run (anvil/driver.py:305-322); no
 * separate reference entry point. */
ANVIL_API int anvil_model_enqueue(anvil_model *m, const anvil_io *inputs, int n_inputs, const anvil_io *outputs,
                                  int n_outputs, anvil_model *after);
ANVIL_API int anvil_model_clear_flags(anvil_model *m);
ANVIL_API int anvil_model_wait(anvil_model *m);

/* Completion tickets, the asynchronous form of anvil_model_wait: anvil_model_record marks everything enqueued on
 * the model's stream so far (it snapshots the device check words on the device and clears them, both in stream
 * order, then records an event) and returns a ticket; anvil_model_wait_ticket blocks until that work is done and
 * maps the checks it raised to a status as anvil_model_wait does, unaffected by work enqueued after the ticket, so a
 * caller can keep the next calls' copies and kernels queued while it waits on an earlier one. At most 64 tickets
 * per model are outstanding (a 65th record fails with ANVIL_E_BAD_ARG); each is waited on once. Backs
 * CompiledModel.submit / PendingRun.wait (asynchronous runs of the reference's CompiledModel.run,
 * anvil/driver.py:305-322); the reference has no asynchronous entry point of its own. */
ANVIL_API int anvil_model_record(anvil_model *m, uint64_t *ticket);
ANVIL_API int anvil_model_wait_ticket(anvil_model *m, uint64_t ticket);

/* Self-test of the device-side wait bound every kernel relies on: launches one block whose warps wait, through
 * the same bounded mbarrier wait, on a barrier nothing arrives on, with a limit of `wait_ns` (at most the kernels'
 * own 2 s). The wait gives up and raises the timeout flag, so the call returns ANVIL_E_TIMEOUT after about wait_ns,
 * and the model (its stream and context) stays usable. No reference counterpart: the reference's analogue is the
 * simulators' timeout_cycles (anvil/runtime/api.py:104-124). */
ANVIL_API int anvil_model_selftest_timeout(anvil_model *m, uint64_t wait_ns);

/* Read/write raw arena bytes (tests and keep="all" readback). */
ANVIL_API int anvil_model_read(anvil_model *m, uint64_t offset, void *host, uint64_t bytes);
ANVIL_API int anvil_model_write(anvil_model *m, uint64_t offset, const void *host, uint64_t bytes);

/* Read raw bytes of the const region, for the stray-write check of a guarded run: a run must leave every const
 * byte as uploaded (the reference's RunOutput.stray_writes, anvil/driver.py:66-71, and JobPlan.stray_writes,
 * anvil/codegen/__init__.py:150-168, check consts and every word outside the plan's buffers). */
ANVIL_API int anvil_model_read_const(anvil_model *m, uint64_t offset, void *host, uint64_t bytes);

/* The launch shape the library chose for prepared op `op` (for summaries and tests): info[0..3] =
 * GEMM: {BN (64 | 128 | 256; 0 for the CUDA-core kernel), CTAs per tile (1, or 2 for CTA-pair 256-row tiles), tiles,
 * CTAs launched}; ATTENTION: {hd, 0, (batch, head, 128-query) work items, CTAs launched}; other kinds: zeros.
 * The reference's counterpart is the per-kernel schedule its summary prints (anvil/driver.py:324-327). */
ANVIL_API int anvil_model_describe(anvil_model *m, int op, int64_t *info);

/* Device pointer of the arena and of the const region (for callers that bring their own device buffers). */
ANVIL_API int anvil_model_arena(anvil_model *m, uint64_t *arena_ptr, uint64_t *const_ptr);

ANVIL_API void anvil_model_free(anvil_model *m);

/* Standalone GEMM + requantize on caller-owned device memory (config 4 sweep; a1/a2 without a graph):
 * out[M, N] = clamp((A[M, K] @ B[K, N] * mult + 2^(shift-1)) >> shift) as int8, with BT = B transposed
 * ([N, K] row-major, K contiguous). Runs on `stream` (cudaStream_t, NULL = legacy default). `flags` takes
 * ANVIL_F_CHECKED / ANVIL_F_SIMT. Bit-exact to requant(matmul_i8(A, B), mult, shift) (anvil/semantics.py:95-103)
 * whenever that raises nothing. The tile shape (64, 128 or 256 columns, single-CTA or CTA-pair 256-row tiles) is
 * chosen by how evenly the tiles fill the SMs. The call synchronises `stream` and reports the kernel's device
 * status in every mode: ANVIL_E_OVERFLOW (checked mode) or ANVIL_E_TIMEOUT (a bounded device wait gave up). Each
 * host thread has its own status words, so calls from several threads do not share them. */
ANVIL_API int anvil_gemm_requant(const int8_t *A, const int8_t *BT, int8_t *out, int64_t M, int64_t N, int64_t K,
                       int32_t mult, int32_t shift, uint32_t flags, void *stream);

/* anvil_gemm_requant without any device allocation. No counterpart in the reference: it exists for callers of
 * this library that cannot allocate device memory themselves or let a library do it (a host framework that owns
 * every device allocation, a process where cudaMalloc is not permitted). Same arguments, result and error codes as
 * anvil_gemm_requant; the caller passes A, BT and out. The kernel's only other device memory is a file-scope
 * static array of 16 32-bit words (64 bytes) that every GPU loading the library holds until the process exits; the
 * GEMM uses 4 of them as its overflow / index / timeout status words and the call fails with ANVIL_E_BAD_ARG if it
 * ever needed more than the array holds. The first call on a device does a one-time set-up there (it looks up the
 * array's device address and the kernels' shared-memory limits), so make that first call before any stream capture;
 * first calls from several host threads on one device are safe (one set-up runs, the others wait for it).
 * All calls share the array: it is cleared at the start of each call, and calls that overlap on the GPU (other
 * streams, other host threads) race on it. The call synchronises `stream` before it returns. */
ANVIL_API int anvil_gemm_requant_noalloc(const int8_t *A, const int8_t *BT, int8_t *out, int64_t M, int64_t N,
                                         int64_t K, int32_t mult, int32_t shift, uint32_t flags, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* ANVIL_CUDA_H */
