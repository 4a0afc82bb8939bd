/*
 * mcke_sm100.h -- C-ABI of libmcke_sm100a.so, the B200 (sm_100a) kernel library
 * that replaces mini-cuda-kernel-engine's kernel layer (the .cu files of its kernels/ directory).
 *
 * Every entry point is a plain C function over caller-owned device pointers,
 * int64 extents and enum ints, enqueued on an explicit CUDA stream.  None
 * synchronises, none allocates device memory (scratch is caller-provided and
 * sized by a *_workspace_bytes query), and each returns an mcke_status code:
 * the numbering is the reference's StatusCode (include/mcke/core/status.hpp:42).
 * The message of the last failing call on the calling thread is available from
 * mcke_sm100_last_error_string().
 *
 * Error behaviour follows the reference launchers: empty extents return OK
 * without a launch; negative extents, null pointers, an output aliasing an
 * input, an illegal vector width, misalignment and extents beyond launch limits
 * return MCKE_INVALID_ARGUMENT; an unsupported variant is rejected, never
 * silently downgraded.  A failed CUDA launch returns MCKE_CUDA_ERROR.
 *
 * Each declaration names the reference interface it replaces (path:line within
 * mini-cuda-kernel-engine).  The C++ launchers of include/mcke/kernels/kernels.hpp
 * become thin wrappers over these (mini-cuda-kernel-engine_b200/integration/kernels_sm100.cpp).
 */
#ifndef MCKE_SM100_H_
#define MCKE_SM100_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same type as cudaStream_t (struct CUstream_st*), declared without CUDA headers. */
typedef struct CUstream_st* mcke_stream_t;

/* include/mcke/core/status.hpp:42 StatusCode, same values. */
typedef enum {
  MCKE_OK = 0,
  MCKE_OUT_OF_MEMORY = 1,
  MCKE_INVALID_ARGUMENT = 2,
  MCKE_FAILED_PRECONDITION = 3,
  MCKE_UNIMPLEMENTED = 4,
  MCKE_INTERNAL = 5,
  MCKE_CUDA_ERROR = 6
} mcke_status;

/* include/mcke/kernels/kernels.hpp:65 Activation, same values. */
typedef enum { MCKE_ACT_NONE = 0, MCKE_ACT_RELU = 1, MCKE_ACT_GELU_ERF = 2, MCKE_ACT_GELU_TANH = 3 } mcke_activation;
/* include/mcke/kernels/kernels.hpp:153 ReduceKind, same values. */
typedef enum { MCKE_REDUCE_SUM = 0, MCKE_REDUCE_MAX = 1, MCKE_REDUCE_MEAN = 2 } mcke_reduce_kind;
/* include/mcke/kernels/kernels.hpp:180 ReduceVariant, same values. */
typedef enum { MCKE_REDUCE_SMEM_TREE = 0, MCKE_REDUCE_WARP_SHUFFLE = 1, MCKE_REDUCE_TWO_PASS = 2 } mcke_reduce_variant;
/* Flags of the full-vector reduce's _ex entry points (new).
 * MCKE_REDUCE_EARLY_READ: the caller guarantees that x is not written by the
 * kernel enqueued immediately before the call on the same stream.  The kernel
 * then reads x before waiting for that kernel and waits only before its first
 * write, so back-to-back reduces overlap (one call's fold and exchange with the
 * next call's read of x).  Every earlier writer of x has completed by then:
 * each kernel of this library lets its successor start only after its own
 * wait, and kernels launched without programmatic serialization (torch,
 * cuBLAS, memcpy) complete before their successor starts.  Same result, same
 * bits as without the flag. */
#define MCKE_REDUCE_EARLY_READ 1u
/* include/mcke/kernels/kernels.hpp:218 SoftmaxVariant, same values.  ONLINE
 * selects the single-read register-resident kernel whenever a row fits
 * (cols % 4 == 0, 16-byte aligned rows, cols <= 16384), else the two-read
 * online kernel. */
typedef enum { MCKE_SOFTMAX_THREE_PASS = 0, MCKE_SOFTMAX_ONLINE = 1 } mcke_softmax_variant;
/* GEMM kernels of this library (the reference's ladder is
 * include/mcke/kernels/gemm_tile.hpp:209 GemmVariant; its kernels are replaced,
 * so its values are not reused).  AUTO picks TCGEN05 for bf16 when the shape
 * meets the TMA rules (K % 8 == 0, N % 8 == 0, 16-byte aligned A and B),
 * else SIMT.  For f32 operands and an f32 output AUTO picks the tensor cores
 * in the 3xTF32 form with the hi/lo split inside the GEMM kernel (no
 * workspace; fp32-level accuracy, not bit-identical to an FFMA loop) when
 * K % 4 == 0, N % 4 == 0 and A and B are 16-byte aligned, else SIMT; SIMT
 * always takes the FFMA kernel. */
/* TCGEN05_WIDE / TCGEN05_NARROW: the tcgen05 kernel with its pair tile forced
 * to 256 x 512 / 256 x 256, one tile per CTA pair at a time (AUTO and TCGEN05
 * choose; shapes that cannot use the pair tile ignore the choice).  The two
 * give bit-identical results.  TCGEN05_SPLIT: the 256 x 512 tile with the
 * split-k schedule wherever it applies (fp32 output, beta == 0, M % 256 == 0,
 * N % 512 == 0): the k-blocks of the tiles past the last whole wave are divided
 * evenly over all CTA pairs and cut tiles are summed in C in k order
 * (deterministic; within the bf16 tolerance of the unsplit result).  AUTO and
 * TCGEN05 use it when at least two whole waves exist and whole waves would
 * leave more than 5% of the pairs idle.  Split launches that run at the same
 * time on one device must be fewer than 128 split launches apart (a captured
 * CUDA graph keeps its launch's flag slot); otherwise one may give up after
 * 2 s and report MCKE_INTERNAL from mcke_sm100_check_device_errors(). */
typedef enum {
  MCKE_GEMM_AUTO = 0,
  MCKE_GEMM_SIMT = 1,
  MCKE_GEMM_TCGEN05 = 2,
  MCKE_GEMM_TCGEN05_WIDE = 3,
  MCKE_GEMM_TCGEN05_NARROW = 4,
  MCKE_GEMM_TCGEN05_SPLIT = 5
} mcke_gemm_variant;
/* Element type of a GEMM output. */
typedef enum { MCKE_DTYPE_F32 = 0, MCKE_DTYPE_BF16 = 2 } mcke_dtype;

/* Result of a full-vector reduce: 16 bytes, device memory. */
typedef struct {
  float sum;      /* sum of all elements, accumulated in double, rounded once */
  float max;      /* largest non-NaN element (-inf if none), bit pattern of x[argmax] */
  int64_t argmax; /* lowest index holding max; -1 when n == 0 or every element is NaN */
} mcke_reduce_result;

/* One shard's partial of a full-vector reduce: 24 bytes, device memory.
 * Partials from several shards are combined, in shard order, by
 * mcke_sm100_reduce_combine. */
typedef struct {
  double sum;
  float max;
  int32_t reserved;
  int64_t argmax; /* global index (index_base already added), -1 if none */
} mcke_reduce_partial;

/* What ptxas produced for one GEMM kernel (include/mcke/kernels/kernels.hpp:293). */
typedef struct {
  int regs_per_thread;
  size_t static_smem_bytes;
  size_t dynamic_smem_bytes;
  size_t local_bytes; /* > 0 means spilling */
  int threads_per_block;
  int max_blocks_per_sm_api;
} mcke_gemm_attrs;

/* ---- library ------------------------------------------------------------ */

/* Version of this ABI (major * 10000 + minor * 100 + patch). */
int mcke_sm100_version(void);
/* Message of the last failing call on this thread ("" if none). */
const char* mcke_sm100_last_error_string(void);
/* Synchronises `stream`, then reads and clears the device-side watchdog word of
 * the current device: 0 if no kernel of this library gave up on a bounded wait
 * since the last call, else MCKE_INTERNAL with the site in the message. */
int mcke_sm100_check_device_errors(mcke_stream_t stream);
/* Diagnostic with no counterpart in the reference: enqueues a one-thread kernel
 * that waits on a barrier nothing arrives on, so its bounded wait (2 s) expires
 * and records itself; the next mcke_sm100_check_device_errors() then returns
 * MCKE_INTERNAL naming site 9 (a site no other wait uses), and the context stays usable.  For testing the
 * failure path of the library's bounded waits without faulting a GPU. */
int mcke_sm100_watchdog_selftest(mcke_stream_t stream);

/* No counterpart in the reference.  Every kernel of this library starts by
 * waiting for the grid launched before it on its stream to complete
 * (griddepcontrol.wait) before it touches global memory, so it may be launched
 * with programmatic dependent launch: its launch and CTA start-up then overlap
 * the tail of the kernel before it (about 2 us per launch back to back on B200).
 * On by default, or off when the environment sets MCKE_PDL=0 at the first launch;
 * this call sets it for the whole process (0 = plain launches) and returns the
 * previous setting.  Results are the same either way. */
int mcke_sm100_set_programmatic_launch(int enable);

/* ---- vector add (toolchain smoke test) ------------------------------------ */

/* Replaces kernels.hpp:59 launch_vector_add_f32 (kernels/elementwise.cu:65):
 * out[i] = a[i] + b[i], one IEEE add per element. */
int mcke_sm100_vector_add_f32(const float* a, const float* b, float* out, size_t n,
                              mcke_stream_t stream);

/* ---- bias + activation: y[r][c] = act(x[r][c] + bias[c]) ---------------- */

/* Replaces kernels.hpp:102 launch_bias_act_f32 (kernels/bias_act.cu:269).
 * vector_width in {1,2,4}; cols % vector_width == 0; x, y, bias aligned to
 * 4*vector_width bytes; x != y.  max_row_blocks > 0 caps the row-direction
 * grid (the reference's starvation knob); 0 = automatic. */
int mcke_sm100_bias_act_f32(const float* x, const float* bias, float* y, int64_t rows,
                            int64_t cols, int act, int vector_width, int max_row_blocks,
                            mcke_stream_t stream);
/* New (no counterpart in the reference): `count` independent fp32 bias +
 * activation jobs in one launch, as the executor's grouped level schedule
 * issues them.  Each job is mcke_sm100_bias_act_f32(x, bias, y, rows, cols,
 * act, vector_width 4, max_row_blocks 0) with cols % 512 == 0 and x, bias, y
 * 16-byte aligned; same bits as one such call per job.  The jobs run at the
 * same time, so no job's y may overlap any job's x, bias or y (its own x
 * included).  `jobs` is a host array; count 1 .. MCKE_BIAS_ACT_GROUP_MAX;
 * empty jobs (rows or cols 0) are skipped.  Anything else is
 * MCKE_INVALID_ARGUMENT, checked before any launch. */
#define MCKE_BIAS_ACT_GROUP_MAX 16
typedef struct {
  const float* x;
  const float* bias;
  float* y;
  int64_t rows;
  int64_t cols;
} mcke_bias_act_job;
int mcke_sm100_bias_act_f32_group(const mcke_bias_act_job* jobs, int count, int act, mcke_stream_t stream);
/* Replaces kernels.hpp:129 launch_bias_add_f32 (bias_act with MCKE_ACT_NONE). */
int mcke_sm100_bias_add_f32(const float* x, const float* bias, float* y, int64_t rows,
                            int64_t cols, int vector_width, mcke_stream_t stream);
/* Replaces kernels.hpp:133 launch_activation_f32 (n % vector_width == 0). */
int mcke_sm100_activation_f32(const float* x, float* y, int64_t n, int act, int vector_width,
                              mcke_stream_t stream);
/* New (bf16 path of the same op): x, y bfloat16 [rows, cols] (raw 16-bit
 * patterns), bias float32 [cols]; math in float, one round-to-nearest-even on
 * store.  cols % 8 == 0 and 16-byte aligned x, y take the 8-wide path; any
 * other shape takes a scalar path. */
int mcke_sm100_bias_act_bf16(const uint16_t* x, const float* bias, uint16_t* y, int64_t rows,
                             int64_t cols, int act, mcke_stream_t stream);

/* ---- row softmax over the last dim -------------------------------------- */

/* Replaces kernels.hpp:220 launch_row_softmax_f32 (kernels/softmax.cu:177). */
int mcke_sm100_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols, int variant,
                           mcke_stream_t stream);

/* ---- reductions ---------------------------------------------------------- */

/* Replaces kernels.hpp:198 row_reduce_workspace_bytes. */
size_t mcke_sm100_reduce_row_workspace_bytes(int64_t rows, int64_t cols, int variant);
/* Replaces kernels.hpp:204/209 launch_row_reduce_f32 (both overloads; pass
 * workspace = NULL, workspace_bytes = 0 for the 7-argument form, which makes
 * MCKE_REDUCE_TWO_PASS return MCKE_UNIMPLEMENTED as the reference does). */
int mcke_sm100_reduce_row_f32(const float* x, float* out, int64_t rows, int64_t cols, int kind,
                              int variant, void* workspace, size_t workspace_bytes,
                              mcke_stream_t stream);

/* Full-vector reduce (new; the reference's nearest interface is the rows = 1
 * case of kernels.hpp:209).  Workspace size for n elements. */
size_t mcke_sm100_reduce_full_workspace_bytes(int64_t n);
/* sum, max and argmax of x[0..n) in one read of x.  Deterministic: the combine
 * order depends on n only. */
int mcke_sm100_reduce_full_f32(const float* x, int64_t n, mcke_reduce_result* out,
                               void* workspace, size_t workspace_bytes, mcke_stream_t stream);
/* mcke_sm100_reduce_full_f32 with flags (0 or MCKE_REDUCE_EARLY_READ; other
 * bits are rejected with MCKE_INVALID_ARGUMENT). */
int mcke_sm100_reduce_full_f32_ex(const float* x, int64_t n, mcke_reduce_result* out,
                                  void* workspace, size_t workspace_bytes, unsigned flags,
                                  mcke_stream_t stream);
/* The same over one shard x[0..n) whose first element has global index
 * index_base; writes one mcke_reduce_partial. */
int mcke_sm100_reduce_full_partial_f32(const float* x, int64_t n, int64_t index_base,
                                       mcke_reduce_partial* out, void* workspace,
                                       size_t workspace_bytes, mcke_stream_t stream);
/* Combines `count` partials (device memory, shard order) into one result. */
int mcke_sm100_reduce_combine(const mcke_reduce_partial* partials, int64_t count,
                              mcke_reduce_result* out, mcke_stream_t stream);
/* New (sharded full reduce, one process per GPU): this rank reduces its shard
 * x[0..n) (global index of x[0] = index_base), stores its 24-byte partial into
 * slot `rank` of every rank's exchange buffer over peer memory, waits (bounded,
 * 1 s) for all ranks' slots in its own buffer and writes the combined result,
 * folded in rank order.  One kernel per call and no workspace: the pass-1
 * partials go to this rank's own buffer, and the CTA that finishes last folds them.
 * peer_buffers: DEVICE array of `world` pointers to the ranks' exchange
 * buffers as mapped in this process (this rank's own at index `rank`), each
 * mcke_sm100_reduce_p2p_buffer_bytes(world) bytes (2 * world 64-byte exchange
 * slots, then 444 slots for this rank's pass-1 partials, then an epoch
 * counter and the CTAs' arrival count; every 8-byte word of a slot carries 4 data bytes and the epoch, so
 * no fence orders data and flag), zeroed before first use.  epoch: 1, 2, 3,
 * ... < 2^32, one per call, the same on every rank; or 0 on every call: the
 * kernel then takes the next value of the counter in this rank's buffer and
 * advances it (what a captured CUDA graph needs, since it replays its launch
 * arguments).  Calls of one rank are ordered on one stream.  Every rank must
 * make the call for each epoch; a rank that does not arrive makes the others
 * give up after 1 s with argmax -1 and MCKE_INTERNAL from
 * mcke_sm100_check_device_errors(). */
size_t mcke_sm100_reduce_p2p_buffer_bytes(int world);
int mcke_sm100_reduce_full_p2p_f32(const float* x, int64_t n, int64_t index_base,
                                   void* const* peer_buffers, int world, int rank, uint64_t epoch,
                                   mcke_reduce_result* out, mcke_stream_t stream);
/* mcke_sm100_reduce_full_p2p_f32 with flags (0 or MCKE_REDUCE_EARLY_READ;
 * other bits are rejected with MCKE_INVALID_ARGUMENT). */
int mcke_sm100_reduce_full_p2p_f32_ex(const float* x, int64_t n, int64_t index_base,
                                      void* const* peer_buffers, int world, int rank, uint64_t epoch,
                                      mcke_reduce_result* out, unsigned flags, mcke_stream_t stream);
/* New, a measuring aid (no counterpart in the reference): the same call, which
 * also records when its phases happened, as %globaltimer nanoseconds, into
 * `stamps` (8 words of device memory, 8-byte aligned; n > 0).  The caller sets
 * words 0, 1, 3 to UINT64_MAX and 2, 4 to 0 before the call:
 *   [0] min over CTAs: entry (before waiting for the previous grid's memory)
 *   [1] min over CTAs: streaming starts      [2] max: the last CTA starts
 *   [3] min over CTAs: a block partial is done [4] max: the last one is done
 *   [5] the last CTA has folded the block partials (the shard partial)
 *   [6] the ranks' partials are combined and the result is stored
 *   [7] the last CTA's arrival on the counter has returned (it knows it is last).
 * Same result and the same bits as mcke_sm100_reduce_full_p2p_f32. */
int mcke_sm100_reduce_full_p2p_f32_timeline(const float* x, int64_t n, int64_t index_base,
                                            void* const* peer_buffers, int world, int rank, uint64_t epoch,
                                            mcke_reduce_result* out, uint64_t* stamps, mcke_stream_t stream);
/* Set-up helpers for exchange buffers shared between processes (CUDA IPC).
 * create: cudaMalloc + zero + IPC handle (64 bytes written to handle_out);
 * open: map a peer's handle in this process; close: unmap (opened = 1) or free. */
int mcke_sm100_ipc_buffer_create(size_t bytes, void** dev_ptr, void* handle_out);
int mcke_sm100_ipc_buffer_open(const void* handle, void** dev_ptr);
int mcke_sm100_ipc_buffer_close(void* dev_ptr, int opened);
/* No counterpart in the reference.  mcke_sm100_reduce_full_f32 for callers that
 * cannot allocate device memory -- for example a host runtime whose memory
 * manager owns every device allocation, or a foreign-language binding that
 * holds only its own input and output buffers -- and so cannot pass a
 * workspace.  Same result as mcke_sm100_reduce_full_f32; allocates nothing.
 * Its scratch is a fixed 10,656-byte array (444 partials of 24 bytes, one per
 * block of the kernel's largest grid) inside the library, which every GPU that
 * loads the library keeps until the process exits; a request needing more
 * partials than that is rejected with MCKE_INVALID_ARGUMENT (the grid never
 * needs more, so every n fits).  The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress) with that device current and
 * keeps it for the life of the process; make that first call before any stream
 * capture, and do not call this entry point on a device after resetting it
 * (cudaDeviceReset), which leaves the kept address stale.  All calls share the one array: calls that overlap on the
 * GPU (other streams, other host threads) race and must be serialised by the
 * caller.  Nothing in the array needs to start at zero. */
int mcke_sm100_reduce_full_f32_noalloc(const float* x, int64_t n, mcke_reduce_result* out,
                                       mcke_stream_t stream);

/* ---- GEMM: C[M,N] = alpha * A[M,K] @ B[K,N] + beta * C, row-major -------- */

/* Replaces kernels.hpp:265 launch_gemm_f32 (kernels/gemm.cu:829).  beta == 0
 * never reads C; k == 0 writes beta * C.  variant: AUTO (tensor cores where
 * the shape allows, see above) or SIMT. */
int mcke_sm100_gemm_f32(const float* a, const float* b, float* c, int64_t m, int64_t n,
                        int64_t k, float alpha, float beta, int variant, mcke_stream_t stream);
/* New: float32 GEMM on the tensor cores (3xTF32): A and B are each split into
 * hi (low 13 mantissa bits cleared) and lo = x - hi parts, and the tcgen05
 * kernel accumulates A_hi*B_lo + A_lo*B_hi + A_hi*B_hi in fp32 -- fp32-level
 * accuracy (relative error ~1e-6, not bit-identical to an FFMA loop) at
 * tensor-core speed.  c = act(alpha * A@B + beta * C + bias[col]), float32;
 * bias may be NULL.  Needs K % 4 == 0, N % 4 == 0 and 16-byte aligned A and B;
 * other shapes are rejected (use mcke_sm100_gemm_f32).  With a workspace of
 * mcke_sm100_gemm_f32_tc_workspace_bytes(m, n, k) bytes (256-byte aligned;
 * 8 * (M*K + K*N), rounded) two split passes write the parts there first; with
 * workspace = NULL and workspace_bytes = 0 the GEMM kernel splits its tiles in
 * shared memory itself (the same bits, no workspace, ~5% slower at 8192^3).
 * Same contract as launch_gemm_f32 (kernels.hpp:265) otherwise: beta == 0
 * never reads C, k == 0 writes act(beta * C + bias). */
size_t mcke_sm100_gemm_f32_tc_workspace_bytes(int64_t m, int64_t n, int64_t k);
int mcke_sm100_gemm_f32_tc(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                           float alpha, float beta, const float* bias, int act, void* workspace,
                           size_t workspace_bytes, mcke_stream_t stream);
/* New: bf16 inputs (raw 16-bit patterns), float32 accumulation and output. */
int mcke_sm100_gemm_bf16(const uint16_t* a, const uint16_t* b, float* c, int64_t m, int64_t n,
                         int64_t k, float alpha, float beta, int variant, mcke_stream_t stream);
/* New: bf16 GEMM with a fused epilogue, c = act(alpha * A@B + beta * C + bias[col]),
 * c of type c_dtype (float32, or bfloat16 rounded once).  bias may be NULL;
 * beta must be 0 for a bf16 output. */
int mcke_sm100_gemm_bf16_ex(const uint16_t* a, const uint16_t* b, void* c, int c_dtype,
                            int64_t m, int64_t n, int64_t k, float alpha, float beta,
                            const float* bias, int act, int variant, mcke_stream_t stream);
/* Replaces kernels.hpp:301 gemm_kernel_attrs: attributes of the kernel that
 * (variant, dtype) selects for a large aligned shape. */
int mcke_sm100_gemm_kernel_attrs(int variant, int in_dtype, mcke_gemm_attrs* out);

/* The schedule mcke_sm100_gemm_bf16_ex(variant, c_dtype) takes for an m x n x k
 * product on a GPU with `sm_count` SMs, assuming 16-byte aligned A, B and C
 * and beta == 0: host arithmetic only (no device is touched), for tests and
 * for callers that size work to whole waves. */
typedef struct {
  int kernel;         /* 0: CUDA-core kernel, 1: tcgen05 one CTA per tile, 2: tcgen05 CTA pairs */
  int tile_m, tile_n; /* output tile */
  int64_t tiles;      /* tiles of C */
  int64_t ctas;       /* CTAs launched */
  int split_dp_tiles; /* split-k schedule: tiles run whole before it (0 when not split) */
  int split_kblocks;  /* split-k schedule: 64-deep k-blocks per CTA pair after them; 0 = not split */
} mcke_gemm_plan;
int mcke_sm100_gemm_plan(int64_t m, int64_t n, int64_t k, int variant, int c_dtype, int sm_count,
                         mcke_gemm_plan* out);

/* ---- roofline denominators (replace bench/stream_triad.cu and bench/fma_peak.cu) ----
 * Measurement probes, timed by the caller: a = b + scalar * c (12 bytes per
 * element moved) and a = b (8 bytes per element) with 128-bit streaming loads
 * and evict-first stores; n % 4 == 0 and 16-byte aligned arrays. */
int mcke_sm100_peak_triad_f32(float* a, const float* b, const float* c, float scalar, int64_t n,
                              mcke_stream_t stream);
int mcke_sm100_peak_copy_f32(float* a, const float* b, int64_t n, mcke_stream_t stream);
/* FFMA throughput: `threads` threads (a multiple of 256; the suggested count,
 * 8 blocks of 256 per SM, comes from mcke_sm100_peak_fma_threads) each run 8
 * independent chains acc = fma(acc, 0.999, 1.0) for `iters` steps from
 * seed[thread] and store one sum to out[thread]: 16 flop per thread per step. */
int64_t mcke_sm100_peak_fma_threads(void);
int mcke_sm100_peak_fma_f32(const float* seed, float* out, int64_t threads, int iters, mcke_stream_t stream);
/* New (the tcgen05 bf16 peak probe): `ctas` CTAs (one per SM:
 * mcke_sm100_peak_mma_ctas()) each issue `iters` k-blocks of four
 * tcgen05.mma.cta_group::1.kind::f16 instructions (M = 128, N = 256, K = 16,
 * bf16 operands, fp32 accumulator in TMEM) from one shared-memory stage, with no
 * loads: the tensor pipe's rate for this library's own GEMM instruction.
 * mcke_sm100_peak_mma_flops(ctas, iters) is the work of one call.  Its
 * completion wait is bounded (site 10 in mcke_sm100_check_device_errors). */
int64_t mcke_sm100_peak_mma_ctas(void);
double mcke_sm100_peak_mma_flops(int64_t ctas, int iters);
int mcke_sm100_peak_mma_bf16(int64_t ctas, int iters, mcke_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MCKE_SM100_H_ */
