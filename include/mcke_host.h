/*
 * mcke_host.h -- C-ABI of libmcke_host.so, the C++ host layer (Graph, Op,
 * GraphExecutor with the multi-GPU sharding pass) over libmcke_sm100a.so.
 *
 * The reference exposes this layer only as C++ (mini-cuda-kernel-engine
 * include/mcke/graph/graph.hpp:109 Graph, include/mcke/graph/op.hpp:99 Op and
 * :180-303 GemmOp/BiasActOp/ReduceOp/SoftmaxOp, include/mcke/graph/executor.hpp:283
 * GraphExecutor); the C++ headers under mini-cuda-kernel-engine_b200/host/include
 * keep those names.  These C entry points wrap them for callers without a C++
 * toolchain (Python's ctypes in this repository's tests and bench).  Objects
 * are opaque handles; every function returns an mcke_status code and the
 * message of the last failure on the calling thread is available from
 * mcke_host_last_error_string().
 */
#ifndef MCKE_HOST_H_
#define MCKE_HOST_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mcke_graph mcke_graph;
typedef struct mcke_executor mcke_executor;

/* Tensor placement hints for graph inputs (mcke::Placement). */
enum { MCKE_PLACE_REPLICATED = 0, MCKE_PLACE_ROW_SPLIT = 1, MCKE_PLACE_COL_SPLIT = 2 };
/* Element types (mcke::DType): 0 f32, 2 bf16, 4 u8. */

const char* mcke_host_last_error_string(void);

/* Graph construction (graph.hpp:109 add_input / add_node / mark_output / finalize). */
mcke_graph* mcke_graph_create(void);
void mcke_graph_destroy(mcke_graph* g);
int mcke_graph_add_input(mcke_graph* g, const char* name, const int64_t* dims, int rank, int dtype,
                         int placement, uint32_t* id_out);
/* GemmOp (op.hpp:180): bias < 0 for none; act is mcke_activation; out_dtype 0 f32 / 2 bf16;
 * variant is the reference's GemmVariant value (8 = kTcgen05Bf16, ignored for bf16 operands). */
int mcke_graph_add_gemm(mcke_graph* g, const char* name, uint32_t a, uint32_t b, int64_t bias, float alpha,
                        int act, int out_dtype, int variant, uint32_t* out);
/* BiasActOp (op.hpp:230): vector_width 0 = widest legal. */
int mcke_graph_add_bias_act(mcke_graph* g, const char* name, uint32_t x, uint32_t bias, int act,
                            int vector_width, uint32_t* out);
/* SoftmaxOp (op.hpp:290). */
int mcke_graph_add_softmax(mcke_graph* g, const char* name, uint32_t x, int variant, uint32_t* out);
/* ReduceOp (op.hpp:260). */
int mcke_graph_add_reduce_row(mcke_graph* g, const char* name, uint32_t x, int kind, int variant, uint32_t* out);
/* FullReduceOp (new): 16-byte result {float sum; float max; int64 argmax}. */
int mcke_graph_add_reduce_full(mcke_graph* g, const char* name, uint32_t x, uint32_t* out);
int mcke_graph_mark_output(mcke_graph* g, uint32_t t);
int mcke_graph_finalize(mcke_graph* g);
/* The reference's cost model (include/mcke/graph/cost_model.hpp): the sum over
 * the graph's nodes of max(flops / peak, bytes / bandwidth) on the graph's
 * global shapes, in ms -- a sequential lower bound for one run on one device.
 * Peaks in TFLOP/s and GB/s, both > 0. */
int mcke_graph_roofline_ms(const mcke_graph* g, double peak_tflops, double peak_gbs, double* ms_out);

/* GraphExecutor (executor.hpp:283) over `num_devices` GPUs. */
mcke_executor* mcke_executor_create(mcke_graph* g, const int* devices, int num_devices, int streams_per_device);
/* As mcke_executor_create, with option flags:
 *   MCKE_EXECUTOR_CUDA_GRAPH  capture the first run into one CUDA graph per GPU
 *                             and replay it (devices all distinct or one GPU repeated);
 *   MCKE_EXECUTOR_POISON      fill intermediates with 0xFF before each run (tests);
 *   MCKE_EXECUTOR_NCCL_EXCHANGE  on distinct GPUs, all-gather a full reduce's partials
 *                             with NCCL instead of the one-kernel peer-to-peer combine. */
#define MCKE_EXECUTOR_CUDA_GRAPH 1u
#define MCKE_EXECUTOR_POISON 2u
#define MCKE_EXECUTOR_NCCL_EXCHANGE 4u
/*   MCKE_EXECUTOR_BUDDY       take each device's arena from a BuddyAllocator of
 *                             that device with 4 GiB slabs (mcke/memory/buddy_allocator.hpp;
 *                             the reference's DeviceAllocator interface, executor.hpp:285),
 *                             owned by this handle;
 *   MCKE_EXECUTOR_VALIDATE    keep host copies of the inputs for
 *                             mcke_executor_validate_numerics (ExecutorOptions::validate_numerics). */
#define MCKE_EXECUTOR_BUDDY 8u
#define MCKE_EXECUTOR_VALIDATE 16u
mcke_executor* mcke_executor_create_ex(mcke_graph* g, const int* devices, int num_devices, int streams_per_device,
                                       unsigned flags);
/* As mcke_executor_create_ex with the stream schedule (mcke::SchedulePolicy:
 * 0 sequential, 1 level-parallel, 2 chain-greedy; schedule.hpp:49 of the
 * reference; 3 level-grouped, added: stream 0 level by level, a level's fp32
 * bias + activation nodes in grouped launches) and the memory policy (mcke::MemoryPolicy: 0 alloc-per-tensor,
 * 2 reuse-same-stream, 3 reuse-happens-before; memory_plan.hpp:67). */
mcke_executor* mcke_executor_create_policy(mcke_graph* g, const int* devices, int num_devices, int num_streams,
                                           unsigned flags, int schedule, int memory);
void mcke_executor_destroy(mcke_executor* e);
/* Planning only (placement, streams, memory): touches no GPU. */
int mcke_executor_plan_dry(mcke_executor* e);
int mcke_executor_plan(mcke_executor* e);
int mcke_executor_set_input(mcke_executor* e, uint32_t t, const void* host, size_t bytes);
int mcke_executor_run_async(mcke_executor* e);
int mcke_executor_synchronize(mcke_executor* e);
int mcke_executor_copy_output(mcke_executor* e, uint32_t t, void* host, size_t bytes);
/* Device time of the last run in ms (fork-to-join events, max over devices); synchronises. */
int mcke_executor_last_run_ms(mcke_executor* e, float* ms_out);
/* Writes a NUL-terminated plan description (placements, streams, waits, arena sizes). */
int mcke_executor_describe(mcke_executor* e, char* buf, size_t len);
/* Placement of tensor t after planning (MCKE_PLACE_*), its stream (node output), arena bytes. */
int mcke_executor_placement(mcke_executor* e, uint32_t t, int* placement_out);
int mcke_executor_arena_bytes(mcke_executor* e, int device_index, size_t* bytes_out);
int mcke_executor_num_events(mcke_executor* e, size_t* out);
/* Launch items of the plan, in enqueue order (after plan_dry or plan): their
 * number, and the number of nodes in the largest (1 unless the schedule is
 * level-grouped). */
int mcke_executor_launch_items(mcke_executor* e, size_t* items_out, size_t* largest_out);
/* The numerics gate (executor.hpp:268 of the reference, GraphExecutor::validate_numerics):
 * replays the graph under every schedule x memory policy x {eager, CUDA graph}
 * on this executor's devices, `repeats` runs each, and compares all outputs bit
 * for bit with a sequential, alloc-per-tensor, eager golden run and each
 * configuration with its own first run.  Needs MCKE_EXECUTOR_VALIDATE and every
 * input set.  *passed = 1 or 0, *configs = configurations compared; detail
 * receives the first mismatch (configuration, output, word, both words). */
int mcke_executor_validate_numerics(mcke_executor* e, int repeats, int* passed, int* configs, char* detail,
                                    size_t len);
/* Statistics of device entry `device_index`'s allocator (mcke::AllocatorStats). */
typedef struct {
  uint64_t alloc_calls, free_calls, raw_malloc_calls, raw_free_calls;
  uint64_t bytes_reserved, bytes_in_use, bytes_requested, peak_bytes_in_use;
  char name[24];
} mcke_alloc_stats;
int mcke_executor_alloc_stats(mcke_executor* e, int device_index, mcke_alloc_stats* out);

#ifdef __cplusplus
}
#endif
#endif /* MCKE_HOST_H_ */
