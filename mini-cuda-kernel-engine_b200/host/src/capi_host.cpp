// capi_host.cpp -- extern "C" wrappers of the C++ host layer (include/mcke_host.h).
#include "mcke_host.h"

#include <algorithm>
#include <cstring>
#include <memory>
#include <string>

#include "mcke/graph/cost_model.hpp"
#include "mcke/graph/executor.hpp"
#include "mcke/memory/buddy_allocator.hpp"

struct mcke_graph {
  mcke::Graph g;
};
struct mcke_executor {
  // declared before `ex`, so the executor (which returns its arenas to them)
  // goes first
  std::vector<std::unique_ptr<mcke::BuddyAllocator>> allocs;
  std::unique_ptr<mcke::GraphExecutor> ex;
};

namespace {
thread_local std::string g_err;

int ret(const mcke::Status& s) {
  if (s.ok()) return 0;
  g_err = s.to_string();
  return static_cast<int>(s.code());
}

template <typename T>
int ret_ids(const mcke::StatusOr<std::vector<mcke::TensorId>>& r, uint32_t* out) {
  if (!r.ok()) return ret(r.status());
  if (out) *out = r.value().at(0);
  return 0;
}

int add(mcke_graph* g, const char* name, mcke::OpPtr op, std::vector<mcke::TensorId> in, uint32_t* out) {
  if (!g) {
    g_err = "null graph";
    return static_cast<int>(mcke::StatusCode::kInvalidArgument);
  }
  auto r = g->g.add_node(name ? name : "node", std::move(op), std::move(in));
  return ret_ids<void>(r, out);
}

mcke::DType dtype_of(int v) { return static_cast<mcke::DType>(v); }
}  // namespace

extern "C" {

const char* mcke_host_last_error_string(void) { return g_err.c_str(); }

mcke_graph* mcke_graph_create(void) { return new mcke_graph(); }
void mcke_graph_destroy(mcke_graph* g) { delete g; }

int mcke_graph_add_input(mcke_graph* g, const char* name, const int64_t* dims, int rank, int dtype, int placement,
                         uint32_t* id_out) {
  if (!g || !dims || rank < 1 || placement < 0 || placement > 2 || (dtype != 0 && dtype != 2 && dtype != 4)) {
    g_err = "mcke_graph_add_input: bad argument";
    return static_cast<int>(mcke::StatusCode::kInvalidArgument);
  }
  mcke::TensorDesc d;
  d.shape = mcke::Shape(std::vector<std::int64_t>(dims, dims + rank));
  d.dtype = dtype_of(dtype);
  d.name = name ? name : "input";
  d.placement = static_cast<mcke::Placement>(placement);
  const auto id = g->g.add_input(d);
  if (id_out) *id_out = id;
  return 0;
}

int mcke_graph_add_gemm(mcke_graph* g, const char* name, uint32_t a, uint32_t b, int64_t bias, float alpha, int act,
                        int out_dtype, int variant, uint32_t* out) {
  mcke::GemmParams p;
  p.alpha = alpha;
  p.act = static_cast<mcke::kernels::Activation>(act);
  p.out_dtype = dtype_of(out_dtype);
  p.variant = static_cast<mcke::kernels::GemmVariant>(variant);
  std::vector<mcke::TensorId> in{a, b};
  if (bias >= 0) in.push_back(static_cast<mcke::TensorId>(bias));
  return add(g, name, std::make_unique<mcke::GemmOp>(p), in, out);
}

int mcke_graph_add_bias_act(mcke_graph* g, const char* name, uint32_t x, uint32_t bias, int act, int vector_width,
                            uint32_t* out) {
  mcke::BiasActParams p;
  p.act = static_cast<mcke::BiasActParams::Act>(act);
  p.vector_width = vector_width;
  return add(g, name, std::make_unique<mcke::BiasActOp>(p), {x, bias}, out);
}

int mcke_graph_add_softmax(mcke_graph* g, const char* name, uint32_t x, int variant, uint32_t* out) {
  mcke::SoftmaxParams p;
  p.variant = static_cast<mcke::SoftmaxParams::Variant>(variant);
  return add(g, name, std::make_unique<mcke::SoftmaxOp>(p), {x}, out);
}

int mcke_graph_add_reduce_row(mcke_graph* g, const char* name, uint32_t x, int kind, int variant, uint32_t* out) {
  mcke::ReduceParams p;
  p.kind = static_cast<mcke::ReduceParams::Kind>(kind);
  p.variant = static_cast<mcke::ReduceParams::Variant>(variant);
  return add(g, name, std::make_unique<mcke::ReduceOp>(p), {x}, out);
}

int mcke_graph_add_reduce_full(mcke_graph* g, const char* name, uint32_t x, uint32_t* out) {
  return add(g, name, std::make_unique<mcke::FullReduceOp>(), {x}, out);
}

int mcke_graph_mark_output(mcke_graph* g, uint32_t t) { return g ? ret(g->g.mark_output(t)) : 2; }
int mcke_graph_finalize(mcke_graph* g) { return g ? ret(g->g.finalize()) : 2; }

int mcke_graph_roofline_ms(const mcke_graph* g, double peak_tflops, double peak_gbs, double* ms_out) {
  if (!g || !ms_out || !(peak_tflops > 0.0) || !(peak_gbs > 0.0)) return 2;
  *ms_out = mcke::graph_roofline_ms(g->g, mcke::Roofline{peak_tflops * 1e12, peak_gbs * 1e9});
  return 0;
}

mcke_executor* mcke_executor_create_policy(mcke_graph* g, const int* devices, int num_devices, int num_streams,
                                           unsigned flags, int schedule, int memory) {
  if (!g || !devices || num_devices < 1 || schedule < 0 || schedule > 3 || memory < 0 || memory > 3) return nullptr;
  mcke::ExecutorOptions o;
  o.devices.assign(devices, devices + num_devices);
  o.num_streams = num_streams > 0 ? num_streams : 4;
  o.use_graph = (flags & MCKE_EXECUTOR_CUDA_GRAPH) != 0;
  o.poison_buffers = (flags & MCKE_EXECUTOR_POISON) != 0;
  o.p2p_exchange = (flags & MCKE_EXECUTOR_NCCL_EXCHANGE) == 0;
  o.validate_numerics = (flags & MCKE_EXECUTOR_VALIDATE) != 0;
  o.schedule = static_cast<mcke::SchedulePolicy>(schedule);
  o.memory = static_cast<mcke::MemoryPolicy>(memory);
  auto* e = new mcke_executor();
  if (flags & MCKE_EXECUTOR_BUDDY) {
    // 4 GiB slabs: config 5's ~3.6 GB arena is one buddy block of a slab
    mcke::BuddyConfig bc;
    bc.slab_bytes = std::size_t{1} << 32;
    for (int d = 0; d < num_devices; ++d) {
      e->allocs.push_back(std::make_unique<mcke::BuddyAllocator>(devices[d], bc));
      o.allocators.push_back(e->allocs.back().get());
    }
  }
  e->ex = std::make_unique<mcke::GraphExecutor>(g->g, o);
  return e;
}

mcke_executor* mcke_executor_create_ex(mcke_graph* g, const int* devices, int num_devices, int streams_per_device,
                                       unsigned flags) {
  return mcke_executor_create_policy(g, devices, num_devices, streams_per_device, flags,
                                     static_cast<int>(mcke::SchedulePolicy::kChainGreedy),
                                     static_cast<int>(mcke::MemoryPolicy::kReuseHappensBefore));
}

mcke_executor* mcke_executor_create(mcke_graph* g, const int* devices, int num_devices, int streams_per_device) {
  return mcke_executor_create_ex(g, devices, num_devices, streams_per_device, 0);
}

void mcke_executor_destroy(mcke_executor* e) { delete e; }

#define EX_CHECK(e)                                        \
  if (!(e) || !(e)->ex) {                                  \
    g_err = "null executor";                               \
    return static_cast<int>(mcke::StatusCode::kInvalidArgument); \
  }

int mcke_executor_plan_dry(mcke_executor* e) { EX_CHECK(e); return ret(e->ex->plan_dry()); }
int mcke_executor_plan(mcke_executor* e) { EX_CHECK(e); return ret(e->ex->plan()); }
int mcke_executor_set_input(mcke_executor* e, uint32_t t, const void* host, size_t bytes) {
  EX_CHECK(e);
  return ret(e->ex->set_input(t, host, bytes));
}
int mcke_executor_run_async(mcke_executor* e) { EX_CHECK(e); return ret(e->ex->run_async()); }
int mcke_executor_synchronize(mcke_executor* e) { EX_CHECK(e); return ret(e->ex->synchronize()); }
int mcke_executor_copy_output(mcke_executor* e, uint32_t t, void* host, size_t bytes) {
  EX_CHECK(e);
  return ret(e->ex->copy_output_to_host(t, host, bytes));
}
int mcke_executor_last_run_ms(mcke_executor* e, float* ms_out) {
  EX_CHECK(e);
  auto r = e->ex->last_run_ms();
  if (!r.ok()) return ret(r.status());
  if (ms_out) *ms_out = *r;
  return 0;
}
int mcke_executor_describe(mcke_executor* e, char* buf, size_t len) {
  EX_CHECK(e);
  const std::string s = e->ex->describe();
  if (buf && len) {
    const size_t n = s.size() < len - 1 ? s.size() : len - 1;
    std::memcpy(buf, s.data(), n);
    buf[n] = '\0';
  }
  return 0;
}
int mcke_executor_placement(mcke_executor* e, uint32_t t, int* placement_out) {
  EX_CHECK(e);
  if (placement_out) *placement_out = static_cast<int>(e->ex->tensor_plan(t).placement);
  return 0;
}
int mcke_executor_arena_bytes(mcke_executor* e, int device_index, size_t* bytes_out) {
  EX_CHECK(e);
  if (bytes_out) *bytes_out = e->ex->arena_bytes(device_index);
  return 0;
}
int mcke_executor_num_events(mcke_executor* e, size_t* out) {
  EX_CHECK(e);
  if (out) *out = e->ex->num_events();
  return 0;
}
int mcke_executor_launch_items(mcke_executor* e, size_t* items_out, size_t* largest_out) {
  EX_CHECK(e);
  std::size_t largest = 0;
  for (std::size_t i = 0; i < e->ex->num_launch_items(); ++i)
    largest = std::max(largest, e->ex->launch_item(i).size());
  if (items_out) *items_out = e->ex->num_launch_items();
  if (largest_out) *largest_out = largest;
  return 0;
}
int mcke_executor_validate_numerics(mcke_executor* e, int repeats, int* passed, int* configs, char* detail,
                                    size_t len) {
  EX_CHECK(e);
  auto r = e->ex->validate_numerics(repeats);
  if (!r.ok()) return ret(r.status());
  if (passed) *passed = r->passed ? 1 : 0;
  if (configs) *configs = r->configs_compared;
  if (detail && len) {
    const size_t n = r->detail.size() < len - 1 ? r->detail.size() : len - 1;
    std::memcpy(detail, r->detail.data(), n);
    detail[n] = '\0';
  }
  return 0;
}
int mcke_executor_alloc_stats(mcke_executor* e, int device_index, mcke_alloc_stats* out) {
  EX_CHECK(e);
  const auto& al = e->ex->options().allocators;
  if (device_index < 0 || device_index >= static_cast<int>(al.size()) || !al[device_index] || !out) {
    g_err = "mcke_executor_alloc_stats: no allocator for that device entry";
    return static_cast<int>(mcke::StatusCode::kInvalidArgument);
  }
  const mcke::AllocatorStats st = al[device_index]->stats();
  out->alloc_calls = st.alloc_calls;
  out->free_calls = st.free_calls;
  out->raw_malloc_calls = st.raw_malloc_calls;
  out->raw_free_calls = st.raw_free_calls;
  out->bytes_reserved = st.bytes_reserved;
  out->bytes_in_use = st.bytes_in_use;
  out->bytes_requested = st.bytes_requested;
  out->peak_bytes_in_use = st.peak_bytes_in_use;
  const std::string_view nm = al[device_index]->name();
  const size_t n = nm.size() < sizeof(out->name) - 1 ? nm.size() : sizeof(out->name) - 1;
  std::memcpy(out->name, nm.data(), n);
  out->name[n] = '\0';
  return 0;
}

}  // extern "C"
