// mcke/graph/executor.hpp -- plans and replays a Graph over one or more GPUs.
//
// Mirrors mini-cuda-kernel-engine include/mcke/graph/executor.hpp:283-372
// (GraphExecutor: plan / set_input / run_async / synchronize, ExecutorOptions
// :115) and adds the sharding pass of a B200 box:
//
//   plan()  1. placement: every tensor is Replicated, RowSplit or ColSplit over
//              the executor's D devices, decided in topological order --
//                GEMM     A row-split            -> C row-split (B replicated)
//                         A replicated           -> C column-split (B, bias
//                                                   stored column-sliced)
//                BiasAct  follows X (a column-split X slices the bias)
//                Softmax / Reduce(row)  row-split (a replicated input is split)
//                FullReduce  each device reduces its contiguous range; the
//                         24-byte partials are all-gathered with NCCL and
//                         combined in device order on every device
//              so no collective moves activations: the only exchange is the
//              reduction's partials;
//           2. streams: per device, a node inherits the stream of its first
//              producer unless a sibling already did (chain-greedy), else the
//              least-recently-used stream; an event is recorded after a
//              producer and waited on by each consumer on another stream.
//              Launch items: one node each in topological order, or
//              (kLevelGrouped) stream 0 level by level, a level's groupable
//              fp32 bias + activation nodes gathered into grouped launches;
//           3. memory: per device one arena; graph inputs and outputs own
//              their bytes, intermediates reuse a freed block of the same
//              stream (stream order makes that reuse race-free), counting in
//              launch items (an item's outputs are placed before anything it
//              reads is freed); scratch is one block per stream sized by the
//              largest workspace_bytes();
//           4. allocation (one cudaMalloc per device), NCCL communicators
//              (only if some node exchanges), streams and events.
//   run_async()  enqueues every node on every device; never synchronises.
//              With ExecutorOptions::use_graph the first call captures that
//              enqueue into one CUDA graph per GPU (stream capture from each
//              device's stream 0, forked to its other streams by events; the
//              NCCL exchange is captured with it) and launches it; later calls
//              only launch the instantiated graphs: one host call per GPU
//              instead of one per node and event.  Pointers are fixed at plan
//              time (arena offsets), so a replay reads the current inputs.
//
// plan_dry() runs steps 1-3 without touching CUDA, for tests on a host with
// no GPU.
//
// Memory.  Each device's arena is one block taken from that device's
// DeviceAllocator (ExecutorOptions::allocators, or the allocator passed to the
// reference-shaped constructor; executor.hpp:285 of the reference takes one)
// on the device's stream 0, and returned to it when the executor goes away;
// with no allocator the executor cudaMallocs the arena itself.  Inside the
// arena the memory plan gives every tensor its offset (MemoryPolicy).
//
// Launches.  plan() also builds, once, every node's per-device OpContext and
// input/output Tensor vectors (pointers are fixed at plan time), so an eager
// run_async only issues event waits, launches and event records.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <optional>
#include <string>
#include <vector>

#include "mcke/core/device.hpp"
#include "mcke/graph/graph.hpp"
#include "mcke/graph/memory_plan.hpp"
#include "mcke/graph/schedule.hpp"
#include "mcke/memory/allocator.hpp"

namespace mcke {

struct ExecutorOptions {
  // include/mcke/graph/executor.hpp:115 of the reference, same names:
  SchedulePolicy schedule = SchedulePolicy::kChainGreedy;
  MemoryPolicy memory = MemoryPolicy::kReuseHappensBefore;
  int num_streams = 4;           // streams per device
  bool validate_numerics = false;  // keep host copies of inputs for validate_numerics()
  bool poison_buffers = false;     // fill intermediates with poison_pattern before each run
  std::uint32_t poison_pattern = 0x7F7F7F7Fu;
  // Added for one process driving a box:
  std::vector<int> devices{0};
  // One allocator per entry of `devices` (null or missing: the executor
  // cudaMallocs that device's arena itself).  Not owned.
  std::vector<DeviceAllocator*> allocators;
  // Capture the first run_async into CUDA graphs and replay them.  Needs a
  // device list that is all distinct GPUs or one GPU repeated.
  bool use_graph = false;
  // Distinct GPUs: exchange a full reduce's partials with the one-kernel
  // peer-to-peer combine (needs peer access between every pair; otherwise,
  // or when false, NCCL all-gathers them).
  bool p2p_exchange = true;
};

// Index of the first differing 32-bit word, or `bytes` when identical.
// Compared as integers: a float compare calls NaN != NaN and -0 == +0.
[[nodiscard]] std::size_t first_bit_mismatch(const void* a, const void* b, std::size_t bytes);

// Outcome of the numerics gate (include/mcke/graph/executor.hpp:149 of the reference).
struct NumericsResult {
  bool passed = false;
  int configs_compared = 0;
  int repeats = 0;
  std::size_t elements_compared = 0;
  std::string detail;  // on failure: config, tensor, word index, both words in hex
};

struct TensorPlan {
  Placement placement = Placement::kReplicated;
  std::vector<std::int64_t> offset;      // per device, bytes into that device's arena
  std::vector<Shape> local_shape;        // per device
  std::vector<std::int64_t> row_begin;   // per device (RowSplit) / column begin (ColSplit)
  std::size_t local_bytes(int d) const;
  DType dtype = DType::kF32;
};

class GraphExecutor {
 public:
  explicit GraphExecutor(Graph& g, ExecutorOptions opts = {});
  // The reference's constructor (include/mcke/graph/executor.hpp:285): the
  // executor owns `graph`, runs on `device.index`, and takes its arena from
  // `alloc` (which must outlive the executor).
  GraphExecutor(Graph graph, DeviceAllocator& alloc, DeviceInfo device, ExecutorOptions opts = {});
  ~GraphExecutor();
  GraphExecutor(const GraphExecutor&) = delete;
  GraphExecutor& operator=(const GraphExecutor&) = delete;

  [[nodiscard]] Status plan_dry();
  [[nodiscard]] Status plan();
  // Host data of the WHOLE tensor (row-major); the executor scatters the
  // slice each device owns.  Synchronous copies (setup, not the hot path).
  [[nodiscard]] Status set_input(TensorId t, const void* host, std::size_t bytes);
  [[nodiscard]] Status run_async();
  [[nodiscard]] Status synchronize();
  // Device time of the last run_async, in ms: on each device, from an event
  // recorded before the first node to one recorded after every stream joined;
  // the maximum over devices.  Synchronises.
  [[nodiscard]] StatusOr<float> last_run_ms();
  // Gathers a graph output's shards into host memory (whole tensor).
  [[nodiscard]] Status copy_output_to_host(TensorId t, void* host, std::size_t bytes);

  // The numerics gate (include/mcke/graph/executor.hpp:268-278 of the
  // reference): replays the graph under every {schedule} x {memory policy} x
  // {eager, CUDA-graph replay} configuration on this executor's devices, each
  // in a fresh executor fed the inputs given to set_input (which needs
  // opts.validate_numerics), `repeats` runs each, and compares every graph
  // output bit for bit against a golden run (kSequential, kAllocPerTensor,
  // eager) and each configuration against its own first run.
  [[nodiscard]] StatusOr<NumericsResult> validate_numerics(int repeats = 3);

  [[nodiscard]] const TensorPlan& tensor_plan(TensorId t) const { return tplan_.at(t); }
  [[nodiscard]] int stream_of(NodeId n) const { return node_stream_.at(n); }
  // Launch items in enqueue order: one node each, or (kLevelGrouped) the
  // nodes one grouped launch runs together.  The memory plan treats an item
  // as one step: its nodes run at the same time.
  [[nodiscard]] std::size_t num_launch_items() const { return items_.size(); }
  [[nodiscard]] const std::vector<NodeId>& launch_item(std::size_t i) const { return items_.at(i); }
  [[nodiscard]] int launch_item_of(NodeId n) const { return item_of_.at(n); }
  [[nodiscard]] std::size_t arena_bytes(int device_index) const { return arena_bytes_.at(device_index); }
  [[nodiscard]] int num_devices() const { return static_cast<int>(opts_.devices.size()); }
  [[nodiscard]] const ExecutorOptions& options() const noexcept { return opts_; }
  [[nodiscard]] const DeviceInfo& device_info() const noexcept { return device_; }
  [[nodiscard]] std::size_t num_events() const { return event_edges_; }
  [[nodiscard]] std::string describe() const;

 private:
  struct Impl;
  [[nodiscard]] Status place();
  [[nodiscard]] Status assign_streams();
  [[nodiscard]] int groupable_act(NodeId nid) const;
  [[nodiscard]] Status plan_memory();
  [[nodiscard]] Tensor local_tensor(TensorId t, int d) const;
  [[nodiscard]] Status enqueue(bool capturing);
  [[nodiscard]] Status capture();
  [[nodiscard]] Status build_launches();

  std::optional<Graph> owned_;  // the graph, when the executor was given it by value
  Graph& g_;
  ExecutorOptions opts_;
  DeviceInfo device_;
  std::vector<std::pair<TensorId, std::vector<char>>> input_cache_;  // validate_numerics only
  std::vector<TensorPlan> tplan_;
  std::vector<int> node_stream_;                 // same stream index on every device
  std::vector<std::vector<int>> waits_;          // per node: producer nodes on other streams
  std::vector<bool> record_after_;               // per node: record an event after it
  std::vector<std::size_t> arena_bytes_;         // per device
  std::vector<std::vector<std::int64_t>> scratch_offset_;   // [device][stream index]
  std::vector<std::size_t> scratch_bytes_;                   // per stream index
  std::vector<std::vector<std::int64_t>> exchange_offset_;  // [device][node] (or -1)
  std::vector<bool> view_rows_;  // per node: input 0 is a replicated tensor read as local rows
  std::vector<std::vector<NodeId>> items_;  // launch items in enqueue order
  std::vector<int> item_of_;                // per node: its launch item
  std::size_t event_edges_ = 0;
  bool planned_ = false;
  std::unique_ptr<Impl> impl_;
};

}  // namespace mcke
