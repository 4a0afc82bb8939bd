// executor.cpp -- the sharding pass, stream assignment, memory plan and replay.
#include "mcke/graph/executor.hpp"

#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstring>

namespace mcke {
namespace {

constexpr std::size_t kAlign = 256;
std::size_t align_up(std::size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

const char* placement_name(Placement p) {
  switch (p) {
    case Placement::kReplicated: return "replicated";
    case Placement::kRowSplit: return "row-split";
    case Placement::kColSplit: return "col-split";
  }
  return "?";
}

// Split extent of a tensor under a placement: the flattened rows for rank >= 2,
// the elements for rank 1, the columns for a column split.
std::int64_t split_extent(const Shape& s, Placement p) {
  if (p == Placement::kColSplit) return s.cols();
  return s.rank() >= 2 ? s.rows() : s.numel();
}

Status nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return OkStatus();
  return InternalError(std::string(what) + ": " + ncclGetErrorString(r));
}

}  // namespace

std::size_t TensorPlan::local_bytes(int d) const {
  return static_cast<std::size_t>(local_shape.at(d).numel()) * dtype_size(dtype);
}

struct GraphExecutor::Impl {
  struct Dev {
    int device = 0;
    void* arena = nullptr;
    DeviceAllocator* alloc = nullptr;  // where the arena came from (null: cudaMalloc)
    Allocation arena_block;
    std::vector<rt::Stream> streams;
    std::vector<rt::Event> node_events;  // indexed by NodeId (only where recorded)
    std::vector<rt::Event> done;         // one per stream: end of the previous run
    rt::Event t_start, t_end;            // timing events around one run (stream 0)
    std::vector<rt::Event> exchange_ready;  // per exchanging node: this shard's partial is written
    std::vector<rt::Event> exchange_done;   // per exchanging node: this device's copies are done
    rt::Event fork, join;                // graph capture: fan-out from / back to the origin stream
    ncclComm_t comm = nullptr;
  };
  std::vector<Dev> devs;
  bool ran_once = false;
  bool peer_copy = false;
  // Peer-to-peer exchange: per exchanging node and device, the exchange
  // buffer and the device table of all devices' buffers.
  bool p2p = false;
  std::vector<std::vector<void*>> p2p_buf;    // [node][device]
  std::vector<std::vector<void*>> p2p_table;  // [node][device]
  // Graph mode: one instantiated graph per capture group (a GPU); origin[i] is
  // the device entry whose stream 0 launches execs[i] and carries its timing.
  std::vector<cudaGraphExec_t> execs;
  std::vector<int> origins;
  // Per node, built once by build_launches(): each device's context and
  // tensors, and where each device gathers the exchanged partials.
  struct NodeLaunch {
    std::vector<OpContext> ctx;
    std::vector<std::vector<Tensor>> ins, outs;
    std::vector<void*> gathered;
  };
  std::vector<NodeLaunch> launches;
  ~Impl() {
    for (std::size_t nid = 0; nid < p2p_buf.size(); ++nid)
      for (std::size_t d = 0; d < p2p_buf[nid].size(); ++d) {
        rt::DeviceGuard g(devs[d].device);
        if (p2p_buf[nid][d]) cudaFree(p2p_buf[nid][d]);
        if (p2p_table[nid][d]) cudaFree(p2p_table[nid][d]);
      }
    for (std::size_t i = 0; i < execs.size(); ++i) {
      rt::DeviceGuard g(devs[origins[i]].device);
      cudaGraphExecDestroy(execs[i]);
    }
    for (Dev& d : devs) {
      rt::DeviceGuard g(d.device);
      if (d.comm) ncclCommDestroy(d.comm);
      if (d.arena && d.alloc) {
        // the last run's work may still be in flight on any of the streams
        for (auto& st : d.streams) static_cast<void>(st.synchronize());
        static_cast<void>(d.alloc->deallocate(d.arena_block, d.streams.empty() ? nullptr : d.streams[0].native()));
      } else if (d.arena) {
        cudaFree(d.arena);
      }
    }
  }
};

GraphExecutor::GraphExecutor(Graph& g, ExecutorOptions opts) : g_(g), opts_(std::move(opts)) {
  device_.index = opts_.devices.empty() ? 0 : opts_.devices[0];
}

GraphExecutor::GraphExecutor(Graph graph, DeviceAllocator& alloc, DeviceInfo device, ExecutorOptions opts)
    : owned_(std::move(graph)), g_(*owned_), opts_(std::move(opts)), device_(std::move(device)) {
  opts_.devices = {device_.index};
  opts_.allocators = {&alloc};
}

GraphExecutor::~GraphExecutor() = default;

std::size_t first_bit_mismatch(const void* a, const void* b, std::size_t bytes) {
  const auto* x = static_cast<const unsigned char*>(a);
  const auto* y = static_cast<const unsigned char*>(b);
  for (std::size_t i = 0; i + 4 <= bytes; i += 4) {
    std::uint32_t u, v;
    std::memcpy(&u, x + i, 4);
    std::memcpy(&v, y + i, 4);
    if (u != v) return i / 4;
  }
  for (std::size_t i = bytes / 4 * 4; i < bytes; ++i)
    if (x[i] != y[i]) return i / 4;
  return bytes;
}

// ------------------------------------------------------------- placement

Status GraphExecutor::place() {
  const int D = num_devices();
  if (D < 1) return InvalidArgumentError("ExecutorOptions.devices is empty");
  const std::size_t T = g_.num_tensors();
  tplan_.assign(T, TensorPlan{});
  std::vector<bool> locked(T, false);      // a consumer has been planned against this placement
  std::vector<bool> row_view(T, false);    // replicated intermediate read as local rows
  view_rows_.assign(g_.num_nodes(), false);
  for (TensorId t = 0; t < T; ++t) {
    tplan_[t].dtype = g_.tensor(t).dtype;
    tplan_[t].placement = (D > 1 && g_.is_input(t)) ? g_.tensor(t).placement : Placement::kReplicated;
  }
  auto P = [&](TensorId t) { return tplan_[t].placement; };
  // Re-place a graph input that no planned consumer depends on yet.
  auto require = [&](TensorId t, Placement want, const Node& n) -> Status {
    if (P(t) == want) {
      locked[t] = true;
      return OkStatus();
    }
    if (!g_.is_input(t) || locked[t])
      return FailedPreconditionError("node '" + n.name + "' needs tensor '" + g_.tensor(t).name + "' " +
                                     placement_name(want) + " but it is already " + placement_name(P(t)) +
                                     "; that would need a collective this executor does not insert");
    if (want == Placement::kColSplit && g_.tensor(t).shape.rank() != 2 && g_.tensor(t).shape.rank() != 1)
      return FailedPreconditionError("node '" + n.name + "': only rank-1/2 tensors can be column-split");
    tplan_[t].placement = want;
    locked[t] = true;
    return OkStatus();
  };

  if (D > 1) {
    for (NodeId nid : g_.topo_order()) {
      const Node& n = g_.node(nid);
      const std::string_view type = n.op->type_name();
      Placement out = Placement::kReplicated;
      if (type == "Gemm") {
        const TensorId a = n.inputs[0], b = n.inputs[1];
        if (P(a) == Placement::kRowSplit) {
          MCKE_RETURN_IF_ERROR(require(b, Placement::kReplicated, n));
          if (n.inputs.size() == 3) MCKE_RETURN_IF_ERROR(require(n.inputs[2], Placement::kReplicated, n));
          out = Placement::kRowSplit;
        } else if (P(a) == Placement::kReplicated) {
          locked[a] = true;
          MCKE_RETURN_IF_ERROR(require(b, Placement::kColSplit, n));
          // a rank-1 bias column-splits element-wise, which is its row split
          if (n.inputs.size() == 3) MCKE_RETURN_IF_ERROR(require(n.inputs[2], Placement::kColSplit, n));
          out = Placement::kColSplit;
        } else {
          return FailedPreconditionError("node '" + n.name + "': a column-split A would need an all-gather");
        }
      } else if (type == "BiasAct") {
        const TensorId x = n.inputs[0], bias = n.inputs[1];
        if (P(x) == Placement::kColSplit) {
          MCKE_RETURN_IF_ERROR(require(bias, Placement::kColSplit, n));
          out = Placement::kColSplit;
        } else {
          if (P(x) == Placement::kReplicated) {
            if (g_.is_input(x) && !locked[x]) MCKE_RETURN_IF_ERROR(require(x, Placement::kRowSplit, n));
            else row_view[x] = locked[x] = view_rows_[nid] = true;
          }
          MCKE_RETURN_IF_ERROR(require(bias, Placement::kReplicated, n));
          out = Placement::kRowSplit;
        }
      } else if (type == "Softmax" || type == "Reduce" || type == "FullReduce") {
        const TensorId x = n.inputs[0];
        if (P(x) == Placement::kColSplit)
          return FailedPreconditionError("node '" + n.name + "' reduces rows of a column-split tensor; that needs "
                                         "an all-gather this executor does not insert");
        if (P(x) == Placement::kReplicated) {
          if (g_.is_input(x) && !locked[x]) MCKE_RETURN_IF_ERROR(require(x, Placement::kRowSplit, n));
          else row_view[x] = locked[x] = view_rows_[nid] = true;
        }
        locked[x] = true;
        out = (type == "FullReduce") ? Placement::kReplicated : Placement::kRowSplit;
      } else {
        return UnimplementedError("node '" + n.name + "': no sharding rule for op " + std::string(type));
      }
      for (TensorId o : n.outputs) tplan_[o].placement = out;
    }
  }
  // Local shapes.
  for (TensorId t = 0; t < T; ++t) {
    TensorPlan& tp = tplan_[t];
    const Shape& s = g_.tensor(t).shape;
    tp.local_shape.assign(D, s);
    tp.row_begin.assign(D, 0);
    tp.offset.assign(D, -1);
    if (tp.placement == Placement::kReplicated) continue;
    const std::int64_t E = split_extent(s, tp.placement);
    if (E < D)
      return FailedPreconditionError("tensor '" + g_.tensor(t).name + "' has " + std::to_string(E) +
                                     " rows/columns to split over " + std::to_string(D) + " devices");
    for (int d = 0; d < D; ++d) {
      const std::int64_t b = E * d / D, e = E * (d + 1) / D;
      tp.row_begin[d] = b;
      if (tp.placement == Placement::kColSplit)
        tp.local_shape[d] = s.rank() == 1 ? Shape{e - b} : Shape{s.rows(), e - b};
      else
        tp.local_shape[d] = s.rank() >= 2 ? Shape{e - b, s.cols()} : Shape{e - b};
    }
  }
  // Row views of replicated intermediates use the row split of the consumer's
  // other operands; record the boundaries so local_tensor can offset into them.
  for (TensorId t = 0; t < T; ++t) {
    if (!row_view[t]) continue;
    const Shape& s = g_.tensor(t).shape;
    const std::int64_t E = s.rank() >= 2 ? s.rows() : s.numel();
    for (int d = 0; d < D; ++d) tplan_[t].row_begin[d] = E * d / D;
  }
  return OkStatus();
}

// ------------------------------------------------------------ streams

Status GraphExecutor::assign_streams() {
  const int S = std::max(1, opts_.num_streams);
  const std::size_t N = g_.num_nodes();
  node_stream_.assign(N, 0);
  waits_.assign(N, {});
  record_after_.assign(N, false);
  if (opts_.schedule == SchedulePolicy::kLevelParallel) {
    // level = longest path from a graph input; each level dealt round-robin
    std::vector<int> level(N, 0);
    int max_level = 0;
    for (NodeId nid : g_.topo_order()) {
      for (TensorId t : g_.node(nid).inputs) {
        const NodeId p = g_.producer(t);
        if (p != kInvalidNode) level[nid] = std::max(level[nid], level[p] + 1);
      }
      max_level = std::max(max_level, level[nid]);
    }
    std::vector<int> next(static_cast<std::size_t>(max_level) + 1, 0);
    for (NodeId nid : g_.topo_order()) node_stream_[nid] = next[level[nid]]++ % S;
  } else if (opts_.schedule == SchedulePolicy::kChainGreedy) {
    std::vector<bool> donated(N, false);
    std::vector<std::int64_t> last_use(S, -1);
    std::int64_t tick = 0;
    for (NodeId nid : g_.topo_order()) {
      const Node& n = g_.node(nid);
      int s = -1;
      for (TensorId t : n.inputs) {
        const NodeId p = g_.producer(t);
        if (p != kInvalidNode && !donated[p]) {
          donated[p] = true;
          s = node_stream_[p];
          break;
        }
      }
      if (s < 0) s = static_cast<int>(std::min_element(last_use.begin(), last_use.end()) - last_use.begin());
      node_stream_[nid] = s;
      last_use[s] = tick++;
    }
  }  // kSequential: every node stays on stream 0
  event_edges_ = 0;
  for (NodeId nid : g_.topo_order()) {
    const Node& n = g_.node(nid);
    for (TensorId t : n.inputs) {
      const NodeId p = g_.producer(t);
      if (p == kInvalidNode || node_stream_[p] == node_stream_[nid]) continue;
      if (std::find(waits_[nid].begin(), waits_[nid].end(), static_cast<int>(p)) != waits_[nid].end()) continue;
      waits_[nid].push_back(static_cast<int>(p));
      record_after_[p] = true;
      ++event_edges_;
    }
  }
  // Launch items: one node each in topological order, or (kLevelGrouped) level
  // by level with the groupable bias + activation nodes of a level gathered,
  // per activation, into items of up to kBiasActGroupMax nodes.
  items_.clear();
  item_of_.assign(N, -1);
  if (opts_.schedule != SchedulePolicy::kLevelGrouped) {
    for (NodeId nid : g_.topo_order()) {
      item_of_[nid] = static_cast<int>(items_.size());
      items_.push_back({nid});
    }
    return OkStatus();
  }
  std::vector<int> level(N, 0);
  int max_level = 0;
  for (NodeId nid : g_.topo_order()) {
    for (TensorId t : g_.node(nid).inputs) {
      const NodeId p = g_.producer(t);
      if (p != kInvalidNode) level[nid] = std::max(level[nid], level[p] + 1);
    }
    max_level = std::max(max_level, level[nid]);
  }
  std::vector<std::vector<NodeId>> by_level(static_cast<std::size_t>(max_level) + 1);
  for (NodeId nid : g_.topo_order()) by_level[level[nid]].push_back(nid);
  for (const auto& nodes : by_level) {
    int open[4] = {-1, -1, -1, -1};  // the item still taking nodes, per activation
    for (NodeId nid : nodes) {
      const int act = groupable_act(nid);
      if (act < 0) {
        item_of_[nid] = static_cast<int>(items_.size());
        items_.push_back({nid});
        continue;
      }
      int& it = open[act];
      if (it < 0 || static_cast<int>(items_[it].size()) == kernels::kBiasActGroupMax) {
        it = static_cast<int>(items_.size());
        items_.emplace_back();
      }
      item_of_[nid] = it;
      items_[it].push_back(nid);
    }
  }
  return OkStatus();
}

// The activation (0-3) of a bias + activation node the grouped kernel can run
// on every device -- fp32, vector width 4 or automatic, no row-block limit,
// local rows x cols with cols % 512 == 0 -- else -1.  (Operand alignment is
// checked again at launch; a group that fails it runs node by node.)
int GraphExecutor::groupable_act(NodeId nid) const {
  const Node& n = g_.node(nid);
  const auto* op = dynamic_cast<const BiasActOp*>(n.op.get());
  if (!op || n.inputs.size() != 2 || n.outputs.size() != 1 || view_rows_[nid]) return -1;
  const BiasActParams& p = op->params();
  if ((p.vector_width != 0 && p.vector_width != 4) || p.max_row_blocks != 0) return -1;
  const TensorId x = n.inputs[0];
  if (g_.tensor(x).dtype != DType::kF32 || g_.tensor(n.outputs[0]).dtype != DType::kF32) return -1;
  for (int d = 0; d < num_devices(); ++d) {
    const Shape& sh = tplan_[x].local_shape[d];
    if (sh.rank() != 2 || sh.rows() <= 0 || sh.cols() <= 0 || sh.cols() % 512 != 0) return -1;
  }
  return static_cast<int>(p.act);
}

// ------------------------------------------------------------- memory

Status GraphExecutor::plan_memory() {
  if (opts_.memory == MemoryPolicy::kReuseTopoNaive)
    return UnimplementedError("MemoryPolicy::kReuseTopoNaive is unsafe under parallel schedules and not offered");
  const bool reuse = opts_.memory != MemoryPolicy::kAllocPerTensor;
  const int D = num_devices();
  const int S = std::max(1, opts_.num_streams);
  const auto& order = g_.topo_order();
  const std::size_t T = g_.num_tensors();
  // Positions are launch items: the nodes of one item run at the same time.
  std::vector<std::int64_t> pos(g_.num_nodes(), 0);
  for (NodeId nid : order) pos[nid] = item_of_[nid];
  // Last use and the set of streams touching each tensor.
  std::vector<std::int64_t> last(T, -1);
  std::vector<bool> single_stream(T, true);
  std::vector<int> home(T, -1);
  for (TensorId t = 0; t < T; ++t) {
    const NodeId p = g_.producer(t);
    if (p != kInvalidNode) {
      home[t] = node_stream_[p];
      last[t] = pos[p];
    }
    for (NodeId c : g_.consumers(t)) {
      last[t] = std::max(last[t], pos[c]);
      if (home[t] >= 0 && node_stream_[c] != home[t]) single_stream[t] = false;
    }
  }
  arena_bytes_.assign(D, 0);
  scratch_offset_.assign(D, std::vector<std::int64_t>(S, 0));
  scratch_bytes_.assign(S, 0);
  exchange_offset_.assign(D, std::vector<std::int64_t>(g_.num_nodes(), -1));
  // Scratch per stream: the largest workspace any node on it needs (any device).
  for (NodeId nid : order) {
    const Node& n = g_.node(nid);
    for (int d = 0; d < D; ++d) {
      std::vector<TensorDesc> in;
      for (TensorId t : n.inputs) {
        TensorDesc desc = g_.tensor(t);
        desc.shape = tplan_[t].local_shape[d];
        in.push_back(desc);
      }
      scratch_bytes_[node_stream_[nid]] = std::max(scratch_bytes_[node_stream_[nid]], n.op->workspace_bytes(in));
    }
  }
  for (int d = 0; d < D; ++d) {
    std::size_t bump = 0;
    struct Block {
      std::size_t off, size;
      int stream;
      bool free;
    };
    std::vector<Block> blocks;
    std::vector<int> block_of(T, -1);
    auto fresh = [&](std::size_t bytes) {
      const std::size_t off = bump;
      bump += align_up(std::max<std::size_t>(bytes, 1));
      return off;
    };
    for (TensorId t = 0; t < T; ++t)  // inputs and outputs own their bytes
      if (g_.is_input(t) || g_.is_output(t)) tplan_[t].offset[d] = static_cast<std::int64_t>(fresh(tplan_[t].local_bytes(d)));
    for (std::size_t i = 0; i < items_.size(); ++i) {
     // every output of the item first, then the frees: no node of an item
     // may take a block another node of the same item still reads
     for (NodeId nid : items_[i]) {
      const Node& n = g_.node(nid);
      const int s = node_stream_[n.id];
      for (TensorId o : n.outputs) {
        if (tplan_[o].offset[d] >= 0) continue;
        const std::size_t need = align_up(std::max<std::size_t>(tplan_[o].local_bytes(d), 1));
        int best = -1;
        if (reuse && single_stream[o])
          for (std::size_t b = 0; b < blocks.size(); ++b)
            if (blocks[b].free && blocks[b].stream == s && blocks[b].size >= need &&
                (best < 0 || blocks[b].size < blocks[best].size))
              best = static_cast<int>(b);
        if (best < 0) {
          blocks.push_back({fresh(need), need, single_stream[o] ? s : -1, false});
          best = static_cast<int>(blocks.size()) - 1;
        }
        blocks[best].free = false;
        block_of[o] = best;
        tplan_[o].offset[d] = static_cast<std::int64_t>(blocks[best].off);
      }
     }
     for (NodeId nid : items_[i]) {
      const Node& n = g_.node(nid);
      // Free intermediates whose last use was this item (same-stream blocks only).
      for (TensorId t : n.inputs)
        if (block_of[t] >= 0 && last[t] == static_cast<std::int64_t>(i) && blocks[block_of[t]].stream >= 0)
          blocks[block_of[t]].free = true;
      for (TensorId o : n.outputs)
        if (block_of[o] >= 0 && last[o] == static_cast<std::int64_t>(i) && blocks[block_of[o]].stream >= 0)
          blocks[block_of[o]].free = true;
     }
    }
    // Exchange buffers: own partial + all devices' partials, per exchanging node.
    for (NodeId nid : order) {
      const std::size_t eb = g_.node(nid).op->exchange_bytes();
      if (eb == 0) continue;
      exchange_offset_[d][nid] = static_cast<std::int64_t>(fresh(eb * static_cast<std::size_t>(D + 1)));
    }
    for (int s = 0; s < S; ++s) scratch_offset_[d][s] = static_cast<std::int64_t>(fresh(scratch_bytes_[s]));
    arena_bytes_[d] = bump;
  }
  return OkStatus();
}

Status GraphExecutor::plan_dry() {
  if (!g_.finalized()) MCKE_RETURN_IF_ERROR(g_.finalize());
  MCKE_RETURN_IF_ERROR(place());
  MCKE_RETURN_IF_ERROR(assign_streams());
  MCKE_RETURN_IF_ERROR(plan_memory());
  return OkStatus();
}

Status GraphExecutor::plan() {
  MCKE_RETURN_IF_ERROR(plan_dry());
  impl_ = std::make_unique<Impl>();
  const int D = num_devices();
  const int S = std::max(1, opts_.num_streams);
  impl_->devs.resize(D);
  bool any_exchange = false;
  for (NodeId nid : g_.topo_order()) any_exchange |= g_.node(nid).op->exchange_bytes() > 0;
  if (opts_.poison_buffers) {
    const std::uint32_t p = opts_.poison_pattern;
    if (((p >> 8) & 0xFFu) != (p & 0xFFu) || ((p >> 16) & 0xFFu) != (p & 0xFFu) || (p >> 24) != (p & 0xFFu))
      return InvalidArgumentError("poison_pattern must repeat one byte (e.g. 0x7F7F7F7F)");
  }
  if (!opts_.allocators.empty() && static_cast<int>(opts_.allocators.size()) != D)
    return InvalidArgumentError("ExecutorOptions.allocators: one per device entry (" + std::to_string(D) +
                                "), got " + std::to_string(opts_.allocators.size()));
  for (int d = 0; d < D; ++d) {
    auto& dv = impl_->devs[d];
    dv.device = opts_.devices[d];
    rt::DeviceGuard guard(dv.device);
    for (int s = 0; s < S; ++s) {
      auto st = rt::Stream::create(dv.device);
      MCKE_RETURN_IF_ERROR(st.status());
      dv.streams.push_back(std::move(*st));
      auto ev = rt::Event::create(dv.device);
      MCKE_RETURN_IF_ERROR(ev.status());
      dv.done.push_back(std::move(*ev));
    }
    const std::size_t bytes = std::max<std::size_t>(arena_bytes_[d], kAlign);
    dv.alloc = opts_.allocators.empty() ? nullptr : opts_.allocators[d];
    if (dv.alloc) {
      auto a = dv.alloc->allocate(bytes, dv.streams[0].native());
      if (!a.ok())
        return Status(a.status().code(), "arena of " + std::to_string(bytes) + " bytes on device " +
                                             std::to_string(dv.device) + " from " + std::string(dv.alloc->name()) +
                                             ": " + a.status().message());
      if (reinterpret_cast<std::uintptr_t>(a->ptr) % kAlign != 0)
        return InternalError(std::string(dv.alloc->name()) + " returned a block not aligned to 256 bytes");
      dv.arena_block = *a;
      dv.arena = a->ptr;
    } else {
      const cudaError_t e = cudaMalloc(&dv.arena, bytes);
      if (e != cudaSuccess)
        return OutOfMemoryError("arena of " + std::to_string(arena_bytes_[d]) + " bytes on device " +
                                std::to_string(dv.device) + ": " + cudaGetErrorString(e));
    }
    if (opts_.use_graph) {
      auto f = rt::Event::create(dv.device);
      MCKE_RETURN_IF_ERROR(f.status());
      dv.fork = std::move(*f);
      auto j = rt::Event::create(dv.device);
      MCKE_RETURN_IF_ERROR(j.status());
      dv.join = std::move(*j);
    }
    auto t0 = rt::Event::create(dv.device, rt::Event::Kind::kTiming);
    MCKE_RETURN_IF_ERROR(t0.status());
    dv.t_start = std::move(*t0);
    auto t1 = rt::Event::create(dv.device, rt::Event::Kind::kTiming);
    MCKE_RETURN_IF_ERROR(t1.status());
    dv.t_end = std::move(*t1);
    dv.node_events.resize(g_.num_nodes());
    for (NodeId nid = 0; nid < g_.num_nodes(); ++nid)
      if (record_after_[nid]) {
        auto ev = rt::Event::create(dv.device);
        MCKE_RETURN_IF_ERROR(ev.status());
        dv.node_events[nid] = std::move(*ev);
      }
  }
  // NCCL needs distinct devices; a device list that repeats a GPU (several
  // shards on one GPU) exchanges partials with device-to-device copies ordered
  // by events instead.
  std::vector<int> sorted = opts_.devices;
  std::sort(sorted.begin(), sorted.end());
  impl_->peer_copy = std::adjacent_find(sorted.begin(), sorted.end()) != sorted.end();
  if (any_exchange && D > 1) {
    for (auto& dv : impl_->devs) {
      dv.exchange_ready.resize(g_.num_nodes());
      dv.exchange_done.resize(g_.num_nodes());
      for (NodeId nid = 0; nid < g_.num_nodes(); ++nid)
        if (g_.node(nid).op->exchange_bytes() > 0) {
          auto ev = rt::Event::create(dv.device);
          MCKE_RETURN_IF_ERROR(ev.status());
          dv.exchange_ready[nid] = std::move(*ev);
          auto ev2 = rt::Event::create(dv.device);
          MCKE_RETURN_IF_ERROR(ev2.status());
          dv.exchange_done[nid] = std::move(*ev2);
        }
    }
  }
  if (any_exchange && D > 1 && !impl_->peer_copy && opts_.p2p_exchange) {
    bool can = true;
    for (int a = 0; a < D && can; ++a)
      for (int b = 0; b < D && can; ++b) {
        int ok = 0;
        if (a != b && (cudaDeviceCanAccessPeer(&ok, opts_.devices[a], opts_.devices[b]) != cudaSuccess || !ok)) can = false;
      }
    cudaGetLastError();
    if (can) {
      for (int a = 0; a < D; ++a) {
        rt::DeviceGuard g(opts_.devices[a]);
        for (int b = 0; b < D; ++b) {
          if (a == b) continue;
          const cudaError_t e = cudaDeviceEnablePeerAccess(opts_.devices[b], 0);
          if (e != cudaSuccess && e != cudaErrorPeerAccessAlreadyEnabled)
            return InternalError(std::string("cudaDeviceEnablePeerAccess: ") + cudaGetErrorString(e));
          cudaGetLastError();
        }
      }
      const std::size_t bytes = kernels::reduce_p2p_buffer_bytes(D);
      impl_->p2p_buf.assign(g_.num_nodes(), std::vector<void*>(D, nullptr));
      impl_->p2p_table.assign(g_.num_nodes(), std::vector<void*>(D, nullptr));
      for (NodeId nid = 0; nid < g_.num_nodes(); ++nid) {
        if (g_.node(nid).op->exchange_bytes() == 0) continue;
        for (int d = 0; d < D; ++d) {
          rt::DeviceGuard g(opts_.devices[d]);
          MCKE_CUDA_RETURN_IF_ERROR(cudaMalloc(&impl_->p2p_buf[nid][d], bytes));
          MCKE_CUDA_RETURN_IF_ERROR(cudaMemset(impl_->p2p_buf[nid][d], 0, bytes));
        }
        for (int d = 0; d < D; ++d) {
          rt::DeviceGuard g(opts_.devices[d]);
          MCKE_CUDA_RETURN_IF_ERROR(cudaMalloc(&impl_->p2p_table[nid][d], D * sizeof(void*)));
          MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpy(impl_->p2p_table[nid][d], impl_->p2p_buf[nid].data(), D * sizeof(void*),
                                               cudaMemcpyHostToDevice));
        }
      }
      impl_->p2p = true;
    }
  }
  if (any_exchange && D > 1 && !impl_->peer_copy && !impl_->p2p) {
    std::vector<ncclComm_t> comms(D);
    MCKE_RETURN_IF_ERROR(nccl_status(ncclCommInitAll(comms.data(), D, opts_.devices.data()), "ncclCommInitAll"));
    for (int d = 0; d < D; ++d) impl_->devs[d].comm = comms[d];
  }
  MCKE_RETURN_IF_ERROR(build_launches());
  planned_ = true;
  return OkStatus();
}

// Every node's per-device OpContext and input/output tensors, once: the
// pointers are fixed by the memory plan and the arenas.
Status GraphExecutor::build_launches() {
  const int D = num_devices();
  impl_->launches.assign(g_.num_nodes(), {});
  for (NodeId nid : g_.topo_order()) {
    const Node& n = g_.node(nid);
    const int s = node_stream_[nid];
    auto& L = impl_->launches[nid];
    L.ctx.resize(D);
    L.ins.resize(D);
    L.outs.resize(D);
    L.gathered.assign(D, nullptr);
    for (int d = 0; d < D; ++d) {
      auto& dv = impl_->devs[d];
      OpContext& c = L.ctx[d];
      c.stream = dv.streams[s].native();
      c.device = dv.device;
      c.workspace = scratch_bytes_[s] ? static_cast<char*>(dv.arena) + scratch_offset_[d][s] : nullptr;
      c.workspace_bytes = scratch_bytes_[s];
      c.shard = d;
      c.num_shards = D;
      for (TensorId t : n.inputs) {
        Tensor x = local_tensor(t, d);
        // A replicated intermediate consumed row-wise: view this device's rows.
        if (view_rows_[nid] && t == n.inputs[0]) {
          const Shape& full = g_.tensor(t).shape;
          const std::int64_t E = full.rank() >= 2 ? full.rows() : full.numel();
          const std::int64_t inner = full.rank() >= 2 ? full.cols() : 1;
          const std::int64_t b = E * d / D, e = E * (d + 1) / D;
          x.data = static_cast<char*>(x.data) + b * inner * static_cast<std::int64_t>(dtype_size(x.dtype));
          x.shape = full.rank() >= 2 ? Shape{e - b, inner} : Shape{e - b};
        }
        L.ins[d].push_back(x);
      }
      for (TensorId t : n.outputs) L.outs[d].push_back(local_tensor(t, d));
      // Range shards of a full reduce: global index of this device's first element.
      if (!n.inputs.empty()) {
        const TensorPlan& tp = tplan_[n.inputs[0]];
        const Shape& full = g_.tensor(n.inputs[0]).shape;
        const std::int64_t inner = full.rank() >= 2 ? full.cols() : 1;
        if (tp.placement == Placement::kRowSplit || view_rows_[nid])
          c.index_base = (full.rank() >= 2 ? full.rows() : full.numel()) * d / D * inner;
      }
      if (exchange_offset_[d][nid] >= 0) c.exchange = static_cast<char*>(dv.arena) + exchange_offset_[d][nid];
      if (impl_->p2p && !impl_->p2p_table.empty() && impl_->p2p_table[nid][d])
        c.p2p_peers = static_cast<void* const*>(impl_->p2p_table[nid][d]);
    }
    const std::size_t eb = n.op->exchange_bytes();
    if (eb > 0)
      for (int d = 0; d < D; ++d)
        L.gathered[d] = D > 1 ? static_cast<char*>(L.ctx[d].exchange) + eb : L.ctx[d].exchange;
  }
  return OkStatus();
}

Tensor GraphExecutor::local_tensor(TensorId t, int d) const {
  const TensorPlan& tp = tplan_[t];
  Tensor x;
  x.dtype = tp.dtype;
  x.device = opts_.devices[d];
  x.shape = tp.local_shape[d];
  x.data = impl_ ? static_cast<char*>(impl_->devs[d].arena) + tp.offset[d] : nullptr;
  return x;
}

Status GraphExecutor::run_async() {
  if (!planned_) return FailedPreconditionError("run_async: plan() has not succeeded");
  if (!opts_.use_graph) {
    MCKE_RETURN_IF_ERROR(enqueue(false));
    impl_->ran_once = true;
    return OkStatus();
  }
  if (impl_->execs.empty()) MCKE_RETURN_IF_ERROR(capture());
  // Stream order on each origin stream serialises replays, so a replay never
  // overwrites a block that the previous one is still reading.
  for (std::size_t i = 0; i < impl_->execs.size(); ++i) {
    auto& dv = impl_->devs[impl_->origins[i]];
    rt::DeviceGuard g(dv.device);
    MCKE_RETURN_IF_ERROR(dv.t_start.record(dv.streams[0]));
    MCKE_CUDA_RETURN_IF_ERROR(cudaGraphLaunch(impl_->execs[i], dv.streams[0].native()));
    MCKE_RETURN_IF_ERROR(dv.t_end.record(dv.streams[0]));
  }
  impl_->ran_once = true;
  return OkStatus();
}

Status GraphExecutor::capture() {
  const int D = num_devices();
  const int S = std::max(1, opts_.num_streams);
  std::vector<std::vector<int>> groups;
  if (D > 1 && impl_->peer_copy) {
    // Repeated GPUs exchange with event-ordered copies between the entries:
    // that only captures when every entry is on one GPU (one capture).
    for (int d = 1; d < D; ++d)
      if (impl_->devs[d].device != impl_->devs[0].device)
        return InvalidArgumentError("use_graph: the device list must be distinct GPUs or one GPU repeated");
    groups.emplace_back();
    for (int d = 0; d < D; ++d) groups[0].push_back(d);
  } else {
    for (int d = 0; d < D; ++d) groups.push_back({d});
  }
  // Every group's capture is open before any node is enqueued: the NCCL
  // exchange of a sharded reduce is one group call over all GPUs.
  std::vector<int> begun;
  auto abort_captures = [&](Status st) {
    for (int gi : begun) {
      auto& o = impl_->devs[groups[gi][0]];
      rt::DeviceGuard g(o.device);
      cudaGraph_t partial = nullptr;
      cudaStreamEndCapture(o.streams[0].native(), &partial);
      if (partial) cudaGraphDestroy(partial);
    }
    cudaGetLastError();
    return st;
  };
  for (std::size_t gi = 0; gi < groups.size(); ++gi) {
    auto& o = impl_->devs[groups[gi][0]];
    rt::DeviceGuard g(o.device);
    cudaError_t e = cudaStreamBeginCapture(o.streams[0].native(), cudaStreamCaptureModeRelaxed);
    if (e != cudaSuccess) return abort_captures(InternalError(std::string("cudaStreamBeginCapture: ") + cudaGetErrorString(e)));
    begun.push_back(static_cast<int>(gi));
    Status st = o.fork.record(o.streams[0]);
    for (int d : groups[gi])
      for (int s = 0; s < S && st.ok(); ++s)
        if (d != groups[gi][0] || s != 0) st = impl_->devs[d].streams[s].wait(o.fork);
    if (!st.ok()) return abort_captures(st);
  }
  Status st = enqueue(true);
  if (!st.ok()) return abort_captures(st);
  for (auto& grp : groups) {
    auto& o = impl_->devs[grp[0]];
    for (std::size_t k = 1; k < grp.size() && st.ok(); ++k) {
      auto& dv = impl_->devs[grp[k]];
      st = dv.join.record(dv.streams[0]);
      if (st.ok()) st = o.streams[0].wait(dv.join);
    }
    if (!st.ok()) return abort_captures(st);
  }
  std::vector<cudaGraph_t> graphs;
  for (int gi : begun) {
    auto& o = impl_->devs[groups[gi][0]];
    rt::DeviceGuard g(o.device);
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(o.streams[0].native(), &graph);
    if (e != cudaSuccess || !graph) {
      st = InternalError(std::string("cudaStreamEndCapture: ") + cudaGetErrorString(e));
      break;
    }
    graphs.push_back(graph);
  }
  if (st.ok()) {
    for (std::size_t gi = 0; gi < graphs.size(); ++gi) {
      rt::DeviceGuard g(impl_->devs[groups[gi][0]].device);
      cudaGraphExec_t exec = nullptr;
      const cudaError_t e = cudaGraphInstantiate(&exec, graphs[gi], 0);
      if (e != cudaSuccess) {
        st = InternalError(std::string("cudaGraphInstantiate: ") + cudaGetErrorString(e));
        break;
      }
      impl_->execs.push_back(exec);
      impl_->origins.push_back(groups[gi][0]);
    }
  }
  for (std::size_t gi = 0; gi < graphs.size(); ++gi) {
    rt::DeviceGuard g(impl_->devs[groups[gi][0]].device);
    cudaGraphDestroy(graphs[gi]);
  }
  if (!st.ok()) {
    for (std::size_t i = 0; i < impl_->execs.size(); ++i) {
      rt::DeviceGuard g(impl_->devs[impl_->origins[i]].device);
      cudaGraphExecDestroy(impl_->execs[i]);
    }
    impl_->execs.clear();
    impl_->origins.clear();
    cudaGetLastError();
  }
  return st;
}

Status GraphExecutor::enqueue(bool /*capturing*/) {
  const int D = num_devices();
  const int S = std::max(1, opts_.num_streams);
  // Each run starts after every stream of the previous run finished (join),
  // so a reused block is never overwritten while a reader is still running.
  // (A captured run needs no such wait: graph launches on one stream are
  // ordered.)
  // (The previous run ended with stream 0 waiting for every other stream, so
  // t_start, recorded on stream 0 and waited on by the others, already orders
  // this run after all of it.)
  for (auto& dv : impl_->devs) {
    MCKE_RETURN_IF_ERROR(dv.t_start.record(dv.streams[0]));
    for (int s = 1; s < S; ++s) MCKE_RETURN_IF_ERROR(dv.streams[s].wait(dv.t_start));
    if (opts_.poison_buffers) {
      rt::DeviceGuard g(dv.device);
      const int d = static_cast<int>(&dv - impl_->devs.data());
      for (TensorId t = 0; t < g_.num_tensors(); ++t)
        if (!g_.is_input(t))
          MCKE_CUDA_RETURN_IF_ERROR(cudaMemsetAsync(static_cast<char*>(dv.arena) + tplan_[t].offset[d],
                                                    static_cast<int>(opts_.poison_pattern & 0xFFu),
                                                    tplan_[t].local_bytes(d), dv.streams[0].native()));
      MCKE_RETURN_IF_ERROR(dv.done[0].record(dv.streams[0]));
      for (int s = 1; s < S; ++s) MCKE_RETURN_IF_ERROR(dv.streams[s].wait(dv.done[0]));
    }
  }
  // One device's launch of one node.
  auto launch_one = [&](NodeId nid, int d) -> Status {
    Node& n = g_.node(nid);
    const auto& L = impl_->launches[nid];
    rt::DeviceGuard g(impl_->devs[d].device);
    const Status st = n.op->launch(L.ctx[d], L.ins[d], L.outs[d]);
    if (!st.ok())
      return Status(st.code(), "node '" + n.name + "' on device " + std::to_string(L.ctx[d].device) + ": " + st.message());
    return OkStatus();
  };
  for (const std::vector<NodeId>& item : items_) {
    const NodeId nid = item[0];
    Node& n = g_.node(nid);
    const int s = node_stream_[nid];
    auto& L = impl_->launches[nid];
    const std::vector<OpContext>& ctx = L.ctx;
    const auto& outs = L.outs;
    for (NodeId m : item)
      for (int d = 0; d < D; ++d)
        for (int p : waits_[m]) MCKE_RETURN_IF_ERROR(impl_->devs[d].streams[s].wait(impl_->devs[d].node_events[p]));
    if (item.size() > 1) {
      // A grouped item (kLevelGrouped): the bias + activation nodes of one
      // level, one launch per device; node by node if an operand turns out
      // misaligned (the plan already treats the nodes as concurrent, so
      // running them in turn is safe too).
      const auto act = static_cast<const BiasActOp*>(n.op.get())->params().act;
      const kernels::Activation ka = act == BiasActParams::Act::kRelu      ? kernels::Activation::kRelu
                                     : act == BiasActParams::Act::kGeluErf  ? kernels::Activation::kGeluErf
                                     : act == BiasActParams::Act::kGeluTanh ? kernels::Activation::kGeluTanh
                                                                             : kernels::Activation::kNone;
      for (int d = 0; d < D; ++d) {
        kernels::BiasActJob jobs[kernels::kBiasActGroupMax];
        bool grouped = item.size() <= static_cast<std::size_t>(kernels::kBiasActGroupMax);
        for (std::size_t k = 0; grouped && k < item.size(); ++k) {
          const auto& Lk = impl_->launches[item[k]];
          const Tensor& x = Lk.ins[d][0];
          jobs[k] = {x.data_as<float>(), Lk.ins[d][1].data_as<float>(), Lk.outs[d][0].data_as<float>(),
                     x.shape.rows(), x.shape.cols()};
          grouped = jobs[k].x && jobs[k].bias && jobs[k].y &&
                    kernels::bias_act_groupable(jobs[k].x, jobs[k].bias, jobs[k].y, jobs[k].cols);
        }
        if (grouped) {
          rt::DeviceGuard g(impl_->devs[d].device);
          const Status st = kernels::launch_bias_act_f32_group(jobs, static_cast<int>(item.size()), ka, ctx[d].stream);
          if (!st.ok())
            return Status(st.code(), "group of " + std::to_string(item.size()) + " nodes from '" + n.name +
                                         "' on device " + std::to_string(ctx[d].device) + ": " + st.message());
        } else {
          for (NodeId m : item) MCKE_RETURN_IF_ERROR(launch_one(m, d));
        }
      }
      for (NodeId m : item)
        if (record_after_[m])
          for (auto& dv : impl_->devs) MCKE_RETURN_IF_ERROR(dv.node_events[m].record(dv.streams[s]));
      continue;
    }
    for (int d = 0; d < D; ++d) MCKE_RETURN_IF_ERROR(launch_one(nid, d));
    const std::size_t eb = n.op->exchange_bytes();
    if (eb > 0 && !(impl_->p2p && D > 1)) {
      const std::vector<void*>& gathered = L.gathered;
      if (D > 1 && impl_->peer_copy) {
        // Every shard's partial lands in every device's gathered buffer, in
        // shard order; each copy waits on the event recorded after the partial.
        for (int d = 0; d < D; ++d)
          MCKE_RETURN_IF_ERROR(impl_->devs[d].exchange_ready[nid].record(impl_->devs[d].streams[s]));
        for (int e = 0; e < D; ++e) {
          auto& de = impl_->devs[e];
          for (int d = 0; d < D; ++d) {
            MCKE_RETURN_IF_ERROR(de.streams[s].wait(impl_->devs[d].exchange_ready[nid]));
            rt::DeviceGuard g(de.device);
            char* dst = static_cast<char*>(gathered[e]) + d * eb;
            if (de.device == impl_->devs[d].device)  // (the form a stream capture accepts)
              MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpyAsync(dst, ctx[d].exchange, eb, cudaMemcpyDeviceToDevice,
                                                        de.streams[s].native()));
            else
              MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpyPeerAsync(dst, de.device, ctx[d].exchange, impl_->devs[d].device,
                                                            eb, de.streams[s].native()));
          }
        }
        // No shard may overwrite its partial (next run) before every peer has
        // copied it: each device's stream waits for all devices' copies.
        for (int e = 0; e < D; ++e)
          MCKE_RETURN_IF_ERROR(impl_->devs[e].exchange_done[nid].record(impl_->devs[e].streams[s]));
        for (int d = 0; d < D; ++d)
          for (int e = 0; e < D; ++e)
            if (e != d) MCKE_RETURN_IF_ERROR(impl_->devs[d].streams[s].wait(impl_->devs[e].exchange_done[nid]));
      } else if (D > 1) {
        MCKE_RETURN_IF_ERROR(nccl_status(ncclGroupStart(), "ncclGroupStart"));
        for (int d = 0; d < D; ++d) {
          rt::DeviceGuard g(impl_->devs[d].device);
          MCKE_RETURN_IF_ERROR(nccl_status(ncclAllGather(ctx[d].exchange, gathered[d], eb, ncclUint8,
                                                         impl_->devs[d].comm, ctx[d].stream),
                                           "ncclAllGather"));
        }
        MCKE_RETURN_IF_ERROR(nccl_status(ncclGroupEnd(), "ncclGroupEnd"));
      }
      for (int d = 0; d < D; ++d) {
        rt::DeviceGuard g(impl_->devs[d].device);
        MCKE_RETURN_IF_ERROR(n.op->finish(ctx[d], gathered[d], outs[d]));
      }
    }
    if (record_after_[nid])
      for (auto& dv : impl_->devs) MCKE_RETURN_IF_ERROR(dv.node_events[nid].record(dv.streams[s]));
  }
  for (auto& dv : impl_->devs) {
    for (int s = 0; s < S; ++s) MCKE_RETURN_IF_ERROR(dv.done[s].record(dv.streams[s]));
    for (int s = 1; s < S; ++s) MCKE_RETURN_IF_ERROR(dv.streams[0].wait(dv.done[s]));
    MCKE_RETURN_IF_ERROR(dv.t_end.record(dv.streams[0]));
  }
  return OkStatus();
}

StatusOr<float> GraphExecutor::last_run_ms() {
  if (!impl_ || !impl_->ran_once) return FailedPreconditionError("last_run_ms: nothing has run");
  float worst = 0.f;
  for (std::size_t d = 0; d < impl_->devs.size(); ++d) {
    // In graph mode only the origins record timing events outside a capture.
    if (opts_.use_graph &&
        std::find(impl_->origins.begin(), impl_->origins.end(), static_cast<int>(d)) == impl_->origins.end())
      continue;
    auto& dv = impl_->devs[d];
    MCKE_RETURN_IF_ERROR(dv.t_end.synchronize());
    auto ms = rt::Event::elapsed_ms(dv.t_start, dv.t_end);
    MCKE_RETURN_IF_ERROR(ms.status());
    worst = std::max(worst, *ms);
  }
  return worst;
}

Status GraphExecutor::synchronize() {
  if (!impl_) return FailedPreconditionError("synchronize: not planned");
  for (auto& dv : impl_->devs)
    for (auto& s : dv.streams) MCKE_RETURN_IF_ERROR(s.synchronize());
  return OkStatus();
}

Status GraphExecutor::set_input(TensorId t, const void* host, std::size_t bytes) {
  if (!planned_) return FailedPreconditionError("set_input: plan() has not succeeded");
  if (!g_.is_input(t)) return InvalidArgumentError("set_input: tensor is not a graph input");
  const TensorDesc& desc = g_.tensor(t);
  const std::size_t es = dtype_size(desc.dtype);
  if (bytes != static_cast<std::size_t>(desc.shape.numel()) * es)
    return InvalidArgumentError("set_input: expected " + std::to_string(desc.shape.numel() * es) + " bytes");
  if (opts_.validate_numerics) {
    const char* h = static_cast<const char*>(host);
    auto it = std::find_if(input_cache_.begin(), input_cache_.end(), [&](const auto& e) { return e.first == t; });
    if (it == input_cache_.end()) input_cache_.push_back({t, std::vector<char>(h, h + bytes)});
    else it->second.assign(h, h + bytes);
  }
  const TensorPlan& tp = tplan_[t];
  for (int d = 0; d < num_devices(); ++d) {
    rt::DeviceGuard g(impl_->devs[d].device);
    char* dst = static_cast<char*>(impl_->devs[d].arena) + tp.offset[d];
    const char* src = static_cast<const char*>(host);
    if (tp.placement == Placement::kReplicated) {
      MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
    } else if (tp.placement == Placement::kRowSplit) {
      const std::int64_t inner = desc.shape.rank() >= 2 ? desc.shape.cols() : 1;
      MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpy(dst, src + tp.row_begin[d] * inner * es, tp.local_bytes(d),
                                           cudaMemcpyHostToDevice));
    } else {
      const std::int64_t R = desc.shape.rank() == 1 ? 1 : desc.shape.rows();
      const std::int64_t C = desc.shape.cols();
      const std::int64_t w = tp.local_shape[d].cols();
      MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpy2D(dst, w * es, src + tp.row_begin[d] * es, C * es, w * es, R,
                                             cudaMemcpyHostToDevice));
    }
  }
  return OkStatus();
}

Status GraphExecutor::copy_output_to_host(TensorId t, void* host, std::size_t bytes) {
  if (!planned_) return FailedPreconditionError("copy_output_to_host: plan() has not succeeded");
  const TensorDesc& desc = g_.tensor(t);
  const std::size_t es = dtype_size(desc.dtype);
  if (bytes != static_cast<std::size_t>(desc.shape.numel()) * es)
    return InvalidArgumentError("copy_output_to_host: expected " + std::to_string(desc.shape.numel() * es) + " bytes");
  MCKE_RETURN_IF_ERROR(synchronize());
  const TensorPlan& tp = tplan_[t];
  char* dst = static_cast<char*>(host);
  const int D = tp.placement == Placement::kReplicated ? 1 : num_devices();
  for (int d = 0; d < D; ++d) {
    rt::DeviceGuard g(impl_->devs[d].device);
    const char* src = static_cast<const char*>(impl_->devs[d].arena) + tp.offset[d];
    if (tp.placement == Placement::kReplicated) {
      MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    } else if (tp.placement == Placement::kRowSplit) {
      const std::int64_t inner = desc.shape.rank() >= 2 ? desc.shape.cols() : 1;
      MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpy(dst + tp.row_begin[d] * inner * es, src, tp.local_bytes(d),
                                           cudaMemcpyDeviceToHost));
    } else {
      const std::int64_t R = desc.shape.rank() == 1 ? 1 : desc.shape.rows();
      const std::int64_t C = desc.shape.cols();
      const std::int64_t w = tp.local_shape[d].cols();
      MCKE_CUDA_RETURN_IF_ERROR(cudaMemcpy2D(dst + tp.row_begin[d] * es, C * es, src, w * es, w * es, R,
                                             cudaMemcpyDeviceToHost));
    }
  }
  return OkStatus();
}

// ------------------------------------------------------------- numerics gate

namespace {
const char* schedule_name(SchedulePolicy p) {
  switch (p) {
    case SchedulePolicy::kSequential: return "sequential";
    case SchedulePolicy::kLevelParallel: return "level-parallel";
    case SchedulePolicy::kChainGreedy: return "chain-greedy";
    case SchedulePolicy::kLevelGrouped: return "level-grouped";
  }
  return "?";
}
const char* memory_name(MemoryPolicy p) {
  switch (p) {
    case MemoryPolicy::kAllocPerTensor: return "alloc-per-tensor";
    case MemoryPolicy::kReuseTopoNaive: return "reuse-topo-naive";
    case MemoryPolicy::kReuseSameStream: return "reuse-same-stream";
    case MemoryPolicy::kReuseHappensBefore: return "reuse-happens-before";
  }
  return "?";
}
std::string hex32(const std::vector<char>& v, std::size_t word) {
  std::uint32_t u = 0;
  std::memcpy(&u, v.data() + word * 4, std::min<std::size_t>(4, v.size() - word * 4));
  char buf[16];
  std::snprintf(buf, sizeof(buf), "0x%08x", u);
  return buf;
}
}  // namespace

StatusOr<NumericsResult> GraphExecutor::validate_numerics(int repeats) {
  if (!opts_.validate_numerics)
    return FailedPreconditionError("validate_numerics: needs ExecutorOptions::validate_numerics (set_input keeps "
                                   "host copies of the inputs only then)");
  if (repeats < 1) repeats = 1;
  for (TensorId t = 0; t < g_.num_tensors(); ++t)
    if (g_.is_input(t) && std::none_of(input_cache_.begin(), input_cache_.end(), [&](const auto& e) { return e.first == t; }))
      return FailedPreconditionError("validate_numerics: input '" + g_.tensor(t).name + "' was never set");
  struct Config {
    SchedulePolicy schedule;
    MemoryPolicy memory;
    bool graph;
  };
  std::vector<Config> configs{{SchedulePolicy::kSequential, MemoryPolicy::kAllocPerTensor, false}};  // golden
  for (SchedulePolicy sp : {SchedulePolicy::kSequential, SchedulePolicy::kLevelParallel, SchedulePolicy::kChainGreedy,
                            SchedulePolicy::kLevelGrouped})
    for (MemoryPolicy mp : {MemoryPolicy::kAllocPerTensor, MemoryPolicy::kReuseSameStream, MemoryPolicy::kReuseHappensBefore})
      for (bool gr : {false, true})
        if (sp != SchedulePolicy::kSequential || mp != MemoryPolicy::kAllocPerTensor || gr)
          configs.push_back({sp, mp, gr});
  NumericsResult res;
  res.repeats = repeats;
  const auto& outs = g_.outputs();
  std::vector<std::vector<char>> golden;
  for (std::size_t ci = 0; ci < configs.size(); ++ci) {
    const Config& c = configs[ci];
    const std::string cname = std::string(schedule_name(c.schedule)) + "/" + memory_name(c.memory) + "/" +
                              (c.graph ? "graph" : "eager");
    ExecutorOptions o = opts_;
    o.schedule = c.schedule;
    o.memory = c.memory;
    o.use_graph = c.graph;
    o.validate_numerics = false;
    GraphExecutor ex(g_, o);
    const Status ps = ex.plan();
    if (!ps.ok()) return Status(ps.code(), "validate_numerics [" + cname + "] plan: " + ps.message());
    for (const auto& [t, bytes] : input_cache_) MCKE_RETURN_IF_ERROR(ex.set_input(t, bytes.data(), bytes.size()));
    std::vector<std::vector<char>> first;
    for (int r = 0; r < repeats; ++r) {
      MCKE_RETURN_IF_ERROR(ex.run_async());
      MCKE_RETURN_IF_ERROR(ex.synchronize());
      for (std::size_t oi = 0; oi < outs.size(); ++oi) {
        const TensorDesc& d = g_.tensor(outs[oi]);
        std::vector<char> buf(static_cast<std::size_t>(d.shape.numel()) * dtype_size(d.dtype));
        MCKE_RETURN_IF_ERROR(ex.copy_output_to_host(outs[oi], buf.data(), buf.size()));
        const std::vector<char>* want = nullptr;
        const char* against = nullptr;
        if (r == 0 && ci > 0) {
          want = &golden[oi];
          against = "the golden run (sequential/alloc-per-tensor/eager)";
        } else if (r > 0) {
          want = &first[oi];
          against = "its own first run";
        }
        if (want) {
          const std::size_t w = first_bit_mismatch(buf.data(), want->data(), buf.size());
          res.elements_compared += buf.size() / 4;
          if (w != buf.size()) {
            res.passed = false;
            res.configs_compared = static_cast<int>(ci);
            res.detail = "[" + cname + "] run " + std::to_string(r) + ", output '" + d.name + "', word " +
                         std::to_string(w) + ": " + hex32(buf, w) + " against " + hex32(*want, w) + " in " + against;
            return res;
          }
        }
        if (r == 0) first.push_back(std::move(buf));
      }
    }
    if (ci == 0) golden = first;
  }
  res.passed = true;
  res.configs_compared = static_cast<int>(configs.size());
  return res;
}

std::string GraphExecutor::describe() const {
  // Plain string building (no iostreams): this library is loaded next to other
  // C++ runtimes in one process, and the description must not depend on their
  // stream machinery.
  std::string s = "devices=" + std::to_string(num_devices()) +
                  " num_streams=" + std::to_string(opts_.num_streams) +
                  " cross_stream_events=" + std::to_string(event_edges_) + "\n";
  for (NodeId nid : g_.topo_order()) {
    const Node& n = g_.node(nid);
    s += "node " + n.name + " (" + std::string(n.op->type_name()) + ") stream=" + std::to_string(node_stream_[nid]) +
         " waits=[";
    for (std::size_t i = 0; i < waits_[nid].size(); ++i) s += (i ? "," : "") + g_.node(waits_[nid][i]).name;
    s += "]\n";
  }
  for (TensorId t = 0; t < g_.num_tensors(); ++t)
    s += "tensor " + g_.tensor(t).name + " " + g_.tensor(t).shape.to_string() + " " +
         placement_name(tplan_[t].placement) + " local0=" + tplan_[t].local_shape[0].to_string() +
         " offset0=" + std::to_string(tplan_[t].offset[0]) + "\n";
  for (int d = 0; d < num_devices(); ++d) s += "arena[" + std::to_string(d) + "]=" + std::to_string(arena_bytes_[d]) + "\n";
  return s;
}

}  // namespace mcke
