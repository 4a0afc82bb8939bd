// CPU fuzz of the executor's memory plan (the reference fuzzes its own plan for
// buffer races, tests/test_graph_host.cpp:1183-1391).  Random DAGs of bias+act
// and softmax nodes over one shape are planned dry under every schedule, both
// reuse policies and 1, 2 or 4 streams; then, for every two tensors whose
// bytes overlap in the arena, stream order must put one tensor's whole life
// (its producer and every reader) before the other's producer:
//   * both lives on one stream, and
//   * the earlier life's last step in an earlier launch item than the later
//     producer (the nodes of one grouped launch run at the same time, so the
//     same item does not count as before).
// Half the graphs have 512-column tensors, so the level-grouped schedule
// forms grouped launches; the run fails if none formed.
// Graph inputs and outputs must overlap nothing.  No GPU is touched.
// Prints "OK" and exits 0, or prints the first violation and exits 1.
#include <cstdint>
#include <cstdio>
#include <memory>
#include <random>
#include <string>
#include <utility>
#include <vector>

#include "mcke/graph/executor.hpp"

namespace {

using namespace mcke;

struct Built {
  Graph g;
  int nodes = 0;
};

// A random DAG: `n` nodes, each reading one earlier 2-D tensor (all one shape)
// through bias+act or softmax; every tensor nobody reads becomes an output.
void build(Built& b, std::mt19937& rng, int n) {
  const std::int64_t rows = 16 + static_cast<std::int64_t>(rng() % 8) * 16;
  const std::int64_t cols = rng() % 2 ? 512 * (1 + static_cast<std::int64_t>(rng() % 2))
                                      : 64 + static_cast<std::int64_t>(rng() % 4) * 64;
  TensorDesc xd;
  xd.shape = Shape{rows, cols};
  xd.name = "x";
  std::vector<TensorId> pool{b.g.add_input(xd)};
  if (rng() % 2) {
    xd.name = "x2";
    pool.push_back(b.g.add_input(xd));
  }
  for (int i = 0; i < n; ++i) {
    // prefer recent tensors, so chains form as well as fan-outs
    const std::size_t back = std::min<std::size_t>(pool.size(), 1 + rng() % 4);
    const TensorId src = pool[pool.size() - 1 - rng() % back];
    StatusOr<std::vector<TensorId>> out = InternalError("unset");
    if (rng() % 3) {
      TensorDesc bd;
      bd.shape = Shape{cols};
      bd.name = "b" + std::to_string(i);
      const TensorId bias = b.g.add_input(bd);
      BiasActParams p;
      p.act = BiasActParams::Act::kGeluTanh;
      out = b.g.add_node("bias" + std::to_string(i), std::make_unique<BiasActOp>(p), {src, bias});
    } else {
      out = b.g.add_node("softmax" + std::to_string(i), std::make_unique<SoftmaxOp>(SoftmaxParams{}), {src});
    }
    if (out.ok()) pool.push_back((*out)[0]);
  }
  b.nodes = static_cast<int>(b.g.num_nodes());
}

}  // namespace

namespace {

// 0 when every overlap is ordered; else prints the first violation.
int check(const Graph& g, const GraphExecutor& ex, const std::string& what, long* overlaps) {
  std::vector<int> pos(g.num_nodes());
  for (NodeId n = 0; n < static_cast<NodeId>(g.num_nodes()); ++n) pos[n] = ex.launch_item_of(n);
  auto life = [&](TensorId t) {
    std::vector<NodeId> l{g.producer(t)};
    for (NodeId c : g.consumers(t)) l.push_back(c);
    return l;
  };
  // every step of a's life before b's producer, on b's producer's stream
  auto before = [&](TensorId a, TensorId b) {
    const NodeId pb = g.producer(b);
    for (NodeId n : life(a))
      if (ex.stream_of(n) != ex.stream_of(pb) || pos[n] >= pos[pb]) return false;
    return true;
  };
  const TensorId T = static_cast<TensorId>(g.num_tensors());
  for (TensorId t1 = 0; t1 < T; ++t1) {
    for (TensorId t2 = t1 + 1; t2 < T; ++t2) {
      const TensorPlan& a = ex.tensor_plan(t1);
      const TensorPlan& b = ex.tensor_plan(t2);
      const std::int64_t ab = static_cast<std::int64_t>(a.local_bytes(0));
      const std::int64_t bb = static_cast<std::int64_t>(b.local_bytes(0));
      if (ab == 0 || bb == 0) continue;
      if (!(a.offset[0] < b.offset[0] + bb && b.offset[0] < a.offset[0] + ab)) continue;
      ++*overlaps;
      if (g.is_input(t1) || g.is_output(t1) || g.is_input(t2) || g.is_output(t2)) {
        std::printf("%s: graph input/output tensor %u shares bytes with %u\n", what.c_str(), t1, t2);
        return 1;
      }
      if (!before(t1, t2) && !before(t2, t1)) {
        std::printf("%s: tensors %u and %u share bytes without stream order\n", what.c_str(), t1, t2);
        return 1;
      }
    }
  }
  return 0;
}

}  // namespace

int main() {
  long overlaps = 0, plans = 0, grouped = 0;
  const SchedulePolicy schedules[] = {SchedulePolicy::kSequential, SchedulePolicy::kLevelParallel,
                                      SchedulePolicy::kChainGreedy, SchedulePolicy::kLevelGrouped};
  const MemoryPolicy memories[] = {MemoryPolicy::kReuseSameStream, MemoryPolicy::kReuseHappensBefore};
  for (unsigned seed = 0; seed < 150; ++seed) {
    std::mt19937 rng(seed);
    Built b;
    build(b, rng, 4 + static_cast<int>(rng() % 24));
    for (TensorId t = 0; t < static_cast<TensorId>(b.g.num_tensors()); ++t)
      if (!b.g.is_input(t) && b.g.consumers(t).empty() && !b.g.mark_output(t).ok()) {
        std::printf("seed %u: mark_output failed\n", seed);
        return 1;
      }
    if (!b.g.finalize().ok()) {
      std::printf("seed %u: finalize failed\n", seed);
      return 1;
    }
    for (SchedulePolicy sp : schedules)
      for (MemoryPolicy mp : memories)
        for (int streams : {1, 2, 4}) {
          ExecutorOptions o;
          o.schedule = sp;
          o.memory = mp;
          o.num_streams = streams;
          GraphExecutor ex(b.g, std::move(o));
          const Status st = ex.plan_dry();
          const std::string what = "seed " + std::to_string(seed) + " schedule " +
                                   std::to_string(static_cast<int>(sp)) + " memory " +
                                   std::to_string(static_cast<int>(mp)) + " streams " + std::to_string(streams);
          if (!st.ok()) {
            std::printf("%s: plan_dry: %s\n", what.c_str(), st.message().c_str());
            return 1;
          }
          ++plans;
          for (std::size_t i = 0; i < ex.num_launch_items(); ++i) grouped += ex.launch_item(i).size() > 1;
          if (check(b.g, ex, what, &overlaps)) return 1;
        }
  }
  if (overlaps == 0 || grouped == 0) {
    std::printf("no plan reused memory or grouped a launch: the fuzz exercised nothing\n");
    return 1;
  }
  std::printf("%ld plans, %ld grouped launches, %ld overlapping tensor pairs, all ordered\nOK\n", plans, grouped,
              overlaps);
  return 0;
}
