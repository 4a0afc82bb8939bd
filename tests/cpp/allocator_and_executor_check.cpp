// CPU check of the host layer's allocator surface (no GPU is touched):
//   * BuddyAllocator over host slabs: alignment, block sizes, splitting and
//     buddy merging, the slab cap, the bypass path, stats and validate();
//   * GraphExecutor built through the reference's constructor
//     GraphExecutor(Graph, DeviceAllocator&, DeviceInfo, ExecutorOptions)
//     (include/mcke/graph/executor.hpp:285 of the reference), planned dry.
// Prints "OK" and exits 0, or prints the failed check and exits 1.
#include <cstdio>
#include <cstdint>
#include <set>
#include <vector>

#include "mcke/graph/executor.hpp"
#include "mcke/memory/buddy_allocator.hpp"

#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::printf("FAILED line %d: %s\n", __LINE__, #c);           \
      return 1;                                                    \
    }                                                              \
  } while (0)

int main() {
  using namespace mcke;
  BuddyConfig cfg;
  cfg.slab_bytes = std::size_t{1} << 20;  // 1 MiB slabs, 256-byte minimum blocks
  cfg.min_block = 256;
  cfg.max_slabs = 2;
  BuddyAllocator buddy(0, cfg, make_host_slab_source());
  rt::StreamHandle s = nullptr;

  // sizes round up to powers of two, blocks are aligned to their size within the slab
  std::vector<Allocation> live;
  const std::size_t sizes[] = {1, 255, 256, 257, 1000, 4096, 70000, 300000};
  for (std::size_t b : sizes) {
    auto a = buddy.allocate(b, s);
    CHECK(a.ok());
    CHECK(a->bytes >= b && (a->bytes & (a->bytes - 1)) == 0 && a->bytes >= 256);
    CHECK(reinterpret_cast<std::uintptr_t>(a->ptr) % kDeviceAlignment == 0);
    CHECK(a->requested_bytes == b);
    live.push_back(*a);
  }
  CHECK(buddy.validate().ok());
  // no two live blocks overlap
  for (std::size_t i = 0; i < live.size(); ++i)
    for (std::size_t j = i + 1; j < live.size(); ++j) {
      const auto* a0 = static_cast<char*>(live[i].ptr);
      const auto* b0 = static_cast<char*>(live[j].ptr);
      CHECK(a0 + live[i].bytes <= b0 || b0 + live[j].bytes <= a0);
    }
  AllocatorStats st = buddy.stats();
  CHECK(st.alloc_calls == 8 && st.raw_malloc_calls == 1 && st.bytes_reserved == cfg.slab_bytes);
  CHECK(st.bytes_requested == 1 + 255 + 256 + 257 + 1000 + 4096 + 70000 + 300000);
  CHECK(st.internal_waste() == st.bytes_in_use - st.bytes_requested);
  // freeing everything merges the slab back into one block
  for (const Allocation& a : live) CHECK(buddy.deallocate(a, s).ok());
  CHECK(buddy.validate().ok());
  st = buddy.stats();
  CHECK(st.bytes_in_use == 0 && st.largest_free_block == cfg.slab_bytes && st.free_calls == 8);

  // a second slab when the first is full, and no third (max_slabs = 2)
  auto big1 = buddy.allocate(cfg.slab_bytes, s);
  auto big2 = buddy.allocate(cfg.slab_bytes / 2 + 1, s);
  CHECK(big1.ok() && big2.ok() && big2->slab_id != big1->slab_id);
  CHECK(buddy.stats().raw_malloc_calls == 2);
  auto none = buddy.allocate(cfg.slab_bytes, s);
  CHECK(!none.ok() && none.status().code() == StatusCode::kOutOfMemory && buddy.stats().oom_events == 1);
  // larger than a slab: bypass
  auto by = buddy.allocate(3 * cfg.slab_bytes, s);
  CHECK(by.ok() && by->slab_id == kBypassSlabId && buddy.stats().raw_malloc_calls == 3);
  CHECK(buddy.validate().ok());
  CHECK(buddy.deallocate(*by, s).ok() && buddy.deallocate(*big1, s).ok() && buddy.deallocate(*big2, s).ok());
  CHECK(!buddy.deallocate(*big2, s).ok());  // double free is refused
  CHECK(buddy.trim().ok() && buddy.stats().bytes_reserved == 0);
  CHECK(buddy.validate().ok());

  // the reference-shaped executor constructor
  Graph g;
  TensorDesc xd;
  xd.shape = Shape({512, 256});
  xd.dtype = DType::kBF16;
  xd.name = "X";
  TensorDesc wd = xd;
  wd.shape = Shape({256, 1024});
  wd.name = "W";
  const TensorId x = g.add_input(xd);
  const TensorId w = g.add_input(wd);
  GemmParams gp;
  gp.variant = kernels::GemmVariant::kTcgen05Bf16;
  auto y = g.add_node("gemm", std::make_unique<GemmOp>(gp), {x, w});
  CHECK(y.ok());
  SoftmaxParams sp;
  auto p = g.add_node("softmax", std::make_unique<SoftmaxOp>(sp), {y->at(0)});
  CHECK(p.ok());
  CHECK(g.mark_output(p->at(0)).ok());
  CHECK(g.finalize().ok());
  RawDeviceAllocator raw(3);
  DeviceInfo info;
  info.index = 3;
  info.sm_count = 148;
  ExecutorOptions opts;
  opts.num_streams = 2;
  GraphExecutor ex(std::move(g), raw, info, opts);
  CHECK(ex.options().devices.size() == 1 && ex.options().devices[0] == 3);
  CHECK(ex.options().allocators.size() == 1 && ex.options().allocators[0] == &raw);
  CHECK(ex.device_info().sm_count == 148);
  CHECK(ex.plan_dry().ok());
  CHECK(ex.arena_bytes(0) >= static_cast<std::size_t>(512 * 1024 * 4 * 2));
  CHECK(raw.stats().alloc_calls == 0);  // planning dry touches no allocator

  // the numerics gate refuses to run without cached inputs
  auto gate = ex.validate_numerics(1);
  CHECK(!gate.ok() && gate.status().code() == StatusCode::kFailedPrecondition);

  CHECK(first_bit_mismatch("abcdefgh", "abcdefgh", 8) == 8);
  CHECK(first_bit_mismatch("abcdefgh", "abcdxfgh", 8) == 1);
  const float pz = 0.0f, nz = -0.0f;
  CHECK(first_bit_mismatch(&pz, &nz, 4) == 0);  // bit identity, not float equality
  std::printf("OK\n");
  return 0;
}
