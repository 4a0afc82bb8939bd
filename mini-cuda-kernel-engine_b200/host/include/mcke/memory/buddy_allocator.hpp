// mcke/memory/buddy_allocator.hpp -- a stream-ordered buddy allocator for one device.
//
// Stands where mini-cuda-kernel-engine include/mcke/memory/buddy_allocator.hpp:146
// (BuddyAllocator) stands: a DeviceAllocator that reserves large slabs from the
// driver and carves them into power-of-two blocks, so after warm-up no
// allocate() reaches cudaMalloc.  It is written for this repository (the
// reference's allocator algorithms are not part of the kernel path); the
// interface and the stream-ordered reuse rules are the reference's:
//
//   * a block freed on stream S may be handed out again at once for use on S;
//   * for any other stream it is parked with an event recorded on S at
//     deallocate() and rejoins the free lists (merging with its buddy) once that
//     event has completed; a request that finds nothing else free takes a
//     same-stream parked block, then reserves a new slab, then (last resort)
//     waits for parked blocks' events (counted as blocking_drains);
//   * requests larger than a slab bypass the slabs (one cudaMalloc each).
//
// Blocks are min_block << k bytes (k = 0 .. log2(slab_bytes / min_block)), a
// block of size s starts at an offset that is a multiple of s within its slab,
// and a block's buddy is at offset ^ s.  One instance serves one device: it
// makes that device current around its CUDA calls.  Not thread-safe (one host
// thread drives an executor).
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <memory>
#include <set>
#include <vector>

#include "mcke/memory/allocator.hpp"

namespace mcke {

// Where slabs come from: device memory (cudaMalloc on the allocator's device)
// or, for tests on a host without a GPU, host memory (no events: a freed block
// is reusable at once).
class SlabSource {
 public:
  virtual ~SlabSource() = default;
  [[nodiscard]] virtual StatusOr<void*> reserve(std::size_t bytes) = 0;
  virtual void release(void* p) = 0;
  [[nodiscard]] virtual bool on_device() const = 0;
};
[[nodiscard]] std::unique_ptr<SlabSource> make_device_slab_source(int device);
[[nodiscard]] std::unique_ptr<SlabSource> make_host_slab_source();

struct BuddyConfig {
  std::size_t slab_bytes = std::size_t{1} << 30;  // a power of two
  std::size_t min_block = kDeviceAlignment;      // a power of two, >= kDeviceAlignment
  int max_slabs = 64;
};

class BuddyAllocator final : public DeviceAllocator {
 public:
  // `source` defaults to device memory of `device`.
  explicit BuddyAllocator(int device = 0, BuddyConfig cfg = {}, std::unique_ptr<SlabSource> source = nullptr);
  ~BuddyAllocator() override;
  BuddyAllocator(const BuddyAllocator&) = delete;
  BuddyAllocator& operator=(const BuddyAllocator&) = delete;

  StatusOr<Allocation> allocate(std::size_t bytes, rt::StreamHandle stream) override;
  Status deallocate(const Allocation& a, rt::StreamHandle stream) override;
  Status trim() override;
  Status settle_pending() override;
  [[nodiscard]] AllocatorStats stats() const override;
  [[nodiscard]] std::string_view name() const override { return "buddy"; }
  [[nodiscard]] Status validate() const override;
  [[nodiscard]] int device() const noexcept { return device_; }
  [[nodiscard]] std::size_t parked_blocks() const noexcept { return parked_.size(); }

 private:
  struct Slab {
    void* base = nullptr;
    std::vector<std::set<std::size_t>> free_by_order;  // offsets of free blocks
    std::map<std::size_t, int> live;                   // offset -> order of blocks handed out
  };
  struct Parked {
    std::uint32_t slab;
    std::size_t off;
    int order;
    rt::StreamHandle stream;
    void* event;  // cudaEvent_t recorded on `stream` at deallocate (device sources only),
                  // shared by the pieces of a parked block split for its own stream
  };

  [[nodiscard]] int order_for(std::size_t bytes) const;
  [[nodiscard]] std::size_t block_bytes(int order) const { return cfg_.min_block << order; }
  void insert_free(std::uint32_t slab, std::size_t off, int order);  // with buddy merging
  [[nodiscard]] bool take_free(int order, std::uint32_t* slab, std::size_t* off);
  void split_to(std::uint32_t slab, std::size_t off, int from, int to, bool to_parked, const Parked* like);
  Status settle(bool block);
  void drop_event(void* ev);  // one parked entry fewer uses the event; destroyed at zero
  [[nodiscard]] Allocation hand_out(std::uint32_t slab, std::size_t off, int order, std::size_t requested);

  int device_;
  BuddyConfig cfg_;
  int max_order_ = 0;
  std::unique_ptr<SlabSource> src_;
  std::vector<Slab> slabs_;
  std::vector<Parked> parked_;
  std::map<void*, std::size_t> bypass_;  // pointer -> bytes
  std::map<void*, int> event_refs_;      // parked entries sharing each recorded event
  AllocatorStats stats_{};
};

}  // namespace mcke
