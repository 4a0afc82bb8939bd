// mcke/memory/allocator.hpp -- the device-allocator interface, per device.
//
// Mirrors mini-cuda-kernel-engine include/mcke/memory/allocator.hpp
// (Allocation :104, AllocatorStats :124, DeviceAllocator :163,
// RawDeviceAllocator :222): the same value type, statistics and virtual
// interface, so an allocator written against the reference's header (its
// BuddyAllocator or FreeListAllocator) plugs into this GraphExecutor
// unchanged.  What changes is that an allocator here belongs to one device:
// it is constructed with a device index and makes that device current around
// every CUDA call it issues, so one host thread can drive one allocator per
// GPU of a box (the executor takes one per device).
//
// Stream-ordered contract (the reference's): allocate(bytes, stream) hands
// out a block the caller will use on `stream`; deallocate(a, stream) names the
// stream on which the last work using the block was enqueued.  A block may be
// handed out again at once for use on that same stream (stream order makes it
// safe); for another stream only after that work has completed.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <string_view>

#include "mcke/core/status.hpp"
#include "mcke/runtime/stream.hpp"

namespace mcke {

// Every block is aligned to at least this many bytes (a TMA tensor map wants
// 16; 256 keeps every tensor carved from a block 16-byte aligned as well).
inline constexpr std::size_t kDeviceAlignment = 256;

// slab_id of a block served directly by the device malloc (not from a slab).
inline constexpr std::uint32_t kBypassSlabId = 0xFFFFFFFFu;

struct Allocation {
  void* ptr = nullptr;
  std::size_t bytes = 0;            // usable size of the block handed out
  std::size_t requested_bytes = 0;  // what the caller asked for
  std::uint32_t slab_id = 0;        // which reserved slab it came from
  std::uint32_t block_id = 0;       // implementation-defined

  [[nodiscard]] bool valid() const noexcept { return ptr != nullptr; }
  [[nodiscard]] std::size_t internal_waste() const noexcept { return bytes - requested_bytes; }
};

struct AllocatorStats {
  std::uint64_t alloc_calls = 0;
  std::uint64_t free_calls = 0;
  std::uint64_t raw_malloc_calls = 0;  // device mallocs actually issued
  std::uint64_t raw_free_calls = 0;
  std::uint64_t oom_events = 0;
  std::uint64_t deferred_reuses = 0;   // blocks parked until another stream's work completed
  std::uint64_t blocking_drains = 0;

  std::size_t bytes_reserved = 0;
  std::size_t bytes_in_use = 0;
  std::size_t bytes_requested = 0;
  std::size_t peak_bytes_in_use = 0;
  std::size_t largest_free_block = 0;

  [[nodiscard]] std::size_t internal_waste() const noexcept {
    return bytes_in_use >= bytes_requested ? bytes_in_use - bytes_requested : 0;
  }
  [[nodiscard]] double utilisation() const noexcept {
    return bytes_reserved ? static_cast<double>(bytes_requested) / static_cast<double>(bytes_reserved) : 0.0;
  }
  [[nodiscard]] std::string to_string() const;
};

class DeviceAllocator {
 public:
  virtual ~DeviceAllocator() = default;
  // At least `bytes`, aligned to kDeviceAlignment, for use on `stream`.
  [[nodiscard]] virtual StatusOr<Allocation> allocate(std::size_t bytes, rt::StreamHandle stream) = 0;
  // `stream`: where the last work using the block was enqueued.
  virtual Status deallocate(const Allocation& a, rt::StreamHandle stream) = 0;
  // Returns unused reserved memory to the driver (synchronising; never inside a timed region).
  virtual Status trim() { return OkStatus(); }
  // Reclaims parked blocks whose last stream's work has completed, releasing nothing.
  virtual Status settle_pending() { return OkStatus(); }
  [[nodiscard]] virtual AllocatorStats stats() const = 0;
  [[nodiscard]] virtual std::string_view name() const = 0;
  // Walks internal structures and checks invariants (tests only).
  [[nodiscard]] virtual Status validate() const { return OkStatus(); }
};

// Every allocate() is a cudaMalloc on this allocator's device, every
// deallocate() a cudaFree (which waits for the device).
class RawDeviceAllocator final : public DeviceAllocator {
 public:
  explicit RawDeviceAllocator(int device = 0) : device_(device) {}
  StatusOr<Allocation> allocate(std::size_t bytes, rt::StreamHandle stream) override;
  Status deallocate(const Allocation& a, rt::StreamHandle stream) override;
  [[nodiscard]] AllocatorStats stats() const override { return stats_; }
  [[nodiscard]] std::string_view name() const override { return "raw(cudaMalloc)"; }
  [[nodiscard]] int device() const noexcept { return device_; }

 private:
  int device_;
  AllocatorStats stats_{};
};

}  // namespace mcke
