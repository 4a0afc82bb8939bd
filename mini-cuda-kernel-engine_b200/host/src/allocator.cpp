// allocator.cpp -- DeviceInfo queries, the raw and the buddy device allocators.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <sstream>

#include "mcke/core/device.hpp"
#include "mcke/memory/buddy_allocator.hpp"

namespace mcke {

// ---------------------------------------------------------------- devices

int device_count() {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

StatusOr<DeviceInfo> query_device(int index) {
  cudaDeviceProp p{};
  const cudaError_t e = cudaGetDeviceProperties(&p, index);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return CudaError(std::string("query_device(") + std::to_string(index) + "): " + cudaGetErrorString(e));
  }
  DeviceInfo d;
  d.index = index;
  d.name = p.name;
  d.cc_major = p.major;
  d.cc_minor = p.minor;
  d.sm_count = p.multiProcessorCount;
  d.max_threads_per_sm = p.maxThreadsPerMultiProcessor;
  d.max_threads_per_block = p.maxThreadsPerBlock;
  d.warps_per_sm = p.maxThreadsPerMultiProcessor / 32;
  d.regs_per_sm = p.regsPerMultiprocessor;
  d.regs_per_block = p.regsPerBlock;
  d.max_blocks_per_sm = p.maxBlocksPerMultiProcessor;
  d.global_mem_bytes = p.totalGlobalMem;
  d.shared_mem_per_block = p.sharedMemPerBlock;
  d.shared_mem_per_block_optin = p.sharedMemPerBlockOptin;
  d.shared_mem_per_sm = p.sharedMemPerMultiprocessor;
  d.l2_cache_bytes = p.l2CacheSize;
  d.memory_bus_width_bits = p.memoryBusWidth;
  int clk = 0;
  if (cudaDeviceGetAttribute(&clk, cudaDevAttrMemoryClockRate, index) == cudaSuccess) d.memory_clock_khz = clk;
  cudaGetLastError();
  d.supports_cooperative_launch = p.cooperativeLaunch != 0;
  int pools = 0;
  if (cudaDeviceGetAttribute(&pools, cudaDevAttrMemoryPoolsSupported, index) == cudaSuccess)
    d.supports_mem_pools = pools != 0;
  cudaGetLastError();
  d.async_engine_count = p.asyncEngineCount;
  return d;
}

std::string DeviceInfo::describe() const {
  std::ostringstream o;
  o << "device " << index << " (" << name << "), cc " << cc_major << "." << cc_minor << ", " << sm_count << " SMs, "
    << (global_mem_bytes >> 20) << " MiB, L2 " << (l2_cache_bytes >> 20) << " MiB, smem/block opt-in "
    << (shared_mem_per_block_optin >> 10) << " KiB";
  return o.str();
}

std::string AllocatorStats::to_string() const {
  std::ostringstream o;
  o << "allocs=" << alloc_calls << " frees=" << free_calls << " raw_mallocs=" << raw_malloc_calls
    << " raw_frees=" << raw_free_calls << " oom=" << oom_events << " deferred=" << deferred_reuses
    << " drains=" << blocking_drains << " reserved=" << bytes_reserved << " in_use=" << bytes_in_use
    << " requested=" << bytes_requested << " peak=" << peak_bytes_in_use << " largest_free=" << largest_free_block;
  return o.str();
}

// ---------------------------------------------------------------- raw

StatusOr<Allocation> RawDeviceAllocator::allocate(std::size_t bytes, rt::StreamHandle) {
  ++stats_.alloc_calls;
  const std::size_t b = std::max<std::size_t>((bytes + kDeviceAlignment - 1) / kDeviceAlignment * kDeviceAlignment,
                                              kDeviceAlignment);
  rt::DeviceGuard g(device_);
  void* p = nullptr;
  const cudaError_t e = cudaMalloc(&p, b);
  if (e != cudaSuccess) {
    cudaGetLastError();
    ++stats_.oom_events;
    return OutOfMemoryError("raw allocator: cudaMalloc(" + std::to_string(b) + ") on device " +
                            std::to_string(device_) + ": " + cudaGetErrorString(e));
  }
  ++stats_.raw_malloc_calls;
  stats_.bytes_reserved += b;
  stats_.bytes_in_use += b;
  stats_.bytes_requested += bytes;
  stats_.peak_bytes_in_use = std::max(stats_.peak_bytes_in_use, stats_.bytes_in_use);
  Allocation a;
  a.ptr = p;
  a.bytes = b;
  a.requested_bytes = bytes;
  a.slab_id = kBypassSlabId;
  return a;
}

Status RawDeviceAllocator::deallocate(const Allocation& a, rt::StreamHandle) {
  if (!a.valid()) return InvalidArgumentError("raw allocator: deallocate of an invalid allocation");
  ++stats_.free_calls;
  rt::DeviceGuard g(device_);
  MCKE_CUDA_RETURN_IF_ERROR(cudaFree(a.ptr));  // waits for the device, so any stream is safe
  ++stats_.raw_free_calls;
  stats_.bytes_reserved -= a.bytes;
  stats_.bytes_in_use -= a.bytes;
  stats_.bytes_requested -= a.requested_bytes;
  return OkStatus();
}

// ---------------------------------------------------------------- slab sources

namespace {
class DeviceSlabs final : public SlabSource {
 public:
  explicit DeviceSlabs(int device) : device_(device) {}
  StatusOr<void*> reserve(std::size_t bytes) override {
    rt::DeviceGuard g(device_);
    void* p = nullptr;
    const cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
      cudaGetLastError();
      return OutOfMemoryError("buddy allocator: cudaMalloc(" + std::to_string(bytes) + ") on device " +
                              std::to_string(device_) + ": " + cudaGetErrorString(e));
    }
    return p;
  }
  void release(void* p) override {
    rt::DeviceGuard g(device_);
    cudaFree(p);
  }
  bool on_device() const override { return true; }

 private:
  int device_;
};

class HostSlabs final : public SlabSource {
 public:
  StatusOr<void*> reserve(std::size_t bytes) override {
    void* p = std::aligned_alloc(kDeviceAlignment, (bytes + kDeviceAlignment - 1) / kDeviceAlignment * kDeviceAlignment);
    if (!p) return OutOfMemoryError("buddy allocator (host slabs): out of memory");
    return p;
  }
  void release(void* p) override { std::free(p); }
  bool on_device() const override { return false; }
};

bool pow2(std::size_t v) { return v && !(v & (v - 1)); }
}  // namespace

std::unique_ptr<SlabSource> make_device_slab_source(int device) { return std::make_unique<DeviceSlabs>(device); }
std::unique_ptr<SlabSource> make_host_slab_source() { return std::make_unique<HostSlabs>(); }

// ---------------------------------------------------------------- buddy

BuddyAllocator::BuddyAllocator(int device, BuddyConfig cfg, std::unique_ptr<SlabSource> source)
    : device_(device), cfg_(cfg), src_(std::move(source)) {
  if (!pow2(cfg_.min_block) || cfg_.min_block < kDeviceAlignment) cfg_.min_block = kDeviceAlignment;
  if (!pow2(cfg_.slab_bytes) || cfg_.slab_bytes < cfg_.min_block) {
    std::size_t s = cfg_.min_block;
    while (s < cfg_.slab_bytes) s <<= 1;
    cfg_.slab_bytes = s;
  }
  while ((cfg_.min_block << max_order_) < cfg_.slab_bytes) ++max_order_;
  if (!src_) src_ = make_device_slab_source(device);
}

BuddyAllocator::~BuddyAllocator() {
  static_cast<void>(settle(true));
  for (auto& s : slabs_)
    if (s.base) src_->release(s.base);
  for (auto& [p, b] : bypass_) src_->release(p);
}

int BuddyAllocator::order_for(std::size_t bytes) const {
  int k = 0;
  while (block_bytes(k) < bytes) ++k;
  return k;
}

void BuddyAllocator::insert_free(std::uint32_t slab, std::size_t off, int order) {
  auto& fl = slabs_[slab].free_by_order;
  while (order < max_order_) {
    const std::size_t buddy = off ^ block_bytes(order);
    auto it = fl[order].find(buddy);
    if (it == fl[order].end()) break;
    fl[order].erase(it);
    off = std::min(off, buddy);
    ++order;
  }
  fl[order].insert(off);
}

bool BuddyAllocator::take_free(int order, std::uint32_t* slab, std::size_t* off) {
  // smallest free block of at least `order`, lowest slab and offset first
  for (int k = order; k <= max_order_; ++k)
    for (std::uint32_t s = 0; s < slabs_.size(); ++s) {
      auto& fl = slabs_[s].free_by_order[k];
      if (fl.empty()) continue;
      const std::size_t o = *fl.begin();
      fl.erase(fl.begin());
      split_to(s, o, k, order, false, nullptr);
      *slab = s;
      *off = o;
      return true;
    }
  return false;
}

// Splits block (off, from) down to (off, to); the upper halves go back to the
// free lists, or -- when the block came from the parked list -- stay parked
// with the same stream and (shared) event.
void BuddyAllocator::split_to(std::uint32_t slab, std::size_t off, int from, int to, bool to_parked,
                              const Parked* like) {
  while (from > to) {
    --from;
    const std::size_t upper = off + block_bytes(from);
    if (to_parked) {
      Parked p = *like;
      p.slab = slab;
      p.off = upper;
      p.order = from;
      if (p.event) ++event_refs_[p.event];
      parked_.push_back(p);
    } else {
      insert_free(slab, upper, from);
    }
  }
}

void BuddyAllocator::drop_event(void* ev) {
  if (!ev) return;
  auto it = event_refs_.find(ev);
  if (it == event_refs_.end() || --it->second > 0) return;
  event_refs_.erase(it);
  rt::DeviceGuard g(device_);
  cudaEventDestroy(static_cast<cudaEvent_t>(ev));
}

Allocation BuddyAllocator::hand_out(std::uint32_t slab, std::size_t off, int order, std::size_t requested) {
  slabs_[slab].live[off] = order;
  Allocation a;
  a.ptr = static_cast<char*>(slabs_[slab].base) + off;
  a.bytes = block_bytes(order);
  a.requested_bytes = requested;
  a.slab_id = slab;
  a.block_id = static_cast<std::uint32_t>(off / cfg_.min_block);
  stats_.bytes_in_use += a.bytes;
  stats_.bytes_requested += requested;
  stats_.peak_bytes_in_use = std::max(stats_.peak_bytes_in_use, stats_.bytes_in_use);
  return a;
}

// Returns parked blocks whose event has completed (all of them when `block`,
// waiting for each) to the free lists.
Status BuddyAllocator::settle(bool block) {
  std::vector<Parked> keep;
  for (Parked& p : parked_) {
    bool done = p.event == nullptr;
    if (!done) {
      rt::DeviceGuard g(device_);
      const cudaError_t e = block ? cudaEventSynchronize(static_cast<cudaEvent_t>(p.event))
                                  : cudaEventQuery(static_cast<cudaEvent_t>(p.event));
      if (e == cudaSuccess) {
        done = true;
      } else if (e != cudaErrorNotReady) {
        cudaGetLastError();
        return CudaError(std::string("buddy allocator: event: ") + cudaGetErrorString(e));
      } else {
        cudaGetLastError();
      }
      if (done) drop_event(p.event);
    }
    if (done) insert_free(p.slab, p.off, p.order);
    else keep.push_back(p);
  }
  parked_.swap(keep);
  return OkStatus();
}

Status BuddyAllocator::settle_pending() { return settle(false); }

StatusOr<Allocation> BuddyAllocator::allocate(std::size_t bytes, rt::StreamHandle stream) {
  ++stats_.alloc_calls;
  const std::size_t want = std::max<std::size_t>(bytes, 1);
  if (want > cfg_.slab_bytes) {  // bypass: one device malloc of its own
    const std::size_t b = (want + kDeviceAlignment - 1) / kDeviceAlignment * kDeviceAlignment;
    auto p = src_->reserve(b);
    if (!p.ok()) {
      ++stats_.oom_events;
      return p.status();
    }
    ++stats_.raw_malloc_calls;
    bypass_[*p] = b;
    stats_.bytes_reserved += b;
    stats_.bytes_in_use += b;
    stats_.bytes_requested += bytes;
    stats_.peak_bytes_in_use = std::max(stats_.peak_bytes_in_use, stats_.bytes_in_use);
    Allocation a;
    a.ptr = *p;
    a.bytes = b;
    a.requested_bytes = bytes;
    a.slab_id = kBypassSlabId;
    return a;
  }
  const int order = order_for(want);
  MCKE_RETURN_IF_ERROR(settle(false));
  std::uint32_t slab = 0;
  std::size_t off = 0;
  if (take_free(order, &slab, &off)) return hand_out(slab, off, order, bytes);
  // a block parked by this same stream: stream order already makes it safe
  int best = -1;
  for (std::size_t i = 0; i < parked_.size(); ++i)
    if (parked_[i].stream == stream && parked_[i].order >= order &&
        (best < 0 || parked_[i].order < parked_[best].order))
      best = static_cast<int>(i);
  if (best >= 0) {
    Parked p = parked_[best];
    parked_.erase(parked_.begin() + best);
    ++stats_.deferred_reuses;
    split_to(p.slab, p.off, p.order, order, true, &p);
    drop_event(p.event);
    return hand_out(p.slab, p.off, order, bytes);
  }
  if (static_cast<int>(slabs_.size()) < cfg_.max_slabs) {
    auto base = src_->reserve(cfg_.slab_bytes);
    if (base.ok()) {
      ++stats_.raw_malloc_calls;
      stats_.bytes_reserved += cfg_.slab_bytes;
      Slab s;
      s.base = *base;
      s.free_by_order.assign(static_cast<std::size_t>(max_order_) + 1, {});
      s.free_by_order[static_cast<std::size_t>(max_order_)].insert(0);
      slabs_.push_back(std::move(s));
      if (take_free(order, &slab, &off)) return hand_out(slab, off, order, bytes);
    }
  }
  if (!parked_.empty()) {  // last resort: wait for other streams' parked blocks
    ++stats_.blocking_drains;
    MCKE_RETURN_IF_ERROR(settle(true));
    if (take_free(order, &slab, &off)) return hand_out(slab, off, order, bytes);
  }
  ++stats_.oom_events;
  return OutOfMemoryError("buddy allocator: no block of " + std::to_string(block_bytes(order)) + " bytes on device " +
                          std::to_string(device_) + " (" + std::to_string(slabs_.size()) + " slabs of " +
                          std::to_string(cfg_.slab_bytes) + " bytes)");
}

Status BuddyAllocator::deallocate(const Allocation& a, rt::StreamHandle stream) {
  if (!a.valid()) return InvalidArgumentError("buddy allocator: deallocate of an invalid allocation");
  ++stats_.free_calls;
  if (a.slab_id == kBypassSlabId) {
    auto it = bypass_.find(a.ptr);
    if (it == bypass_.end()) return InvalidArgumentError("buddy allocator: unknown bypass block");
    if (src_->on_device()) {  // the block may still be in use on `stream`
      rt::DeviceGuard g(device_);
      MCKE_CUDA_RETURN_IF_ERROR(cudaStreamSynchronize(stream));
    }
    src_->release(a.ptr);
    ++stats_.raw_free_calls;
    stats_.bytes_reserved -= it->second;
    stats_.bytes_in_use -= it->second;
    stats_.bytes_requested -= a.requested_bytes;
    bypass_.erase(it);
    return OkStatus();
  }
  if (a.slab_id >= slabs_.size()) return InvalidArgumentError("buddy allocator: unknown slab");
  Slab& s = slabs_[a.slab_id];
  const std::size_t off = static_cast<std::size_t>(static_cast<char*>(a.ptr) - static_cast<char*>(s.base));
  auto it = s.live.find(off);
  if (it == s.live.end()) return InvalidArgumentError("buddy allocator: double free or foreign pointer");
  const int order = it->second;
  s.live.erase(it);
  stats_.bytes_in_use -= block_bytes(order);
  stats_.bytes_requested -= a.requested_bytes;
  Parked p{a.slab_id, off, order, stream, nullptr};
  if (src_->on_device()) {
    rt::DeviceGuard g(device_);
    cudaEvent_t ev = nullptr;
    MCKE_CUDA_RETURN_IF_ERROR(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
    const cudaError_t e = cudaEventRecord(ev, stream);
    if (e != cudaSuccess) {
      cudaEventDestroy(ev);
      return rt::cuda_status(e, "buddy allocator: cudaEventRecord");
    }
    p.event = ev;
    event_refs_[ev] = 1;
    parked_.push_back(p);
  } else {
    insert_free(p.slab, p.off, p.order);
  }
  return OkStatus();
}

Status BuddyAllocator::trim() {
  MCKE_RETURN_IF_ERROR(settle(true));
  for (std::size_t i = 0; i < slabs_.size(); ++i) {
    Slab& s = slabs_[i];
    if (!s.base || !s.live.empty()) continue;
    if (s.free_by_order[static_cast<std::size_t>(max_order_)].count(0) == 0) continue;
    src_->release(s.base);
    s.base = nullptr;
    for (auto& fl : s.free_by_order) fl.clear();
    ++stats_.raw_free_calls;
    stats_.bytes_reserved -= cfg_.slab_bytes;
  }
  return OkStatus();
}

AllocatorStats BuddyAllocator::stats() const {
  AllocatorStats st = stats_;
  st.largest_free_block = 0;
  for (const Slab& s : slabs_)
    for (int k = max_order_; k >= 0; --k)
      if (!s.free_by_order[static_cast<std::size_t>(k)].empty()) {
        st.largest_free_block = std::max(st.largest_free_block, block_bytes(k));
        break;
      }
  return st;
}

Status BuddyAllocator::validate() const {
  std::size_t in_use = 0;
  for (std::size_t si = 0; si < slabs_.size(); ++si) {
    const Slab& s = slabs_[si];
    if (!s.base) continue;
    // every byte of the slab is covered by exactly one live, free or parked block
    std::vector<std::pair<std::size_t, std::size_t>> spans;
    for (auto& [off, k] : s.live) {
      spans.push_back({off, block_bytes(k)});
      in_use += block_bytes(k);
    }
    for (int k = 0; k <= max_order_; ++k)
      for (std::size_t off : s.free_by_order[static_cast<std::size_t>(k)]) {
        if (off % block_bytes(k) != 0) return InternalError("buddy: free block misaligned");
        if (k < max_order_ && s.free_by_order[static_cast<std::size_t>(k)].count(off ^ block_bytes(k)))
          return InternalError("buddy: two free buddies left unmerged");
        spans.push_back({off, block_bytes(k)});
      }
    for (const Parked& p : parked_)
      if (p.slab == si) spans.push_back({p.off, block_bytes(p.order)});
    std::sort(spans.begin(), spans.end());
    std::size_t at = 0;
    for (auto& [off, len] : spans) {
      if (off != at) return InternalError("buddy: blocks overlap or leave a gap in slab " + std::to_string(si));
      at = off + len;
    }
    if (at != cfg_.slab_bytes) return InternalError("buddy: slab " + std::to_string(si) + " not fully covered");
  }
  for (auto& [p, b] : bypass_) in_use += b;
  if (in_use != stats_.bytes_in_use) return InternalError("buddy: bytes_in_use does not match the live blocks");
  return OkStatus();
}

}  // namespace mcke
