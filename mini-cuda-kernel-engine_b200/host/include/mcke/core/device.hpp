// mcke/core/device.hpp -- what the executor needs to know about a GPU.
//
// Mirrors mini-cuda-kernel-engine include/mcke/core/device.hpp:29-125
// (DeviceInfo with the same field names, query_device, device_count), so the
// reference's GraphExecutor(Graph, DeviceAllocator&, DeviceInfo, ...) call
// compiles against this tree.  On a B200 query_device(i) reports 148 SMs,
// cc 10.0, 227 KiB of opt-in shared memory per block and a 126 MB L2.
#pragma once

#include <cstddef>
#include <string>

#include "mcke/core/status.hpp"

namespace mcke {

struct DeviceInfo {
  int index = 0;
  std::string name = "unqueried";
  int cc_major = 0;
  int cc_minor = 0;

  int sm_count = 0;
  int max_threads_per_sm = 0;
  int max_threads_per_block = 0;
  int warps_per_sm = 0;
  int regs_per_sm = 0;
  int regs_per_block = 0;
  int max_blocks_per_sm = 0;

  std::size_t global_mem_bytes = 0;
  std::size_t shared_mem_per_block = 0;
  std::size_t shared_mem_per_block_optin = 0;
  std::size_t shared_mem_per_sm = 0;
  int l2_cache_bytes = 0;
  int memory_bus_width_bits = 0;
  int memory_clock_khz = 0;

  bool supports_cooperative_launch = false;
  bool supports_mem_pools = false;
  int async_engine_count = 0;

  // Nominal DRAM bandwidth from the clock and bus width (2 transfers a clock);
  // the rooflines of this repository use measured figures instead.
  [[nodiscard]] double peak_dram_gb_s() const {
    return 2.0 * static_cast<double>(memory_clock_khz) * 1e3 * (static_cast<double>(memory_bus_width_bits) / 8.0) /
           1e9;
  }
  [[nodiscard]] int compute_capability() const { return cc_major * 10 + cc_minor; }
  [[nodiscard]] std::string describe() const;
};

// Visible CUDA devices (0 when none).
[[nodiscard]] int device_count();
// Snapshot of device `index`.
[[nodiscard]] StatusOr<DeviceInfo> query_device(int index = 0);

}  // namespace mcke
