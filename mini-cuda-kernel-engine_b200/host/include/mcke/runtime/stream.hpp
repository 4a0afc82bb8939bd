// mcke/runtime/stream.hpp -- per-device CUDA streams and events (mcke::rt).
//
// Mirrors mini-cuda-kernel-engine include/mcke/runtime/stream.hpp:55-305
// (StreamHandle = cudaStream_t; non-blocking priority streams; Event with a
// dependency-only or timing kind; Stream::wait) and adds what that single-GPU
// API lacked: every Stream and Event knows its device and makes it current
// around the CUDA calls it issues, so one host thread can drive all GPUs of a
// box and order work across them with events (cudaStreamWaitEvent accepts an
// event recorded on another device).
#pragma once

#include <cuda_runtime.h>

#include <string>
#include <utility>

#include "mcke/core/status.hpp"

namespace mcke::rt {

using StreamHandle = cudaStream_t;

[[nodiscard]] inline Status cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return OkStatus();
  return CudaError(std::string(what) + ": " + cudaGetErrorString(e));
}

#define MCKE_CUDA_RETURN_IF_ERROR(expr) MCKE_RETURN_IF_ERROR(::mcke::rt::cuda_status((expr), #expr))

// Makes `device` current for the lifetime of the guard and restores the
// previous device afterwards.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    cudaGetDevice(&prev_);
    if (device != prev_) cudaSetDevice(device);
    dev_ = device;
  }
  ~DeviceGuard() {
    if (dev_ != prev_) cudaSetDevice(prev_);
  }
  DeviceGuard(const DeviceGuard&) = delete;
  DeviceGuard& operator=(const DeviceGuard&) = delete;

 private:
  int prev_ = 0, dev_ = 0;
};

[[nodiscard]] StatusOr<int> device_count();

class Event;

class Stream {
 public:
  Stream() = default;
  // Non-blocking stream on `device`; priority as cudaDeviceGetStreamPriorityRange
  // reports (lower = higher priority), clamped into range.
  [[nodiscard]] static StatusOr<Stream> create(int device, int priority = 0);
  [[nodiscard]] static Stream wrap(StreamHandle h, int device) { return Stream(h, device, false); }
  ~Stream() { reset(); }
  Stream(Stream&& o) noexcept { *this = std::move(o); }
  Stream& operator=(Stream&& o) noexcept {
    if (this != &o) {
      reset();
      handle_ = std::exchange(o.handle_, nullptr);
      device_ = o.device_;
      owned_ = std::exchange(o.owned_, false);
    }
    return *this;
  }
  Stream(const Stream&) = delete;
  Stream& operator=(const Stream&) = delete;

  [[nodiscard]] StreamHandle native() const noexcept { return handle_; }
  [[nodiscard]] int device() const noexcept { return device_; }
  [[nodiscard]] Status wait(const Event& e) const;  // this stream waits for e (any device)
  [[nodiscard]] Status synchronize() const;

 private:
  Stream(StreamHandle h, int device, bool owned) : handle_(h), device_(device), owned_(owned) {}
  void reset();
  StreamHandle handle_ = nullptr;
  int device_ = 0;
  bool owned_ = false;
};

class Event {
 public:
  enum class Kind { kDependency, kTiming };
  Event() = default;
  [[nodiscard]] static StatusOr<Event> create(int device, Kind kind = Kind::kDependency);
  ~Event() { reset(); }
  Event(Event&& o) noexcept { *this = std::move(o); }
  Event& operator=(Event&& o) noexcept {
    if (this != &o) {
      reset();
      handle_ = std::exchange(o.handle_, nullptr);
      device_ = o.device_;
      kind_ = o.kind_;
    }
    return *this;
  }
  Event(const Event&) = delete;
  Event& operator=(const Event&) = delete;

  [[nodiscard]] Status record(const Stream& s) const;
  [[nodiscard]] Status synchronize() const;
  [[nodiscard]] cudaEvent_t native() const noexcept { return handle_; }
  [[nodiscard]] int device() const noexcept { return device_; }
  // Milliseconds between two timing events (both recorded and complete).
  [[nodiscard]] static StatusOr<float> elapsed_ms(const Event& start, const Event& stop);

 private:
  void reset();
  cudaEvent_t handle_ = nullptr;
  int device_ = 0;
  Kind kind_ = Kind::kDependency;
};

}  // namespace mcke::rt
