// runtime.cpp -- mcke::rt streams and events (per device).
#include "mcke/runtime/stream.hpp"

namespace mcke::rt {

StatusOr<int> device_count() {
  int n = 0;
  const cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return CudaError(std::string("cudaGetDeviceCount: ") + cudaGetErrorString(e));
  return n;
}

StatusOr<Stream> Stream::create(int device, int priority) {
  DeviceGuard g(device);
  int lo = 0, hi = 0;
  MCKE_CUDA_RETURN_IF_ERROR(cudaDeviceGetStreamPriorityRange(&lo, &hi));
  // lo is the least urgent (numerically largest), hi the most urgent.
  if (priority > lo) priority = lo;
  if (priority < hi) priority = hi;
  cudaStream_t s = nullptr;
  MCKE_CUDA_RETURN_IF_ERROR(cudaStreamCreateWithPriority(&s, cudaStreamNonBlocking, priority));
  return Stream(s, device, true);
}

void Stream::reset() {
  if (owned_ && handle_) {
    DeviceGuard g(device_);
    cudaStreamDestroy(handle_);
  }
  handle_ = nullptr;
  owned_ = false;
}

Status Stream::wait(const Event& e) const {
  DeviceGuard g(device_);
  MCKE_CUDA_RETURN_IF_ERROR(cudaStreamWaitEvent(handle_, e.native(), 0));
  return OkStatus();
}

Status Stream::synchronize() const {
  DeviceGuard g(device_);
  MCKE_CUDA_RETURN_IF_ERROR(cudaStreamSynchronize(handle_));
  return OkStatus();
}

StatusOr<Event> Event::create(int device, Kind kind) {
  DeviceGuard g(device);
  cudaEvent_t e = nullptr;
  const unsigned flags = (kind == Kind::kDependency) ? cudaEventDisableTiming : cudaEventDefault;
  MCKE_CUDA_RETURN_IF_ERROR(cudaEventCreateWithFlags(&e, flags));
  Event ev;
  ev.handle_ = e;
  ev.device_ = device;
  ev.kind_ = kind;
  return ev;
}

void Event::reset() {
  if (handle_) {
    DeviceGuard g(device_);
    cudaEventDestroy(handle_);
  }
  handle_ = nullptr;
}

Status Event::record(const Stream& s) const {
  DeviceGuard g(s.device());
  MCKE_CUDA_RETURN_IF_ERROR(cudaEventRecord(handle_, s.native()));
  return OkStatus();
}

Status Event::synchronize() const {
  MCKE_CUDA_RETURN_IF_ERROR(cudaEventSynchronize(handle_));
  return OkStatus();
}

StatusOr<float> Event::elapsed_ms(const Event& start, const Event& stop) {
  float ms = 0.f;
  MCKE_CUDA_RETURN_IF_ERROR(cudaEventElapsedTime(&ms, start.handle_, stop.handle_));
  return ms;
}

}  // namespace mcke::rt
