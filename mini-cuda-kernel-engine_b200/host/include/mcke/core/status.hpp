// mcke/core/status.hpp -- the error model of the host API.
//
// Same names, codes and meaning as mini-cuda-kernel-engine
// include/mcke/core/status.hpp:42-190 (StatusCode values, Status, StatusOr<T>,
// the *Error constructors, MCKE_RETURN_IF_ERROR), so code written against the
// reference compiles against this header unchanged.  The numeric codes are
// also the C-ABI's mcke_status values (include/mcke_sm100.h).
#pragma once

#include <cstdint>
#include <optional>
#include <stdexcept>
#include <string>
#include <string_view>
#include <utility>

namespace mcke {

enum class StatusCode : std::uint8_t {
  kOk = 0,
  kOutOfMemory,
  kInvalidArgument,
  kFailedPrecondition,
  kUnimplemented,
  kInternal,
  kCudaError,
};

[[nodiscard]] constexpr std::string_view to_string(StatusCode c) noexcept {
  switch (c) {
    case StatusCode::kOk: return "Ok";
    case StatusCode::kOutOfMemory: return "OutOfMemory";
    case StatusCode::kInvalidArgument: return "InvalidArgument";
    case StatusCode::kFailedPrecondition: return "FailedPrecondition";
    case StatusCode::kUnimplemented: return "Unimplemented";
    case StatusCode::kInternal: return "Internal";
    case StatusCode::kCudaError: return "CudaError";
  }
  return "Unknown";
}

class [[nodiscard]] Status {
 public:
  Status() = default;
  Status(StatusCode code, std::string message) : code_(code), message_(std::move(message)) {}
  [[nodiscard]] bool ok() const noexcept { return code_ == StatusCode::kOk; }
  [[nodiscard]] StatusCode code() const noexcept { return code_; }
  [[nodiscard]] const std::string& message() const noexcept { return message_; }
  [[nodiscard]] std::string to_string() const {
    return ok() ? std::string("Ok") : std::string(mcke::to_string(code_)) + ": " + message_;
  }
  void throw_if_error() const {
    if (!ok()) throw std::runtime_error(to_string());
  }

 private:
  StatusCode code_ = StatusCode::kOk;
  std::string message_;
};

[[nodiscard]] inline Status OkStatus() { return {}; }
[[nodiscard]] inline Status OutOfMemoryError(std::string m) { return {StatusCode::kOutOfMemory, std::move(m)}; }
[[nodiscard]] inline Status InvalidArgumentError(std::string m) { return {StatusCode::kInvalidArgument, std::move(m)}; }
[[nodiscard]] inline Status FailedPreconditionError(std::string m) {
  return {StatusCode::kFailedPrecondition, std::move(m)};
}
[[nodiscard]] inline Status UnimplementedError(std::string m) { return {StatusCode::kUnimplemented, std::move(m)}; }
[[nodiscard]] inline Status InternalError(std::string m) { return {StatusCode::kInternal, std::move(m)}; }
[[nodiscard]] inline Status CudaError(std::string m) { return {StatusCode::kCudaError, std::move(m)}; }

template <typename T>
class [[nodiscard]] StatusOr {
 public:
  StatusOr(Status s) : status_(std::move(s)) {  // NOLINT: implicit by design
    if (status_.ok()) status_ = InternalError("StatusOr constructed from an OK Status without a value");
  }
  StatusOr(T v) : value_(std::move(v)) {}  // NOLINT
  [[nodiscard]] bool ok() const noexcept { return status_.ok(); }
  [[nodiscard]] const Status& status() const noexcept { return status_; }
  T& value() & { check(); return *value_; }
  const T& value() const& { check(); return *value_; }
  T&& value() && { check(); return std::move(*value_); }
  T* operator->() { check(); return &*value_; }
  const T* operator->() const { check(); return &*value_; }
  T& operator*() & { check(); return *value_; }

 private:
  void check() const {
    if (!value_) throw std::runtime_error("StatusOr has no value: " + status_.to_string());
  }
  Status status_;
  std::optional<T> value_;
};

#define MCKE_STATUS_CONCAT_INNER(a, b) a##b
#define MCKE_STATUS_CONCAT(a, b) MCKE_STATUS_CONCAT_INNER(a, b)
#define MCKE_RETURN_IF_ERROR(expr)                                    \
  do {                                                                \
    ::mcke::Status MCKE_STATUS_CONCAT(_mcke_s_, __LINE__) = (expr);   \
    if (!MCKE_STATUS_CONCAT(_mcke_s_, __LINE__).ok())                 \
      return MCKE_STATUS_CONCAT(_mcke_s_, __LINE__);                  \
  } while (0)

}  // namespace mcke
