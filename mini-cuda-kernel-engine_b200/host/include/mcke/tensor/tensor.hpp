// mcke/tensor/tensor.hpp -- dtypes, shapes and non-owning device tensor views.
//
// Mirrors mini-cuda-kernel-engine include/mcke/core/dtype.hpp:33 (DType values),
// include/mcke/tensor/shape.hpp:42 (rows() = product of the leading dims,
// cols() = last dim, :139/:144) and include/mcke/tensor/tensor.hpp:114
// (data_as<T>() returns nullptr on a dtype mismatch, :153).  Adds the device
// index a multi-GPU executor needs and a bf16 element type (the reference
// declares kBF16 but gives it no C++ type).
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace mcke {

enum class DType : std::uint8_t { kF32 = 0, kF16, kBF16, kI32, kU8, kCount };

[[nodiscard]] constexpr std::size_t dtype_size(DType t) noexcept {
  switch (t) {
    case DType::kF32: return 4;
    case DType::kF16: return 2;
    case DType::kBF16: return 2;
    case DType::kI32: return 4;
    case DType::kU8: return 1;
    default: return 0;
  }
}

// bfloat16 storage (raw bits; arithmetic happens in the kernels).
struct bf16 {
  std::uint16_t bits;
};

template <typename T> struct DTypeOf;
template <> struct DTypeOf<float> { static constexpr DType value = DType::kF32; };
template <> struct DTypeOf<bf16> { static constexpr DType value = DType::kBF16; };
template <> struct DTypeOf<std::int32_t> { static constexpr DType value = DType::kI32; };
template <> struct DTypeOf<std::uint8_t> { static constexpr DType value = DType::kU8; };

class Shape {
 public:
  Shape() = default;
  Shape(std::initializer_list<std::int64_t> d) : dims_(d) {}
  explicit Shape(std::vector<std::int64_t> d) : dims_(std::move(d)) {}
  [[nodiscard]] int rank() const noexcept { return static_cast<int>(dims_.size()); }
  [[nodiscard]] std::int64_t operator[](int i) const { return dims_.at(static_cast<std::size_t>(i)); }
  [[nodiscard]] std::int64_t numel() const noexcept {
    std::int64_t n = 1;
    for (auto d : dims_) n *= d;
    return n;
  }
  [[nodiscard]] std::int64_t cols() const noexcept { return dims_.empty() ? 1 : dims_.back(); }
  [[nodiscard]] std::int64_t rows() const noexcept {
    std::int64_t n = 1;
    for (std::size_t i = 0; i + 1 < dims_.size(); ++i) n *= dims_[i];
    return n;
  }
  [[nodiscard]] const std::vector<std::int64_t>& dims() const noexcept { return dims_; }
  [[nodiscard]] bool operator==(const Shape& o) const { return dims_ == o.dims_; }
  [[nodiscard]] std::string to_string() const {
    std::string s = "[";
    for (std::size_t i = 0; i < dims_.size(); ++i) s += (i ? "," : "") + std::to_string(dims_[i]);
    return s + "]";
  }

 private:
  std::vector<std::int64_t> dims_;
};

// A non-owning view of device memory.
struct Tensor {
  void* data = nullptr;
  Shape shape;
  DType dtype = DType::kF32;
  int device = 0;

  template <typename T>
  [[nodiscard]] T* data_as() const noexcept {
    return dtype == DTypeOf<T>::value ? static_cast<T*>(data) : nullptr;
  }
  [[nodiscard]] std::size_t nbytes() const noexcept {
    return static_cast<std::size_t>(shape.numel()) * dtype_size(dtype);
  }
};

}  // namespace mcke
