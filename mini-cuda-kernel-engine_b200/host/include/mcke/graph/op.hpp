// mcke/graph/op.hpp -- the operator interface and the four hot-path ops.
//
// Mirrors mini-cuda-kernel-engine include/mcke/graph/op.hpp:72-303: OpContext
// (stream + scratch, :72), OpCost (:91), Op with launch / infer / cost /
// workspace_bytes (:99-122), and GemmOp, BiasActOp, ReduceOp, SoftmaxOp with
// their Params structs.  Differences, all additive:
//   * infer() works on TensorDesc (shape + dtype) so bf16 tensors flow through
//     the graph; the reference's ops are f32-only;
//   * OpContext carries the device and the shard index/count the sharding
//     pass assigned;
//   * GemmParams can fuse a bias and an activation into the GEMM epilogue and
//     choose a bf16 output (the tcgen05 kernel);
//   * FullReduceOp (sum/max/argmax of a whole tensor) is new; it reduces its
//     shard, the executor all-gathers the 24-byte partials (exchange_bytes /
//     finish), and each device combines them in shard order.
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <vector>

#include "mcke/core/status.hpp"
#include "mcke/kernels/kernels.hpp"
#include "mcke/runtime/stream.hpp"
#include "mcke/tensor/tensor.hpp"

namespace mcke {

using TensorId = std::uint32_t;
using NodeId = std::uint32_t;
inline constexpr TensorId kInvalidTensor = 0xFFFFFFFFu;
inline constexpr NodeId kInvalidNode = 0xFFFFFFFFu;

// How a tensor is laid out over the executor's devices.
enum class Placement : std::uint8_t {
  kReplicated,  // every device holds the whole tensor
  kRowSplit,    // device d holds rows [R*d/D, R*(d+1)/D) of rows() x cols()
  kColSplit,    // device d holds columns [C*d/D, C*(d+1)/D)
};

struct TensorDesc {
  Shape shape;
  DType dtype = DType::kF32;
  std::string name;
  Placement placement = Placement::kReplicated;  // a hint for graph inputs
};

struct OpContext {
  rt::StreamHandle stream = {};
  int device = 0;
  void* workspace = nullptr;
  std::size_t workspace_bytes = 0;
  int shard = 0;        // this device's index among the executor's devices
  int num_shards = 1;
  std::int64_t index_base = 0;  // flat index of this shard's first element (range shards)
  void* exchange = nullptr;     // exchange_bytes() of device scratch for the partial
  // Set when the executor exchanges this node's partials peer to peer: a
  // device array of the shards' exchange buffers; the op then does the whole
  // step (no exchange/finish).
  void* const* p2p_peers = nullptr;
};

struct OpCost {
  std::uint64_t flops = 0;
  std::uint64_t bytes = 0;
  [[nodiscard]] double arithmetic_intensity() const {
    return bytes ? static_cast<double>(flops) / static_cast<double>(bytes) : 0.0;
  }
};

class Op {
 public:
  virtual ~Op() = default;
  [[nodiscard]] virtual std::string_view type_name() const = 0;
  // Enqueue on ctx.stream.  Must not synchronise.
  [[nodiscard]] virtual Status launch(const OpContext& ctx, const std::vector<Tensor>& inputs,
                                      const std::vector<Tensor>& outputs) = 0;
  // Output descriptors from input descriptors (build time).
  [[nodiscard]] virtual StatusOr<std::vector<TensorDesc>> infer(const std::vector<TensorDesc>& inputs) const = 0;
  [[nodiscard]] virtual OpCost cost(const std::vector<TensorDesc>& inputs) const = 0;
  [[nodiscard]] virtual std::size_t workspace_bytes(const std::vector<TensorDesc>&) const { return 0; }
  // Bytes each shard contributes to an all-gather after launch(); 0 = none.
  [[nodiscard]] virtual std::size_t exchange_bytes() const { return 0; }
  // Runs after the all-gather with num_shards * exchange_bytes() gathered bytes.
  [[nodiscard]] virtual Status finish(const OpContext&, const void* /*gathered*/,
                                      const std::vector<Tensor>& /*outputs*/) {
    return OkStatus();
  }
};

using OpPtr = std::unique_ptr<Op>;

struct GemmParams {
  float alpha = 1.f;
  float beta = 0.f;  // must be 0 in a graph (C is not a graph input), as in the reference
  using Variant = kernels::GemmVariant;
  // f32 inputs: the reference's ladder (FFMA kernel) or kTcgen05Tf32x3 (tensor
  // cores, which also takes bias/act); bf16 inputs always use kTcgen05Bf16.
  Variant variant = Variant::kTiledRegBlock;
  kernels::GemmTile tile{};
  // Epilogue fusion (new): inputs are [A, B] or [A, B, bias]; act applied last.
  kernels::Activation act = kernels::Activation::kNone;
  DType out_dtype = DType::kF32;  // kBF16 allowed for bf16 inputs
};

class GemmOp final : public Op {
 public:
  explicit GemmOp(GemmParams p) : p_(p) {}
  [[nodiscard]] std::string_view type_name() const override { return "Gemm"; }
  [[nodiscard]] Status launch(const OpContext&, const std::vector<Tensor>&, const std::vector<Tensor>&) override;
  [[nodiscard]] StatusOr<std::vector<TensorDesc>> infer(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] OpCost cost(const std::vector<TensorDesc>&) const override;
  // kTcgen05Tf32x3: the hi/lo split of A and B; 0 otherwise.
  [[nodiscard]] std::size_t workspace_bytes(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] const GemmParams& params() const { return p_; }

 private:
  GemmParams p_;
};

struct BiasActParams {
  enum class Act { kNone, kRelu, kGeluErf, kGeluTanh } act = Act::kGeluErf;
  int vector_width = 0;    // 0 = widest legal (max_vector_width_f32)
  int max_row_blocks = 0;  // 0 = automatic grid
};

class BiasActOp final : public Op {
 public:
  explicit BiasActOp(BiasActParams p) : p_(p) {}
  [[nodiscard]] std::string_view type_name() const override { return "BiasAct"; }
  [[nodiscard]] const BiasActParams& params() const noexcept { return p_; }
  [[nodiscard]] Status launch(const OpContext&, const std::vector<Tensor>&, const std::vector<Tensor>&) override;
  [[nodiscard]] StatusOr<std::vector<TensorDesc>> infer(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] OpCost cost(const std::vector<TensorDesc>&) const override;

 private:
  BiasActParams p_;
};

struct ReduceParams {
  enum class Kind { kSum, kMax, kMean } kind = Kind::kSum;
  int axis = -1;
  enum class Variant { kSmemTree, kWarpShuffle, kTwoPass } variant = Variant::kWarpShuffle;
};

class ReduceOp final : public Op {
 public:
  explicit ReduceOp(ReduceParams p) : p_(p) {}
  [[nodiscard]] std::string_view type_name() const override { return "Reduce"; }
  [[nodiscard]] Status launch(const OpContext&, const std::vector<Tensor>&, const std::vector<Tensor>&) override;
  [[nodiscard]] StatusOr<std::vector<TensorDesc>> infer(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] OpCost cost(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] std::size_t workspace_bytes(const std::vector<TensorDesc>&) const override;

 private:
  ReduceParams p_;
};

struct SoftmaxParams {
  int axis = -1;
  enum class Variant { kThreePass, kOnlineOnePass } variant = Variant::kOnlineOnePass;
};

class SoftmaxOp final : public Op {
 public:
  explicit SoftmaxOp(SoftmaxParams p) : p_(p) {}
  [[nodiscard]] std::string_view type_name() const override { return "Softmax"; }
  [[nodiscard]] Status launch(const OpContext&, const std::vector<Tensor>&, const std::vector<Tensor>&) override;
  [[nodiscard]] StatusOr<std::vector<TensorDesc>> infer(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] OpCost cost(const std::vector<TensorDesc>&) const override;

 private:
  SoftmaxParams p_;
};

// Whole-tensor sum / max / argmax; output is one 16-byte result
// {float sum; float max; int64 argmax} (DType kU8, shape {16}).
class FullReduceOp final : public Op {
 public:
  [[nodiscard]] std::string_view type_name() const override { return "FullReduce"; }
  [[nodiscard]] Status launch(const OpContext&, const std::vector<Tensor>&, const std::vector<Tensor>&) override;
  [[nodiscard]] StatusOr<std::vector<TensorDesc>> infer(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] OpCost cost(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] std::size_t workspace_bytes(const std::vector<TensorDesc>&) const override;
  [[nodiscard]] std::size_t exchange_bytes() const override { return 24; }
  [[nodiscard]] Status finish(const OpContext&, const void* gathered, const std::vector<Tensor>&) override;
};

}  // namespace mcke
