// ops.cpp -- infer / cost / launch for the hot-path ops.
//
// Shape rules, build-time rejections and cost models follow the reference's
// src/graph/ops_gemm.cpp:15-96 (beta != 0 rejected, variant/tile pairing
// checked, 2MNK flops, (MK+KN+MN) x element bytes), ops_bias_act.cpp:63-130
// (bias rank 1 matching the last dim, vector-width rule on cols, flops per
// element {1, 2, 22, 10} for {none, relu, gelu_erf, gelu_tanh}, bytes
// (2n + cols) x 4), ops_reduce.cpp:54-133 (last axis only, rows(cols-1) flops,
// 0 for max) and ops_softmax.cpp:27-83 (5 flops per element, 2n x 4 bytes).
#include <algorithm>

#include "mcke/graph/op.hpp"

namespace mcke {
namespace {

kernels::Activation to_kernel(BiasActParams::Act a) {
  switch (a) {
    case BiasActParams::Act::kNone: return kernels::Activation::kNone;
    case BiasActParams::Act::kRelu: return kernels::Activation::kRelu;
    case BiasActParams::Act::kGeluErf: return kernels::Activation::kGeluErf;
    case BiasActParams::Act::kGeluTanh: return kernels::Activation::kGeluTanh;
  }
  return kernels::Activation::kNone;
}

std::uint64_t act_flops(kernels::Activation a) {
  switch (a) {
    case kernels::Activation::kNone: return 1;
    case kernels::Activation::kRelu: return 2;
    case kernels::Activation::kGeluErf: return 22;
    case kernels::Activation::kGeluTanh: return 10;
  }
  return 0;
}

bool last_axis(int axis, int rank) { return axis == -1 || axis == rank - 1; }

}  // namespace

// ---------------------------------------------------------------- GemmOp

StatusOr<std::vector<TensorDesc>> GemmOp::infer(const std::vector<TensorDesc>& in) const {
  if (in.size() != 2 && in.size() != 3)
    return InvalidArgumentError("GemmOp: expects inputs (A, B) or (A, B, bias), got " + std::to_string(in.size()));
  const Shape& a = in[0].shape;
  const Shape& b = in[1].shape;
  if (a.rank() != 2 || b.rank() != 2) return InvalidArgumentError("GemmOp: A and B must be rank 2");
  if (a[1] != b[0])
    return InvalidArgumentError("GemmOp: inner dimensions disagree -- A is " + a.to_string() + " and B is " +
                                b.to_string());
  if (in[0].dtype != in[1].dtype) return InvalidArgumentError("GemmOp: A and B must have the same dtype");
  if (in[0].dtype != DType::kF32 && in[0].dtype != DType::kBF16)
    return InvalidArgumentError("GemmOp: operands must be f32 or bf16");
  if (p_.beta != 0.0f)
    return UnimplementedError("GemmOp: beta != 0 reads C, a third input the graph does not model");
  if (in.size() == 3 && (in[2].shape.rank() != 1 || in[2].shape[0] != b[1] || in[2].dtype != DType::kF32))
    return InvalidArgumentError("GemmOp: bias must be f32 of shape [N]");
  const bool bf16 = in[0].dtype == DType::kBF16;
  if (!bf16) {
    const bool tc = p_.variant == kernels::GemmVariant::kTcgen05Tf32x3;
    if (p_.out_dtype != DType::kF32) return InvalidArgumentError("GemmOp: f32 operands give an f32 output");
    if (!tc && (in.size() == 3 || p_.act != kernels::Activation::kNone))
      return InvalidArgumentError("GemmOp: epilogue fusion with f32 operands needs kTcgen05Tf32x3");
    if (p_.variant == kernels::GemmVariant::kTcgen05Bf16)
      return InvalidArgumentError("GemmOp: kTcgen05Bf16 needs bf16 operands");
    if (p_.variant == kernels::GemmVariant::kCublasRef)
      return UnimplementedError("GemmOp: the cuBLAS comparison row is not part of this library");
    if (!kernels::gemm_tile_is_supported(p_.variant, p_.tile))
      return InvalidArgumentError("GemmOp: tile is not defined for this variant (kTiledSmem requires (32,32,32,1,1); "
                                  "the register-blocked variants require (128,128,8,8,8))");
  } else if (p_.out_dtype != DType::kF32 && p_.out_dtype != DType::kBF16) {
    return InvalidArgumentError("GemmOp: output must be f32 or bf16");
  }
  TensorDesc out;
  out.shape = Shape{a[0], b[1]};
  out.dtype = bf16 ? p_.out_dtype : DType::kF32;
  return std::vector<TensorDesc>{out};
}

OpCost GemmOp::cost(const std::vector<TensorDesc>& in) const {
  OpCost c;
  if (in.size() < 2) return c;
  const std::uint64_t m = in[0].shape[0], k = in[0].shape[1], n = in[1].shape[1];
  const std::uint64_t e = dtype_size(in[0].dtype);
  const std::uint64_t eo = in[0].dtype == DType::kBF16 ? dtype_size(p_.out_dtype) : 4;
  c.flops = 2ull * m * n * k;
  c.bytes = (m * k + k * n) * e + m * n * eo + (in.size() == 3 ? n * 4 : 0);
  return c;
}

std::size_t GemmOp::workspace_bytes(const std::vector<TensorDesc>& in) const {
  if (in.size() < 2 || in[0].dtype != DType::kF32 || p_.variant != kernels::GemmVariant::kTcgen05Tf32x3) return 0;
  return kernels::gemm_f32_tc_workspace_bytes(in[0].shape[0], in[1].shape[1], in[0].shape[1]);
}

Status GemmOp::launch(const OpContext& ctx, const std::vector<Tensor>& in, const std::vector<Tensor>& out) {
  if ((in.size() != 2 && in.size() != 3) || out.size() != 1)
    return InvalidArgumentError("GemmOp::launch: expects 2 or 3 inputs and 1 output");
  const std::int64_t m = in[0].shape[0], k = in[0].shape[1], n = in[1].shape[1];
  if (in[0].dtype == DType::kF32) {
    const float* a = in[0].data_as<float>();
    const float* b = in[1].data_as<float>();
    float* c = out[0].data_as<float>();
    if (!a || !b || !c) return InvalidArgumentError("GemmOp::launch: a tensor is undefined or not f32");
    if (p_.variant == kernels::GemmVariant::kTcgen05Tf32x3) {
      const float* bias = in.size() == 3 ? in[2].data_as<float>() : nullptr;
      if (in.size() == 3 && !bias) return InvalidArgumentError("GemmOp::launch: bias is not f32");
      return kernels::launch_gemm_f32_tc(a, b, c, m, n, k, p_.alpha, p_.beta, bias, p_.act, ctx.workspace,
                                         ctx.workspace_bytes, ctx.stream);
    }
    return kernels::launch_gemm_f32(a, b, c, m, n, k, p_.alpha, p_.beta, p_.variant, p_.tile, ctx.stream);
  }
  const bf16* a = in[0].data_as<bf16>();
  const bf16* b = in[1].data_as<bf16>();
  const float* bias = in.size() == 3 ? in[2].data_as<float>() : nullptr;
  if (!a || !b || !out[0].data || (in.size() == 3 && !bias))
    return InvalidArgumentError("GemmOp::launch: a tensor is undefined or has the wrong dtype");
  return kernels::launch_gemm_bf16(reinterpret_cast<const std::uint16_t*>(a), reinterpret_cast<const std::uint16_t*>(b),
                                   out[0].data, out[0].dtype, m, n, k, p_.alpha, p_.beta, bias, p_.act, ctx.stream);
}

// ------------------------------------------------------------- BiasActOp

StatusOr<std::vector<TensorDesc>> BiasActOp::infer(const std::vector<TensorDesc>& in) const {
  if (in.size() != 2) return InvalidArgumentError("BiasActOp: expects 2 inputs (x, bias)");
  if (in[1].shape.rank() != 1) return InvalidArgumentError("BiasActOp: bias must be rank 1");
  if (in[1].shape[0] != in[0].shape.cols())
    return InvalidArgumentError("BiasActOp: bias length " + std::to_string(in[1].shape[0]) +
                                " does not match x's last dimension " + std::to_string(in[0].shape.cols()));
  if (in[1].dtype != DType::kF32) return InvalidArgumentError("BiasActOp: bias must be f32");
  if (in[0].dtype != DType::kF32 && in[0].dtype != DType::kBF16)
    return InvalidArgumentError("BiasActOp: x must be f32 or bf16");
  const int vw = p_.vector_width;
  if (vw != 0 && vw != 1 && vw != 2 && vw != 4)
    return InvalidArgumentError("BiasActOp: vector_width must be 0 (auto), 1, 2 or 4");
  if (vw > 1 && in[0].shape.cols() % vw != 0)
    return InvalidArgumentError("BiasActOp: cols " + std::to_string(in[0].shape.cols()) +
                                " is not a multiple of vector_width " + std::to_string(vw));
  TensorDesc out = in[0];
  out.name.clear();
  out.placement = Placement::kReplicated;
  return std::vector<TensorDesc>{out};
}

OpCost BiasActOp::cost(const std::vector<TensorDesc>& in) const {
  OpCost c;
  if (in.empty()) return c;
  const std::uint64_t n = in[0].shape.numel(), cols = in[0].shape.cols();
  c.flops = n * act_flops(to_kernel(p_.act));
  c.bytes = 2ull * n * dtype_size(in[0].dtype) + cols * 4;
  return c;
}

Status BiasActOp::launch(const OpContext& ctx, const std::vector<Tensor>& in, const std::vector<Tensor>& out) {
  if (in.size() != 2 || out.size() != 1) return InvalidArgumentError("BiasActOp::launch: expects 2 inputs and 1 output");
  const std::int64_t rows = in[0].shape.rows(), cols = in[0].shape.cols();
  const float* bias = in[1].data_as<float>();
  if (in[0].dtype == DType::kBF16) {
    const bf16* x = in[0].data_as<bf16>();
    bf16* y = out[0].data_as<bf16>();
    if (!x || !y || !bias) return InvalidArgumentError("BiasActOp::launch: a tensor is undefined or has the wrong dtype");
    return kernels::launch_bias_act_bf16(reinterpret_cast<const std::uint16_t*>(x), bias,
                                         reinterpret_cast<std::uint16_t*>(y), rows, cols, to_kernel(p_.act), ctx.stream);
  }
  const float* x = in[0].data_as<float>();
  float* y = out[0].data_as<float>();
  if (!x || !y || !bias) return InvalidArgumentError("BiasActOp::launch: a tensor is undefined or not f32");
  // The minimum over every pointer the kernel vector-loads or -stores.
  const int vw = p_.vector_width != 0
                     ? p_.vector_width
                     : std::min({kernels::max_vector_width_f32(x, cols), kernels::max_vector_width_f32(y, cols),
                                 kernels::max_vector_width_f32(bias, cols)});
  return kernels::launch_bias_act_f32(x, bias, y, rows, cols, to_kernel(p_.act), vw, ctx.stream, p_.max_row_blocks);
}

// ------------------------------------------------------------- ReduceOp

StatusOr<std::vector<TensorDesc>> ReduceOp::infer(const std::vector<TensorDesc>& in) const {
  if (in.size() != 1) return InvalidArgumentError("ReduceOp: expects exactly 1 input");
  if (!last_axis(p_.axis, in[0].shape.rank()))
    return InvalidArgumentError("ReduceOp: only the last axis can be reduced");
  if (in[0].dtype != DType::kF32) return InvalidArgumentError("ReduceOp: x must be f32");
  TensorDesc out;
  const auto& d = in[0].shape.dims();
  out.shape = d.size() <= 1 ? Shape{1} : Shape(std::vector<std::int64_t>(d.begin(), d.end() - 1));
  return std::vector<TensorDesc>{out};
}

OpCost ReduceOp::cost(const std::vector<TensorDesc>& in) const {
  OpCost c;
  if (in.empty()) return c;
  const std::uint64_t rows = in[0].shape.rows(), cols = in[0].shape.cols();
  c.flops = p_.kind == ReduceParams::Kind::kMax ? 0 : rows * (cols > 0 ? cols - 1 : 0);
  c.bytes = (rows * cols + rows) * 4;
  return c;
}

std::size_t ReduceOp::workspace_bytes(const std::vector<TensorDesc>& in) const {
  if (in.empty()) return 0;
  return kernels::row_reduce_workspace_bytes(in[0].shape.rows(), in[0].shape.cols(),
                                             static_cast<kernels::ReduceVariant>(p_.variant));
}

Status ReduceOp::launch(const OpContext& ctx, const std::vector<Tensor>& in, const std::vector<Tensor>& out) {
  if (in.size() != 1 || out.size() != 1) return InvalidArgumentError("ReduceOp::launch: expects 1 input and 1 output");
  const float* x = in[0].data_as<float>();
  float* o = out[0].data_as<float>();
  if (!x || !o) return InvalidArgumentError("ReduceOp::launch: a tensor is undefined or not f32");
  return kernels::launch_row_reduce_f32(x, o, in[0].shape.rows(), in[0].shape.cols(),
                                        static_cast<kernels::ReduceKind>(p_.kind),
                                        static_cast<kernels::ReduceVariant>(p_.variant),
                                        static_cast<float*>(ctx.workspace), ctx.workspace_bytes, ctx.stream);
}

// ------------------------------------------------------------ SoftmaxOp

StatusOr<std::vector<TensorDesc>> SoftmaxOp::infer(const std::vector<TensorDesc>& in) const {
  if (in.size() != 1) return InvalidArgumentError("SoftmaxOp: expects exactly 1 input");
  if (!last_axis(p_.axis, in[0].shape.rank()))
    return InvalidArgumentError("SoftmaxOp: only the last axis is supported (row-wise kernels)");
  if (in[0].dtype != DType::kF32) return InvalidArgumentError("SoftmaxOp: x must be f32");
  TensorDesc out = in[0];
  out.name.clear();
  out.placement = Placement::kReplicated;
  return std::vector<TensorDesc>{out};
}

OpCost SoftmaxOp::cost(const std::vector<TensorDesc>& in) const {
  OpCost c;
  if (in.empty()) return c;
  const std::uint64_t n = in[0].shape.numel();
  c.flops = 5ull * n;
  c.bytes = 2ull * n * 4;
  return c;
}

Status SoftmaxOp::launch(const OpContext& ctx, const std::vector<Tensor>& in, const std::vector<Tensor>& out) {
  if (in.size() != 1 || out.size() != 1) return InvalidArgumentError("SoftmaxOp::launch: expects 1 input and 1 output");
  const float* x = in[0].data_as<float>();
  float* y = out[0].data_as<float>();
  if (!x || !y) return InvalidArgumentError("SoftmaxOp::launch: a tensor is undefined or not f32");
  return kernels::launch_row_softmax_f32(x, y, in[0].shape.rows(), in[0].shape.cols(),
                                         static_cast<kernels::SoftmaxVariant>(p_.variant), ctx.stream);
}

// ---------------------------------------------------------- FullReduceOp

StatusOr<std::vector<TensorDesc>> FullReduceOp::infer(const std::vector<TensorDesc>& in) const {
  if (in.size() != 1) return InvalidArgumentError("FullReduceOp: expects exactly 1 input");
  if (in[0].dtype != DType::kF32) return InvalidArgumentError("FullReduceOp: x must be f32");
  TensorDesc out;
  out.shape = Shape{16};
  out.dtype = DType::kU8;
  return std::vector<TensorDesc>{out};
}

OpCost FullReduceOp::cost(const std::vector<TensorDesc>& in) const {
  OpCost c;
  if (in.empty()) return c;
  const std::uint64_t n = in[0].shape.numel();
  c.flops = n > 0 ? n - 1 : 0;
  c.bytes = n * 4 + 16;
  return c;
}

std::size_t FullReduceOp::workspace_bytes(const std::vector<TensorDesc>& in) const {
  return in.empty() ? 0 : kernels::reduce_full_workspace_bytes(in[0].shape.numel());
}

Status FullReduceOp::launch(const OpContext& ctx, const std::vector<Tensor>& in, const std::vector<Tensor>& outs) {
  if (in.size() != 1) return InvalidArgumentError("FullReduceOp::launch: expects 1 input");
  const float* x = in[0].data_as<float>();
  if (!x && in[0].shape.numel() > 0) return InvalidArgumentError("FullReduceOp::launch: x undefined or not f32");
  if (ctx.p2p_peers) {
    if (outs.size() != 1 || !outs[0].data) return InvalidArgumentError("FullReduceOp::launch: no output");
    return kernels::launch_reduce_full_p2p_f32(x, in[0].shape.numel(), ctx.index_base, ctx.p2p_peers,
                                               ctx.num_shards, ctx.shard, outs[0].data, ctx.stream);
  }
  if (!ctx.exchange) return InternalError("FullReduceOp::launch: no exchange buffer planned");
  return kernels::launch_reduce_full_partial_f32(x, in[0].shape.numel(), ctx.index_base, ctx.exchange, ctx.workspace,
                                                 ctx.workspace_bytes, ctx.stream);
}

Status FullReduceOp::finish(const OpContext& ctx, const void* gathered, const std::vector<Tensor>& out) {
  if (out.size() != 1 || !out[0].data) return InvalidArgumentError("FullReduceOp::finish: no output");
  return kernels::launch_reduce_combine(gathered, ctx.num_shards, out[0].data, ctx.stream);
}

}  // namespace mcke
