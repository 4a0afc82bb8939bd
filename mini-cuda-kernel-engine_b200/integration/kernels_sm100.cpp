// kernels_sm100.cpp -- the reference-side binding: mini-cuda-kernel-engine's
// kernel launcher API (its include/mcke/kernels/kernels.hpp) implemented over
// libmcke_sm100a.so.
//
// A maintainer of the reference drops this file into its tree in place of
// kernels/*.cu, keeps every header and every caller unchanged (the Op classes
// of src/graph/ops_*.cpp, the benches), and links libmcke_sm100a.so.  It is
// compiled against the reference's own headers, so it uses the reference's
// Status/StatusOr, enums and GemmTile; it contains no kernels.  This
// repository compiles it against the reference tree in its CPU tests
// (tests/test_integration_shim.py) to keep the signatures honest.
#include <string>

#include "mcke/kernels/kernels.hpp"  // the reference's header
#include "mcke_sm100.h"              // this library's C-ABI

namespace mcke::kernels {
namespace {

// The C-ABI's codes are the reference's StatusCode values.
Status to_status(int rc) {
  if (rc == MCKE_OK) return OkStatus();
  return Status(static_cast<StatusCode>(rc), mcke_sm100_last_error_string());
}

mcke_stream_t st(rt::StreamHandle s) { return reinterpret_cast<mcke_stream_t>(s); }

}  // namespace

Status launch_vector_add_f32(const float* a, const float* b, float* out, std::size_t n, rt::StreamHandle stream) {
  return to_status(mcke_sm100_vector_add_f32(a, b, out, n, st(stream)));
}

Status launch_bias_act_f32(const float* x, const float* bias, float* y, std::int64_t rows, std::int64_t cols,
                           Activation act, int vector_width, rt::StreamHandle stream, int max_row_blocks) {
  return to_status(mcke_sm100_bias_act_f32(x, bias, y, rows, cols, static_cast<int>(act), vector_width,
                                           max_row_blocks, st(stream)));
}

Status launch_bias_add_f32(const float* x, const float* bias, float* y, std::int64_t rows, std::int64_t cols,
                           int vector_width, rt::StreamHandle stream) {
  return to_status(mcke_sm100_bias_add_f32(x, bias, y, rows, cols, vector_width, st(stream)));
}

Status launch_activation_f32(const float* x, float* y, std::int64_t n, Activation act, int vector_width,
                             rt::StreamHandle stream) {
  return to_status(mcke_sm100_activation_f32(x, y, n, static_cast<int>(act), vector_width, st(stream)));
}

std::size_t row_reduce_workspace_bytes(std::int64_t rows, std::int64_t cols, ReduceVariant variant) noexcept {
  return mcke_sm100_reduce_row_workspace_bytes(rows, cols, static_cast<int>(variant));
}

Status launch_row_reduce_f32(const float* x, float* out, std::int64_t rows, std::int64_t cols, ReduceKind kind,
                             ReduceVariant variant, rt::StreamHandle stream) {
  return to_status(mcke_sm100_reduce_row_f32(x, out, rows, cols, static_cast<int>(kind), static_cast<int>(variant),
                                             nullptr, 0, st(stream)));
}

Status launch_row_reduce_f32(const float* x, float* out, std::int64_t rows, std::int64_t cols, ReduceKind kind,
                             ReduceVariant variant, float* workspace, std::size_t workspace_bytes,
                             rt::StreamHandle stream) {
  return to_status(mcke_sm100_reduce_row_f32(x, out, rows, cols, static_cast<int>(kind), static_cast<int>(variant),
                                             workspace, workspace_bytes, st(stream)));
}

Status launch_row_softmax_f32(const float* x, float* y, std::int64_t rows, std::int64_t cols,
                              SoftmaxVariant variant, rt::StreamHandle stream) {
  return to_status(mcke_sm100_softmax_f32(x, y, rows, cols, static_cast<int>(variant), st(stream)));
}

Status launch_gemm_f32(const float* a, const float* b, float* c, std::int64_t m, std::int64_t n, std::int64_t k,
                       float alpha, float beta, GemmVariant variant, GemmTile tile, rt::StreamHandle stream) {
  // The reference's (variant, tile) contract is kept: an unsupported pair is
  // rejected (gemm_tile_is_supported is the reference's own predicate); every
  // accepted fp32 variant runs the library's sm_100a FFMA kernel.
  if (variant == GemmVariant::kCublasRef)
    return UnimplementedError("launch_gemm_f32: the cuBLAS ceiling row is not part of libmcke_sm100a");
  if (!gemm_tile_is_supported(variant, tile))
    return InvalidArgumentError("launch_gemm_f32: tile is not one this variant is defined for; no fallback is applied");
  return to_status(mcke_sm100_gemm_f32(a, b, c, m, n, k, alpha, beta, MCKE_GEMM_AUTO, st(stream)));
}

StatusOr<GemmKernelAttrs> gemm_kernel_attrs(GemmVariant variant, GemmTile tile) {
  if (variant == GemmVariant::kCublasRef)
    return UnimplementedError("gemm_kernel_attrs: cuBLAS's kernels are not part of libmcke_sm100a");
  if (!gemm_tile_is_supported(variant, tile)) return InvalidArgumentError("gemm_kernel_attrs: unsupported tile");
  mcke_gemm_attrs a{};
  const int rc = mcke_sm100_gemm_kernel_attrs(MCKE_GEMM_SIMT, MCKE_DTYPE_F32, &a);
  if (rc != MCKE_OK) return to_status(rc);
  GemmKernelAttrs out;
  out.regs_per_thread = a.regs_per_thread;
  out.static_smem_bytes = a.static_smem_bytes;
  out.local_bytes = a.local_bytes;
  out.threads_per_block = a.threads_per_block;
  out.max_blocks_per_sm_api = a.max_blocks_per_sm_api;
  return out;
}

}  // namespace mcke::kernels
