// kernels.cpp -- mcke::kernels launchers as thin wrappers over the C-ABI of
// libmcke_sm100a.so (include/mcke_sm100.h).  Argument checks that the
// reference's launchers make and the C-ABI does not (the GEMM variant/tile
// pairing, include/mcke/kernels/gemm_tile.hpp:239 in the reference) live here.
#include "mcke/kernels/kernels.hpp"

#include "mcke_sm100.h"

namespace mcke::kernels {

Status from_capi(int rc) {
  if (rc == MCKE_OK) return OkStatus();
  return Status(static_cast<StatusCode>(rc), mcke_sm100_last_error_string());
}

namespace {
mcke_stream_t st(rt::StreamHandle s) { return reinterpret_cast<mcke_stream_t>(s); }
}  // namespace

bool gemm_tile_is_supported(GemmVariant v, const GemmTile& t) {
  switch (v) {
    case GemmVariant::kNaive:
    case GemmVariant::kNaiveUncoalesced:
    case GemmVariant::kCublasRef:
    case GemmVariant::kTcgen05Bf16:
    case GemmVariant::kTcgen05Tf32x3:
      return true;  // these own no GemmTile
    case GemmVariant::kTiledSmem:
      return t.bm == 32 && t.bn == 32 && t.bk == 32 && t.tm == 1 && t.tn == 1;
    default:
      return t.bm == 128 && t.bn == 128 && t.bk == 8 && t.tm == 8 && t.tn == 8;
  }
}

Status launch_bias_act_f32(const float* x, const float* bias, float* y, std::int64_t rows, std::int64_t cols,
                           Activation act, int vector_width, rt::StreamHandle stream, int max_row_blocks) {
  return from_capi(mcke_sm100_bias_act_f32(x, bias, y, rows, cols, static_cast<int>(act), vector_width,
                                           max_row_blocks, st(stream)));
}

Status launch_bias_act_f32_group(const BiasActJob* jobs, int count, Activation act, rt::StreamHandle stream) {
  static_assert(sizeof(BiasActJob) == sizeof(mcke_bias_act_job) && kBiasActGroupMax == MCKE_BIAS_ACT_GROUP_MAX,
                "the job layout is the C-ABI's");
  if (count < 1 || count > kBiasActGroupMax || !jobs) return InvalidArgumentError("launch_bias_act_f32_group: count");
  mcke_bias_act_job c[kBiasActGroupMax];
  for (int k = 0; k < count; ++k) c[k] = {jobs[k].x, jobs[k].bias, jobs[k].y, jobs[k].rows, jobs[k].cols};
  return from_capi(mcke_sm100_bias_act_f32_group(c, count, static_cast<int>(act), st(stream)));
}

Status launch_bias_add_f32(const float* x, const float* bias, float* y, std::int64_t rows, std::int64_t cols,
                           int vector_width, rt::StreamHandle stream) {
  return from_capi(mcke_sm100_bias_add_f32(x, bias, y, rows, cols, vector_width, st(stream)));
}

Status launch_activation_f32(const float* x, float* y, std::int64_t n, Activation act, int vector_width,
                             rt::StreamHandle stream) {
  return from_capi(mcke_sm100_activation_f32(x, y, n, static_cast<int>(act), vector_width, st(stream)));
}

Status launch_bias_act_bf16(const std::uint16_t* x, const float* bias, std::uint16_t* y, std::int64_t rows,
                            std::int64_t cols, Activation act, rt::StreamHandle stream) {
  return from_capi(mcke_sm100_bias_act_bf16(x, bias, y, rows, cols, static_cast<int>(act), st(stream)));
}

std::size_t row_reduce_workspace_bytes(std::int64_t rows, std::int64_t cols, ReduceVariant variant) noexcept {
  return mcke_sm100_reduce_row_workspace_bytes(rows, cols, static_cast<int>(variant));
}

Status launch_row_reduce_f32(const float* x, float* out, std::int64_t rows, std::int64_t cols, ReduceKind kind,
                             ReduceVariant variant, rt::StreamHandle stream) {
  return launch_row_reduce_f32(x, out, rows, cols, kind, variant, nullptr, 0, stream);
}

Status launch_row_reduce_f32(const float* x, float* out, std::int64_t rows, std::int64_t cols, ReduceKind kind,
                             ReduceVariant variant, float* workspace, std::size_t workspace_bytes,
                             rt::StreamHandle stream) {
  return from_capi(mcke_sm100_reduce_row_f32(x, out, rows, cols, static_cast<int>(kind),
                                             static_cast<int>(variant), workspace, workspace_bytes, st(stream)));
}

std::size_t reduce_full_workspace_bytes(std::int64_t n) noexcept { return mcke_sm100_reduce_full_workspace_bytes(n); }

Status launch_reduce_full_f32(const float* x, std::int64_t n, void* out, void* workspace,
                              std::size_t workspace_bytes, rt::StreamHandle stream) {
  return from_capi(mcke_sm100_reduce_full_f32(x, n, static_cast<mcke_reduce_result*>(out), workspace,
                                              workspace_bytes, st(stream)));
}

Status launch_reduce_full_partial_f32(const float* x, std::int64_t n, std::int64_t index_base, void* partial,
                                      void* workspace, std::size_t workspace_bytes, rt::StreamHandle stream) {
  return from_capi(mcke_sm100_reduce_full_partial_f32(x, n, index_base, static_cast<mcke_reduce_partial*>(partial),
                                                      workspace, workspace_bytes, st(stream)));
}

std::size_t reduce_p2p_buffer_bytes(int world) noexcept { return mcke_sm100_reduce_p2p_buffer_bytes(world); }

Status launch_reduce_full_p2p_f32(const float* x, std::int64_t n, std::int64_t index_base, void* const* peer_buffers,
                                  int world, int rank, void* out, rt::StreamHandle stream) {
  return from_capi(mcke_sm100_reduce_full_p2p_f32(x, n, index_base, peer_buffers, world, rank, 0,
                                                  static_cast<mcke_reduce_result*>(out), st(stream)));
}

Status launch_reduce_combine(const void* partials, std::int64_t count, void* out, rt::StreamHandle stream) {
  return from_capi(mcke_sm100_reduce_combine(static_cast<const mcke_reduce_partial*>(partials), count,
                                             static_cast<mcke_reduce_result*>(out), st(stream)));
}

Status launch_row_softmax_f32(const float* x, float* y, std::int64_t rows, std::int64_t cols,
                              SoftmaxVariant variant, rt::StreamHandle stream) {
  return from_capi(mcke_sm100_softmax_f32(x, y, rows, cols, static_cast<int>(variant), st(stream)));
}

Status launch_gemm_f32(const float* a, const float* b, float* c, std::int64_t m, std::int64_t n, std::int64_t k,
                       float alpha, float beta, GemmVariant variant, GemmTile tile, rt::StreamHandle stream) {
  if (variant == GemmVariant::kCublasRef)
    return UnimplementedError("launch_gemm_f32: the cuBLAS comparison row is not part of this library");
  if (variant == GemmVariant::kTcgen05Bf16)
    return InvalidArgumentError("launch_gemm_f32: kTcgen05Bf16 takes bf16 operands (launch_gemm_bf16)");
  if (variant == GemmVariant::kTcgen05Tf32x3)  // no workspace: the GEMM kernel splits its tiles itself
    return from_capi(mcke_sm100_gemm_f32_tc(a, b, c, m, n, k, alpha, beta, nullptr, 0, nullptr, 0, st(stream)));
  if (!gemm_tile_is_supported(variant, tile))
    return InvalidArgumentError("launch_gemm_f32: tile is not one the variant is defined for; no fallback is applied");
  return from_capi(mcke_sm100_gemm_f32(a, b, c, m, n, k, alpha, beta, MCKE_GEMM_AUTO, st(stream)));
}

std::size_t gemm_f32_tc_workspace_bytes(std::int64_t m, std::int64_t n, std::int64_t k) noexcept {
  return mcke_sm100_gemm_f32_tc_workspace_bytes(m, n, k);
}

Status launch_gemm_f32_tc(const float* a, const float* b, float* c, std::int64_t m, std::int64_t n, std::int64_t k,
                          float alpha, float beta, const float* bias, Activation act, void* workspace,
                          std::size_t workspace_bytes, rt::StreamHandle stream) {
  return from_capi(mcke_sm100_gemm_f32_tc(a, b, c, m, n, k, alpha, beta, bias, static_cast<int>(act), workspace,
                                          workspace_bytes, st(stream)));
}

Status launch_gemm_bf16(const std::uint16_t* a, const std::uint16_t* b, void* c, DType c_dtype, std::int64_t m,
                        std::int64_t n, std::int64_t k, float alpha, float beta, const float* bias, Activation act,
                        rt::StreamHandle stream) {
  if (c_dtype != DType::kF32 && c_dtype != DType::kBF16)
    return InvalidArgumentError("launch_gemm_bf16: output must be f32 or bf16");
  return from_capi(mcke_sm100_gemm_bf16_ex(a, b, c, c_dtype == DType::kBF16 ? MCKE_DTYPE_BF16 : MCKE_DTYPE_F32, m,
                                           n, k, alpha, beta, bias, static_cast<int>(act), MCKE_GEMM_AUTO,
                                           st(stream)));
}

StatusOr<GemmKernelAttrs> gemm_kernel_attrs(GemmVariant variant, GemmTile tile) {
  if (variant == GemmVariant::kCublasRef)
    return UnimplementedError("gemm_kernel_attrs: cuBLAS's kernels are not part of this library");
  if (!gemm_tile_is_supported(variant, tile)) return InvalidArgumentError("gemm_kernel_attrs: unsupported tile");
  mcke_gemm_attrs a{};
  const bool tc = variant == GemmVariant::kTcgen05Bf16;
  MCKE_RETURN_IF_ERROR(from_capi(mcke_sm100_gemm_kernel_attrs(tc ? MCKE_GEMM_TCGEN05 : MCKE_GEMM_SIMT,
                                                              tc ? MCKE_DTYPE_BF16 : MCKE_DTYPE_F32, &a)));
  GemmKernelAttrs out;
  out.regs_per_thread = a.regs_per_thread;
  out.static_smem_bytes = a.static_smem_bytes + a.dynamic_smem_bytes;
  out.local_bytes = a.local_bytes;
  out.threads_per_block = a.threads_per_block;
  out.max_blocks_per_sm_api = a.max_blocks_per_sm_api;
  return out;
}

}  // namespace mcke::kernels
