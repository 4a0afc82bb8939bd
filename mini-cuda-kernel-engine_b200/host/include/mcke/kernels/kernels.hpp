// mcke/kernels/kernels.hpp -- C++ launchers of the sm_100a kernel library.
//
// Same names, signatures, enums and error behaviour as mini-cuda-kernel-engine
// include/mcke/kernels/kernels.hpp:59-302 (launch_bias_act_f32 :102,
// launch_bias_add_f32 :129, launch_activation_f32 :133, max_vector_width_f32
// :143, row_reduce_workspace_bytes :198, launch_row_reduce_f32 :204/:209,
// launch_row_softmax_f32 :220, launch_gemm_f32 :265, gemm_kernel_attrs :301)
// and the GemmVariant/GemmTile vocabulary of include/mcke/kernels/gemm_tile.hpp.
// Each launcher is a thin wrapper over the C-ABI in include/mcke_sm100.h; none
// synchronises or allocates.  New entries (bf16 bias+act, bf16 GEMM with a
// fused epilogue, the full-vector reduce) follow the same conventions.
#pragma once

#include <cstddef>
#include <cstdint>

#include "mcke/core/status.hpp"
#include "mcke/runtime/stream.hpp"
#include "mcke/tensor/tensor.hpp"

namespace mcke::kernels {

enum class Activation : std::uint8_t { kNone, kRelu, kGeluErf, kGeluTanh };
enum class ReduceKind : std::uint8_t { kSum, kMax, kMean };
enum class ReduceVariant : std::uint8_t { kSmemTree, kWarpShuffle, kTwoPass };
enum class SoftmaxVariant : std::uint8_t { kThreePass, kOnlineOnePass };

// Append-only, as the reference's enum is (gemm_tile.hpp:209).  The reference's
// fp32 ladder values all run this library's sm_100a FFMA kernel (their kernels
// are replaced); kCublasRef is not on this path and returns Unimplemented;
// kTcgen05Bf16 is the tensor-core kernel and takes bf16 operands.
enum class GemmVariant : std::uint8_t {
  kNaive, kTiledSmem, kTiledRegBlock, kWarpTile, kCublasRef,
  kWarpTileNoDbuf, kWarpTileVec4, kNaiveUncoalesced,
  kTcgen05Bf16,
  kTcgen05Tf32x3,  // new: f32 operands on the tensor cores (3xTF32)
};

// The reference's tile descriptor; validated exactly as the reference does
// (only the (32,32,32,1,1) tile for kTiledSmem and (128,128,8,8,8) for the
// register-blocked variants are accepted), then ignored: the sm_100a kernels
// carry their own tiles.
struct GemmTile {
  int bm = 128, bn = 128, bk = 8;
  int tm = 8, tn = 8;
};
[[nodiscard]] bool gemm_tile_is_supported(GemmVariant v, const GemmTile& t);

[[nodiscard]] Status launch_bias_act_f32(const float* x, const float* bias, float* y, std::int64_t rows,
                                        std::int64_t cols, Activation act, int vector_width,
                                        rt::StreamHandle stream, int max_row_blocks = 0);
[[nodiscard]] Status launch_bias_add_f32(const float* x, const float* bias, float* y, std::int64_t rows,
                                        std::int64_t cols, int vector_width, rt::StreamHandle stream);
[[nodiscard]] Status launch_activation_f32(const float* x, float* y, std::int64_t n, Activation act,
                                          int vector_width, rt::StreamHandle stream);
[[nodiscard]] inline int max_vector_width_f32(const void* p, std::int64_t cols) noexcept {
  const auto addr = reinterpret_cast<std::uintptr_t>(p);
  for (int w = 4; w > 1; w >>= 1)
    if (cols % w == 0 && addr % (sizeof(float) * static_cast<std::size_t>(w)) == 0) return w;
  return 1;
}
// Independent fp32 bias + activation jobs in one launch (no counterpart in
// the reference; the executor's grouped level schedule): each job is
// launch_bias_act_f32 with vector width 4 on cols % 512 == 0 and 16-byte
// aligned operands, and no job's y overlaps any job's operands.
struct BiasActJob {
  const float* x = nullptr;
  const float* bias = nullptr;
  float* y = nullptr;
  std::int64_t rows = 0, cols = 0;
};
inline constexpr int kBiasActGroupMax = 16;
[[nodiscard]] Status launch_bias_act_f32_group(const BiasActJob* jobs, int count, Activation act,
                                              rt::StreamHandle stream);
// True when a job qualifies for launch_bias_act_f32_group.
[[nodiscard]] inline bool bias_act_groupable(const void* x, const void* bias, const void* y,
                                             std::int64_t cols) noexcept {
  const auto a = [](const void* p) { return reinterpret_cast<std::uintptr_t>(p) % 16 == 0; };
  return cols > 0 && cols % 512 == 0 && a(x) && a(bias) && a(y);
}
// bf16 x/y (raw 16-bit patterns), float bias.
[[nodiscard]] Status launch_bias_act_bf16(const std::uint16_t* x, const float* bias, std::uint16_t* y,
                                         std::int64_t rows, std::int64_t cols, Activation act,
                                         rt::StreamHandle stream);

[[nodiscard]] std::size_t row_reduce_workspace_bytes(std::int64_t rows, std::int64_t cols,
                                                    ReduceVariant variant) noexcept;
[[nodiscard]] Status launch_row_reduce_f32(const float* x, float* out, std::int64_t rows, std::int64_t cols,
                                          ReduceKind kind, ReduceVariant variant, rt::StreamHandle stream);
[[nodiscard]] Status launch_row_reduce_f32(const float* x, float* out, std::int64_t rows, std::int64_t cols,
                                          ReduceKind kind, ReduceVariant variant, float* workspace,
                                          std::size_t workspace_bytes, rt::StreamHandle stream);

// Full-vector sum/max/argmax; `out` is a 16-byte device result
// {float sum; float max; int64 argmax}.
[[nodiscard]] std::size_t reduce_full_workspace_bytes(std::int64_t n) noexcept;
[[nodiscard]] Status launch_reduce_full_f32(const float* x, std::int64_t n, void* out, void* workspace,
                                           std::size_t workspace_bytes, rt::StreamHandle stream);
// One shard's 24-byte partial {double sum; float max; int32; int64 argmax}.
[[nodiscard]] Status launch_reduce_full_partial_f32(const float* x, std::int64_t n, std::int64_t index_base,
                                                   void* partial, void* workspace, std::size_t workspace_bytes,
                                                   rt::StreamHandle stream);
// New: one rank's step of a sharded full reduce with the peer-to-peer combine
// (epoch taken from the counter in this rank's exchange buffer).
[[nodiscard]] std::size_t reduce_p2p_buffer_bytes(int world) noexcept;
[[nodiscard]] Status launch_reduce_full_p2p_f32(const float* x, std::int64_t n, std::int64_t index_base,
                                                void* const* peer_buffers, int world, int rank, void* out,
                                                rt::StreamHandle stream);
[[nodiscard]] Status launch_reduce_combine(const void* partials, std::int64_t count, void* out,
                                          rt::StreamHandle stream);

[[nodiscard]] Status launch_row_softmax_f32(const float* x, float* y, std::int64_t rows, std::int64_t cols,
                                           SoftmaxVariant variant, rt::StreamHandle stream);

// The reference's FFMA variants (kNaive .. kWarpTileVec4) run this
// library's f32 AUTO choice: the tensor cores in the 3xTF32 form (hi/lo split
// inside the GEMM kernel, no workspace) when K % 4 == 0, N % 4 == 0 and A, B
// are 16-byte aligned, else the FFMA kernel; kTcgen05Tf32x3 asks for the
// tensor-core form outright (other shapes rejected).
[[nodiscard]] Status launch_gemm_f32(const float* a, const float* b, float* c, std::int64_t m, std::int64_t n,
                                    std::int64_t k, float alpha, float beta, GemmVariant variant,
                                    GemmTile tile, rt::StreamHandle stream);
// bf16 A[M,K] @ B[K,N] with a fused epilogue c = act(alpha*acc + beta*C + bias[col]),
// C float32 or bfloat16 (beta must be 0 for bf16).
// New: f32 GEMM on the tensor cores (3xTF32), c = act(alpha * A@B + beta * C +
// bias); the workspace holds the hi/lo split of A and B (nullptr and 0: the
// GEMM kernel splits its tiles itself).
[[nodiscard]] std::size_t gemm_f32_tc_workspace_bytes(std::int64_t m, std::int64_t n, std::int64_t k) noexcept;
[[nodiscard]] Status launch_gemm_f32_tc(const float* a, const float* b, float* c, std::int64_t m, std::int64_t n,
                                        std::int64_t k, float alpha, float beta, const float* bias, Activation act,
                                        void* workspace, std::size_t workspace_bytes, rt::StreamHandle stream);
[[nodiscard]] Status launch_gemm_bf16(const std::uint16_t* a, const std::uint16_t* b, void* c, DType c_dtype,
                                     std::int64_t m, std::int64_t n, std::int64_t k, float alpha, float beta,
                                     const float* bias, Activation act, rt::StreamHandle stream);

struct GemmKernelAttrs {
  int regs_per_thread = 0;
  std::size_t static_smem_bytes = 0;
  std::size_t local_bytes = 0;
  int threads_per_block = 0;
  int max_blocks_per_sm_api = 0;
};
[[nodiscard]] StatusOr<GemmKernelAttrs> gemm_kernel_attrs(GemmVariant variant, GemmTile tile);

// Maps a C-ABI status code (and the library's last message) to a Status.
[[nodiscard]] Status from_capi(int rc);

}  // namespace mcke::kernels
