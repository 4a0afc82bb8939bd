// gemm_epilogue.cuh -- the element-wise tail shared by every GEMM kernel of the
// library: v = act(alpha * acc + beta * C + bias[col]), stored as float32 or
// bfloat16.  beta == 0 never reads C (kernels/gemm.cu:91 store_c in the
// reference), which is also what makes a bf16 output legal (beta must be 0).
#pragma once

#include "mcke_common.cuh"

namespace mcke_sm100 {

struct EpilogueParams {
  float alpha;
  float beta;
  const float* bias;  // [N] or nullptr
  int act;            // mcke_activation
  int out_bf16;       // 0: float32 C, 1: bfloat16 C
  int vec_ok;         // 1: N % 4 == 0 and C 16-byte (f32) / 8-byte (bf16) aligned
};

__device__ __forceinline__ float epi_value(const EpilogueParams& ep, float acc, float prev,
                                           int64_t col) {
  float v = ep.alpha * acc;
  if (ep.beta != 0.0f) v = fmaf(ep.beta, prev, v);
  if (ep.bias) v += __ldg(ep.bias + col);
  return act_dispatch(ep.act, v);
}

// Four consecutive columns gn..gn+3 of row gm.
__device__ __forceinline__ void epilogue_store4(const EpilogueParams& ep, void* c, int64_t M,
                                                int64_t N, int64_t gm, int64_t gn, float a0,
                                                float a1, float a2, float a3) {
  (void)M;
  if (gn >= N) return;
  const int64_t base = gm * N + gn;
  if (ep.vec_ok && gn + 3 < N) {
    if (ep.out_bf16) {
      uint16_t* cb = static_cast<uint16_t*>(c);
      const uint32_t lo = pack_bf16x2(epi_value(ep, a0, 0.f, gn), epi_value(ep, a1, 0.f, gn + 1));
      const uint32_t hi = pack_bf16x2(epi_value(ep, a2, 0.f, gn + 2), epi_value(ep, a3, 0.f, gn + 3));
      *reinterpret_cast<uint2*>(cb + base) = make_uint2(lo, hi);
    } else {
      float* cf = static_cast<float*>(c);
      float4 prev = make_float4(0.f, 0.f, 0.f, 0.f);
      if (ep.beta != 0.0f) prev = *reinterpret_cast<const float4*>(cf + base);
      *reinterpret_cast<float4*>(cf + base) =
          make_float4(epi_value(ep, a0, prev.x, gn), epi_value(ep, a1, prev.y, gn + 1),
                      epi_value(ep, a2, prev.z, gn + 2), epi_value(ep, a3, prev.w, gn + 3));
    }
    return;
  }
  const float acc[4] = {a0, a1, a2, a3};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (gn + j >= N) break;
    if (ep.out_bf16) {
      static_cast<uint16_t*>(c)[base + j] = to_bf16(epi_value(ep, acc[j], 0.f, gn + j));
    } else {
      float* cf = static_cast<float*>(c);
      const float prev = (ep.beta != 0.0f) ? cf[base + j] : 0.0f;
      cf[base + j] = epi_value(ep, acc[j], prev, gn + j);
    }
  }
}

// Host side: kernels of the library.
int launch_gemm_simt(const void* a, const void* b, void* c, int64_t m, int64_t n, int64_t k,
                     bool bf16_in, const EpilogueParams& ep, cudaStream_t s,
                     const void** kernel_out);
// tile: 0 = choose the pair tile, 1 = 256 x 256, 2 = 256 x 512.
int launch_gemm_tcgen05(const uint16_t* a, const uint16_t* b, void* c, int64_t m, int64_t n,
                        int64_t k, const EpilogueParams& ep, cudaStream_t s,
                        const void** kernel_out, std::size_t* smem_out, int tile = 0);
bool tcgen05_shape_ok(const void* a, const void* b, const void* c, int64_t m, int64_t n, int64_t k,
                      bool out_bf16);
// fp32 GEMM on the tensor cores in the 3xTF32 form (split kernels, then the
// tcgen05 kernel); workspace holds the hi/lo parts of A and B.
// Host-only view of a bf16 tcgen05 launch's schedule (mcke_sm100_gemm_plan).
struct TcSchedule {
  bool pair, wide;
  int tile_m, tile_n;
  int64_t tiles, ctas;
  int split_dp_tiles, split_kblocks;
};
TcSchedule tc_schedule(int64_t m, int64_t n, int64_t k, int tile, bool out_bf16, int sms);

std::size_t gemm_tf32x3_workspace_bytes(int64_t m, int64_t n, int64_t k);
int launch_gemm_tf32x3(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                       const EpilogueParams& ep, void* workspace, cudaStream_t s, const void** kernel_out,
                       std::size_t* smem_out);
// The same product with the hi/lo split inside the GEMM kernel (no workspace).
int launch_gemm_tf32x3_split(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                             const EpilogueParams& ep, cudaStream_t s, const void** kernel_out, std::size_t* smem_out);

}  // namespace mcke_sm100
