// gemm_simt.cu -- CUDA-core GEMM, C = act(alpha * A @ B + beta * C + bias).
//
// Replaces mini-cuda-kernel-engine kernels/gemm.cu's fp32 ladder (launcher
// :829, register-blocked kernel :370, store_c :91).  This is the library's fp32
// path (FFMA, fp32 accumulation) and the fallback for bf16 shapes that the
// TMA-fed tensor-core kernel cannot take (K or N not a multiple of 8,
// unaligned operands, K == 0).
//
// Tiling: a 256-thread block owns a 128 x 128 tile of C and walks K in slabs
// of 16.  Each thread accumulates an 8 x 8 micro-tile held as 2 x 2 sub-tiles
// of 4 x 4 spaced 64 apart, so its fragment reads from shared memory are two
// float4 per operand per k and hit distinct banks.  A is stored k-major
// (transposed) in shared memory so both fragments are float4 reads.  Shared
// memory is double-buffered: slab s+1 is fetched into registers while slab s is
// multiplied, then stored to the other buffer -- one barrier per slab.
// Out-of-range rows/columns/k are zero-filled on load and masked on store, so
// any shape is correct; the float4 global path needs K % 4 == 0, N % 4 == 0 and
// 16-byte aligned operands and is chosen only then.
#include "mcke_common.cuh"
#include "gemm_epilogue.cuh"

namespace mcke_sm100 {
namespace {

constexpr int BM = 128, BN = 128, BK = 16;
constexpr int kThreads = 256;
constexpr int APAD = 4;

template <typename T>
__device__ __forceinline__ float ld_elem(const T* p);
template <>
__device__ __forceinline__ float ld_elem<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float ld_elem<uint16_t>(const uint16_t* p) { return from_bf16(__ldg(p)); }

template <typename T, bool VEC>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_simt_kernel(const T* __restrict__ a, const T* __restrict__ b, void* __restrict__ c,
                     int64_t M, int64_t N, int64_t K, EpilogueParams ep) {
  pdl_entry();
  __shared__ __align__(16) float As[2][BK][BM + APAD];
  __shared__ __align__(16) float Bs[2][BK][BN];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = static_cast<int64_t>(blockIdx.y) * BM;
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * BN;

  // Loader mapping.  A slab 128 x 16: thread loads rows (tid>>2) and
  // (tid>>2)+64, 4 consecutive k at (tid&3)*4.  B slab 16 x 128: thread loads
  // k rows (tid>>5) and (tid>>5)+8, 4 consecutive n at (tid&31)*4.
  const int a_row = tid >> 2, a_k = (tid & 3) * 4;
  const int b_k = tid >> 5, b_col = (tid & 31) * 4;

  float ra[2][4], rb[2][4];
  auto fetch = [&](int64_t k0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t gm = m0 + a_row + 64 * h;
      const int64_t gk = k0 + a_k;
      if (VEC && gm < M && gk + 3 < K) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(a + gm * K + gk));
        ra[h][0] = v.x; ra[h][1] = v.y; ra[h][2] = v.z; ra[h][3] = v.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          ra[h][j] = (gm < M && gk + j < K) ? ld_elem<T>(a + gm * K + gk + j) : 0.0f;
      }
      const int64_t bk = k0 + b_k + 8 * h;
      const int64_t bn = n0 + b_col;
      if (VEC && bk < K && bn + 3 < N) {
        const float4 v = __ldg(reinterpret_cast<const float4*>(b + bk * N + bn));
        rb[h][0] = v.x; rb[h][1] = v.y; rb[h][2] = v.z; rb[h][3] = v.w;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j)
          rb[h][j] = (bk < K && bn + j < N) ? ld_elem<T>(b + bk * N + bn + j) : 0.0f;
      }
    }
  };
  auto stash = [&](int buf) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
#pragma unroll
      for (int j = 0; j < 4; ++j) As[buf][a_k + j][a_row + 64 * h] = ra[h][j];
      *reinterpret_cast<float4*>(&Bs[buf][b_k + 8 * h][b_col]) =
          make_float4(rb[h][0], rb[h][1], rb[h][2], rb[h][3]);
    }
  };

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  const int64_t slabs = (K + BK - 1) / BK;
  if (slabs > 0) {
    fetch(0);
    stash(0);
  }
  __syncthreads();
  for (int64_t s = 0; s < slabs; ++s) {
    const int buf = static_cast<int>(s & 1);
    if (s + 1 < slabs) fetch((s + 1) * BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float af[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float bf[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(af[i], bf[j], acc[i][j]);
    }
    if (s + 1 < slabs) stash(buf ^ 1);
    __syncthreads();
  }

  // Epilogue: rows ty*4+i and 64+ty*4+i, columns tx*4+j and 64+tx*4+j.
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int64_t gm = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (gm >= M) continue;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int64_t gn = n0 + h * 64 + tx * 4;
      epilogue_store4(ep, c, M, N, gm, gn, acc[i][4 * h], acc[i][4 * h + 1], acc[i][4 * h + 2],
                      acc[i][4 * h + 3]);
    }
  }
}

}  // namespace

int launch_gemm_simt(const void* a, const void* b, void* c, int64_t m, int64_t n, int64_t k,
                     bool bf16_in, const EpilogueParams& ep, cudaStream_t s,
                     const void** kernel_out) {
  const int64_t gx = (n + BN - 1) / BN, gy = (m + BM - 1) / BM;
  if (gx > 2147483647LL || gy > 65535)
    return fail(MCKE_INVALID_ARGUMENT, "gemm (simt): extents exceed the grid limits");
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy), 1u);
  if (bf16_in) {
    if (kernel_out) *kernel_out = reinterpret_cast<const void*>(&gemm_simt_kernel<uint16_t, false>);
    if (m > 0 && n > 0)
      launch_async(gemm_simt_kernel<uint16_t, false>, grid, kThreads, 0, s, static_cast<const uint16_t*>(a), static_cast<const uint16_t*>(b), c, m, n, k, ep);
  } else {
    const bool vec = (k % 4 == 0) && (n % 4 == 0) && aligned(a, 16) && aligned(b, 16);
    if (vec) {
      if (kernel_out) *kernel_out = reinterpret_cast<const void*>(&gemm_simt_kernel<float, true>);
      if (m > 0 && n > 0)
        launch_async(gemm_simt_kernel<float, true>, grid, kThreads, 0, s, static_cast<const float*>(a), static_cast<const float*>(b), c, m, n, k, ep);
    } else {
      if (kernel_out) *kernel_out = reinterpret_cast<const void*>(&gemm_simt_kernel<float, false>);
      if (m > 0 && n > 0)
        launch_async(gemm_simt_kernel<float, false>, grid, kThreads, 0, s, static_cast<const float*>(a), static_cast<const float*>(b), c, m, n, k, ep);
    }
  }
  return MCKE_OK;
}

}  // namespace mcke_sm100
