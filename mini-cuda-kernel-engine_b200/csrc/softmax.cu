// softmax.cu -- numerically stable row softmax over the last dim.
//
// Replaces mini-cuda-kernel-engine kernels/softmax.cu (launcher :177, kernels
// :112 and :152; online-softmax algebra include/mcke/kernels/softmax_online.hpp).
//
// The reference reads each row two or three times.  Here the whole row is
// held in registers, so x is read ONCE and y written once (1R + 1W, the HBM
// floor for this op):
//   * cols <= 2048  : one warp per row, NV float4 per lane (NV = cols/128
//                     rounded up to a power of two) all loaded before any math,
//                     max and sum by xor-shuffle butterflies -- no shared
//                     memory, no barrier.  At config 2's 32768 x 1024 this runs
//                     at 0.99 of the measured copy rate in steady state (41.2 us
//                     per launch back to back); a per-warp ring of bulk
//                     asynchronous copies through shared memory, the first
//                     design, took 47.0 us (and 43.0 against 40.9 us timed
//                     alone after an L2 flush);
//   * cols <= 16384 : one 256-thread block per row, NV float4 per thread, two
//                     one-barrier block combines (max, then sum);
//   * anything else (cols % 4 != 0, unaligned rows, longer rows): one block per
//     row running the reference's two algorithms with scalar loads -- the
//     online (max, sum) single statistics pass plus a write pass (2R + 1W), or
//     the three-pass form (3R + 1W) when that variant is asked for.
// Every path computes exp(x - max) with expf and scales by the reciprocal of
// the float sum.
#include <cfloat>
#include <mutex>

#include "mcke_common.cuh"

namespace mcke_sm100 {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float max4(float4 v) { return fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)); }

__device__ __forceinline__ float4 exp4_sub(float4 v, float m) {
  return make_float4(expf(v.x - m), expf(v.y - m), expf(v.z - m), expf(v.w - m));
}

// One warp per row; the row lives in NV float4 registers per lane, all loaded
// before any arithmetic.  kExact: cols == 128 * NV, so no load or store needs a
// bound check (48 instead of 62 registers at NV = 8: five resident CTAs per SM
// instead of four).
template <int NV, bool kExact>
__global__ void __launch_bounds__(kThreads) softmax_warp_row_kernel(const float* __restrict__ x,
                                                                    float* __restrict__ y,
                                                                    int64_t rows, int64_t cols) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t c = static_cast<int64_t>(i * 32 + lane) * 4;
    v[i] = (kExact || c < cols) ? ld_stream_f4(xr + c) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NV; ++i) m = fmaxf(m, max4(v[i]));
  m = warp_max(m);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = exp4_sub(v[i], m);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  s = warp_sum(s);
  const float r = 1.0f / s;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t c = static_cast<int64_t>(i * 32 + lane) * 4;
    if (kExact || c < cols) st_stream_f4(yr + c, make_float4(v[i].x * r, v[i].y * r, v[i].z * r, v[i].w * r));
  }
}

// Block-wide combine of one float per thread; every thread gets the result.
template <bool kMax>
__device__ __forceinline__ float block_all(float v, float* red) {
  v = kMax ? warp_max(v) : warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = red[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) t = kMax ? fmaxf(t, red[w]) : t + red[w];
  return t;
}

// One block per row; the row lives in NV float4 registers per thread.
template <int NV>
__global__ void __launch_bounds__(kThreads) softmax_block_row_kernel(const float* __restrict__ x,
                                                                     float* __restrict__ y,
                                                                     int64_t cols) {
  pdl_entry();
  __shared__ float red_max[kWarps];
  __shared__ float red_sum[kWarps];
  const int64_t row = blockIdx.x;
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t c = static_cast<int64_t>(i * kThreads + threadIdx.x) * 4;
    v[i] = (c < cols) ? ld_stream_f4(xr + c) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
  }
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < NV; ++i) m = fmaxf(m, max4(v[i]));
  m = block_all<true>(m, red_max);
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    v[i] = exp4_sub(v[i], m);
    s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  s = block_all<false>(s, red_sum);
  const float r = 1.0f / s;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t c = static_cast<int64_t>(i * kThreads + threadIdx.x) * 4;
    if (c < cols) st_stream_f4(yr + c, make_float4(v[i].x * r, v[i].y * r, v[i].z * r, v[i].w * r));
  }
}

// Online (max, sum) state: sum is relative to max.  The empty state is
// (-inf, 0); combining with it returns the other operand unchanged, so no
// exp(-inf - -inf) = NaN can arise from padding.
struct Online {
  float m, d;
};
__device__ __forceinline__ Online online_combine(Online a, Online b) {
  if (a.d == 0.0f && a.m == -INFINITY) return b;
  if (b.d == 0.0f && b.m == -INFINITY) return a;
  const float m = fmaxf(a.m, b.m);
  return Online{m, a.d * expf(a.m - m) + b.d * expf(b.m - m)};
}
__device__ __forceinline__ Online online_add(Online s, float v) {
  if (v == -INFINITY) return s;  // contributes exp(-inf) = 0 against any finite max
  if (v > s.m) return Online{v, s.d * expf(s.m - v) + 1.0f};
  return Online{s.m, s.d + expf(v - s.m)};
}

__global__ void __launch_bounds__(kThreads) softmax_online_generic_kernel(const float* __restrict__ x,
                                                                          float* __restrict__ y,
                                                                          int64_t cols) {
  pdl_entry();
  __shared__ Online red[kWarps];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * cols;
  Online st{-INFINITY, 0.0f};
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) st = online_add(st, x[base + c]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    Online other{__shfl_xor_sync(0xffffffffu, st.m, o), __shfl_xor_sync(0xffffffffu, st.d, o)};
    st = online_combine(st, other);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = st;
  __syncthreads();
  Online t = red[0];
#pragma unroll
  for (int w = 1; w < kWarps; ++w) t = online_combine(t, red[w]);
  const float r = 1.0f / t.d;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) y[base + c] = expf(x[base + c] - t.m) * r;
}

__global__ void __launch_bounds__(kThreads) softmax_three_pass_kernel(const float* __restrict__ x,
                                                                      float* __restrict__ y,
                                                                      int64_t cols) {
  pdl_entry();
  __shared__ float red_max[kWarps];
  __shared__ float red_sum[kWarps];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * cols;
  float m = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) m = fmaxf(m, x[base + c]);
  m = block_all<true>(m, red_max);
  float s = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) s += expf(x[base + c] - m);
  s = block_all<false>(s, red_sum);
  const float r = 1.0f / s;
  for (int64_t c = threadIdx.x; c < cols; c += kThreads) y[base + c] = expf(x[base + c] - m) * r;
}

}  // namespace

namespace {
template <int NV>
void launch_warp_rows(unsigned g, cudaStream_t s, const float* x, float* y, int64_t rows, int64_t cols) {
  if (cols == 128 * NV) launch_async(softmax_warp_row_kernel<NV, true>, g, kThreads, 0, s, x, y, rows, cols);
  else launch_async(softmax_warp_row_kernel<NV, false>, g, kThreads, 0, s, x, y, rows, cols);
}
}  // namespace
}  // namespace mcke_sm100

using namespace mcke_sm100;

extern "C" int mcke_sm100_softmax_f32(const float* x, float* y, int64_t rows, int64_t cols,
                                      int variant, mcke_stream_t stream) {
  static const char* who = "mcke_sm100_softmax_f32";
  clear_error();
  if (rows == 0 || cols == 0) return MCKE_OK;
  if (rows < 0 || cols < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (!x || !y) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (x == y) return fail(MCKE_INVALID_ARGUMENT, "%s: in-place (x == y) is not supported", who);
  if (variant != MCKE_SOFTMAX_THREE_PASS && variant != MCKE_SOFTMAX_ONLINE)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown variant %d", who, variant);
  if (rows > 2147483647LL) return fail(MCKE_INVALID_ARGUMENT, "%s: rows exceeds the grid limit", who);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec = (cols % 4 == 0) && aligned(x, 16) && aligned(y, 16);
  if (variant == MCKE_SOFTMAX_ONLINE && vec && cols <= 2048) {
    const unsigned g = static_cast<unsigned>((rows + kWarps - 1) / kWarps);
    if (cols <= 128) launch_warp_rows<1>(g, s, x, y, rows, cols);
    else if (cols <= 256) launch_warp_rows<2>(g, s, x, y, rows, cols);
    else if (cols <= 512) launch_warp_rows<4>(g, s, x, y, rows, cols);
    else if (cols <= 1024) launch_warp_rows<8>(g, s, x, y, rows, cols);
    else launch_warp_rows<16>(g, s, x, y, rows, cols);
  } else if (variant == MCKE_SOFTMAX_ONLINE && vec && cols <= 16384) {
    const unsigned g = static_cast<unsigned>(rows);
    if (cols <= 4096) launch_async(softmax_block_row_kernel<4>, g, kThreads, 0, s, x, y, cols);
    else if (cols <= 8192) launch_async(softmax_block_row_kernel<8>, g, kThreads, 0, s, x, y, cols);
    else launch_async(softmax_block_row_kernel<16>, g, kThreads, 0, s, x, y, cols);
  } else if (variant == MCKE_SOFTMAX_ONLINE) {
    launch_async(softmax_online_generic_kernel, static_cast<unsigned>(rows), kThreads, 0, s, x, y, cols);
  } else {
    launch_async(softmax_three_pass_kernel, static_cast<unsigned>(rows), kThreads, 0, s, x, y, cols);
  }
  return check_launch(who);
}
