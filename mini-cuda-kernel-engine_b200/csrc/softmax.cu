// softmax.cu -- numerically stable row softmax over the last dim.
//
// Replaces mini-cuda-kernel-engine kernels/softmax.cu (launcher :177, kernels
// :112 and :152; online-softmax algebra include/mcke/kernels/softmax_online.hpp).
//
// The reference reads each row two or three times.  Here the whole row is
// held in registers, so x is read ONCE and y written once (1R + 1W, the HBM
// floor for this op):
//   * cols <= 1024  : one warp per row fed through shared memory by bulk
//                     asynchronous copies (softmax_stream_row_kernel, below);
//   * cols <= 2048  : one warp per row, NV float4 per lane (NV = cols/128
//                     rounded up to a power of two), max and sum by xor-shuffle
//                     butterflies -- no shared memory, no barrier;
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

// One warp per row; the row lives in NV float4 registers per lane.
template <int NV>
__global__ void __launch_bounds__(kThreads) softmax_warp_row_kernel(const float* __restrict__ x,
                                                                    float* __restrict__ y,
                                                                    int64_t rows, int64_t cols) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * cols;
  float* yr = y + row * cols;
  float4 v[NV];
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int64_t c = static_cast<int64_t>(i * 32 + lane) * 4;
    v[i] = (c < cols) ? ld_stream_f4(xr + c) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
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
    if (c < cols) st_stream_f4(yr + c, make_float4(v[i].x * r, v[i].y * r, v[i].z * r, v[i].w * r));
  }
}

// Streamed variant of the warp-per-row kernel, for rows of at most 1024
// floats.  Each warp owns a ring of kRowStages row buffers in shared memory,
// filled by bulk asynchronous copies (cp.async.bulk, completion counted on one
// mbarrier per buffer), and walks rows gw, gw + W, gw + 2W, ... (W = warps in
// the grid).  A CTA of 8 warps holds 8 x 2 rows = 64 KB of reads in flight
// without holding them in registers, and 3 such CTAs fit on an SM (192 KB in
// flight and 24 warps per SM); the arithmetic is the warp-per-row
// kernel's, reading the row from shared memory instead of global memory.
// Waits are bounded (2 s); on expiry the warp records it in a device word read
// by mcke_sm100_check_device_errors, lets its issued copies land and stops.
constexpr int kRowStages = 2;
constexpr int kRowWarps = 8;                            // warps per CTA
constexpr int kRowThreads = 32 * kRowWarps;
constexpr int kRowBufFloats = 1024;
constexpr std::size_t kRowSmem = static_cast<std::size_t>(kRowWarps) * kRowStages * kRowBufFloats * 4 +
                                 kRowWarps * kRowStages * 8;
constexpr unsigned long long kRowWaitNs = 2000000000ull;

__device__ uint32_t g_softmax_watchdog;

__device__ __forceinline__ uint32_t sm_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool row_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (it == 0) t0 = t;
    else if (t - t0 > kRowWaitNs) return false;
  }
}

template <int NV>
__global__ void __launch_bounds__(kRowThreads) softmax_stream_row_kernel(const float* __restrict__ x,
                                                                      float* __restrict__ y, int64_t rows,
                                                                      int64_t cols) {
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & 31;
  const int w = threadIdx.x >> 5;
  float* bufs = reinterpret_cast<float*>(smem) + static_cast<std::size_t>(w) * kRowStages * kRowBufFloats;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<std::size_t>(kRowWarps) * kRowStages * kRowBufFloats * 4) +
                   w * kRowStages;
  const int64_t W = static_cast<int64_t>(gridDim.x) * kRowWarps;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kRowWarps + w;
  const int64_t mine = rows > gw ? (rows - gw + W - 1) / W : 0;
  const uint32_t row_bytes = static_cast<uint32_t>(cols * 4);
  if (lane == 0) {
    for (int s = 0; s < kRowStages; ++s)
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_addr(bars + s)) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncwarp();
  auto issue = [&](int64_t i) {  // lane 0: my i-th row into buffer i % kRowStages
    const int64_t r = gw + i * W;
    const uint32_t bar = sm_addr(bars + (i % kRowStages));
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(row_bytes) : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     sm_addr(bufs + (i % kRowStages) * kRowBufFloats)),
                 "l"(x + r * cols), "r"(row_bytes), "r"(bar)
                 : "memory");
  };
  if (lane == 0)
    for (int64_t i = 0; i < mine && i < kRowStages; ++i) issue(i);
  int64_t i = 0;
  for (; i < mine; ++i) {
    const int stage = static_cast<int>(i % kRowStages);
    const bool ok = row_wait(sm_addr(bars + stage), static_cast<uint32_t>((i / kRowStages) & 1));
    if (__any_sync(0xffffffffu, !ok)) break;
    const float* row = bufs + stage * kRowBufFloats;
    float4 v[NV];
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = (k * 32 + lane) * 4;
      v[k] = (c < cols) ? *reinterpret_cast<const float4*>(row + c)
                        : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    }
    __syncwarp();
    if (lane == 0 && i + kRowStages < mine) {
      // the row is in registers now; order those reads before the async refill
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(i + kRowStages);
    }
    float m = -INFINITY;
#pragma unroll
    for (int k = 0; k < NV; ++k) m = fmaxf(m, max4(v[k]));
    m = warp_max(m);
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      v[k] = exp4_sub(v[k], m);
      sum += (v[k].x + v[k].y) + (v[k].z + v[k].w);
    }
    sum = warp_sum(sum);
    const float rcp = 1.0f / sum;
    float* yr = y + (gw + i * W) * cols;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = (k * 32 + lane) * 4;
      if (c < cols) st_stream_f4(yr + c, make_float4(v[k].x * rcp, v[k].y * rcp, v[k].z * rcp, v[k].w * rcp));
    }
  }
  if (i < mine && lane == 0) {
    atomicCAS(&g_softmax_watchdog, 0u, 1u);
    for (int64_t k = i; k < mine && k < i + kRowStages; ++k)
      row_wait(sm_addr(bars + (k % kRowStages)), static_cast<uint32_t>((k / kRowStages) & 1));
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

std::mutex g_row_mu;
bool g_row_attr[64] = {};
int ensure_row_smem(const char* who) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(MCKE_CUDA_ERROR, "%s: no usable current device", who);
  std::lock_guard<std::mutex> lk(g_row_mu);
  if (!g_row_attr[dev]) {
    const void* ks[4] = {reinterpret_cast<const void*>(softmax_stream_row_kernel<1>),
                         reinterpret_cast<const void*>(softmax_stream_row_kernel<2>),
                         reinterpret_cast<const void*>(softmax_stream_row_kernel<4>),
                         reinterpret_cast<const void*>(softmax_stream_row_kernel<8>)};
    for (const void* k : ks) {
      const cudaError_t e =
          cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kRowSmem));
      if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "%s: %s", who, cudaGetErrorString(e));
    }
    g_row_attr[dev] = true;
  }
  return MCKE_OK;
}

}  // namespace

// Reads and clears the streamed softmax's watchdog word on the current device.
int read_softmax_watchdog(uint32_t* site) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_softmax_watchdog, sizeof(v));
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "softmax watchdog read: %s", cudaGetErrorString(e));
  if (v != 0) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_softmax_watchdog, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "softmax watchdog clear: %s", cudaGetErrorString(e));
  }
  *site = v;
  return MCKE_OK;
}
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
  if (variant == MCKE_SOFTMAX_ONLINE && vec && cols <= kRowBufFloats) {
    MCKE_RETURN_IF(ensure_row_smem(who));
    // At most 3 CTAs per SM (their rings fill shared memory); fewer for few rows.
    int64_t g = (rows + kRowWarps - 1) / kRowWarps;
    const int64_t cap = 3LL * sm_count();
    if (g > cap) g = cap;
    const unsigned gu = static_cast<unsigned>(g);
    if (cols <= 128) softmax_stream_row_kernel<1><<<gu, kRowThreads, kRowSmem, s>>>(x, y, rows, cols);
    else if (cols <= 256) softmax_stream_row_kernel<2><<<gu, kRowThreads, kRowSmem, s>>>(x, y, rows, cols);
    else if (cols <= 512) softmax_stream_row_kernel<4><<<gu, kRowThreads, kRowSmem, s>>>(x, y, rows, cols);
    else softmax_stream_row_kernel<8><<<gu, kRowThreads, kRowSmem, s>>>(x, y, rows, cols);
  } else if (variant == MCKE_SOFTMAX_ONLINE && vec && cols <= 2048) {
    const unsigned g = static_cast<unsigned>((rows + kWarps - 1) / kWarps);
    if (cols <= 128) softmax_warp_row_kernel<1><<<g, kThreads, 0, s>>>(x, y, rows, cols);
    else if (cols <= 256) softmax_warp_row_kernel<2><<<g, kThreads, 0, s>>>(x, y, rows, cols);
    else if (cols <= 512) softmax_warp_row_kernel<4><<<g, kThreads, 0, s>>>(x, y, rows, cols);
    else if (cols <= 1024) softmax_warp_row_kernel<8><<<g, kThreads, 0, s>>>(x, y, rows, cols);
    else softmax_warp_row_kernel<16><<<g, kThreads, 0, s>>>(x, y, rows, cols);
  } else if (variant == MCKE_SOFTMAX_ONLINE && vec && cols <= 16384) {
    const unsigned g = static_cast<unsigned>(rows);
    if (cols <= 4096) softmax_block_row_kernel<4><<<g, kThreads, 0, s>>>(x, y, cols);
    else if (cols <= 8192) softmax_block_row_kernel<8><<<g, kThreads, 0, s>>>(x, y, cols);
    else softmax_block_row_kernel<16><<<g, kThreads, 0, s>>>(x, y, cols);
  } else if (variant == MCKE_SOFTMAX_ONLINE) {
    softmax_online_generic_kernel<<<static_cast<unsigned>(rows), kThreads, 0, s>>>(x, y, cols);
  } else {
    softmax_three_pass_kernel<<<static_cast<unsigned>(rows), kThreads, 0, s>>>(x, y, cols);
  }
  return check_launch(who);
}
