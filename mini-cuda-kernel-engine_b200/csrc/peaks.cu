// peaks.cu -- the roofline denominators measured by the library's own kernels.
//
// Replaces mini-cuda-kernel-engine bench/stream_triad.cu (the triad
// a[i] = b[i] + s * c[i], 12 bytes per element: the "measured bandwidth") and
// bench/fma_peak.cu (independent contracting FMA chains seeded from device
// memory: the "measured FMA peak").  Here they are library entry points, so
// bench.py times them with CUDA events on the same GPU and in the same run as
// the kernels they grade, next to the copy rate and cuBLAS rate in
// MEASURED_PEAKS.json.
//
// Streaming kernels: 128-bit loads that bypass L1 and evict-first stores, a
// grid of 4 blocks x 256 threads per SM striding over float4s with two float4
// per array in flight per thread (the bias kernel's measured shape); arrays
// must be 16-byte aligned with n % 4 == 0 (the host checks).  FMA kernel: 8
// independent chains per thread of acc = fma(acc, m, b) with m = 0.999,
// b = 1.0 (a contraction toward 1000: never overflows, never subnormal), seeds
// from device memory and one store per thread, so nothing folds away; 8 blocks
// of 256 threads per SM.  The tensor-core probe (the bf16 denominator from this
// library's own MMAs) lives with the GEMM kernel, whose instruction and
// descriptor helpers it uses; its entry points are here with the others.
#include "mcke_common.cuh"

namespace mcke_sm100 {
double mma_peak_flops_per_cta_iter();
int launch_mma_peak(int64_t ctas, int iters, cudaStream_t s);
namespace {

constexpr int kThreads = 256;
constexpr int kChains = 8;

template <bool kTriad>
__global__ void __launch_bounds__(kThreads) stream_kernel(float* __restrict__ a, const float* __restrict__ b,
                                                          const float* __restrict__ c, float s, int64_t n4) {
  pdl_entry();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  for (; i + stride < n4; i += 2 * stride) {
    const float4 b0 = ld_stream_f4(b + 4 * i), b1 = ld_stream_f4(b + 4 * (i + stride));
    float4 r0 = b0, r1 = b1;
    if (kTriad) {
      const float4 c0 = ld_stream_f4(c + 4 * i), c1 = ld_stream_f4(c + 4 * (i + stride));
      r0 = make_float4(fmaf(s, c0.x, b0.x), fmaf(s, c0.y, b0.y), fmaf(s, c0.z, b0.z), fmaf(s, c0.w, b0.w));
      r1 = make_float4(fmaf(s, c1.x, b1.x), fmaf(s, c1.y, b1.y), fmaf(s, c1.z, b1.z), fmaf(s, c1.w, b1.w));
    }
    st_stream_f4(a + 4 * i, r0);
    st_stream_f4(a + 4 * (i + stride), r1);
  }
  if (i < n4) {
    const float4 b0 = ld_stream_f4(b + 4 * i);
    float4 r0 = b0;
    if (kTriad) {
      const float4 c0 = ld_stream_f4(c + 4 * i);
      r0 = make_float4(fmaf(s, c0.x, b0.x), fmaf(s, c0.y, b0.y), fmaf(s, c0.z, b0.z), fmaf(s, c0.w, b0.w));
    }
    st_stream_f4(a + 4 * i, r0);
  }
}

__global__ void __launch_bounds__(kThreads) fma_kernel(const float* __restrict__ seed, float* __restrict__ out,
                                                       int iters) {
  pdl_entry();
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  const float s0 = seed[t];
  float acc[kChains];
#pragma unroll
  for (int j = 0; j < kChains; ++j) acc[j] = s0 + static_cast<float>(j);
  const float m = 0.999f, b = 1.0f;
  // 16 steps (128 FMAs) per loop trip: the counter and branch take ~2% of
  // the issue slots that the FFMA pipe shares
#pragma unroll 16
  for (int it = 0; it < iters; ++it) {
#pragma unroll
    for (int j = 0; j < kChains; ++j) acc[j] = fmaf(acc[j], m, b);
  }
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kChains; ++j) sum += acc[j];
  out[t] = sum;
}

int stream_launch(bool triad, float* a, const float* b, const float* c, float s, int64_t n, cudaStream_t st,
                  const char* who) {
  clear_error();
  if (n == 0) return MCKE_OK;
  if (n < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative length", who);
  if (!a || !b || (triad && !c)) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (n % 4 != 0 || !aligned(a, 16) || !aligned(b, 16) || (triad && !aligned(c, 16)))
    return fail(MCKE_INVALID_ARGUMENT, "%s: needs n %% 4 == 0 and 16-byte aligned arrays", who);
  const int64_t n4 = n / 4;
  int64_t grid = static_cast<int64_t>(sm_count()) * 4;
  const int64_t need = (n4 + kThreads - 1) / kThreads;
  if (need < grid) grid = need;
  if (triad) launch_async(stream_kernel<true>, static_cast<unsigned>(grid), kThreads, 0, st, a, b, c, s, n4);
  else launch_async(stream_kernel<false>, static_cast<unsigned>(grid), kThreads, 0, st, a, b, nullptr, 0.f, n4);
  return check_launch(who);
}

}  // namespace
}  // namespace mcke_sm100

using namespace mcke_sm100;

extern "C" int mcke_sm100_peak_triad_f32(float* a, const float* b, const float* c, float scalar, int64_t n,
                                         mcke_stream_t stream) {
  return stream_launch(true, a, b, c, scalar, n, reinterpret_cast<cudaStream_t>(stream), "mcke_sm100_peak_triad_f32");
}

extern "C" int mcke_sm100_peak_copy_f32(float* a, const float* b, int64_t n, mcke_stream_t stream) {
  return stream_launch(false, a, b, nullptr, 0.f, n, reinterpret_cast<cudaStream_t>(stream),
                       "mcke_sm100_peak_copy_f32");
}

extern "C" int64_t mcke_sm100_peak_fma_threads(void) {
  return static_cast<int64_t>(sm_count()) * 8 * kThreads;
}

extern "C" int mcke_sm100_peak_fma_f32(const float* seed, float* out, int64_t threads, int iters,
                                       mcke_stream_t stream) {
  static const char* who = "mcke_sm100_peak_fma_f32";
  clear_error();
  if (threads == 0 || iters == 0) return MCKE_OK;
  if (threads < 0 || iters < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (!seed || !out) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (threads % kThreads != 0 || threads / kThreads > 2147483647LL)
    return fail(MCKE_INVALID_ARGUMENT, "%s: threads must be a multiple of %d", who, kThreads);
  launch_async(fma_kernel, static_cast<unsigned>(threads / kThreads), kThreads, 0, reinterpret_cast<cudaStream_t>(stream), seed, out, iters);
  return check_launch(who);
}

extern "C" int64_t mcke_sm100_peak_mma_ctas(void) { return static_cast<int64_t>(sm_count()); }

extern "C" double mcke_sm100_peak_mma_flops(int64_t ctas, int iters) {
  return ctas > 0 && iters > 0 ? static_cast<double>(ctas) * iters * mma_peak_flops_per_cta_iter() : 0.0;
}

extern "C" int mcke_sm100_peak_mma_bf16(int64_t ctas, int iters, mcke_stream_t stream) {
  static const char* who = "mcke_sm100_peak_mma_bf16";
  clear_error();
  if (ctas == 0 || iters == 0) return MCKE_OK;
  if (ctas < 0 || iters < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (ctas > 65535) return fail(MCKE_INVALID_ARGUMENT, "%s: at most 65535 CTAs", who);
  MCKE_RETURN_IF(launch_mma_peak(ctas, iters, reinterpret_cast<cudaStream_t>(stream)));
  return check_launch(who);
}
