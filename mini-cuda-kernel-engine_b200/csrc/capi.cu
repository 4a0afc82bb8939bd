// capi.cu -- library-wide entry points of libmcke_sm100a.so and the GEMM
// front door (validation + kernel selection).  The GEMM launchers mirror
// mini-cuda-kernel-engine kernels/gemm.cu:829 launch_gemm_f32: empty M or N is
// OK without a launch, k == 0 is a legal GEMM (C = beta * C), negative
// extents, nulls and an output aliasing an input are rejected.
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

#include "gemm_epilogue.cuh"

namespace mcke_sm100 {

namespace {
thread_local std::string g_last_error;
}

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

void clear_error() { g_last_error.clear(); }

int sm_count() {
  static std::mutex mu;
  static std::vector<int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  std::lock_guard<std::mutex> lk(mu);
  if (static_cast<int>(cache.size()) <= dev) cache.resize(dev + 1, 0);
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

// Programmatic dependent launch: on unless the environment sets MCKE_PDL=0;
// mcke_sm100_set_programmatic_launch() changes it for the process.
std::atomic<int> g_pdl{-1};
bool pdl_enabled() {
  int v = g_pdl.load(std::memory_order_relaxed);
  if (v < 0) {
    const char* e = std::getenv("MCKE_PDL");
    v = (e && e[0] == '0') ? 0 : 1;
    g_pdl.store(v, std::memory_order_relaxed);
  }
  return v != 0;
}

int read_tc_watchdog(uint32_t* site);
int launch_watchdog_selftest(cudaStream_t s);
int read_reduce_watchdog(uint32_t* site);

namespace {

// The variant word of mcke_sm100_gemm_bf16_ex as launch_gemm_tcgen05's tile
// word: bits 0-1 the pair tile (1 = 256 x 256, 2 = 256 x 512), bits 2-3 the
// split-k schedule (1 = never, 2 = where it applies), 0 = choose.
static int tile_word(int variant) {
  return variant == MCKE_GEMM_TCGEN05_WIDE     ? (2 | 4)
         : variant == MCKE_GEMM_TCGEN05_NARROW ? (1 | 4)
         : variant == MCKE_GEMM_TCGEN05_SPLIT  ? (2 | 8)
                                               : 0;
}

int gemm_front(const char* who, const void* a, const void* b, void* c, int64_t m, int64_t n,
               int64_t k, bool bf16_in, int c_dtype, float alpha, float beta, const float* bias,
               int act, int variant, mcke_stream_t stream) {
  clear_error();
  if (m < 0 || n < 0 || k < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (m == 0 || n == 0) return MCKE_OK;
  if (!a || !b || !c) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (a == c || b == c)
    return fail(MCKE_INVALID_ARGUMENT, "%s: output aliases an input, which violates the __restrict__ contract", who);
  if (m > 2147483647LL || n > 2147483647LL || k > 2147483647LL)
    return fail(MCKE_INVALID_ARGUMENT, "%s: extent exceeds INT32_MAX", who);
  if (c_dtype != MCKE_DTYPE_F32 && c_dtype != MCKE_DTYPE_BF16)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown output dtype %d", who, c_dtype);
  const bool out_bf16 = (c_dtype == MCKE_DTYPE_BF16);
  if (out_bf16 && beta != 0.0f)
    return fail(MCKE_INVALID_ARGUMENT, "%s: beta must be 0 for a bf16 output", who);
  if (act < MCKE_ACT_NONE || act > MCKE_ACT_GELU_TANH)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown activation %d", who, act);
  if (variant < MCKE_GEMM_AUTO || variant > MCKE_GEMM_TCGEN05_SPLIT)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown variant %d", who, variant);
  const int tile = tile_word(variant);
  if (tile != 0) variant = MCKE_GEMM_TCGEN05;
  if (!bf16_in && variant == MCKE_GEMM_TCGEN05)
    return fail(MCKE_INVALID_ARGUMENT, "%s: the tcgen05 kernel takes bf16 operands; no fallback is applied", who);

  EpilogueParams ep;
  ep.alpha = alpha;
  ep.beta = beta;
  ep.bias = bias;
  ep.act = act;
  ep.out_bf16 = out_bf16 ? 1 : 0;
  ep.vec_ok = (n % 4 == 0) && aligned(c, out_bf16 ? 8 : 16) ? 1 : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);

  const bool tc_ok = bf16_in && tcgen05_shape_ok(a, b, c, m, n, k, out_bf16);
  if (variant == MCKE_GEMM_TCGEN05 && !tc_ok)
    return fail(MCKE_INVALID_ARGUMENT,
                "%s: the tcgen05 kernel needs k > 0, K %% 8 == 0, N %% 8 == 0 and 16-byte aligned "
                "A and B (TMA); no fallback is applied",
                who);
  // fp32 operands, AUTO: the tensor cores in the 3xTF32 form with the hi/lo
  // split inside the kernel (fp32-level accuracy, no workspace) wherever TMA
  // can describe A and B; SIMT (the FFMA kernel) otherwise or when asked for.
  const bool tf32_ok = !bf16_in && !out_bf16 && variant == MCKE_GEMM_AUTO && k > 0 && k % 4 == 0 && n % 4 == 0 &&
                       aligned(a, 16) && aligned(b, 16);
  if (tc_ok && variant != MCKE_GEMM_SIMT) {
    MCKE_RETURN_IF(launch_gemm_tcgen05(static_cast<const uint16_t*>(a), static_cast<const uint16_t*>(b),
                                       c, m, n, k, ep, s, nullptr, nullptr, tile));
  } else if (tf32_ok) {
    MCKE_RETURN_IF(launch_gemm_tf32x3_split(static_cast<const float*>(a), static_cast<const float*>(b),
                                            static_cast<float*>(c), m, n, k, ep, s, nullptr, nullptr));
  } else {
    MCKE_RETURN_IF(launch_gemm_simt(a, b, c, m, n, k, bf16_in, ep, s, nullptr));
  }
  return check_launch(who);
}

}  // namespace
}  // namespace mcke_sm100

using namespace mcke_sm100;

extern "C" int mcke_sm100_version(void) { return 100; }

extern "C" const char* mcke_sm100_last_error_string(void) { return g_last_error.c_str(); }

extern "C" int mcke_sm100_check_device_errors(mcke_stream_t stream) {
  clear_error();
  const cudaError_t e = cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "check_device_errors: %s", cudaGetErrorString(e));
  uint32_t site = 0;
  MCKE_RETURN_IF(read_tc_watchdog(&site));
  if (site == 9) return fail(MCKE_INTERNAL, "watchdog self-test: its bounded wait expired as intended (site 9)");
  if (site != 0) {
    static const char* const kWhere[] = {"", "producer: free stage", "mma: loaded stage", "mma: free accumulator",
                                         "epilogue: full accumulator", "drain", "split-k: previous contributor's flag",
                                         "epilogue warps' meeting", "split of a stage's raw tiles",
                                         "self-test", "tensor-core peak probe's completion"};
    return fail(MCKE_INTERNAL, "gemm (tcgen05): a bounded wait expired (site %u, %s); the kernel stopped early",
                site, site <= 10 ? kWhere[site] : "unknown");
  }
  MCKE_RETURN_IF(read_reduce_watchdog(&site));
  if (site == 2)
    return fail(MCKE_INTERNAL, "reduce (p2p exchange): a peer's partial did not arrive within 1 s; the result is incomplete");
  if (site != 0)
    return fail(MCKE_INTERNAL,
                "reduce (one-kernel step): a CTA's partial did not arrive within 1 s; the result is incomplete");
return MCKE_OK;
}

extern "C" int mcke_sm100_watchdog_selftest(mcke_stream_t stream) {
  clear_error();
  MCKE_RETURN_IF(launch_watchdog_selftest(reinterpret_cast<cudaStream_t>(stream)));
  return check_launch("mcke_sm100_watchdog_selftest");
}

extern "C" int mcke_sm100_gemm_f32(const float* a, const float* b, float* c, int64_t m, int64_t n,
                                   int64_t k, float alpha, float beta, int variant,
                                   mcke_stream_t stream) {
  return gemm_front("mcke_sm100_gemm_f32", a, b, c, m, n, k, false, MCKE_DTYPE_F32, alpha, beta,
                    nullptr, MCKE_ACT_NONE, variant, stream);
}

extern "C" size_t mcke_sm100_gemm_f32_tc_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  return gemm_tf32x3_workspace_bytes(m, n, k);
}

extern "C" int mcke_sm100_gemm_f32_tc(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                                      float alpha, float beta, const float* bias, int act, void* workspace,
                                      size_t workspace_bytes, mcke_stream_t stream) {
  static const char* who = "mcke_sm100_gemm_f32_tc";
  clear_error();
  if (m < 0 || n < 0 || k < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (m == 0 || n == 0) return MCKE_OK;
  if (!a || !b || !c) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (a == c || b == c)
    return fail(MCKE_INVALID_ARGUMENT, "%s: output aliases an input, which violates the __restrict__ contract", who);
  if (m > 2147483647LL || n > 2147483647LL || k > 2147483647LL)
    return fail(MCKE_INVALID_ARGUMENT, "%s: extent exceeds INT32_MAX", who);
  if (act < MCKE_ACT_NONE || act > MCKE_ACT_GELU_TANH)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown activation %d", who, act);
  EpilogueParams ep;
  ep.alpha = alpha;
  ep.beta = beta;
  ep.bias = bias;
  ep.act = act;
  ep.out_bf16 = 0;
  ep.vec_ok = (n % 4 == 0) && aligned(c, 16) ? 1 : 0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (k == 0) {  // C = act(beta * C + bias): no products to split
    MCKE_RETURN_IF(launch_gemm_simt(a, b, c, m, n, k, false, ep, s, nullptr));
    return check_launch(who);
  }
  if (k % 4 != 0 || n % 4 != 0 || !aligned(a, 16) || !aligned(b, 16))
    return fail(MCKE_INVALID_ARGUMENT,
                "%s: needs K %% 4 == 0, N %% 4 == 0 and 16-byte aligned A and B (TMA rows); no fallback is applied",
                who);
  if (!workspace && workspace_bytes == 0) {  // split inside the GEMM kernel
    MCKE_RETURN_IF(launch_gemm_tf32x3_split(a, b, c, m, n, k, ep, s, nullptr, nullptr));
    return check_launch(who);
  }
  const size_t need = gemm_tf32x3_workspace_bytes(m, n, k);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(MCKE_INVALID_ARGUMENT,
                "%s: needs %zu bytes of 256-byte aligned workspace (got %zu); query "
                "mcke_sm100_gemm_f32_tc_workspace_bytes() first",
                who, need, workspace_bytes);
  MCKE_RETURN_IF(launch_gemm_tf32x3(a, b, c, m, n, k, ep, workspace, s, nullptr, nullptr));
  return check_launch(who);
}

extern "C" int mcke_sm100_gemm_bf16(const uint16_t* a, const uint16_t* b, float* c, int64_t m,
                                    int64_t n, int64_t k, float alpha, float beta, int variant,
                                    mcke_stream_t stream) {
  return gemm_front("mcke_sm100_gemm_bf16", a, b, c, m, n, k, true, MCKE_DTYPE_F32, alpha, beta,
                    nullptr, MCKE_ACT_NONE, variant, stream);
}

extern "C" int mcke_sm100_gemm_bf16_ex(const uint16_t* a, const uint16_t* b, void* c, int c_dtype,
                                       int64_t m, int64_t n, int64_t k, float alpha, float beta,
                                       const float* bias, int act, int variant,
                                       mcke_stream_t stream) {
  return gemm_front("mcke_sm100_gemm_bf16_ex", a, b, c, m, n, k, true, c_dtype, alpha, beta, bias,
                    act, variant, stream);
}

extern "C" int mcke_sm100_gemm_plan(int64_t m, int64_t n, int64_t k, int variant, int c_dtype, int sm_count,
                                    mcke_gemm_plan* out) {
  static const char* who = "mcke_sm100_gemm_plan";
  clear_error();
  if (!out) return fail(MCKE_INVALID_ARGUMENT, "%s: null output", who);
  if (m < 0 || n < 0 || k < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (m > 2147483647LL || n > 2147483647LL || k > 2147483647LL)
    return fail(MCKE_INVALID_ARGUMENT, "%s: extent exceeds INT32_MAX", who);
  if (variant < MCKE_GEMM_AUTO || variant > MCKE_GEMM_TCGEN05_SPLIT)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown variant %d", who, variant);
  if (c_dtype != MCKE_DTYPE_F32 && c_dtype != MCKE_DTYPE_BF16)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown output dtype %d", who, c_dtype);
  if (sm_count < 2) return fail(MCKE_INVALID_ARGUMENT, "%s: sm_count must be at least 2", who);
  const bool tc_ok = k > 0 && k % 8 == 0 && n % 8 == 0;
  const bool want_tc = variant != MCKE_GEMM_AUTO && variant != MCKE_GEMM_SIMT;
  if (want_tc && !tc_ok)
    return fail(MCKE_INVALID_ARGUMENT, "%s: the tcgen05 kernel needs k > 0, K %% 8 == 0 and N %% 8 == 0", who);
  *out = mcke_gemm_plan{};
  if (tc_ok && variant != MCKE_GEMM_SIMT) {
    const TcSchedule r = tc_schedule(m, n, k, tile_word(variant), c_dtype == MCKE_DTYPE_BF16, sm_count);
    out->kernel = r.pair ? 2 : 1;
    out->tile_m = r.tile_m;
    out->tile_n = r.tile_n;
    out->tiles = r.tiles;
    out->ctas = (m == 0 || n == 0) ? 0 : r.ctas;
    out->split_dp_tiles = r.split_dp_tiles;
    out->split_kblocks = r.split_kblocks;
  } else {
    out->kernel = 0;
    out->tile_m = 128;
    out->tile_n = 128;
    out->tiles = ((m + 127) / 128) * ((n + 127) / 128);
    out->ctas = out->tiles;
  }
  return MCKE_OK;
}

extern "C" int mcke_sm100_gemm_kernel_attrs(int variant, int in_dtype, mcke_gemm_attrs* out) {
  static const char* who = "mcke_sm100_gemm_kernel_attrs";
  clear_error();
  if (!out) return fail(MCKE_INVALID_ARGUMENT, "%s: null output", who);
  if (in_dtype != MCKE_DTYPE_F32 && in_dtype != MCKE_DTYPE_BF16)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown dtype %d", who, in_dtype);
  const bool bf16 = (in_dtype == MCKE_DTYPE_BF16);
  const void* kernel = nullptr;
  std::size_t dyn = 0;
  int threads = 0;
  EpilogueParams ep{1.0f, 0.0f, nullptr, 0, 0, 1};
  if (bf16 && variant != MCKE_GEMM_SIMT) {
    // M > 128 selects the 2-CTA pair kernel that large shapes run; N = 0 stops
    // the launcher after the choice (both pair tiles have the same footprint).
    launch_gemm_tcgen05(nullptr, nullptr, nullptr, 8192, 0, 0, ep, nullptr, &kernel, &dyn);
    threads = 320;
  } else if (variant == MCKE_GEMM_TCGEN05) {
    return fail(MCKE_INVALID_ARGUMENT, "%s: the tcgen05 kernel takes bf16 operands", who);
  } else {
    // Aligned operands select the float4 instantiation for f32.
    alignas(16) static float dummy[4];
    launch_gemm_simt(dummy, dummy, nullptr, 0, 0, 4, bf16, ep, nullptr, &kernel);
    threads = 256;
  }
  cudaFuncAttributes fa{};
  cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "%s: %s", who, cudaGetErrorString(e));
  out->regs_per_thread = fa.numRegs;
  out->static_smem_bytes = fa.sharedSizeBytes;
  out->dynamic_smem_bytes = dyn;
  out->local_bytes = fa.localSizeBytes;
  out->threads_per_block = threads;
  if (dyn > 0) cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(dyn));
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&out->max_blocks_per_sm_api, kernel, threads, dyn);
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "%s: %s", who, cudaGetErrorString(e));
  return MCKE_OK;
}

extern "C" int mcke_sm100_set_programmatic_launch(int enable) {
  const int prev = pdl_enabled() ? 1 : 0;
  g_pdl.store(enable ? 1 : 0, std::memory_order_relaxed);
  return prev;
}
