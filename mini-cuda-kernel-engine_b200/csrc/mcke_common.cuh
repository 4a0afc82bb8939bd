// mcke_common.cuh -- shared plumbing of libmcke_sm100a.so: status codes,
// per-thread error messages, launch checks and small device helpers.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "mcke_sm100.h"

namespace mcke_sm100 {

// Records the message of a failing call for mcke_sm100_last_error_string()
// and returns `code`, so call sites read `return fail(MCKE_..., "...")`.
int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

inline bool aligned(const void* p, std::size_t a) {
  return (reinterpret_cast<std::uintptr_t>(p) % a) == 0;
}

// Checks the launch that was just issued (never synchronises).
inline int check_launch(const char* who) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "%s: launch failed: %s", who, cudaGetErrorString(e));
  return MCKE_OK;
}

#define MCKE_RETURN_IF(expr)          \
  do {                                \
    const int _mcke_rc = (expr);      \
    if (_mcke_rc != MCKE_OK) return _mcke_rc; \
  } while (0)

// Number of SMs of the current device (cached per device).
int sm_count();

// ---- launches ------------------------------------------------------------
//
// Programmatic dependent launch.  Every kernel of this library begins with
// pdl_entry(): it waits until the grid launched before it on the stream has
// completed and its memory operations are visible (griddepcontrol.wait), and
// only then touches global memory; it then lets the next grid on the stream be
// scheduled (griddepcontrol.launch_dependents).  Launched with the
// programmatic-stream-serialization attribute (launch_async, on unless
// mcke_sm100_set_programmatic_launch(0) or MCKE_PDL=0), the next kernel's launch
// and CTA start-up overlap the tail of the kernel before it instead of following
// its completion: ~2 us per launch measured back to back on B200.  Without the
// attribute both instructions return at once.  Results do not depend on it.
__device__ __forceinline__ void pdl_entry() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

bool pdl_enabled();

// Launches `kernel` on `s` (programmatic serialization when enabled).  Errors
// are left for check_launch(), like a <<<>>> launch.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_async(void (*kernel)(KArgs...), dim3 grid, dim3 block, std::size_t smem, cudaStream_t s,
                                Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  if (pdl_enabled()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
}

// ---- device helpers ------------------------------------------------------

// Streaming 128-bit global load: read once, do not keep in L1.
__device__ __forceinline__ float4 ld_stream_f4(const float* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

// Streaming 128-bit global store (evict-first).
__device__ __forceinline__ void st_stream_f4(float* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_stream_u4(void* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}

// bfloat16 <-> float on raw 16-bit patterns.  The narrowing is
// round-to-nearest-even through the hardware cvt (NaN stays NaN).
__device__ __forceinline__ float bf16_lo(uint32_t pair) { return __uint_as_float(pair << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t pair) { return __uint_as_float(pair & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint16_t to_bf16(float v) {
  return static_cast<uint16_t>(pack_bf16x2(v, 0.0f) & 0xFFFFu);
}
__device__ __forceinline__ float from_bf16(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

// ---- activations (values of mcke_activation) ------------------------------
//
// Written in forms that keep their relative accuracy where the textbook form
// cancels.  The reference's CPU oracle evaluates
//   gelu_tanh(v) = 0.5 v (1 + tanh(k (v + 0.044715 v^3)))   (double)
//   gelu_erf(v)  = 0.5 v (1 + erf(v / sqrt 2))             (double)
// In float, 1 + tanh(z) and 1 + erf(t) lose every significant bit once z or t
// is moderately negative.  The identities 1 + tanh(z) = 2 / (1 + e^{-2z}) and
// 1 + erf(t) = erfc(-t) give the same function with no cancellation, so the
// kernels agree with the double-precision oracle to a few ulp over the whole
// range instead of only where y is large.
struct ActNone {
  static __device__ __forceinline__ float apply(float v) { return v; }
};
struct ActRelu {
  // (v > 0) ? v : 0 as in the oracle: relu(-0) = +0 and relu(NaN) = +0.
  static __device__ __forceinline__ float apply(float v) { return v > 0.0f ? v : 0.0f; }
};
struct ActGeluErf {
  static __device__ __forceinline__ float apply(float v) {
    return 0.5f * v * erfcf(-0.70710678118654752f * v);
  }
};
struct ActGeluTanh {
  // v / (1 + e^{-2z}), z = sqrt(2/pi) (v + 0.044715 v^3), with e^{-2z} written
  // as 2^t, t = v (c0 + c1 v^2), c0 = -2 sqrt(2/pi) log2(e), c1 = 0.044715 c0:
  // one hardware base-2 exponential (ex2.approx, relative error below 2^-22)
  // and the IEEE divide.  The rounding of t adds at most |t| 2^-24 ln 2 to the
  // exponential's relative error, and the result carries that error times
  // e/(1+e): about 4e-7 at v = -3 (t = 9.7), and 5e-6 only where |v| > 9 and
  // the result is below 1e-30 in magnitude.  Measured on B200 against
  // float64: at most 8.1e-7 relative wherever |result| > 1e-3 (config 1 and a
  // sweep of [-12, 12]), and no element outside 1e-6 relative + 1e-7
  // absolute.  In the bias kernel at config 1, launches back to back:
  // 22.7-22.8 us against 22.6-23.2 us with CUDA's expf.  Once 2^t overflows
  // (v below about -10.5) the quotient is 0 with v's sign; the exact value
  // there is below 1e-45, and the double-precision oracle already returns 0
  // from v of about -6 on.
  static __device__ __forceinline__ float apply(float v) {
    constexpr float c0 = -2.302208198144325f;
    constexpr float c1 = -0.1029432395800235f;
    const float t = v * fmaf(c1, v * v, c0);
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
    return v / (1.0f + e);
  }
};

// GELU (tanh form) for a bf16 output: v / (1 + e^{-2z}) as in ActGeluTanh,
// with e^{-2z} = 2^{v (c0 + c1 v^2)}: c0 = -2 sqrt(2/pi) log2(e) and
// c1 = 0.044715 c0, one hardware base-2 exponential (ex2.approx, ~2 ulp), then
// the fast divide; the result is rounded to bf16's 8 significant bits right
// after.  At the DAG's 8192 x 16384 the bf16 bias+GELU kernel is issue-bound: CUDA's
// accurate expf took it from 94.2 us (fast exponential) to 102.4 us.
struct ActGeluTanhBf16 {
  static __device__ __forceinline__ float apply(float v) {
    constexpr float c0 = -2.302208198144325;
    constexpr float c1 = -0.1029432395800235;
    const float t = v * fmaf(c1, v * v, c0);
    float e;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(t));
    return __fdividef(v, 1.0f + e);
  }
};

template <class F>
__device__ __forceinline__ float4 apply4(float4 v) {
  return make_float4(F::apply(v.x), F::apply(v.y), F::apply(v.z), F::apply(v.w));
}

__device__ __forceinline__ float act_dispatch(int act, float v) {
  switch (act) {
    case MCKE_ACT_RELU: return ActRelu::apply(v);
    case MCKE_ACT_GELU_ERF: return ActGeluErf::apply(v);
    case MCKE_ACT_GELU_TANH: return ActGeluTanh::apply(v);
    default: return v;
  }
}

}  // namespace mcke_sm100
