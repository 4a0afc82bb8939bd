// bias_act.cu -- fused bias + activation, y[r][c] = act(x[r][c] + bias[c]).
//
// Replaces mini-cuda-kernel-engine kernels/bias_act.cu (launchers :269 :296
// :307; validation :208).  One read of x, one write of y, bias read once per
// thread: the op is HBM-bound, so the design is about bytes in flight.
//
// Layout: block = 256 threads over 256*VW consecutive columns (blockIdx.x),
// each thread owning ROWS rows of that column strip per step (blockIdx.y,
// grid-strided).  The loop is software-pipelined: the ROWS loads of the next
// step are issued before the current step's arithmetic and stores, so a
// thread always has a step of loads in flight while it works; the grid holds
// about 4 blocks per SM (each looping over many steps) rather than one block
// per step.  Measured on config 1 (4096 x 4096): 23.8 us -> 21.0 us (0.97 of
// the measured HBM copy rate).  The bias vector is loaded once per thread for
// the whole kernel.  Loads bypass L1 (ld.global.nc.L1::no_allocate) and stores
// are evict-first (st.global.cs): every byte is touched exactly once.
#include "mcke_common.cuh"

namespace mcke_sm100 {
namespace {

constexpr int kThreads = 256;
constexpr int kRows = 4;  // rows per thread per step

template <int VW>
struct Vec;
template <>
struct Vec<1> {
  using T = float;
  static __device__ __forceinline__ T load(const float* p) { return __ldg(p); }
  static __device__ __forceinline__ void store(float* p, T v) { __stcs(p, v); }
  template <class F>
  static __device__ __forceinline__ T act_bias(T v, T b) { return F::apply(v + b); }
  template <class F>
  static __device__ __forceinline__ T act(T v) { return F::apply(v); }
};
template <>
struct Vec<2> {
  using T = float2;
  static __device__ __forceinline__ T load(const float* p) {
    return __ldg(reinterpret_cast<const float2*>(p));
  }
  static __device__ __forceinline__ void store(float* p, T v) {
    __stcs(reinterpret_cast<float2*>(p), v);
  }
  template <class F>
  static __device__ __forceinline__ T act_bias(T v, T b) {
    return make_float2(F::apply(v.x + b.x), F::apply(v.y + b.y));
  }
  template <class F>
  static __device__ __forceinline__ T act(T v) { return make_float2(F::apply(v.x), F::apply(v.y)); }
};
template <>
struct Vec<4> {
  using T = float4;
  static __device__ __forceinline__ T load(const float* p) { return ld_stream_f4(p); }
  static __device__ __forceinline__ void store(float* p, T v) { st_stream_f4(p, v); }
  template <class F>
  static __device__ __forceinline__ T act_bias(T v, T b) {
    return make_float4(F::apply(v.x + b.x), F::apply(v.y + b.y), F::apply(v.z + b.z),
                       F::apply(v.w + b.w));
  }
  template <class F>
  static __device__ __forceinline__ T act(T v) { return apply4<F>(v); }
};

template <int VW, class F>
__global__ void __launch_bounds__(kThreads) bias_act_f32_kernel(const float* __restrict__ x,
                                                                const float* __restrict__ bias,
                                                                float* __restrict__ y,
                                                                int64_t rows, int64_t cols) {
  pdl_entry();
  using V = Vec<VW>;
  const int64_t col = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * VW;
  if (col >= cols) return;
  const typename V::T b = V::load(bias + col);
  const int64_t step = static_cast<int64_t>(gridDim.y) * kRows;
  int64_t r0 = static_cast<int64_t>(blockIdx.y) * kRows;
  typename V::T cur[kRows], nxt[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i)
    if (r0 + i < rows) cur[i] = V::load(x + (r0 + i) * cols + col);
  for (; r0 < rows; r0 += step) {
    const int64_t r1 = r0 + step;
#pragma unroll
    for (int i = 0; i < kRows; ++i)
      if (r1 + i < rows) nxt[i] = V::load(x + (r1 + i) * cols + col);
#pragma unroll
    for (int i = 0; i < kRows; ++i)
      if (r0 + i < rows) V::store(y + (r0 + i) * cols + col, V::template act_bias<F>(cur[i], b));
#pragma unroll
    for (int i = 0; i < kRows; ++i) cur[i] = nxt[i];
  }
}

// Rows whose width is a multiple of 512 (config 1's 4096 x 4096): one warp per
// 512 contiguous floats of a row, each lane loading its four float4 of x and of
// the bias before any arithmetic, one CTA of 8 warps per 4096 floats and no
// loop.  The same arithmetic per element as bias_act_f32_kernel (same bits).
// In steady state (launches back to back) at 4096 x 4096 on B200: 23.2 us per
// launch against 24.0 us for the strip kernel above (timed alone after an L2
// flush the strip kernel is the faster, 22.5 against 24.6 us).  The reference's
// max_row_blocks knob and the narrower vector widths keep the strip kernel.
// The row of a chunk comes from a shift when chunks_per_row is a power of two
// (cpr_shift >= 0; config 1: 8) and from a 32-bit division otherwise: the
// kernel is issue-bound, and a 64-bit division per thread is a ~70-instruction
// subroutine.
// One warp's 512-float chunk w of x[rows, chunks_per_row * 512].
template <class F>
__device__ __forceinline__ void bias_act_chunk(const float* __restrict__ x, const float* __restrict__ bias,
                                               float* __restrict__ y, uint32_t w, uint32_t chunks_per_row,
                                               int cpr_shift) {
  const int lane = threadIdx.x & 31;
  const uint32_t row = cpr_shift >= 0 ? w >> cpr_shift : w / chunks_per_row;
  const int64_t c0 = static_cast<int64_t>(w - row * chunks_per_row) * 512;
  const int64_t base = static_cast<int64_t>(w) * 512;
  float4 v[4], b[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) v[u] = ld_stream_f4(x + base + 4 * (lane + 32 * u));
#pragma unroll
  for (int u = 0; u < 4; ++u) b[u] = __ldg(reinterpret_cast<const float4*>(bias + c0) + lane + 32 * u);
#pragma unroll
  for (int u = 0; u < 4; ++u)
    st_stream_f4(y + base + 4 * (lane + 32 * u), Vec<4>::template act_bias<F>(v[u], b[u]));
}

template <class F>
__global__ void __launch_bounds__(kThreads) bias_act_f32_chunk_kernel(const float* __restrict__ x,
                                                                      const float* __restrict__ bias,
                                                                      float* __restrict__ y, uint32_t chunks,
                                                                      uint32_t chunks_per_row, int cpr_shift) {
  pdl_entry();
  const uint32_t w = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5);
  if (w >= chunks) return;
  bias_act_chunk<F>(x, bias, y, w, chunks_per_row, cpr_shift);
}

// Up to kGroupMax independent jobs of the chunk kernel in one grid: job k
// owns blocks [first_block[k], first_block[k + 1]).  Each chunk runs the same
// code as in bias_act_f32_chunk_kernel, so the bits are the same.
constexpr int kGroupMax = MCKE_BIAS_ACT_GROUP_MAX;
struct BiasActGroup {
  const float* x[kGroupMax];
  const float* bias[kGroupMax];
  float* y[kGroupMax];
  uint32_t chunks[kGroupMax];
  uint32_t per_row[kGroupMax];
  int32_t shift[kGroupMax];
  uint32_t first_block[kGroupMax + 1];
  int count;
};

template <class F>
__global__ void __launch_bounds__(kThreads) bias_act_f32_group_kernel(const __grid_constant__ BiasActGroup G) {
  pdl_entry();
  int k = 0;
  while (k + 1 < G.count && G.first_block[k + 1] <= blockIdx.x) ++k;
  const uint32_t w = (blockIdx.x - G.first_block[k]) * (kThreads / 32) + (threadIdx.x >> 5);
  if (w >= G.chunks[k]) return;
  bias_act_chunk<F>(G.x[k], G.bias[k], G.y[k], w, G.per_row[k], G.shift[k]);
}

// Activation only (the unfused half): flat grid-stride over n / VW vectors.
template <int VW, class F>
__global__ void __launch_bounds__(kThreads) activation_f32_kernel(const float* __restrict__ x,
                                                                  float* __restrict__ y,
                                                                  int64_t n) {
  pdl_entry();
  using V = Vec<VW>;
  const int64_t nv = n / VW;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < nv; i += stride)
    V::store(y + i * VW, V::template act<F>(V::load(x + i * VW)));
}


// bf16 x/y, float bias and math.  8 elements (16 bytes) per thread per row.
template <class F>
__global__ void __launch_bounds__(kThreads) bias_act_bf16x8_kernel(const uint16_t* __restrict__ x,
                                                                   const float* __restrict__ bias,
                                                                   uint16_t* __restrict__ y,
                                                                   int64_t rows, int64_t cols) {
  pdl_entry();
  const int64_t col = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) * 8;
  if (col >= cols) return;
  float b[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) b[j] = __ldg(bias + col + j);
  const int64_t step = static_cast<int64_t>(gridDim.y) * kRows;
  int64_t r0 = static_cast<int64_t>(blockIdx.y) * kRows;
  uint4 cur[kRows], nxt[kRows];
#pragma unroll
  for (int i = 0; i < kRows; ++i)
    if (r0 + i < rows) cur[i] = ld_stream_u4(x + (r0 + i) * cols + col);
  for (; r0 < rows; r0 += step) {  // software-pipelined like the fp32 kernel
    const int64_t r1 = r0 + step;
#pragma unroll
    for (int i = 0; i < kRows; ++i)
      if (r1 + i < rows) nxt[i] = ld_stream_u4(x + (r1 + i) * cols + col);
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
      if (r0 + i >= rows) continue;
      const uint32_t w[4] = {cur[i].x, cur[i].y, cur[i].z, cur[i].w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        o[j] = pack_bf16x2(F::apply(bf16_lo(w[j]) + b[2 * j]), F::apply(bf16_hi(w[j]) + b[2 * j + 1]));
      st_stream_u4(y + (r0 + i) * cols + col, make_uint4(o[0], o[1], o[2], o[3]));
    }
#pragma unroll
    for (int i = 0; i < kRows; ++i) cur[i] = nxt[i];
  }
}

// Any shape: one element per thread, grid-stride over rows*cols.
template <class F>
__global__ void __launch_bounds__(kThreads) bias_act_bf16_scalar_kernel(
    const uint16_t* __restrict__ x, const float* __restrict__ bias, uint16_t* __restrict__ y,
    int64_t rows, int64_t cols) {
  pdl_entry();
  const int64_t n = rows * cols;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < n; i += stride)
    y[i] = to_bf16(F::apply(from_bf16(x[i]) + bias[i % cols]));
}

int validate_2d(const char* who, const void* x, const void* y, int64_t rows, int64_t cols, int vw) {
  if (!x || !y) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (rows < 0 || cols < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (vw != 1 && vw != 2 && vw != 4)
    return fail(MCKE_INVALID_ARGUMENT, "%s: vector_width must be 1, 2 or 4, got %d", who, vw);
  if (cols % vw != 0)
    return fail(MCKE_INVALID_ARGUMENT,
                "%s: cols (%lld) must be a multiple of vector_width (%d); the launcher refuses "
                "rather than silently running narrower",
                who, static_cast<long long>(cols), vw);
  const std::size_t a = sizeof(float) * static_cast<std::size_t>(vw);
  if (!aligned(x, a) || !aligned(y, a))
    return fail(MCKE_INVALID_ARGUMENT, "%s: pointer not %zu-byte aligned", who, a);
  return MCKE_OK;
}

// Grid: columns across blockIdx.x; row steps across blockIdx.y, about 4 blocks
// per SM in all (each looping over its row steps), at most 65535, at least 1.
dim3 grid_2d(int64_t rows, int64_t cols_vec, int max_row_blocks) {
  const int64_t gx = (cols_vec + kThreads - 1) / kThreads;
  int64_t gy = (rows + kRows - 1) / kRows;
  const int64_t cap = (static_cast<int64_t>(sm_count()) * 4 + gx - 1) / (gx > 0 ? gx : 1);
  if (gy > cap) gy = cap;
  if (gy > 65535) gy = 65535;
  if (max_row_blocks > 0 && gy > max_row_blocks) gy = max_row_blocks;
  if (gy < 1) gy = 1;
  return dim3(static_cast<unsigned>(gx > 0 ? gx : 1), static_cast<unsigned>(gy), 1u);
}

template <int VW>
void launch_bias_act(int act, dim3 g, cudaStream_t s, const float* x, const float* b, float* y,
                     int64_t rows, int64_t cols) {
  switch (act) {
    case MCKE_ACT_RELU: launch_async(bias_act_f32_kernel<VW, ActRelu>, g, kThreads, 0, s, x, b, y, rows, cols); break;
    case MCKE_ACT_GELU_ERF: launch_async(bias_act_f32_kernel<VW, ActGeluErf>, g, kThreads, 0, s, x, b, y, rows, cols); break;
    case MCKE_ACT_GELU_TANH: launch_async(bias_act_f32_kernel<VW, ActGeluTanh>, g, kThreads, 0, s, x, b, y, rows, cols); break;
    default: launch_async(bias_act_f32_kernel<VW, ActNone>, g, kThreads, 0, s, x, b, y, rows, cols); break;
  }
}

bool act_ok(int act) { return act >= MCKE_ACT_NONE && act <= MCKE_ACT_GELU_TANH; }

}  // namespace
}  // namespace mcke_sm100

using namespace mcke_sm100;

extern "C" int mcke_sm100_bias_act_f32(const float* x, const float* bias, float* y, int64_t rows,
                                       int64_t cols, int act, int vector_width,
                                       int max_row_blocks, mcke_stream_t stream) {
  static const char* who = "mcke_sm100_bias_act_f32";
  clear_error();
  if (rows == 0 || cols == 0) return MCKE_OK;
  if (!bias) return fail(MCKE_INVALID_ARGUMENT, "%s: null bias", who);
  MCKE_RETURN_IF(validate_2d(who, x, y, rows, cols, vector_width));
  if (!aligned(bias, sizeof(float) * static_cast<std::size_t>(vector_width)))
    return fail(MCKE_INVALID_ARGUMENT, "%s: bias pointer not aligned", who);
  if (x == y) return fail(MCKE_INVALID_ARGUMENT, "%s: in-place (x == y) is not supported", who);
  if (!act_ok(act)) return fail(MCKE_INVALID_ARGUMENT, "%s: unknown activation %d", who, act);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (vector_width == 4 && max_row_blocks == 0 && cols % 512 == 0 && rows * (cols / 512) < (int64_t{1} << 31)) {
    const uint32_t per_row = static_cast<uint32_t>(cols / 512);
    const uint32_t chunks = static_cast<uint32_t>(rows) * per_row;
    const int shift = (per_row & (per_row - 1)) == 0 ? __builtin_ctz(per_row) : -1;
    const unsigned g = (chunks + 7) / 8;
    switch (act) {
      case MCKE_ACT_RELU: launch_async(bias_act_f32_chunk_kernel<ActRelu>, g, kThreads, 0, s, x, bias, y, chunks, per_row, shift); break;
      case MCKE_ACT_GELU_ERF: launch_async(bias_act_f32_chunk_kernel<ActGeluErf>, g, kThreads, 0, s, x, bias, y, chunks, per_row, shift); break;
      case MCKE_ACT_GELU_TANH: launch_async(bias_act_f32_chunk_kernel<ActGeluTanh>, g, kThreads, 0, s, x, bias, y, chunks, per_row, shift); break;
      default: launch_async(bias_act_f32_chunk_kernel<ActNone>, g, kThreads, 0, s, x, bias, y, chunks, per_row, shift); break;
    }
    return check_launch(who);
  }
  const dim3 g = grid_2d(rows, cols / vector_width, max_row_blocks);
  switch (vector_width) {
    case 4: launch_bias_act<4>(act, g, s, x, bias, y, rows, cols); break;
    case 2: launch_bias_act<2>(act, g, s, x, bias, y, rows, cols); break;
    default: launch_bias_act<1>(act, g, s, x, bias, y, rows, cols); break;
  }
  return check_launch(who);
}

namespace {
bool overlaps(const void* a, std::size_t an, const void* b, std::size_t bn) {
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  return an && bn && pa < pb + bn && pb < pa + an;
}
}  // namespace

extern "C" int mcke_sm100_bias_act_f32_group(const mcke_bias_act_job* jobs, int count, int act,
                                             mcke_stream_t stream) {
  static const char* who = "mcke_sm100_bias_act_f32_group";
  clear_error();
  if (!jobs) return fail(MCKE_INVALID_ARGUMENT, "%s: null job array", who);
  if (count < 1 || count > kGroupMax)
    return fail(MCKE_INVALID_ARGUMENT, "%s: count must be 1..%d, got %d", who, kGroupMax, count);
  if (!act_ok(act)) return fail(MCKE_INVALID_ARGUMENT, "%s: unknown activation %d", who, act);
  BiasActGroup G{};
  G.count = count;
  uint64_t blocks = 0;
  for (int k = 0; k < count; ++k) {
    const mcke_bias_act_job& j = jobs[k];
    if (j.rows < 0 || j.cols < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: job %d: negative extent", who, k);
    G.first_block[k] = static_cast<uint32_t>(blocks);
    if (j.rows == 0 || j.cols == 0) continue;  // nothing to do, as for one call
    if (!j.x || !j.bias || !j.y) return fail(MCKE_INVALID_ARGUMENT, "%s: job %d: null pointer", who, k);
    if (j.cols % 512 != 0)
      return fail(MCKE_INVALID_ARGUMENT, "%s: job %d: cols must be a multiple of 512, got %lld", who, k,
                  static_cast<long long>(j.cols));
    if (!aligned(j.x, 16) || !aligned(j.y, 16) || !aligned(j.bias, 16))
      return fail(MCKE_INVALID_ARGUMENT, "%s: job %d: x, bias and y must be 16-byte aligned", who, k);
    const uint64_t per_row = static_cast<uint64_t>(j.cols / 512);
    const uint64_t chunks = static_cast<uint64_t>(j.rows) * per_row;
    if (chunks >= (uint64_t{1} << 31)) return fail(MCKE_INVALID_ARGUMENT, "%s: job %d: too large", who, k);
    G.x[k] = j.x;
    G.bias[k] = j.bias;
    G.y[k] = j.y;
    G.chunks[k] = static_cast<uint32_t>(chunks);
    G.per_row[k] = static_cast<uint32_t>(per_row);
    G.shift[k] = (per_row & (per_row - 1)) == 0 ? __builtin_ctzll(per_row) : -1;
    blocks += (chunks + 7) / 8;
    if (blocks >= (uint64_t{1} << 31)) return fail(MCKE_INVALID_ARGUMENT, "%s: too many blocks", who);
  }
  G.first_block[count] = static_cast<uint32_t>(blocks);
  // The jobs run at the same time: a job's output may overlap no job's
  // input, bias or output (its own input included: no in-place).
  for (int k = 0; k < count; ++k) {
    const std::size_t yb = static_cast<std::size_t>(G.chunks[k]) * 512 * sizeof(float);
    for (int i = 0; i < count; ++i) {
      const std::size_t xb = static_cast<std::size_t>(G.chunks[i]) * 512 * sizeof(float);
      const std::size_t bb = static_cast<std::size_t>(G.per_row[i]) * 512 * sizeof(float);
      if (overlaps(G.y[k], yb, G.x[i], xb) || overlaps(G.y[k], yb, G.bias[i], bb) ||
          (i != k && overlaps(G.y[k], yb, G.y[i], static_cast<std::size_t>(G.chunks[i]) * 512 * sizeof(float))))
        return fail(MCKE_INVALID_ARGUMENT, "%s: job %d's output overlaps job %d's operands", who, k, i);
    }
  }
  if (blocks == 0) return MCKE_OK;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned g = static_cast<unsigned>(blocks);
  switch (act) {
    case MCKE_ACT_RELU: launch_async(bias_act_f32_group_kernel<ActRelu>, g, kThreads, 0, s, G); break;
    case MCKE_ACT_GELU_ERF: launch_async(bias_act_f32_group_kernel<ActGeluErf>, g, kThreads, 0, s, G); break;
    case MCKE_ACT_GELU_TANH: launch_async(bias_act_f32_group_kernel<ActGeluTanh>, g, kThreads, 0, s, G); break;
    default: launch_async(bias_act_f32_group_kernel<ActNone>, g, kThreads, 0, s, G); break;
  }
  return check_launch(who);
}

extern "C" int mcke_sm100_bias_add_f32(const float* x, const float* bias, float* y, int64_t rows,
                                       int64_t cols, int vector_width, mcke_stream_t stream) {
  return mcke_sm100_bias_act_f32(x, bias, y, rows, cols, MCKE_ACT_NONE, vector_width, 0, stream);
}

namespace mcke_sm100 {
namespace {
template <int VW>
void launch_activation(int act, int blocks, cudaStream_t s, const float* x, float* y, int64_t n) {
  switch (act) {
    case MCKE_ACT_RELU: launch_async(activation_f32_kernel<VW, ActRelu>, blocks, kThreads, 0, s, x, y, n); break;
    case MCKE_ACT_GELU_ERF: launch_async(activation_f32_kernel<VW, ActGeluErf>, blocks, kThreads, 0, s, x, y, n); break;
    case MCKE_ACT_GELU_TANH: launch_async(activation_f32_kernel<VW, ActGeluTanh>, blocks, kThreads, 0, s, x, y, n); break;
    default: launch_async(activation_f32_kernel<VW, ActNone>, blocks, kThreads, 0, s, x, y, n); break;
  }
}
}  // namespace
}  // namespace mcke_sm100

extern "C" int mcke_sm100_activation_f32(const float* x, float* y, int64_t n, int act,
                                         int vector_width, mcke_stream_t stream) {
  static const char* who = "mcke_sm100_activation_f32";
  clear_error();
  if (n == 0) return MCKE_OK;
  if (!x || !y) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (n < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (vector_width != 1 && vector_width != 2 && vector_width != 4)
    return fail(MCKE_INVALID_ARGUMENT, "%s: vector_width must be 1, 2 or 4", who);
  if (n % vector_width != 0)
    return fail(MCKE_INVALID_ARGUMENT, "%s: n must be a multiple of vector_width", who);
  const std::size_t a = sizeof(float) * static_cast<std::size_t>(vector_width);
  if (!aligned(x, a) || !aligned(y, a)) return fail(MCKE_INVALID_ARGUMENT, "%s: pointer not aligned", who);
  if (!act_ok(act)) return fail(MCKE_INVALID_ARGUMENT, "%s: unknown activation %d", who, act);
  const int64_t nv = n / vector_width;
  int64_t blocks = (nv + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (vector_width) {
    case 4: launch_activation<4>(act, static_cast<int>(blocks), s, x, y, n); break;
    case 2: launch_activation<2>(act, static_cast<int>(blocks), s, x, y, n); break;
    default: launch_activation<1>(act, static_cast<int>(blocks), s, x, y, n); break;
  }
  return check_launch(who);
}

extern "C" int mcke_sm100_bias_act_bf16(const uint16_t* x, const float* bias, uint16_t* y,
                                        int64_t rows, int64_t cols, int act,
                                        mcke_stream_t stream) {
  static const char* who = "mcke_sm100_bias_act_bf16";
  clear_error();
  if (rows == 0 || cols == 0) return MCKE_OK;
  if (!x || !y || !bias) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (rows < 0 || cols < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (x == y) return fail(MCKE_INVALID_ARGUMENT, "%s: in-place (x == y) is not supported", who);
  if (!act_ok(act)) return fail(MCKE_INVALID_ARGUMENT, "%s: unknown activation %d", who, act);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cols % 8 == 0 && aligned(x, 16) && aligned(y, 16)) {
    const dim3 g = grid_2d(rows, cols / 8, 0);
    switch (act) {
      case MCKE_ACT_RELU: launch_async(bias_act_bf16x8_kernel<ActRelu>, g, kThreads, 0, s, x, bias, y, rows, cols); break;
      case MCKE_ACT_GELU_ERF: launch_async(bias_act_bf16x8_kernel<ActGeluErf>, g, kThreads, 0, s, x, bias, y, rows, cols); break;
      case MCKE_ACT_GELU_TANH: launch_async(bias_act_bf16x8_kernel<ActGeluTanhBf16>, g, kThreads, 0, s, x, bias, y, rows, cols); break;
      default: launch_async(bias_act_bf16x8_kernel<ActNone>, g, kThreads, 0, s, x, bias, y, rows, cols); break;
    }
  } else {
    int64_t blocks = (rows * cols + kThreads - 1) / kThreads;
    const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
    if (blocks > cap) blocks = cap;
    const unsigned gb = static_cast<unsigned>(blocks);
    switch (act) {
      case MCKE_ACT_RELU: launch_async(bias_act_bf16_scalar_kernel<ActRelu>, gb, kThreads, 0, s, x, bias, y, rows, cols); break;
      case MCKE_ACT_GELU_ERF: launch_async(bias_act_bf16_scalar_kernel<ActGeluErf>, gb, kThreads, 0, s, x, bias, y, rows, cols); break;
      case MCKE_ACT_GELU_TANH: launch_async(bias_act_bf16_scalar_kernel<ActGeluTanhBf16>, gb, kThreads, 0, s, x, bias, y, rows, cols); break;
      default: launch_async(bias_act_bf16_scalar_kernel<ActNone>, gb, kThreads, 0, s, x, bias, y, rows, cols); break;
    }
  }
  return check_launch(who);
}

// ---- vector add (toolchain smoke test) -------------------------------------
// out[i] = a[i] + b[i].  Replaces mini-cuda-kernel-engine kernels/elementwise.cu
// (launch_vector_add_f32 :65): the reference's first-light kernel, kept so a
// new machine can be checked end to end with one exact IEEE add per element.
namespace mcke_sm100 {
namespace {
__global__ void __launch_bounds__(kThreads) vector_add_f32_kernel(const float* __restrict__ a,
                                                                  const float* __restrict__ b,
                                                                  float* __restrict__ out, int64_t n,
                                                                  bool vec) {
  pdl_entry();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (vec) {
    for (int64_t i = t; i < n / 4; i += stride) {
      const float4 x = ld_stream_f4(a + 4 * i), y = ld_stream_f4(b + 4 * i);
      st_stream_f4(out + 4 * i, make_float4(x.x + y.x, x.y + y.y, x.z + y.z, x.w + y.w));
    }
    for (int64_t i = (n / 4) * 4 + t; i < n; i += stride) out[i] = a[i] + b[i];
  } else {
    for (int64_t i = t; i < n; i += stride) out[i] = a[i] + b[i];
  }
}
}  // namespace
}  // namespace mcke_sm100

extern "C" int mcke_sm100_vector_add_f32(const float* a, const float* b, float* out, size_t n,
                                         mcke_stream_t stream) {
  static const char* who = "mcke_sm100_vector_add_f32";
  clear_error();
  if (n == 0) return MCKE_OK;
  if (!a || !b || !out) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  const bool vec = aligned(a, 16) && aligned(b, 16) && aligned(out, 16);
  int64_t blocks = (static_cast<int64_t>(n) / (vec ? 4 : 1) + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  launch_async(vector_add_f32_kernel, static_cast<unsigned>(blocks), kThreads, 0, reinterpret_cast<cudaStream_t>(stream), a, b, out, static_cast<int64_t>(n), vec);
  return check_launch(who);
}
