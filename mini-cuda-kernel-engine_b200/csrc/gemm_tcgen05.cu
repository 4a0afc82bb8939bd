// gemm_tcgen05.cu -- bf16 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[M,N] = act(alpha * A[M,K] @ B[K,N] + beta * C + bias[N]),  A, B bf16
//   row-major, fp32 accumulation in tensor memory, C fp32 or bf16.
//
// Replaces the fp32 SIMT ladder of mini-cuda-kernel-engine kernels/gemm.cu
// (launcher :829) for bf16 operands.  Design:
//
// * Persistent: one 192-thread CTA per SM walks output tiles of 128 x 256 in a
//   grouped order (16 tile-rows per group) so that the A row-panels and B
//   column-panels in use at any moment stay in L2.
// * Warp-specialised:
//     warp 0      TMA producer: per 64-deep k-block, one 128 x 64 box of A and
//                 four 64 x 64 boxes of B, 128-byte swizzled, no multicast;
//     warp 1      allocates 512 TMEM columns and issues tcgen05.mma
//                 (M=128, N=256, K=16; A K-major, B N-major) from one lane,
//                 committing each smem stage back to the producer;
//     warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time, the
//                 fused alpha/beta/bias/activation, global stores.
// * Pipelines: a 4-stage shared-memory ring (48 KB per stage) between TMA and
//   MMA, and two 256-column TMEM accumulators between MMA and epilogue, so the
//   epilogue of tile i overlaps the main loop of tile i+1.
// * Every mbarrier wait is bounded (2 s of %globaltimer).  On expiry the CTA
//   records the site in a device word read by mcke_sm100_check_device_errors,
//   raises a shared abort flag so the other roles stop, waits (bounded) for its
//   own TMA loads and MMAs in flight, frees its TMEM and exits.
//
// Tensor-memory and descriptor encodings follow the PTX ISA for tcgen05
// (instruction descriptor for .kind::f16, shared-memory matrix descriptor with
// version 1 and SWIZZLE_128B), written out by hand below.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "gemm_epilogue.cuh"

namespace mcke_sm100 {
namespace {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int STAGES = 4;
constexpr int UMMA_K = 16;
constexpr int A_STAGE_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BOX_BYTES = 64 * BK * 2;    // one 64(N) x 64(K) box, 8 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int TMEM_COLS = 512;  // two accumulators of BN fp32 columns
constexpr int kThreads = 192;
constexpr int kGroupM = 16;
constexpr int kNumBars = 2 * STAGES + 5;
constexpr std::size_t kSmemBytes =
    static_cast<std::size_t>(STAGES) * STAGE_BYTES + 1024 /*align*/ + 256 /*barriers*/;
constexpr unsigned long long kWaitNs = 2000000000ull;

// Sites reported through the watchdog word (1-based).
enum : uint32_t { kSiteProducer = 1, kSiteMmaFull = 2, kSiteMmaEmpty = 3, kSiteEpilogue = 4, kSiteDrain = 5 };

__device__ uint32_t g_tc_watchdog;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  Returns false when another role raised the abort flag
// (honor_abort) or when the wait itself ran past kWaitNs, in which case it
// raises the flag and records `site`.
__device__ __noinline__ bool wait_bounded(uint32_t bar, uint32_t parity, volatile uint32_t* abort_flag,
                                          uint32_t site, bool honor_abort) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (honor_abort && *abort_flag) return false;
      if (gtimer() - t0 > kWaitNs) {
        *abort_flag = 1u;
        atomicCAS(&g_tc_watchdog, 0u, site);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05): start, leading and stride byte
// offsets in 16-byte units, version 1 at bit 46, layout SWIZZLE_128B (2) at
// bits 61-63, base offset 0 (every stage starts on a 1024-byte boundary).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor, .kind::f16: D f32 (bits 4-5 = 1), A bf16 (7-9 = 1),
// B bf16 (10-12 = 1), A K-major (bit 15 = 0), B N-major (bit 16 = 1),
// N >> 3 at bits 17-22, M >> 4 at bits 24-28.
constexpr uint32_t kInstrDesc = (1u << 4) | (1u << 7) | (1u << 10) | (0u << 15) | (1u << 16) |
                                (static_cast<uint32_t>(BN >> 3) << 17) |
                                (static_cast<uint32_t>(BM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kInstrDesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Grouped raster: tiles advance down kGroupM tile-rows before moving right.
__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int& mb, int& nb) {
  const int per_group = kGroupM * num_n;
  const int group = t / per_group;
  const int first_m = group * kGroupM;
  const int gm = min(num_m - first_m, kGroupM);
  const int r = t - group * per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a,
                        const __grid_constant__ CUtensorMap tmap_b, void* __restrict__ c, int M,
                        int N, int K, EpilogueParams ep) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_STAGE_BYTES);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kNumBars);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 4);

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);  // one arrive per epilogue warp
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (M + BM - 1) / BM;
  const int num_n = (N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (K + BK - 1) / BK;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      // Stages that have had a load issued, and the parity of their latest
      // phase, as bit masks (registers, not a local array).
      uint32_t issued_mask = 0, parity_mask = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, kSiteProducer, true)) {
            ok = false;
            break;
          }
          mbar_expect_tx(full_bar(stage), STAGE_BYTES);
          const uint32_t fb = full_bar(stage);
          tma_load_2d(smem_u32(sA + stage * A_STAGE_BYTES), &tmap_a, fb, kb * BK, mb * BM);
#pragma unroll
          for (int j = 0; j < BN / 64; ++j)
            tma_load_2d(smem_u32(sB + stage * B_STAGE_BYTES + j * B_BOX_BYTES), &tmap_b, fb,
                        nb * BN + 64 * j, kb * BK);
          issued_mask |= 1u << stage;
          parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Do not leave with bulk copies still writing this CTA's shared memory.
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s))
            wait_bounded(full_bar(s), (parity_mask >> s) & 1u, abort_flag, kSiteDrain, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int lt = 0;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++lt) {
        const int acc = lt & 1;
        const uint32_t aphase = static_cast<uint32_t>(lt >> 1) & 1u;
        if (!wait_bounded(tempty_bar(acc), aphase ^ 1u, abort_flag, kSiteMmaEmpty, true)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(full_bar(stage), phase, abort_flag, kSiteMmaFull, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b_base = smem_u32(sB + stage * B_STAGE_BYTES);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // A: K-major SW128, +32 bytes per 16-deep step; SBO = 8 rows x 128 B.
            const uint64_t adesc = smem_desc(a_base + k * (UMMA_K * 2), 16, 1024);
            // B: N-major SW128, +16 rows x 128 B per step; LBO = one 64-wide
            // N box (8 KB), SBO = 8 k-rows x 128 B.
            const uint64_t bdesc = smem_desc(b_base + k * (UMMA_K * 128), B_BOX_BYTES, 1024);
            umma_bf16(d_tmem, adesc, bdesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
      }
      // Every MMA this thread issued has completed once drain_bar flips.
      umma_commit(drain_bar);
      wait_bounded(drain_bar, 0u, abort_flag, kSiteDrain, false);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;  // TMEM lanes 32*quad .. 32*quad+31
    int lt = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++lt) {
      const int acc = lt & 1;
      const uint32_t aphase = static_cast<uint32_t>(lt >> 1) & 1u;
      int ok = 1;
      if (lane == 0) ok = wait_bounded(tfull_bar(acc), aphase, abort_flag, kSiteEpilogue, true) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const int64_t gm = static_cast<int64_t>(mb) * BM + quad * 32 + lane;
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                            static_cast<uint32_t>(acc * BN);
#pragma unroll 1
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld32(trow + static_cast<uint32_t>(chunk * 32), r);
        if (gm < M) {
          const int64_t gn0 = static_cast<int64_t>(nb) * BN + chunk * 32;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            epilogue_store4(ep, c, M, N, gm, gn0 + 4 * j, __uint_as_float(r[4 * j]),
                            __uint_as_float(r[4 * j + 1]), __uint_as_float(r[4 * j + 2]),
                            __uint_as_float(r[4 * j + 3]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base),
                 "r"(TMEM_COLS)
                 : "memory");
  }
}

// ---- host side ------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Row-major [rows, cols] bf16 matrix, box {box_cols (inner), box_rows}.
int make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
             uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05): cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05): cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return MCKE_OK;
}

}  // namespace

bool tcgen05_shape_ok(const void* a, const void* b, const void* c, int64_t m, int64_t n, int64_t k,
                      bool out_bf16) {
  (void)c;
  (void)out_bf16;
  return k > 0 && k % 8 == 0 && n % 8 == 0 && m > 0 && m < (1LL << 31) && n < (1LL << 31) &&
         k < (1LL << 31) && aligned(a, 16) && aligned(b, 16);
}

int launch_gemm_tcgen05(const uint16_t* a, const uint16_t* b, void* c, int64_t m, int64_t n,
                        int64_t k, const EpilogueParams& ep, cudaStream_t s,
                        const void** kernel_out, std::size_t* smem_out) {
  if (kernel_out) *kernel_out = reinterpret_cast<const void*>(&gemm_tcgen05_kernel);
  if (smem_out) *smem_out = kSmemBytes;
  if (m == 0 || n == 0) return MCKE_OK;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05): no device");
  static bool attr_set[64] = {};
  if (dev < 64 && !attr_set[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(gemm_tcgen05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05): %s", cudaGetErrorString(e));
    attr_set[dev] = true;
  }
  CUtensorMap ta, tb;
  MCKE_RETURN_IF(make_map(&ta, a, static_cast<uint64_t>(m), static_cast<uint64_t>(k), 64, BM));
  MCKE_RETURN_IF(make_map(&tb, b, static_cast<uint64_t>(k), static_cast<uint64_t>(n), 64, BK));
  const int64_t tiles = ((m + BM - 1) / BM) * ((n + BN - 1) / BN);
  if (tiles > 2147483647LL) return fail(MCKE_INVALID_ARGUMENT, "gemm (tcgen05): too many tiles");
  int grid = sm_count();
  if (tiles < grid) grid = static_cast<int>(tiles);
  gemm_tcgen05_kernel<<<grid, kThreads, kSmemBytes, s>>>(ta, tb, c, static_cast<int>(m),
                                                         static_cast<int>(n), static_cast<int>(k), ep);
  return MCKE_OK;
}

int read_tc_watchdog(uint32_t* site) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tc_watchdog, sizeof(v));
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "watchdog read: %s", cudaGetErrorString(e));
  if (v != 0) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_tc_watchdog, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "watchdog clear: %s", cudaGetErrorString(e));
  }
  *site = v;
  return MCKE_OK;
}

}  // namespace mcke_sm100
