// gemm_tcgen05.cu -- bf16 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   C[M,N] = act(alpha * A[M,K] @ B[K,N] + beta * C + bias[N]),  A, B bf16
//   row-major, fp32 accumulation in tensor memory, C fp32 or bf16.
//
// Replaces the fp32 SIMT ladder of mini-cuda-kernel-engine kernels/gemm.cu
// (launcher :829) for bf16 operands.  One kernel template, two shapes:
//
//   single (kPair = false): one CTA per SM owns a 128 x 256 output tile and
//     issues tcgen05.mma.cta_group::1 (M=128, N=256, K=16); 4-stage ring of
//     48 KB stages (A 128x64, B 64x256).
//   pair   (kPair = true):  a cluster of two CTAs on two SMs owns a 256 x 256
//     tile.  Each CTA loads its own 128 rows of A and its own 128 columns of B
//     (no multicast: every TMA load targets this CTA's shared memory and
//     signals the leader CTA's barrier, .cta_group::2); the leader issues
//     tcgen05.mma.cta_group::2 (M=256, N=256), which reads A and B from both
//     CTAs' shared memory and accumulates each CTA's 128 rows in that CTA's
//     tensor memory.  Stages are 32 KB per CTA, so the ring is 6 deep, and each
//     SM moves a third less data from L2 per flop than the single shape.
//
// Roles (both shapes): warp 0 = TMA producer (one lane), warp 1 = TMEM
// allocator and MMA issuer (one lane, leader CTA only), warps 2..9 = epilogue
// (two warps per TMEM lane quadrant, alternating 32-column chunks).  Two
// 256-column TMEM accumulators let the epilogue of one tile overlap the main
// loop of the next.  Tiles are walked persistently in a grouped order (16 tile
// rows per group) so the A row panels and B column panels in use stay in L2.
//
// The epilogue is a compile-time functor (output type, bias, activation): the
// 32 values of a chunk are independent, so one warp per scheduler still has
// enough instruction-level parallelism to keep up with the main loop.
//
// Every mbarrier wait is bounded (2 s of %globaltimer).  On expiry the CTA
// records the site in a device word read by mcke_sm100_check_device_errors,
// raises a shared abort flag so its other roles stop, waits (bounded) for
// its own TMA loads and MMAs in flight, frees its TMEM and exits; both CTAs of
// a pair always meet at the final cluster barrier.
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

constexpr int BK = 64;
constexpr int UMMA_K = 16;
constexpr int B_BOX_BYTES = 64 * BK * 2;  // one 64(N) x 64(K) box, 8 KB
constexpr int TMEM_COLS = 512;            // two accumulators of 256 fp32 columns
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // 320
constexpr int kGroupM = 16;
constexpr unsigned long long kWaitNs = 2000000000ull;

template <bool kPair>
struct Cfg {
  static constexpr int BM = 128;                      // rows of A per CTA
  static constexpr int BN = 256;                      // output columns per tile
  static constexpr int TILE_M = kPair ? 2 * BM : BM;  // output rows per tile
  static constexpr int B_COLS = kPair ? BN / 2 : BN;  // columns of B per CTA
  static constexpr int STAGES = kPair ? 6 : 4;
  static constexpr int A_STAGE = BM * BK * 2;
  static constexpr int B_STAGE = B_COLS * BK * 2;
  static constexpr int STAGE = A_STAGE + B_STAGE;
  static constexpr int TX = kPair ? 2 * STAGE : STAGE;  // bytes landing on the leader's full barrier
  static constexpr int EPI_ARRIVALS = kPair ? 2 * kEpiWarps : kEpiWarps;
  static constexpr int NUM_BARS = 2 * STAGES + 5;
  static constexpr std::size_t SMEM = static_cast<std::size_t>(STAGES) * STAGE + 1024 + 256;
  // Instruction descriptor, .kind::f16: D f32 (bits 4-5 = 1), A bf16 (7-9 = 1),
  // B bf16 (10-12 = 1), A K-major (bit 15 = 0), B N-major (bit 16 = 1),
  // N >> 3 at bits 17-22, M >> 4 at bits 24-28.
  static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | (0u << 15) | (1u << 16) |
                                    (static_cast<uint32_t>(BN >> 3) << 17) |
                                    (static_cast<uint32_t>(TILE_M >> 4) << 24);
};
static_assert(Cfg<false>::SMEM <= 232448 && Cfg<true>::SMEM <= 232448, "shared memory budget");

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
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory variable in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
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
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
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

// Bounded wait on a barrier of this CTA.  Returns false when another role
// raised the abort flag (honor_abort) or when the wait itself ran past
// kWaitNs, in which case it raises the flag and records `site`.
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

// TMA tile load into this CTA's shared memory, completing on a barrier of this
// CTA (single) or of the leader CTA of the pair (.cta_group::2).  Never multicast.
template <bool kPair>
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x, int y) {
  if constexpr (kPair) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
  } else {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
        : "memory");
  }
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

template <bool kPair>
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  if constexpr (kPair) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(Cfg<true>::IDESC), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(Cfg<false>::IDESC), "r"(accumulate)
        : "memory");
  }
}

// Arrive on `bar` (same shared-memory offset) once every MMA this thread has
// issued so far has completed: in this CTA (single), or in both CTAs of the
// pair (mask 0b11).
template <bool kPair>
__device__ __forceinline__ void umma_commit_all(uint32_t bar) {
  if constexpr (kPair) {
    const uint16_t mask = 0x3;
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"(mask)
        : "memory");
  } else {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
  }
}
// Arrive on this CTA's `bar` only.
template <bool kPair>
__device__ __forceinline__ void umma_commit_self(uint32_t bar) {
  if constexpr (kPair)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

template <bool kPair>
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem) {
  if constexpr (kPair) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  } else {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
}
template <bool kPair>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr) {
  if constexpr (kPair)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(TMEM_COLS) : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(TMEM_COLS) : "memory");
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

// ---- compile-time epilogue ----------------------------------------------------

template <int kAct>
__device__ __forceinline__ float epi_act(float v) {
  if constexpr (kAct == MCKE_ACT_RELU) return ActRelu::apply(v);
  else if constexpr (kAct == MCKE_ACT_GELU_ERF) return ActGeluErf::apply(v);
  else if constexpr (kAct == MCKE_ACT_GELU_TANH) return ActGeluTanh::apply(v);
  else return v;
}

// 32 accumulator values of row gm, columns gn0 .. gn0+31.
// `fast`: C 16-byte aligned, N % 8 == 0 and bias (if any) 16-byte aligned.
template <bool kBf16Out, bool kBias, int kAct>
__device__ __forceinline__ void epi_chunk(const EpilogueParams& ep, void* c, int N, int64_t gm, int gn0,
                                          const uint32_t (&r)[32], bool fast) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = ep.alpha * __uint_as_float(r[j]);
  const int64_t base = gm * N + gn0;
  if (fast && gn0 + 32 <= N) {
    if constexpr (!kBf16Out) {
      if (ep.beta != 0.0f) {
        const float4* pc = reinterpret_cast<const float4*>(static_cast<const float*>(c) + base);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 p = pc[q];
          v[4 * q] = fmaf(ep.beta, p.x, v[4 * q]);
          v[4 * q + 1] = fmaf(ep.beta, p.y, v[4 * q + 1]);
          v[4 * q + 2] = fmaf(ep.beta, p.z, v[4 * q + 2]);
          v[4 * q + 3] = fmaf(ep.beta, p.w, v[4 * q + 3]);
        }
      }
    }
    if constexpr (kBias) {
      const float4* pb = reinterpret_cast<const float4*>(ep.bias + gn0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = __ldg(pb + q);
        v[4 * q] += b.x;
        v[4 * q + 1] += b.y;
        v[4 * q + 2] += b.z;
        v[4 * q + 3] += b.w;
      }
    }
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = epi_act<kAct>(v[j]);
    if constexpr (kBf16Out) {
      uint4* pc = reinterpret_cast<uint4*>(static_cast<uint16_t*>(c) + base);
#pragma unroll
      for (int q = 0; q < 4; ++q)
        pc[q] = make_uint4(pack_bf16x2(v[8 * q], v[8 * q + 1]), pack_bf16x2(v[8 * q + 2], v[8 * q + 3]),
                           pack_bf16x2(v[8 * q + 4], v[8 * q + 5]), pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
    } else {
      float4* pc = reinterpret_cast<float4*>(static_cast<float*>(c) + base);
#pragma unroll
      for (int q = 0; q < 8; ++q) pc[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
    return;
  }
  // Ragged right edge or unaligned operands: element by element (fully
  // unrolled so v[] stays in registers).
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (gn0 + j >= N) continue;
    float x = v[j];
    if constexpr (!kBf16Out) {
      if (ep.beta != 0.0f) x = fmaf(ep.beta, static_cast<const float*>(c)[base + j], x);
    }
    if constexpr (kBias) x += __ldg(ep.bias + gn0 + j);
    x = epi_act<kAct>(x);
    if constexpr (kBf16Out) static_cast<uint16_t*>(c)[base + j] = to_bf16(x);
    else static_cast<float*>(c)[base + j] = x;
  }
}

// ---- the kernel -------------------------------------------------------------------

template <bool kPair, bool kBf16Out, bool kBias, int kAct>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        void* __restrict__ c, int M, int N, int K, EpilogueParams ep, int fast) {
  using C = Cfg<kPair>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + C::STAGES * C::A_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + C::STAGES * C::B_STAGE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * C::STAGES + 4);

  const int warp = __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0);
  const int lane = threadIdx.x & 31;
  uint32_t rank = 0u;
  if constexpr (kPair) rank = cluster_rank();
  const bool leader = (rank == 0);

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), C::EPI_ARRIVALS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
  }
  if (warp == 1) tmem_alloc<kPair>(smem_u32(tmem_slot));
  tc_fence_before();
  if constexpr (kPair) cluster_sync_all();  // barriers of both CTAs exist before any remote use
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (M + C::TILE_M - 1) / C::TILE_M;
  const int num_n = (N + C::BN - 1) / C::BN;
  const int num_tiles = num_m * num_n;
  const int kblocks = (K + BK - 1) / BK;
  const int unit = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
  const int units = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);

  if (warp == 0) {
    // ---------------- TMA producer (every CTA) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0, parity_mask = 0;  // for the drain on abort (leader)
      bool ok = true;
      for (int t = unit; t < num_tiles && ok; t += units) {
        int mb, nb;
        tile_coords(t, num_m, num_n, mb, nb);
        const int row0 = mb * C::TILE_M + static_cast<int>(rank) * C::BM;
        const int col0 = nb * C::BN + static_cast<int>(rank) * C::B_COLS;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, kSiteProducer, true)) {
            ok = false;
            break;
          }
          uint32_t fb = full_bar(stage);
          if (leader) mbar_expect_tx(fb, C::TX);
          if constexpr (kPair) fb = map_to_rank(fb, 0);
          tma_load_2d<kPair>(smem_u32(sA + stage * C::A_STAGE), &tmap_a, fb, kb * BK, row0);
#pragma unroll
          for (int j = 0; j < C::B_COLS / 64; ++j)
            tma_load_2d<kPair>(smem_u32(sB + stage * C::B_STAGE + j * B_BOX_BYTES), &tmap_b, fb, col0 + 64 * j,
                               kb * BK);
          issued_mask |= 1u << stage;
          parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {
        // Do not leave with bulk copies still landing (their bytes complete
        // on the leader's full barriers).
        for (int s = 0; s < C::STAGES; ++s)
          if (issued_mask & (1u << s))
            wait_bounded(full_bar(s), (parity_mask >> s) & 1u, abort_flag, kSiteDrain, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int lt = 0;
      for (int t = unit; t < num_tiles && ok; t += units, ++lt) {
        const int acc = lt & 1;
        const uint32_t aphase = static_cast<uint32_t>(lt >> 1) & 1u;
        if (!wait_bounded(tempty_bar(acc), aphase ^ 1u, abort_flag, kSiteMmaEmpty, true)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::BN);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!wait_bounded(full_bar(stage), phase, abort_flag, kSiteMmaFull, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(sA + stage * C::A_STAGE);
          const uint32_t b_base = smem_u32(sB + stage * C::B_STAGE);
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            // A: K-major SW128, +32 bytes per 16-deep step; SBO = 8 rows x 128 B.
            const uint64_t adesc = smem_desc(a_base + k * (UMMA_K * 2), 16, 1024);
            // B: N-major SW128, +16 rows x 128 B per step; LBO = one 64-wide
            // N box (8 KB), SBO = 8 k-rows x 128 B.
            const uint64_t bdesc = smem_desc(b_base + k * (UMMA_K * 128), B_BOX_BYTES, 1024);
            umma_bf16<kPair>(d_tmem, adesc, bdesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit_all<kPair>(empty_bar(stage));
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_all<kPair>(tfull_bar(acc));
      }
      // Every MMA this thread issued has completed once drain_bar flips.
      umma_commit_self<kPair>(drain_bar);
      wait_bounded(drain_bar, 0u, abort_flag, kSiteDrain, false);
    }
    __syncwarp();
  } else {
    // ---------------- epilogue (warps 2..9, every CTA) ----------------
    const int quad = warp & 3;             // TMEM lanes 32*quad .. 32*quad+31
    const int half = (warp - 2) >> 2;      // which alternate 32-column chunks
    uint32_t tempty_leader0 = tempty_bar(0);
    if constexpr (kPair) tempty_leader0 = map_to_rank(tempty_leader0, 0);
    int lt = 0;
    for (int t = unit; t < num_tiles; t += units, ++lt) {
      const int acc = lt & 1;
      const uint32_t aphase = static_cast<uint32_t>(lt >> 1) & 1u;
      int ok = 1;
      if (lane == 0) ok = wait_bounded(tfull_bar(acc), aphase, abort_flag, kSiteEpilogue, true) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int mb, nb;
      tile_coords(t, num_m, num_n, mb, nb);
      const int64_t gm = static_cast<int64_t>(mb) * C::TILE_M + static_cast<int>(rank) * C::BM + quad * 32 + lane;
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * C::BN);
#pragma unroll 1
      for (int chunk = half; chunk < C::BN / 32; chunk += 2) {
        uint32_t r[32];
        tmem_ld32(trow + static_cast<uint32_t>(chunk * 32), r);
        if (gm < M) epi_chunk<kBf16Out, kBias, kAct>(ep, c, N, gm, nb * C::BN + chunk * 32, r, fast != 0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) mbar_arrive_cluster(tempty_leader0 + 8u * acc);
        else mbar_arrive(tempty_bar(acc));
      }
    }
  }

  __syncthreads();
  if constexpr (kPair) cluster_sync_all();  // the leader's MMAs have drained before either CTA frees TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc<kPair>(tmem_base);
  }
}

// ---- host side ------------------------------------------------------------------

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

using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, void*, int, int, int, EpilogueParams, int);

template <bool kPair, bool kBf16, bool kBias>
KernelFn pick_act(int act) {
  switch (act) {
    case MCKE_ACT_RELU: return gemm_tcgen05_kernel<kPair, kBf16, kBias, MCKE_ACT_RELU>;
    case MCKE_ACT_GELU_ERF: return gemm_tcgen05_kernel<kPair, kBf16, kBias, MCKE_ACT_GELU_ERF>;
    case MCKE_ACT_GELU_TANH: return gemm_tcgen05_kernel<kPair, kBf16, kBias, MCKE_ACT_GELU_TANH>;
    default: return gemm_tcgen05_kernel<kPair, kBf16, kBias, MCKE_ACT_NONE>;
  }
}

template <bool kPair>
KernelFn pick(bool bf16, bool bias, int act) {
  if (bf16) return bias ? pick_act<kPair, true, true>(act) : pick_act<kPair, true, false>(act);
  return bias ? pick_act<kPair, false, true>(act) : pick_act<kPair, false, false>(act);
}

// Clusters of two that can be resident at once on this device (cached).
int max_pairs(KernelFn k) {
  static std::mutex mu;
  static int cache[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  if (dev >= 0 && dev < 64 && cache[dev] > 0) return cache[dev];
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * (sm_count() / 2), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg<true>::SMEM;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, reinterpret_cast<const void*>(k), &cfg) != cudaSuccess || n <= 0) {
    cudaGetLastError();
    n = sm_count() / 2;
  }
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

bool ensure_smem_attr(KernelFn k, std::size_t bytes) {
  // One attribute call per (kernel, device); cheap enough to keep a small table.
  static std::mutex mu;
  static const void* done_k[256];
  static int done_d[256];
  static int n_done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n_done; ++i)
    if (done_k[i] == reinterpret_cast<const void*>(k) && done_d[i] == dev) return true;
  if (cudaFuncSetAttribute(reinterpret_cast<const void*>(k), cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes)) != cudaSuccess)
    return false;
  if (n_done < 256) {
    done_k[n_done] = reinterpret_cast<const void*>(k);
    done_d[n_done] = dev;
    ++n_done;
  }
  return true;
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
  // A pair tile is 256 rows; below that the single-CTA shape wastes less.
  const bool pair = m > Cfg<false>::BM;
  const bool has_bias = ep.bias != nullptr;
  KernelFn kfn = pair ? pick<true>(ep.out_bf16 != 0, has_bias, ep.act) : pick<false>(ep.out_bf16 != 0, has_bias, ep.act);
  const std::size_t smem = pair ? Cfg<true>::SMEM : Cfg<false>::SMEM;
  if (kernel_out) *kernel_out = reinterpret_cast<const void*>(kfn);
  if (smem_out) *smem_out = smem;
  if (m == 0 || n == 0) return MCKE_OK;
  if (!ensure_smem_attr(kfn, smem)) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05): cannot set shared memory size");
  CUtensorMap ta, tb;
  MCKE_RETURN_IF(make_map(&ta, a, static_cast<uint64_t>(m), static_cast<uint64_t>(k), 64, Cfg<false>::BM));
  MCKE_RETURN_IF(make_map(&tb, b, static_cast<uint64_t>(k), static_cast<uint64_t>(n), 64, BK));
  const int fast = aligned(c, 16) && n % 8 == 0 && (!has_bias || aligned(ep.bias, 16)) ? 1 : 0;
  const int tile_m = pair ? Cfg<true>::TILE_M : Cfg<false>::TILE_M;
  const int64_t tiles = ((m + tile_m - 1) / tile_m) * ((n + 255) / 256);
  if (tiles > 2147483647LL) return fail(MCKE_INVALID_ARGUMENT, "gemm (tcgen05): too many tiles");
  const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
  if (!pair) {
    int grid = sm_count();
    if (tiles < grid) grid = static_cast<int>(tiles);
    kfn<<<grid, kThreads, smem, s>>>(ta, tb, c, mi, ni, ki, ep, fast);
    return MCKE_OK;
  }
  int pairs = max_pairs(kfn);
  if (tiles < pairs) pairs = static_cast<int>(tiles);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, ta, tb, c, mi, ni, ki, ep, fast);
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05 pair): launch failed: %s", cudaGetErrorString(e));
  return MCKE_OK;
}

namespace {
// Watchdog self-test: one thread waits on an mbarrier that nothing arrives on.
// The bounded wait gives up after its limit, records kSiteSelfTest and the
// kernel returns normally, so the context stays usable.
constexpr uint32_t kSiteSelfTest = 6;
__global__ void watchdog_selftest_kernel() {
  __shared__ uint64_t bar;
  __shared__ uint32_t abort_word;
  if (threadIdx.x != 0) return;
  abort_word = 0u;
  mbar_init(smem_u32(&bar), 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  wait_bounded(smem_u32(&bar), 0u, &abort_word, kSiteSelfTest, false);
}
}  // namespace

int launch_watchdog_selftest(cudaStream_t s) {
  watchdog_selftest_kernel<<<1, 32, 0, s>>>();
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
