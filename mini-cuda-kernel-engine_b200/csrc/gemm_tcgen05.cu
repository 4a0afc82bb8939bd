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
// fp32 operands (kTf32 = true) take the same template through .kind::tf32 in
// the 3xTF32 form: each operand is split into hi = its value with the low 13
// mantissa bits cleared (exact in tf32) and lo = value - hi, and every k-step
// issues A_hi*B_lo + A_lo*B_hi + A_hi*B_hi into the fp32 accumulator, which
// recovers fp32-level accuracy (the dropped lo*lo term and the tf32 rounding
// of lo are ~2^-22 relative).  Rows of 128 bytes hold 32 fp32 values, so a
// k-block is 32 deep and an MMA step 8 deep; a stage holds A, B, A_lo and
// B_lo (64 KB per CTA in the pair shape, 3 stages).  Two ways to split:
//   * kSplit = false: a split pass writes hi and lo of A and of B^T into a
//     caller workspace beforehand, and B is fed K-major;
//   * kSplit = true: TMA loads the raw fp32 tiles -- A K-major, B N-major as
//     stored in SWIZZLE_128B_BASE32B (128-byte rows of 32 floats whose 32-byte
//     chunks are permuted by (row & 3), the layout an MN-major 32-bit operand
//     needs; with the plain 128-byte swizzle an N-major tf32 B accumulated
//     nothing) -- and the epilogue warps write each stage's lo part in
//     shared memory (below) before the MMA reads it.  The raw tile itself
//     serves as hi: a .kind::tf32 MMA reads the top 19 bits of each 32-bit
//     operand and ignores the low 13, which is exactly hi.  No workspace and
//     no extra passes over A and B; the two give the same bits (a GPU test
//     compares them bit for bit, so hardware that read the low bits would
//     fail it).
//
// Tensor-memory and descriptor encodings follow the PTX ISA for tcgen05
// (instruction descriptor for .kind::f16 / .kind::tf32, shared-memory matrix
// descriptor with version 1 and SWIZZLE_128B or SWIZZLE_128B_BASE32B), written
// out by hand below.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <mutex>

#include "gemm_epilogue.cuh"

namespace mcke_sm100 {
namespace {

constexpr int TMEM_COLS = 512;            // two accumulators of 256 fp32 columns
constexpr int kEpiWarps = 8;
constexpr int kThreads = 64 + 32 * kEpiWarps;  // 320
constexpr int kGroupM = 16;
constexpr unsigned long long kWaitNs = 2000000000ull;

template <bool kPair, bool kTf32 = false, bool kWide = false, bool kSplit = false>
struct Cfg {
  static_assert(!kWide || (kPair && !kTf32), "the wide tile is a bf16 pair shape");
  static_assert(!kSplit || kTf32, "the in-kernel hi/lo split is a 3xTF32 shape");
  static constexpr int ELEM = kTf32 ? 4 : 2;          // operand bytes
  static constexpr int BK = 128 / ELEM;               // k-block: one 128-byte swizzle row
  static constexpr int UMMA_K = 32 / ELEM;            // k per MMA: 32 bytes of a row
  static constexpr int BOX_COLS = 128 / ELEM;         // B box: one swizzle row of N
  static constexpr int B_BOX_BYTES = BOX_COLS * BK * ELEM;
  static_assert(B_BOX_BYTES == 128 * BK, "a B box is BK rows of 128 bytes");
  static constexpr int OPS = kTf32 ? 2 : 1;           // hi (+ lo) copies of each operand
  static constexpr int BM = 128;                      // rows of A per CTA
  static constexpr int MMA_N = 256;                   // columns per MMA instruction
  static constexpr int BN = kWide ? 512 : 256;        // output columns per tile
  static constexpr int NH = BN / MMA_N;               // MMA instructions per k-step (N halves)
  static constexpr int NACC = kWide ? 1 : 2;          // TMEM accumulators (512 columns in all)
  static constexpr int TILE_M = kPair ? 2 * BM : BM;  // output rows per tile
  static constexpr int B_COLS = kPair ? BN / 2 : BN;  // columns of B per CTA
  static constexpr int B_HALF_COLS = B_COLS / NH;     // this CTA's columns of one MMA's B
  static constexpr int A_STAGE = BM * BK * ELEM;
  static constexpr int B_STAGE = B_COLS * BK * ELEM;
  static constexpr int STAGE = OPS * (A_STAGE + B_STAGE);  // A, B, then A_lo, B_lo
  static constexpr int STAGES = kTf32 ? (kPair ? 3 : 2) : (kWide ? 4 : (kPair ? 6 : 4));
  // k-blocks per tensor-memory accumulation unit: tf32 partial sums are moved
  // to registers every PROMOTE k-blocks (128 k); bf16 accumulates a whole tile.
  static constexpr int PROMOTE = kTf32 ? 4 : 0;
  // bytes landing on a full barrier: the leader's, for both CTAs' loads of a
  // stage; with kSplit each CTA's own, for its raw A and B tiles
  static constexpr int TX = kSplit ? (A_STAGE + B_STAGE) : (kPair ? 2 * STAGE : STAGE);
  static constexpr int EPI_ARRIVALS = kPair ? 2 * kEpiWarps : kEpiWarps;
  // kSplit: one "converted" barrier per stage, on the leader, one arrival per
  // epilogue warp of either CTA
  static constexpr int NUM_BARS = (kSplit ? 3 : 2) * STAGES + 6;
  // bf16 operands: one 32-row x 128-byte output box per epilogue warp, staged
  // for a TMA store (SWIZZLE_128B, 1024-byte aligned after the stages).
  static constexpr int EPI_BOX_BYTES = 32 * 128;
  static constexpr int EPI_STAGE = kTf32 ? 0 : kEpiWarps * EPI_BOX_BYTES;
  static constexpr std::size_t SMEM = static_cast<std::size_t>(STAGES) * STAGE + EPI_STAGE + 1024 + 256;
  // Instruction descriptor, .kind::f16 / .kind::tf32: D f32 (bits 4-5 = 1),
  // A and B bf16 (1) or tf32 (2) at bits 7-9 and 10-12, A K-major (bit 15 = 0),
  // B N-major (bit 16 = 1; bf16) or K-major (0; tf32), N >> 3 at bits 17-22,
  // M >> 4 at bits 24-28.
  static constexpr uint32_t FMT = kTf32 ? 2u : 1u;
  // bf16: B N-major; tf32 with a split pass: B^T, K-major; tf32 split in the
  // kernel: B as stored, N-major (rows of 32 floats, 128B_BASE32B swizzle)
  static constexpr uint32_t B_MN_MAJOR = kTf32 ? (kSplit ? 1u : 0u) : 1u;
  static constexpr uint32_t IDESC = (1u << 4) | (FMT << 7) | (FMT << 10) | (0u << 15) | (B_MN_MAJOR << 16) |
                                    (static_cast<uint32_t>(MMA_N >> 3) << 17) |
                                    (static_cast<uint32_t>(TILE_M >> 4) << 24);
  static_assert(IDESC != 0u && NH >= 1 && B_HALF_COLS > 0 && FMT > 0u && B_MN_MAJOR <= 1u, "configuration");
};
static_assert(Cfg<false>::SMEM <= 232448 && Cfg<true>::SMEM <= 232448, "shared memory budget");
static_assert(Cfg<false, true>::SMEM <= 232448 && Cfg<true, true>::SMEM <= 232448, "shared memory budget");
static_assert(Cfg<true, false, true>::SMEM <= 232448, "shared memory budget");
static_assert(Cfg<true, true>::B_STAGE % 1024 == 0 && Cfg<false, true>::A_STAGE % 1024 == 0, "stage alignment");
static_assert(Cfg<true, true, false, true>::SMEM <= 232448 && Cfg<false, true, false, true>::SMEM <= 232448,
              "shared memory budget");
static_assert(Cfg<true, true, false, true>::A_STAGE % 1024 == 0 && Cfg<true, true, false, true>::B_STAGE % 1024 == 0 &&
                  Cfg<false, true, false, true>::B_STAGE % 1024 == 0,
              "stage alignment");
static_assert(Cfg<true, true, false, true>::STAGES <= Cfg<true, true, false, true>::PROMOTE &&
                  Cfg<false, true, false, true>::STAGES <= Cfg<false, true, false, true>::PROMOTE,
              "the split runs at most one accumulation unit ahead");

// Sites reported through the watchdog word (1-based).
enum : uint32_t {
  kSiteProducer = 1,
  kSiteMmaFull = 2,
  kSiteMmaEmpty = 3,
  kSiteEpilogue = 4,
  kSiteDrain = 5,
  kSiteSplitFlag = 6,  // a split-k tile's flag from the previous contributor
  kSiteEpiMeet = 7,    // the epilogue warps' meeting on their mbarrier
  kSiteConvert = 8,    // 3xTF32 split in the kernel: a stage's raw tiles
  kSiteSelfTest = 9,   // mcke_sm100_watchdog_selftest only
  kSitePeak = 10       // mcke_sm100_peak_mma_bf16: its MMAs' completion
};

__device__ uint32_t g_tc_watchdog;

// ---- split-k schedule (stream-K) ---------------------------------------------
//
// Whole waves of tiles run one tile per CTA pair; the k-blocks of the tiles
// left over are then divided evenly over all pairs, each pair taking one
// contiguous range of (tile, k-block) in tile-major order.  A tile whose range
// is cut between pairs is summed through its own region of C: contributor j
// (in k order) waits until j contributors have written, adds the sum found
// there to its own partial and writes it back (flag j + 1); the last one adds,
// applies the epilogue and stores.  The sum order is fixed by k, so results do
// not depend on timing.  A pair walks its segments from its last tile down:
// the head of a cut tile is the first thing its owner computes and the tail
// the last thing the next pair computes, so waits are short.
//
// Flags: one 32-bit word per (launch slot, tile, CTA rank), (tag << 8) | j
// while in use, reset to 0 by the last contributor; the host gives every
// launch the next slot of the ring and a fresh tag.  Two split launches that
// run at the same time on one device must be fewer than kSplitSlots launches
// apart (a CUDA graph keeps the slot it was captured with); otherwise a
// waiter can miss its flag and give up after 2 s with watchdog site 6.
// 128 slots x 1024 tiles x 2 CTAs x 4 bytes = 1 MiB per device.
constexpr int kSplitSlots = 128;
constexpr int kSplitMaxTiles = 1024;
__device__ uint32_t g_split_flags[kSplitSlots * kSplitMaxTiles * 2];

struct SplitK {
  int tiles_dp;   // tiles [0, tiles_dp) one per pair; the rest split
  int w;          // k-blocks per pair over the split tiles; 0 = no split
  int slot;       // flag slot of this launch
  uint32_t tag;   // 24-bit launch tag, non-zero
};

struct Seg {
  int tile, kb0, kb1;  // k-blocks [kb0, kb1) of tile
};

// The segments of one pair, in the order every role walks them.
struct SegIter {
  int t, units, dp_end, kblocks;
  int64_t g_beg, g;
  __device__ __forceinline__ SegIter(int unit, int units_, int num_tiles, int kblocks_, const SplitK& sk)
      : t(unit), units(units_), kblocks(kblocks_) {
    dp_end = sk.w > 0 ? sk.tiles_dp : num_tiles;
    if (sk.w > 0) {
      const int64_t total = static_cast<int64_t>(num_tiles - dp_end) * kblocks;
      g_beg = min(static_cast<int64_t>(unit) * sk.w, total);
      g = min(g_beg + sk.w, total);
    } else {
      g_beg = g = 0;
    }
  }
  __device__ __forceinline__ bool next(Seg& sg) {
    if (t < dp_end) {
      sg.tile = t;
      sg.kb0 = 0;
      sg.kb1 = kblocks;
      t += units;
      return true;
    }
    if (g > g_beg) {
      const int64_t tl = (g - 1) / kblocks;
      const int64_t ts = tl * kblocks;
      const int64_t s0 = max(ts, g_beg);
      sg.tile = dp_end + static_cast<int>(tl);
      sg.kb0 = static_cast<int>(s0 - ts);
      sg.kb1 = static_cast<int>(g - ts);
      g = s0;
      return true;
    }
    return false;
  }
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}


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

// Bounded wait for a split-tile flag; a timeout is recorded (site 6) and the
// caller carries on, so no CTA is left waiting.
__device__ __noinline__ void split_wait(const uint32_t* flag, uint32_t want) {
  if (ld_acquire_u32(flag) == want) return;
  const unsigned long long t0 = gtimer();
  for (;;) {
    __nanosleep(64);
    if (ld_acquire_u32(flag) == want) return;
    if (gtimer() - t0 > kWaitNs) {
      atomicCAS(&g_tc_watchdog, 0u, kSiteSplitFlag);
      return;
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

// TMA store of one box from this CTA's shared memory, tracked by this
// thread's bulk async-group.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// This thread's bulk stores have completed.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Generic-proxy writes to shared memory become visible to the async proxy.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05): start, leading and stride byte
// offsets in 16-byte units, version 1 at bit 46, the layout at bits 61-63 --
// SWIZZLE_128B (2), or SWIZZLE_128B_BASE32B (1): 128-byte rows whose 32-byte
// chunks are permuted by (row & 3), the layout an MN-major 32-bit operand
// needs -- base offset 0 (every stage starts on a 1024-byte boundary).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint64_t layout = 2) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (layout << 61);
}

template <bool kPair, bool kTf32, bool kSplit = false>
__device__ __forceinline__ void umma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  constexpr uint32_t idesc = Cfg<kPair, kTf32, false, kSplit>::IDESC;
  if constexpr (kPair && kTf32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (kTf32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else if constexpr (kPair) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
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

// A bf16 output takes the GELU (tanh) with one hardware exponential
// (ActGeluTanhBf16, ~2 fp32 ulp before the bf16 rounding): the wide tile's
// epilogue does not overlap the main loop, and with expf it cost the fused
// DAG more than the separate bias kernel did.
template <int kAct, bool kBf16Out = false>
__device__ __forceinline__ float epi_act(float v) {
  if constexpr (kAct == MCKE_ACT_RELU) return ActRelu::apply(v);
  else if constexpr (kAct == MCKE_ACT_GELU_ERF) return ActGeluErf::apply(v);
  else if constexpr (kAct == MCKE_ACT_GELU_TANH && kBf16Out) return ActGeluTanhBf16::apply(v);
  else if constexpr (kAct == MCKE_ACT_GELU_TANH) return ActGeluTanh::apply(v);
  else return v;
}

// 32 accumulator values of row gm, columns gn0 .. gn0+31.
// `fast`: C 16-byte aligned, N % 8 == 0 and bias (if any) 16-byte aligned.
// v: the 32 accumulator values of columns gn0.. of row gm (scaled in place).
template <bool kBf16Out, bool kBias, int kAct>
__device__ __forceinline__ void epi_vals(const EpilogueParams& ep, void* c, int N, int64_t gm, int gn0, float (&v)[32],
                                         bool fast) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = ep.alpha * v[j];
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
    for (int j = 0; j < 32; ++j) v[j] = epi_act<kAct, kBf16Out>(v[j]);
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
    x = epi_act<kAct, kBf16Out>(x);
    if constexpr (kBf16Out) static_cast<uint16_t*>(c)[base + j] = to_bf16(x);
    else static_cast<float*>(c)[base + j] = x;
  }
}

// alpha, bias and activation on 32 values of columns gn0.. (beta == 0; the
// columns past N, clipped by the store, use no bias).  The same arithmetic,
// in the same order, as epi_vals.
template <bool kBias, int kAct, bool kBf16Out>
__device__ __forceinline__ void epi_math(const EpilogueParams& ep, int N, int gn0, float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = ep.alpha * v[j];
  if constexpr (kBias) {
    if (gn0 + 32 <= N) {
      const float4* pb = reinterpret_cast<const float4*>(ep.bias + gn0);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = __ldg(pb + q);
        v[4 * q] += b.x;
        v[4 * q + 1] += b.y;
        v[4 * q + 2] += b.z;
        v[4 * q + 3] += b.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (gn0 + j < N) v[j] += __ldg(ep.bias + gn0 + j);
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = epi_act<kAct, kBf16Out>(v[j]);
}

template <bool kBf16Out, bool kBias, int kAct>
__device__ __forceinline__ void epi_chunk(const EpilogueParams& ep, void* c, int N, int64_t gm, int gn0,
                                          const uint32_t (&r)[32], bool fast) {
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  epi_vals<kBf16Out, kBias, kAct>(ep, c, N, gm, gn0, v, fast);
}

// ---- the kernel -------------------------------------------------------------------

template <bool kPair, bool kTf32, bool kWide, bool kBf16Out, bool kBias, int kAct, bool kSplit = false>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                        const __grid_constant__ CUtensorMap tmap_alo, const __grid_constant__ CUtensorMap tmap_blo,
                        const __grid_constant__ CUtensorMap tmap_c, void* __restrict__ c, int M, int N, int K,
                        EpilogueParams ep, int fast, SplitK sk) {
  pdl_entry();
  using C = Cfg<kPair, kTf32, kWide, kSplit>;
  constexpr int BK = C::BK;
  constexpr int UMMA_K = C::UMMA_K;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  // Stage s: A, B (and A_lo, B_lo) back to back, each a multiple of 1024 bytes.
  auto sA = [&](int st) { return smem + st * C::STAGE; };
  auto sB = [&](int st) { return smem + st * C::STAGE + C::A_STAGE; };
  auto sAlo = [&](int st) { return smem + st * C::STAGE + C::A_STAGE + C::B_STAGE; };
  auto sBlo = [&](int st) { return smem + st * C::STAGE + 2 * C::A_STAGE + C::B_STAGE; };
  uint8_t* epi_stage = smem + C::STAGES * C::STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(epi_stage + C::EPI_STAGE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NUM_BARS);
  volatile uint32_t* abort_flag = tmem_slot + 1;

  const uint32_t bar0 = smem_u32(bars);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (C::STAGES + s); };
  auto tfull_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + a); };
  auto tempty_bar = [&](int a) { return bar0 + 8u * (2 * C::STAGES + 2 + a); };
  const uint32_t drain_bar = bar0 + 8u * (2 * C::STAGES + 4);
  const uint32_t epi_bar = bar0 + 8u * (2 * C::STAGES + 5);  // the eight epilogue warps
  auto conv_bar = [&](int s) { return bar0 + 8u * (2 * C::STAGES + 6 + s); };  // kSplit only

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
    mbar_init(epi_bar, kEpiWarps);
    if constexpr (kSplit)
      for (int s = 0; s < C::STAGES; ++s) {
        mbar_init(conv_bar(s), C::EPI_ARRIVALS);
      }
    *abort_flag = 0u;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_a)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_b)) : "memory");
    if constexpr (kTf32) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_alo)) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_blo)) : "memory");
    } else {
      if (fast & 2) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmap_c)) : "memory");
    }
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
      SegIter it(unit, units, num_tiles, kblocks, sk);
      Seg sg;
      while (ok && it.next(sg)) {
        int mb, nb;
        tile_coords(sg.tile, num_m, num_n, mb, nb);
        const int row0 = mb * C::TILE_M + static_cast<int>(rank) * C::BM;
        const int col0 = nb * C::BN + static_cast<int>(rank) * C::B_COLS;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          if (!wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, kSiteProducer, true)) {
            ok = false;
            break;
          }
          uint32_t fb = full_bar(stage);
          if constexpr (kSplit) {
            // raw fp32 tiles onto this CTA's own barrier (its epilogue warps
            // split them before the leader's MMA reads them): A K-major, B as
            // stored, B_COLS / 32 boxes of 32 columns x 32 k
            mbar_expect_tx(fb, C::TX);
            tma_load_2d<false>(smem_u32(sA(stage)), &tmap_a, fb, kb * BK, row0);
#pragma unroll
            for (int j = 0; j < C::B_COLS / C::BOX_COLS; ++j)
              tma_load_2d<false>(smem_u32(sB(stage) + j * C::B_BOX_BYTES), &tmap_b, fb, col0 + C::BOX_COLS * j, kb * BK);
            issued_mask |= 1u << stage;
            parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
            if (++stage == C::STAGES) {
              stage = 0;
              phase ^= 1u;
            }
            continue;
          }
          if (leader) mbar_expect_tx(fb, C::TX);
          if constexpr (kPair) fb = map_to_rank(fb, 0);
          tma_load_2d<kPair>(smem_u32(sA(stage)), &tmap_a, fb, kb * BK, row0);
          if constexpr (kTf32) {
            // B^T rows col0.. (K-major): one box of B_COLS rows x 32 k
            tma_load_2d<kPair>(smem_u32(sB(stage)), &tmap_b, fb, kb * BK, col0);
            tma_load_2d<kPair>(smem_u32(sAlo(stage)), &tmap_alo, fb, kb * BK, row0);
            tma_load_2d<kPair>(smem_u32(sBlo(stage)), &tmap_blo, fb, kb * BK, col0);
          } else {
            // per MMA half h: this CTA's B_HALF_COLS columns of that half
#pragma unroll
            for (int h = 0; h < C::NH; ++h) {
              const int hc = nb * C::BN + h * C::MMA_N + static_cast<int>(rank) * C::B_HALF_COLS;
#pragma unroll
              for (int j = 0; j < C::B_HALF_COLS / C::BOX_COLS; ++j)
                tma_load_2d<kPair>(smem_u32(sB(stage) + (h * (C::B_HALF_COLS / C::BOX_COLS) + j) * C::B_BOX_BYTES),
                                   &tmap_b, fb, hc + C::BOX_COLS * j, kb * BK);
            }
          }
          issued_mask |= 1u << stage;
          parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && (leader || kSplit)) {
        // Do not leave with bulk copies still landing (their bytes complete
        // on the leader's full barriers; with kSplit on this CTA's own).
        for (int s = 0; s < C::STAGES; ++s)
          if (issued_mask & (1u << s))
            wait_bounded(full_bar(s), (parity_mask >> s) & 1u, abort_flag, kSiteDrain, false);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA) ----------------
    // Accumulation units alternate between the two TMEM accumulators: one unit
    // per tile (bf16), or one per PROMOTE k-blocks (tf32).
    if (lane == 0 && leader) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int lc = 0;
      const int unit_kb = kTf32 ? C::PROMOTE : kblocks;
      SegIter it(unit, units, num_tiles, kblocks, sk);
      Seg sg;
      while (ok && it.next(sg)) {
        for (int kb0 = sg.kb0; kb0 < sg.kb1 && ok; kb0 += unit_kb, ++lc) {
          const int acc = lc % C::NACC;
          const uint32_t aphase = static_cast<uint32_t>(lc / C::NACC) & 1u;
          if (!wait_bounded(tempty_bar(acc), aphase ^ 1u, abort_flag, kSiteMmaEmpty, true)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * C::BN);
          const int kb1 = min(kb0 + unit_kb, sg.kb1);
          for (int kb = kb0; kb < kb1; ++kb) {
            // kSplit: both CTAs' epilogue warps have split the stage
            if (!wait_bounded(kSplit ? conv_bar(stage) : full_bar(stage), phase, abort_flag, kSiteMmaFull, true)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(sA(stage));
            const uint32_t b_base = smem_u32(sB(stage));
#pragma unroll
            for (int k = 0; k < BK / UMMA_K; ++k) {
              const uint32_t accum = (kb != kb0 || k != 0) ? 1u : 0u;
              // A: K-major SW128, +32 bytes per step; SBO = 8 rows x 128 B.
              const uint64_t adesc = smem_desc(a_base + k * 32, 16, 1024);
              if constexpr (kSplit) {
                // B as stored, N-major with the 128B_BASE32B swizzle: +8 k-rows
                // x 128 B per step; LBO = one 32-column box (32 k-rows x 128 B),
                // SBO = 4 k-rows x 128 B (one swizzle atom).  A_hi*B_lo,
                // A_lo*B_hi, then A_hi*B_hi.
                const uint64_t bdesc = smem_desc(b_base + k * 1024, C::B_BOX_BYTES, 512, 1);
                const uint64_t aldesc = smem_desc(smem_u32(sAlo(stage)) + k * 32, 16, 1024);
                const uint64_t bldesc = smem_desc(smem_u32(sBlo(stage)) + k * 1024, C::B_BOX_BYTES, 512, 1);
                umma<kPair, true, true>(d_tmem, adesc, bldesc, accum);
                umma<kPair, true, true>(d_tmem, aldesc, bdesc, 1u);
                umma<kPair, true, true>(d_tmem, adesc, bdesc, 1u);
              } else if constexpr (kTf32) {
                // B^T: K-major like A.  Small terms first: A_hi*B_lo, A_lo*B_hi,
                // then A_hi*B_hi.
                const uint64_t bdesc = smem_desc(b_base + k * 32, 16, 1024);
                const uint64_t aldesc = smem_desc(smem_u32(sAlo(stage)) + k * 32, 16, 1024);
                const uint64_t bldesc = smem_desc(smem_u32(sBlo(stage)) + k * 32, 16, 1024);
                umma<kPair, true>(d_tmem, adesc, bldesc, accum);
                umma<kPair, true>(d_tmem, aldesc, bdesc, 1u);
                umma<kPair, true>(d_tmem, adesc, bdesc, 1u);
              } else {
                // B: N-major SW128, +UMMA_K rows x 128 B per step; LBO = one
                // BOX_COLS-wide N box, SBO = 8 k-rows x 128 B.  One MMA per
                // 256-column half of the tile, into its own TMEM columns.
#pragma unroll
                for (int h = 0; h < C::NH; ++h) {
                  const uint32_t hb = b_base + h * (C::B_HALF_COLS / C::BOX_COLS) * C::B_BOX_BYTES;
                  const uint64_t bdesc = smem_desc(hb + k * (UMMA_K * 128), C::B_BOX_BYTES, 1024);
                  umma<kPair, false>(d_tmem + h * C::MMA_N, adesc, bdesc, accum);
                }
              }
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
    // Wait for accumulation unit lc; false on abort.
    auto wait_unit = [&](int lc) {
      int ok = 1;
      if (lane == 0)
        ok = wait_bounded(tfull_bar(lc % C::NACC), static_cast<uint32_t>(lc / C::NACC) & 1u, abort_flag,
                          kSiteEpilogue, true)
                 ? 1
                 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (ok) tc_fence_after();
      return ok != 0;
    };
    auto release_unit = [&](int lc) {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) mbar_arrive_cluster(tempty_leader0 + 8u * (lc % C::NACC));
        else mbar_arrive(tempty_bar(lc % C::NACC));
      }
    };
    // The eight epilogue warps meet on an mbarrier (one arrival per warp) with
    // the kernel's bounded wait, so a warp that left early on an abort cannot
    // hold the others.
    uint32_t epi_uses = 0;
    auto epi_sync = [&]() {
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(epi_bar);
        wait_bounded(epi_bar, epi_uses & 1u, abort_flag, kSiteEpiMeet, false);
      }
      __syncwarp();
      ++epi_uses;
    };
    // kSplit: these warps also split every stage of this CTA: lo = value -
    // hi, hi being the value with its low 13 mantissa bits cleared, written
    // into the stage's lo buffers at the raw tile's offsets, so the lo tiles
    // have the raw tiles' swizzled layout; the raw tile stays as it is and
    // the MMA reads it as hi (the tensor core ignores a tf32 operand's low 13
    // bits).  A conversion cursor
    // walks (segment, k-block) in the producer's order and runs ahead of the
    // promotions: before waiting for accumulation unit lc the warps have split
    // every k-block of units <= lc + 1.  (The MMA of unit lc + 1 needs its
    // k-blocks split and the accumulator that unit lc - 1's promotion freed;
    // splitting a k-block waits for its stage, which the MMA of a k-block of
    // unit lc or lc + 1 frees -- STAGES <= PROMOTE -- so nothing waits on
    // itself.)  Each warp fences its writes for the async proxy and arrives on
    // the leader's "converted" barrier (CTA-scope release, as a TMA or MMA
    // completion would).  Measured at 8192^3 on B200 (fp32-equivalent
    // TFLOP/s): this form 253-264, and 242-252 on the same boxes when hi was
    // also written back over the raw tile (4096^3: 233 against 219); with a
    // cluster-scope release per arrival 186 (warps stalled on the fence);
    // with one arrival per CTA after a local barrier 162; with 16-deep
    // k-blocks and 6 stages 217 (twice the per-stage synchronisation); with
    // two extra warps doing all the splits 138.  The split-pass path with a
    // caller workspace: 264-272.
    SegIter cit(unit, units, num_tiles, kblocks, sk);
    Seg csg{};
    bool cvalid = kSplit && cit.next(csg);
    int ckb = cvalid ? csg.kb0 : 0, cunit = 0, cin = 0, cstage = 0;
    uint32_t cphase = 0;
    uint32_t conv_leader0 = conv_bar(0);
    if constexpr (kPair) conv_leader0 = map_to_rank(conv_leader0, 0);
    auto convert_stage = [&](int st, uint32_t ph) -> bool {
      int ok = 1;
      if (lane == 0) ok = wait_bounded(full_bar(st), ph, abort_flag, kSiteConvert, true) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) return false;
      mbar_try(full_bar(st), ph);  // every lane observes the completed phase (acquire)
      const int t = static_cast<int>(threadIdx.x) - 64;  // 0 .. 255 over the eight warps
      auto split = [](const float4* raw, float4* lo) {
        const float4 v = *raw;
        float4 h, l;
        h.x = __uint_as_float(__float_as_uint(v.x) & 0xffffe000u);
        h.y = __uint_as_float(__float_as_uint(v.y) & 0xffffe000u);
        h.z = __uint_as_float(__float_as_uint(v.z) & 0xffffe000u);
        h.w = __uint_as_float(__float_as_uint(v.w) & 0xffffe000u);
        l.x = v.x - h.x;
        l.y = v.y - h.y;
        l.z = v.z - h.z;
        l.w = v.w - h.w;
        *lo = l;
      };
      const float4* a = reinterpret_cast<const float4*>(sA(st)) + t;
      float4* alo = reinterpret_cast<float4*>(sAlo(st)) + t;
      const float4* b = reinterpret_cast<const float4*>(sB(st)) + t;
      float4* blo = reinterpret_cast<float4*>(sBlo(st)) + t;
      constexpr int kStride = 32 * kEpiWarps;
      static_assert(C::A_STAGE % (16 * kStride) == 0 && C::B_STAGE % (16 * kStride) == 0, "whole rounds");
#pragma unroll
      for (int j = 0; j < C::A_STAGE / 16 / kStride; ++j) split(a + j * kStride, alo + j * kStride);
#pragma unroll
      for (int j = 0; j < C::B_STAGE / 16 / kStride; ++j) split(b + j * kStride, blo + j * kStride);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        if constexpr (kPair) mbar_arrive_cluster(conv_leader0 + 8u * st);
        else mbar_arrive(conv_bar(st));
      }
      return true;
    };
    auto convert_through = [&](int upto) -> bool {
      while (cvalid && cunit <= upto) {
        if (!convert_stage(cstage, cphase)) return false;
        if (++cstage == C::STAGES) {
          cstage = 0;
          cphase ^= 1u;
        }
        ++ckb;
        if (++cin == C::PROMOTE) {
          cin = 0;
          ++cunit;
        }
        if (ckb == csg.kb1) {
          if (cin != 0) {
            cin = 0;
            ++cunit;
          }
          cvalid = cit.next(csg);
          if (cvalid) ckb = csg.kb0;
        }
      }
      return true;
    };
    int lc = 0;
    SegIter it(unit, units, num_tiles, kblocks, sk);
    Seg sg;
    while (it.next(sg)) {
      int mb, nb;
      tile_coords(sg.tile, num_m, num_n, mb, nb);
      const int64_t gm = static_cast<int64_t>(mb) * C::TILE_M + static_cast<int>(rank) * C::BM + quad * 32 + lane;
      const uint32_t trow = tmem_base + (static_cast<uint32_t>(quad * 32) << 16);
      if constexpr (!kTf32) {
        if (!wait_unit(lc)) break;
        const uint32_t tacc = trow + static_cast<uint32_t>((lc % C::NACC) * C::BN);
        const bool whole = sg.kb0 == 0 && sg.kb1 == kblocks;
        if (!whole) {
          if constexpr (!kBf16Out) {
            // A cut tile (fp32 output, beta = 0, M and N whole tiles: the
            // host splits nothing else).  Contributor j of the tile in k order.
            const int tl = sg.tile - sk.tiles_dp;
            const uint32_t j =
                static_cast<uint32_t>(unit - static_cast<int>(static_cast<int64_t>(tl) * kblocks / sk.w));
            const bool last = sg.kb1 == kblocks;
            uint32_t* flag = g_split_flags + (static_cast<size_t>(sk.slot) * kSplitMaxTiles + sg.tile) * 2 + rank;
            if (j > 0) {
              if (warp == 2 && lane == 0) split_wait(flag, (sk.tag << 8) | j);
              epi_sync();
              if (last && warp == 2 && lane == 0) st_release_u32(flag, 0u);  // every waiter has passed
            }
            // The running sum of value (row r0 + lane, column u*32 + jj) is kept
            // at (row r0 + jj, column u*32 + lane) of the tile's own region of
            // C: 128 contiguous bytes per warp access.
            const int row0 = static_cast<int>(gm) - lane;
            float* region = static_cast<float*>(c) + static_cast<int64_t>(row0) * N + nb * C::BN + lane;
            const uint32_t box = smem_u32(epi_stage) + static_cast<uint32_t>((warp - 2) * C::EPI_BOX_BYTES);
            const uint32_t my_row = box + static_cast<uint32_t>(lane) * 128u;
            const uint32_t sw = static_cast<uint32_t>(lane & 7);
            if (j > 0) {
              // the running sums were written a while ago: bring every line
              // this warp will read into L2 at once (lane l: line of row l)
#pragma unroll
              for (int u = half; u < C::BN / 32; u += 2)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(region - lane + static_cast<int64_t>(lane) * N + u * 32));
            }
#pragma unroll 1
            for (int u = half; u < C::BN / 32; u += 2) {
              uint32_t r[32];
              tmem_ld32(tacc + static_cast<uint32_t>(u * 32), r);
              float v[32];
              float* blk = region + u * 32;
              if (j > 0) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) v[jj] = __ldcg(blk + static_cast<int64_t>(jj) * N) + __uint_as_float(r[jj]);
              } else {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) v[jj] = __uint_as_float(r[jj]);
              }
              if (!last) {
#pragma unroll
                for (int jj = 0; jj < 32; ++jj) __stcg(blk + static_cast<int64_t>(jj) * N, v[jj]);
              } else {
                const int gn0 = nb * C::BN + u * 32;
                if (lane == 0) bulk_wait_read_all();
                __syncwarp();
                epi_math<kBias, kAct, false>(ep, N, gn0, v);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  st_shared_v4(my_row + ((static_cast<uint32_t>(q) ^ sw) << 4), __float_as_uint(v[4 * q]),
                               __float_as_uint(v[4 * q + 1]), __float_as_uint(v[4 * q + 2]),
                               __float_as_uint(v[4 * q + 3]));
                fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                  tma_store_2d(&tmap_c, box, gn0, row0);
                  bulk_commit();
                }
              }
            }
            if (!last) {
              epi_sync();  // all eight warps have written
              if (warp == 2 && lane == 0) {
                __threadfence();
                st_release_u32(flag, (sk.tag << 8) | (j + 1u));
              }
            }
          }
        } else if (fast & 2) {
          // Through shared memory: this thread writes its row of a 32 x 128-byte
          // box (16-byte granule g at g ^ (row & 7): SWIZZLE_128B, and no bank
          // conflicts), then lane 0 stores the box with TMA, clipped at M and N.
          constexpr int UCOLS = kBf16Out ? 64 : 32;  // output columns per box
          const uint32_t box = smem_u32(epi_stage) + static_cast<uint32_t>((warp - 2) * C::EPI_BOX_BYTES);
          const uint32_t my_row = box + static_cast<uint32_t>(lane) * 128u;
          const uint32_t sw = static_cast<uint32_t>(lane & 7);
          const int row0 = static_cast<int>(gm) - lane;
#pragma unroll 1
          for (int u = half; u < C::BN / UCOLS; u += 2) {
            const int gn0 = nb * C::BN + u * UCOLS;
            if (lane == 0) bulk_wait_read_all();  // the previous box has left the buffer
            __syncwarp();
            // one 32-column TMEM load at a time (bf16: two per box), which keeps
            // the erf GELU's registers within the launch's 168
#pragma unroll 1
            for (int sub = 0; sub < UCOLS / 32; ++sub) {
              uint32_t r[32];
              tmem_ld32(tacc + static_cast<uint32_t>(u * UCOLS + sub * 32), r);
              float v[32];
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
              epi_math<kBias, kAct, kBf16Out>(ep, N, gn0 + sub * 32, v);
              if constexpr (kBf16Out) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  const uint32_t g = static_cast<uint32_t>(4 * sub + q);
                  st_shared_v4(my_row + ((g ^ sw) << 4), pack_bf16x2(v[8 * q], v[8 * q + 1]),
                               pack_bf16x2(v[8 * q + 2], v[8 * q + 3]), pack_bf16x2(v[8 * q + 4], v[8 * q + 5]),
                               pack_bf16x2(v[8 * q + 6], v[8 * q + 7]));
                }
              } else {
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  st_shared_v4(my_row + ((static_cast<uint32_t>(q) ^ sw) << 4), __float_as_uint(v[4 * q]),
                               __float_as_uint(v[4 * q + 1]), __float_as_uint(v[4 * q + 2]),
                               __float_as_uint(v[4 * q + 3]));
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0 && row0 < M && gn0 < N) {
              tma_store_2d(&tmap_c, box, gn0, row0);
              bulk_commit();
            }
          }
        } else {
#pragma unroll 1
          for (int chunk = half; chunk < C::BN / 32; chunk += 2) {
            uint32_t r[32];
            tmem_ld32(tacc + static_cast<uint32_t>(chunk * 32), r);
            if (gm < M) epi_chunk<kBf16Out, kBias, kAct>(ep, c, N, gm, nb * C::BN + chunk * 32, r, fast != 0);
          }
        }
        release_unit(lc);
        ++lc;
      } else {
        // Partial sums of PROMOTE k-blocks each, added in fp32 (round to
        // nearest) in registers: 4 chunks x 32 columns per thread.
        float sum[4][32];
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
          for (int j = 0; j < 32; ++j) sum[q][j] = 0.f;
        bool ok = true;
        for (int kb0 = sg.kb0; kb0 < sg.kb1; kb0 += C::PROMOTE, ++lc) {
          if constexpr (kSplit) {
            if (!convert_through(lc + 1)) {
              ok = false;
              break;
            }
          }
          if (!wait_unit(lc)) {
            ok = false;
            break;
          }
          const uint32_t tacc = trow + static_cast<uint32_t>((lc % C::NACC) * C::BN);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint32_t r[32];
            tmem_ld32(tacc + static_cast<uint32_t>((half + 2 * q) * 32), r);
#pragma unroll
            for (int j = 0; j < 32; ++j) sum[q][j] += __uint_as_float(r[j]);
          }
          release_unit(lc);
        }
        if (!ok) break;
        if (gm < M) {
#pragma unroll
          for (int q = 0; q < 4; ++q)
            epi_vals<kBf16Out, kBias, kAct>(ep, c, N, gm, nb * C::BN + (half + 2 * q) * 32, sum[q], fast != 0);
        }
      }
    }
    // the staged boxes have been written before the CTA's shared memory goes
    if constexpr (!kTf32) {
      if ((fast & 2) && lane == 0) bulk_wait_all();
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

// Row-major [rows, cols] bf16 or fp32 matrix, box {box_cols (inner), box_rows}.
// Swizzle: 128-byte rows (the default), or 128-byte rows with 32-byte chunks
// permuted by row (the layout of an MN-major 32-bit MMA operand).
enum class Sw { k128, k128Atom32 };
int make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_cols,
             uint32_t box_rows, bool fp32 = false, Sw sw = Sw::k128) {
  auto fn = encode_fn();
  if (!fn) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05): cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * (fp32 ? 4 : 2)};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        sw == Sw::k128Atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05): cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return MCKE_OK;
}

using KernelFn = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                          const CUtensorMap, void*, int, int, int, EpilogueParams, int, SplitK);

template <bool kPair, bool kTf32, bool kWide, bool kBf16, bool kBias, bool kSplit = false>
KernelFn pick_act(int act) {
  switch (act) {
    case MCKE_ACT_RELU: return gemm_tcgen05_kernel<kPair, kTf32, kWide, kBf16, kBias, MCKE_ACT_RELU, kSplit>;
    case MCKE_ACT_GELU_ERF: return gemm_tcgen05_kernel<kPair, kTf32, kWide, kBf16, kBias, MCKE_ACT_GELU_ERF, kSplit>;
    case MCKE_ACT_GELU_TANH: return gemm_tcgen05_kernel<kPair, kTf32, kWide, kBf16, kBias, MCKE_ACT_GELU_TANH, kSplit>;
    default: return gemm_tcgen05_kernel<kPair, kTf32, kWide, kBf16, kBias, MCKE_ACT_NONE, kSplit>;
  }
}

// bf16 operands: every output type; fp32 operands (3xTF32): fp32 output.
template <bool kPair, bool kTf32, bool kWide = false, bool kSplit = false>
KernelFn pick(bool bf16, bool bias, int act) {
  if constexpr (kTf32) {
    (void)bf16;
    return bias ? pick_act<kPair, true, false, false, true, kSplit>(act)
                : pick_act<kPair, true, false, false, false, kSplit>(act);
  } else {
    if (bf16)
      return bias ? pick_act<kPair, false, kWide, true, true>(act) : pick_act<kPair, false, kWide, true, false>(act);
    return bias ? pick_act<kPair, false, kWide, false, true>(act) : pick_act<kPair, false, kWide, false, false>(act);
  }
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

bool ensure_smem_attr(const void* k, std::size_t bytes) {
  // One attribute call per (kernel, device); cheap enough to keep a small table.
  static std::mutex mu;
  static const void* done_k[256];
  static int done_d[256];
  static int n_done = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lk(mu);
  for (int i = 0; i < n_done; ++i)
    if (done_k[i] == k && done_d[i] == dev) return true;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(bytes)) != cudaSuccess)
    return false;
  if (n_done < 256) {
    done_k[n_done] = k;
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

namespace {

// Whether the 256 x 512 pair tile beats the 256 x 256 one.  Both run in
// waves of one tile per CTA pair.  Per k the wide tile does twice the work at
// kWideMain of the time (a third fewer L2 bytes per flop), but its single
// accumulator leaves the epilogue (TMA stores) un-overlapped, worth about
// kWideEpiK k of main loop.  Fitted on B200 at 8192 x 8192 x {2048, 8192},
// 8192 x 16384 x 4096, 8192 x 4096 x 16384 and 8192 x 2048 x 8192 (wide 13%
// faster at K = 8192, 9% at K = 4096, even at K = 2048).
constexpr double kWideMain = 0.82;
constexpr double kWideEpiK = 350.0;
// The split-k schedule (see SplitK) needs an fp32 output written through TMA
// boxes with beta = 0 (cut tiles keep their running sums in C) and whole tiles
// in M and N; it is chosen when whole waves would leave more than kSplitBelow
// of the pairs idle.
constexpr double kSplitBelow = 0.95;
// ... and when at least kSplitMinWaves whole waves exist: measured on B200,
// the split pays after data-parallel waves (8192 x 4096 x 8192: 5% faster)
// but not in place of them (8192 x {1024, 2048} x 8192: 8-20% slower), where
// pairs no longer walk k together and the cut tiles' sums leave L2.
constexpr int64_t kSplitMinWaves = 2;
bool split_shape_ok(int64_t m, int64_t n, int tile_n, int64_t tiles, bool tma_fp32_out) {
  return tma_fp32_out && m % 256 == 0 && n % tile_n == 0 && tiles <= kSplitMaxTiles;
}
double busy_fraction(int64_t tiles, int64_t units) {
  const int64_t waves = (tiles + units - 1) / units;
  return static_cast<double>(tiles) / static_cast<double>(waves * units);
}
// Time of a tile count in tile-times: whole waves, or the exact share when the
// split schedule will take the launch.
double tile_waves(int64_t tiles, int64_t units, bool split) {
  if (split && busy_fraction(tiles, units) < kSplitBelow && tiles >= kSplitMinWaves * units)
    return static_cast<double>(tiles) / units;
  return static_cast<double>((tiles + units - 1) / units);
}
bool wide_pays(int64_t m, int64_t n, int64_t k, bool can_split, int64_t units) {
  const int64_t rows = (m + 255) / 256;
  const int64_t narrow = rows * ((n + 255) / 256), wide = rows * ((n + 511) / 512);
  const double t_narrow = tile_waves(narrow, units, can_split && split_shape_ok(m, n, 256, narrow, true));
  const double per_wide = 2.0 * (kWideMain + kWideEpiK / static_cast<double>(k > 0 ? k : 1));
  const double t_wide = per_wide * tile_waves(wide, units, can_split && split_shape_ok(m, n, 512, wide, true));
  return t_wide < t_narrow;
}

// The split-k schedule of a pair launch, or none (w = 0).  Whole waves but
// the last run unsplit, so most tiles keep the data-parallel order.
SplitK plan_split(int64_t tiles, int pairs, int64_t k, int tile_n, int64_t m, int64_t n, bool tma_fp32_out,
                  bool force, bool take_slot = true) {
  SplitK sk = {0, 0, 0, 0u};
  if (!split_shape_ok(m, n, tile_n, tiles, tma_fp32_out) || pairs < 2) return sk;
  if (!force && (busy_fraction(tiles, pairs) >= kSplitBelow || tiles < kSplitMinWaves * pairs)) return sk;
  const int64_t kblocks = (k + Cfg<true>::BK - 1) / Cfg<true>::BK;
  const int64_t dp = tiles / pairs >= 2 ? (tiles / pairs - 1) * pairs : 0;
  const int64_t total = (tiles - dp) * kblocks;
  const int64_t w = (total + pairs - 1) / pairs;
  // short ranges, or more contributors to a tile than the flag's 8 bits count
  if (w < 4 || (kblocks + w - 1) / w + 1 >= 255) return sk;
  sk.tiles_dp = static_cast<int>(dp);
  sk.w = static_cast<int>(w);
  if (!take_slot) return sk;
  static std::atomic<uint32_t> launches{0};
  const uint32_t seq = launches.fetch_add(1u, std::memory_order_relaxed);
  sk.slot = static_cast<int>(seq % kSplitSlots);
  sk.tag = (seq / kSplitSlots) % 0xFFFFFFu + 1u;
  return sk;
}

}  // namespace

// The schedule a bf16 launch of this shape takes on a GPU with `sms` SMs
// (one CTA per SM), by the same rules as launch_tc and with no device query:
// A, B and C 16-byte aligned, beta == 0.
TcSchedule tc_schedule(int64_t m, int64_t n, int64_t k, int tile, bool out_bf16, int sms) {
  TcSchedule r{};
  const int tile_sel = tile & 3, split_sel = (tile >> 2) & 3;
  const bool tma_fp32_out = (n % 8 == 0) && !out_bf16;
  const int pairs = sms / 2;
  r.pair = m > Cfg<false>::BM;
  r.wide = r.pair && n >= 512 &&
           (tile_sel == 2 || (tile_sel == 0 && wide_pays(m, n, k, split_sel != 1 && tma_fp32_out, pairs)));
  r.tile_m = r.pair ? 256 : 128;
  r.tile_n = r.wide ? 512 : 256;
  r.tiles = ((m + r.tile_m - 1) / r.tile_m) * ((n + r.tile_n - 1) / r.tile_n);
  if (!r.pair) {
    r.ctas = r.tiles < sms ? r.tiles : sms;
    return r;
  }
  SplitK sk = {0, 0, 0, 0u};
  if (split_sel != 1) sk = plan_split(r.tiles, pairs, k, r.tile_n, m, n, tma_fp32_out, split_sel == 2, false);
  r.split_dp_tiles = sk.tiles_dp;
  r.split_kblocks = sk.w;
  r.ctas = 2 * (sk.w == 0 && r.tiles < pairs ? r.tiles : pairs);
  return r;
}

namespace {

// Common launcher of both operand types: bf16 (a, b) or 3xTF32 (a, b = the hi
// parts, alo, blo = the lo parts).
template <bool kTf32, bool kSplit = false>
int launch_tc(const void* a, const void* b, const void* alo, const void* blo, void* c, int64_t m, int64_t n,
              int64_t k, const EpilogueParams& ep, cudaStream_t s, const void** kernel_out, std::size_t* smem_out,
              int tile = 0) {
  // A pair tile is 256 rows; below that the single-CTA shape wastes less.
  const bool pair = m > Cfg<false, kTf32>::BM;
  const bool has_bias = ep.bias != nullptr;
  // bf16 pairs: 256 x 256 tiles (two TMEM accumulators, epilogue overlapped
  // with the next tile) or 256 x 512 (one accumulator, a third fewer bytes
  // from L2 per flop).  tile bits 0-1: 0 = choose, 1 = 256 x 256, 2 = 256 x 512;
  // bits 2-3, the split-k schedule: 0 = choose, 1 = never, 2 = wherever it applies.
  const int tile_sel = tile & 3, split_sel = (tile >> 2) & 3;
  // C 16-byte aligned rows and bias: vector epilogue (fast bit 0); with
  // beta == 0 and bf16 operands, TMA-store epilogue (bit 1)
  int fast = aligned(c, 16) && n % 8 == 0 && (!has_bias || aligned(ep.bias, 16)) ? 1 : 0;
  if (!kTf32 && fast && ep.beta == 0.0f) fast |= 2;
  const bool tma_fp32_out = (fast & 2) && !ep.out_bf16;
  bool wide = false;
  if constexpr (!kTf32) {
    if (pair && n >= 512)
      wide = tile_sel == 2 || (tile_sel == 0 && wide_pays(m, n, k, split_sel != 1 && tma_fp32_out, sm_count() / 2));
  }
  KernelFn kfn;
  std::size_t smem;
  if constexpr (!kTf32) {
    if (wide) {
      kfn = pick<true, false, true>(ep.out_bf16 != 0, has_bias, ep.act);
      smem = Cfg<true, false, true>::SMEM;
    } else {
      kfn = pair ? pick<true, kTf32>(ep.out_bf16 != 0, has_bias, ep.act)
                 : pick<false, kTf32>(ep.out_bf16 != 0, has_bias, ep.act);
      smem = pair ? Cfg<true, kTf32>::SMEM : Cfg<false, kTf32>::SMEM;
    }
  } else {
    kfn = pair ? pick<true, kTf32, false, kSplit>(ep.out_bf16 != 0, has_bias, ep.act)
               : pick<false, kTf32, false, kSplit>(ep.out_bf16 != 0, has_bias, ep.act);
    smem = pair ? Cfg<true, kTf32, false, kSplit>::SMEM : Cfg<false, kTf32, false, kSplit>::SMEM;
  }
  if (kernel_out) *kernel_out = reinterpret_cast<const void*>(kfn);
  if (smem_out) *smem_out = smem;
  if (m == 0 || n == 0) return MCKE_OK;
  if (!ensure_smem_attr(reinterpret_cast<const void*>(kfn), smem))
    return fail(MCKE_CUDA_ERROR, "gemm (tcgen05): cannot set shared memory size");
  using C1 = Cfg<false, kTf32, false, kSplit>;
  CUtensorMap ta, tb, talo, tblo;
  if constexpr (kSplit) {
    // raw A [m, k] as for the split pass (32 k x 128 rows); raw B [k, n] as
    // stored, boxes of 32 columns x 32 k (the kernel loads its B_COLS columns
    // as B_COLS / 32 of them) in the 32-byte-atom swizzle
    MCKE_RETURN_IF(make_map(&ta, a, static_cast<uint64_t>(m), static_cast<uint64_t>(k), C1::BK, C1::BM, true));
    MCKE_RETURN_IF(make_map(&tb, b, static_cast<uint64_t>(k), static_cast<uint64_t>(n), C1::BOX_COLS, C1::BK, true,
                            Sw::k128Atom32));
    talo = ta;
    tblo = tb;
  } else {
    MCKE_RETURN_IF(make_map(&ta, a, static_cast<uint64_t>(m), static_cast<uint64_t>(k), C1::BK, C1::BM, kTf32));
  }
  if constexpr (kSplit) {
  } else if constexpr (kTf32) {
    // b, blo are B^T [n, k]: boxes of B_COLS rows (pair: 128, single: 256) x 32 k
    const uint32_t bcols = pair ? Cfg<true, true>::B_COLS : Cfg<false, true>::B_COLS;
    MCKE_RETURN_IF(make_map(&tb, b, static_cast<uint64_t>(n), static_cast<uint64_t>(k), C1::BK, bcols, true));
    MCKE_RETURN_IF(make_map(&talo, alo, static_cast<uint64_t>(m), static_cast<uint64_t>(k), C1::BK, C1::BM, true));
    MCKE_RETURN_IF(make_map(&tblo, blo, static_cast<uint64_t>(n), static_cast<uint64_t>(k), C1::BK, bcols, true));
  } else {
    MCKE_RETURN_IF(make_map(&tb, b, static_cast<uint64_t>(k), static_cast<uint64_t>(n), C1::BOX_COLS, C1::BK));
    talo = ta;
    tblo = tb;
  }
  // bf16 operands: the output leaves through shared memory and TMA stores of
  // 32 x 128-byte boxes (fast bit 1) when C is written, not read (beta == 0).
  CUtensorMap tc = ta;
  if (fast & 2) {
    const bool bf16_out = ep.out_bf16 != 0;
    MCKE_RETURN_IF(make_map(&tc, c, static_cast<uint64_t>(m), static_cast<uint64_t>(n), bf16_out ? 64u : 32u, 32u,
                            !bf16_out));
  }
  const int tile_m = pair ? Cfg<true, kTf32>::TILE_M : Cfg<false, kTf32>::TILE_M;
  const int tile_n = wide ? 512 : 256;
  const int64_t tiles = ((m + tile_m - 1) / tile_m) * ((n + tile_n - 1) / tile_n);
  if (tiles > 2147483647LL) return fail(MCKE_INVALID_ARGUMENT, "gemm (tcgen05): too many tiles");
  const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
  SplitK sk = {0, 0, 0, 0u};
  if (!pair) {
    int grid = sm_count();
    if (tiles < grid) grid = static_cast<int>(tiles);
    launch_async(kfn, grid, kThreads, smem, s, ta, tb, talo, tblo, tc, c, mi, ni, ki, ep, fast, sk);
    return MCKE_OK;
  }
  int pairs = max_pairs(kfn);
  if constexpr (!kTf32) {
    if (split_sel != 1) sk = plan_split(tiles, pairs, k, tile_n, m, n, tma_fp32_out, split_sel == 2);
  }
  if (sk.w == 0 && tiles < pairs) pairs = static_cast<int>(tiles);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kfn, ta, tb, talo, tblo, tc, c, mi, ni, ki, ep, fast, sk);
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "gemm (tcgen05 pair): launch failed: %s", cudaGetErrorString(e));
  return MCKE_OK;
}

// hi = x with the low 13 mantissa bits cleared (exact in tf32), lo = x - hi.
__global__ void __launch_bounds__(256) split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi,
                                                         float* __restrict__ lo, int64_t n) {
  pdl_entry();
  const int64_t n4 = n / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = ld_stream_f4(x + 4 * i);
    float4 h, l;
    h.x = __uint_as_float(__float_as_uint(v.x) & 0xffffe000u);
    h.y = __uint_as_float(__float_as_uint(v.y) & 0xffffe000u);
    h.z = __uint_as_float(__float_as_uint(v.z) & 0xffffe000u);
    h.w = __uint_as_float(__float_as_uint(v.w) & 0xffffe000u);
    l.x = v.x - h.x;
    l.y = v.y - h.y;
    l.z = v.z - h.z;
    l.w = v.w - h.w;
    reinterpret_cast<float4*>(hi)[i] = h;
    reinterpret_cast<float4*>(lo)[i] = l;
  }
  for (int64_t i = 4 * n4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const float h = __uint_as_float(__float_as_uint(x[i]) & 0xffffe000u);
    hi[i] = h;
    lo[i] = x[i] - h;
  }
}

// B [k, n] -> B^T hi and lo [n, k]: 32 x 32 tiles through shared memory
// (reads coalesced along n, writes along k).
__global__ void __launch_bounds__(256) split_tf32_transpose_kernel(const float* __restrict__ b,
                                                                   float* __restrict__ hi_t,
                                                                   float* __restrict__ lo_t, int64_t k,
                                                                   int64_t n) {
  pdl_entry();
  __shared__ float tile[32][33];
  const int64_t n0 = static_cast<int64_t>(blockIdx.x) * 32, k0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
#pragma unroll
  for (int r = ty; r < 32; r += 8) {
    const int64_t kk = k0 + r, nn = n0 + tx;
    tile[r][tx] = (kk < k && nn < n) ? __ldg(b + kk * n + nn) : 0.f;
  }
  __syncthreads();
#pragma unroll
  for (int r = ty; r < 32; r += 8) {
    const int64_t nn = n0 + r, kk = k0 + tx;
    if (nn < n && kk < k) {
      const float v = tile[tx][r];
      const float h = __uint_as_float(__float_as_uint(v) & 0xffffe000u);
      hi_t[nn * k + kk] = h;
      lo_t[nn * k + kk] = v - h;
    }
  }
}

constexpr std::size_t kSplitAlign = 1024;
std::size_t split_bytes(int64_t elems) {
  return (static_cast<std::size_t>(elems) * 4 + kSplitAlign - 1) / kSplitAlign * kSplitAlign;
}

}  // namespace

int launch_gemm_tcgen05(const uint16_t* a, const uint16_t* b, void* c, int64_t m, int64_t n,
                        int64_t k, const EpilogueParams& ep, cudaStream_t s,
                        const void** kernel_out, std::size_t* smem_out, int tile) {
  return launch_tc<false>(a, b, nullptr, nullptr, c, m, n, k, ep, s, kernel_out, smem_out, tile);
}

std::size_t gemm_tf32x3_workspace_bytes(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0) return 0;
  return 2 * split_bytes(m * k) + 2 * split_bytes(k * n);
}

int launch_gemm_tf32x3(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                       const EpilogueParams& ep, void* workspace, cudaStream_t s, const void** kernel_out,
                       std::size_t* smem_out) {
  if (m == 0 || n == 0 || k == 0)
    return launch_tc<true>(nullptr, nullptr, nullptr, nullptr, c, 0, 0, 0, ep, s, kernel_out, smem_out);
  char* w = static_cast<char*>(workspace);
  float* ahi = reinterpret_cast<float*>(w);
  float* alo = reinterpret_cast<float*>(w + split_bytes(m * k));
  float* bhi = reinterpret_cast<float*>(w + 2 * split_bytes(m * k));
  float* blo = reinterpret_cast<float*>(w + 2 * split_bytes(m * k) + split_bytes(k * n));
  const int grid = 4 * sm_count();
  launch_async(split_tf32_kernel, grid, 256, 0, s, a, ahi, alo, m * k);
  const dim3 tgrid(static_cast<unsigned>((n + 31) / 32), static_cast<unsigned>((k + 31) / 32));
  if (tgrid.y > 65535u) return fail(MCKE_INVALID_ARGUMENT, "gemm (3xTF32): K too large for the transpose grid");
  launch_async(split_tf32_transpose_kernel, tgrid, 256, 0, s, b, bhi, blo, k, n);
  return launch_tc<true>(ahi, bhi, alo, blo, c, m, n, k, ep, s, kernel_out, smem_out);
}

// fp32 on the tensor cores with the hi/lo split done inside the GEMM kernel:
// no workspace, no split passes.  Needs K % 4 == 0 and N % 4 == 0 (TMA row
// pitches) and 16-byte aligned A and B.
int launch_gemm_tf32x3_split(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                             const EpilogueParams& ep, cudaStream_t s, const void** kernel_out, std::size_t* smem_out) {
  if (m == 0 || n == 0 || k == 0)
    return launch_tc<true, true>(nullptr, nullptr, nullptr, nullptr, c, 0, 0, 0, ep, s, kernel_out, smem_out);
  return launch_tc<true, true>(a, b, nullptr, nullptr, c, m, n, k, ep, s, kernel_out, smem_out);
}

// Watchdog self-test: one thread waits on an mbarrier that nothing arrives on.
// The bounded wait gives up after its limit, records kSiteSelfTest and the
// kernel returns normally, so the context stays usable.
namespace {
__global__ void watchdog_selftest_kernel() {
  pdl_entry();
  __shared__ uint64_t bar;
  __shared__ uint32_t abort_word;
  if (threadIdx.x != 0) return;
  abort_word = 0u;
  mbar_init(smem_u32(&bar), 1);
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  wait_bounded(smem_u32(&bar), 0u, &abort_word, kSiteSelfTest, false);
}
// ---- tensor-core peak probe ------------------------------------------------------
//
// The bf16 roofline denominator measured with this library's own MMAs: one CTA
// per SM issues `iters` k-blocks of the GEMM's single-CTA instruction
// (tcgen05.mma.cta_group::1.kind::f16, M = 128, N = 256, K = 16, fp32
// accumulator in TMEM; four per 64-deep k-block) on one shared-memory stage laid
// out exactly as the GEMM's (A K-major with the 128-byte swizzle, B N-major in
// 64-column boxes), with no loads and no epilogue.  The operands are bf16
// values of magnitude [0.5, 1) with hashed signs and mantissas, so the
// multipliers switch as they do on real data (zeros would draw less power and
// overstate the clock).  2 * 128 * 256 * 16 flop per MMA.
constexpr int kPeakThreads = 128;
constexpr std::size_t kPeakSmem = 120 * 1024;  // more than half an SM's shared memory: one CTA per SM

__global__ void __launch_bounds__(kPeakThreads, 1) mma_peak_kernel(int iters) {
  pdl_entry();
  using C = Cfg<false>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + C::A_STAGE;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sb + C::B_STAGE);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  volatile uint32_t* abort_word = tmem_slot + 1;
  static_assert(C::A_STAGE + C::B_STAGE + 1024 + 64 <= kPeakSmem, "probe shared memory");
  uint32_t* w = reinterpret_cast<uint32_t*>(smem);
  for (int i = static_cast<int>(threadIdx.x); i < (C::A_STAGE + C::B_STAGE) / 4; i += kPeakThreads) {
    uint32_t h = static_cast<uint32_t>(i) * 2654435761u;
    h ^= h >> 15;
    h *= 2246822519u;
    h ^= h >> 13;
    const uint32_t lo = ((h & 1u) << 15) | (126u << 7) | ((h >> 1) & 0x7Fu);
    const uint32_t hi = (((h >> 8) & 1u) << 15) | (126u << 7) | ((h >> 9) & 0x7Fu);
    w[i] = lo | (hi << 16);
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    *abort_word = 0u;
    mbar_init(smem_u32(bar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < 32) tmem_alloc<false>(smem_u32(tmem_slot));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (threadIdx.x == 0) {
    const uint32_t a_base = smem_u32(sa), b_base = smem_u32(sb);
    for (int it = 0; it < iters; ++it) {
#pragma unroll
      for (int k = 0; k < C::BK / C::UMMA_K; ++k) {
        const uint64_t adesc = smem_desc(a_base + k * 32, 16, 1024);
        const uint64_t bdesc = smem_desc(b_base + k * (C::UMMA_K * 128), C::B_BOX_BYTES, 1024);
        umma<false, false>(tmem, adesc, bdesc, (it | k) != 0 ? 1u : 0u);
      }
    }
    // every MMA issued above has completed once the barrier's phase 0 does;
    // on a timeout (recorded, site 10) wait once more before TMEM is freed
    umma_commit_self<false>(smem_u32(bar));
    if (!wait_bounded(smem_u32(bar), 0u, abort_word, kSitePeak, false))
      wait_bounded(smem_u32(bar), 0u, abort_word, kSitePeak, false);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x < 32) tmem_dealloc<false>(tmem);
}
}  // namespace

double mma_peak_flops_per_cta_iter() { return 4.0 * 2.0 * 128.0 * 256.0 * 16.0; }

int launch_mma_peak(int64_t ctas, int iters, cudaStream_t s) {
  if (!ensure_smem_attr(reinterpret_cast<const void*>(mma_peak_kernel), kPeakSmem))
    return fail(MCKE_CUDA_ERROR, "mcke_sm100_peak_mma_bf16: cannot set shared memory size");
  launch_async(mma_peak_kernel, static_cast<unsigned>(ctas), kPeakThreads, kPeakSmem, s, iters);
  return MCKE_OK;
}

int launch_watchdog_selftest(cudaStream_t s) {
  launch_async(watchdog_selftest_kernel, 1, 32, 0, s);
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
