// reduce.cu -- full-vector sum/max/argmax and row-wise sum/max/mean.
//
// Replaces mini-cuda-kernel-engine kernels/reduce.cu (launchers :224 and :285,
// row_reduce_workspace_bytes :213, two_pass_split :65) and the primitives of
// kernels/reduce_ops.cuh (SumOp/MaxOp :38-53, warp_reduce :83, block_reduce
// :103).  Both reductions read their input once with 128-bit streaming loads.
//
// Numerics.  The reference's CPU oracle accumulates sums serially in double and
// rounds once (tests/reference.hpp:154-172); these kernels also accumulate in
// double -- each thread over its own elements, then a fixed-shape combine tree
// -- and round once, so the float result is the oracle's unless the two double
// sums straddle a float rounding boundary.  The combine tree depends only on
// the extents (never on the device or on timing), so results are bitwise
// reproducible run to run.  Max is the std::max fold of the oracle: NaN never
// replaces the running maximum, the identity is -inf.  Argmax is the lowest
// index holding the maximum; each thread visits its elements in increasing
// index order and the combine breaks value ties by index.
#include <cfloat>
#include <cstring>
#include <mutex>

#include "mcke_common.cuh"

namespace mcke_sm100 {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 4;
// Pass-1 grid cap: 8 resident 256-thread blocks on each of a B200's 148 SMs.
// A constant, not a device query, so the combine tree (and therefore every
// bit of the sum) is the same on any GPU.
constexpr int64_t kMaxBlocks = 8 * 148;

struct Part {
  double s;
  float m;
  int32_t reserved;
  long long i;
};
static_assert(sizeof(Part) == sizeof(mcke_reduce_partial), "partial layout");

__device__ __forceinline__ Part part_identity() { return Part{0.0, -INFINITY, 0, -1}; }

__device__ __forceinline__ void part_add(Part& p, float v, long long idx) {
  p.s += static_cast<double>(v);
  if (v > p.m || (p.i < 0 && v == p.m)) {
    p.m = v;
    p.i = idx;
  }
}

__device__ __forceinline__ Part part_combine(const Part& a, const Part& b) {
  Part r;
  r.s = a.s + b.s;
  r.reserved = 0;
  const bool take_b = (b.i >= 0) && (a.i < 0 || b.m > a.m || (b.m == a.m && b.i < a.i));
  r.m = take_b ? b.m : a.m;
  r.i = take_b ? b.i : a.i;
  return r;
}

__device__ __forceinline__ Part part_shfl_xor(const Part& p, int o) {
  Part q;
  q.s = __shfl_xor_sync(0xffffffffu, p.s, o);
  q.m = __shfl_xor_sync(0xffffffffu, p.m, o);
  q.i = __shfl_xor_sync(0xffffffffu, p.i, o);
  q.reserved = 0;
  return q;
}

// Called by all 32 lanes of a warp.  It reconverges them first: lanes that
// left a loop or a branch at different times would otherwise run the FP64
// steps one divergent group at a time.
__device__ __forceinline__ Part warp_butterfly(Part p) {
  __syncwarp();
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) p = part_combine(p, part_shfl_xor(p, o));
  return p;
}

// Fixed-shape block combine: xor butterfly in each warp (every lane ends with
// the same bits: the combine is commutative), then warp 0 runs the same
// butterfly over the warp results (lane w takes warp w's, lanes past the last
// warp the identity).  The result is valid in thread 0 only.
__device__ __forceinline__ Part block_combine(Part p, Part* red) {
  p = warp_butterfly(p);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = p;
  __syncthreads();
  if (threadIdx.x < 32) {
    p = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : part_identity();
    p = warp_butterfly(p);
  }
  return p;
}

// Pass-1 grid of the streamed kernel: one CTA per 16 KB chunk up to 3 per SM
// of a B200 (a constant, so the combine tree is the same on any GPU).
constexpr int64_t kFullCtaCap = 3 * 148;
static_assert(kFullCtaCap < 2 * kThreads && 2 * kThreads / 32 <= 16,
              "the P2P collector polls at most two part slots per thread");
int64_t full_blocks(int64_t n) {
  const int64_t per_block = 4096;  // floats per chunk
  int64_t g = (n + per_block - 1) / per_block;
  if (g > kFullCtaCap) g = kFullCtaCap;
  return g < 1 ? 1 : g;
}

// Pass 1.  Thread g of the grid (G CTAs of 256) reads float4 g, g + 256 G,
// g + 512 G, ... of the 16-byte aligned body, kLoads of them in flight at a
// time (128-bit loads that bypass L1), and accumulates them in per-thread
// increasing index order: the sum in double, the running maximum once per
// float4.  On an update the float4's index and its first element equal to
// the maximum (its own bits, so a -0 ahead of a +0 wins) are remembered; a
// later float4 with an equal maximum never replaces an earlier one, so the
// lowest index survives.  Head and tail elements (outside whole 16-byte
// float4s) go to global thread 0: head first, tail last.  Measured on B200
// (events, L2 flushed, both launches) against the first version, a ring of
// 16 KB bulk copies into shared memory per CTA with two CTA barriers per
// chunk: 2^23 floats 21.5 -> 17.4 us, 2^25 35.8 -> 33.8 us, 2^28 175.1 ->
// 166.9 us (6.43 TB/s): no barrier per chunk, and a round's loads overlap
// the previous round's FP64 adds.
constexpr int kLoads = 4;

__device__ uint32_t g_reduce_watchdog;

// ---- peer-to-peer combine of a sharded full reduce ----------------------------
//
// For one process per GPU: rank r's result slot lives in every rank's exchange
// buffer; a call stores this rank's shard partial into slot `rank` of every
// rank's buffer (peer memory over NVLink), waits (bounded) until each slot of
// its own buffer carries the call's tag and folds the slots in rank order.
// Slots use a low-latency format: each 8-byte word holds 4 bytes of the
// partial and the 4-byte tag (the epoch), and an aligned 8-byte store is
// single-copy atomic, so a reader that sees the tag in all six words has the
// whole partial -- no fence on either side.  Slots are double-buffered by
// epoch parity: a rank can run at most one epoch ahead of a peer that is still
// reading, so the halves never collide.  After the 2 * world exchange slots
// each buffer holds kFullCtaCap slots of the same format for the pass-1
// partials of this rank's own call (only this GPU touches them).
struct LLSlot {
  unsigned long long w[8];  // words 0..5: data | tag << 32; 6, 7 unused
};
static_assert(sizeof(LLSlot) == 64, "slot layout");
constexpr unsigned long long kP2pWaitNs = 1000000000ull;

struct P2pArgs {
  LLSlot* const* peers;  // device table: every rank's buffer as mapped here
  mcke_reduce_result* out;
  uint32_t tag;
  uint32_t parity;
  int world;
  int rank;
  int auto_epoch;  // 1: the epoch is the counter after the part area, advanced by each call
  unsigned long long* stamps;  // null, or the kStamp* phase times of this call (%globaltimer, ns)
};

// Phase times of one call of the one-kernel reduce, for the fixed-cost
// breakdown (mcke_sm100_reduce_full_p2p_f32_timeline).  Min slots start at
// ~0, max slots at 0; the last CTA's slots are plain stores.
enum : int {
  kStampFirstEntry = 0,   // min over CTAs: entry, before the wait for the previous grid
  kStampFirstStart = 1,   // min over CTAs: the previous grid's memory is visible, streaming starts
  kStampLastStart = 2,    // max over CTAs: the last CTA starts streaming (dispatch ramp)
  kStampFirstDone = 3,    // min over CTAs: a CTA has its block partial
  kStampLastDone = 4,     // max over CTAs: the last CTA has its block partial
  kStampFolded = 5,       // the last CTA has folded all block partials (the shard partial)
  kStampExchanged = 6,    // the ranks' partials are combined and the result stored
  kStampCounted = 7,      // the last CTA's arrival has come back: it knows it is last
  kStampWords = 8,
};
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Counter of the automatic epochs: the 64-byte slot after the part area
// (first 8 bytes); the CTAs' arrival count of the current call follows it
// (bytes 8-11, back at 0 between calls).
__device__ __forceinline__ unsigned long long* epoch_counter(const P2pArgs& a) {
  return reinterpret_cast<unsigned long long*>(a.peers[a.rank] + 2 * a.world + kFullCtaCap);
}
__device__ __forceinline__ unsigned int* arrival_count(const P2pArgs& a) {
  return reinterpret_cast<unsigned int*>(epoch_counter(a) + 1);
}

// With automatic epochs, resolve this call's tag (every CTA reads the counter
// before it publishes; CTA 0 advances it only after all CTAs have published).
__device__ __forceinline__ void resolve_tag(P2pArgs& a) {
  if (!a.auto_epoch) return;
  __shared__ uint32_t s_tag;
  if (threadIdx.x == 0) {
    uint32_t t = static_cast<uint32_t>(*reinterpret_cast<volatile unsigned long long*>(epoch_counter(a)) + 1ull);
    s_tag = t == 0u ? 1u : t;  // 0 marks an empty slot
  }
  __syncthreads();
  a.tag = s_tag;
  a.parity = a.tag & 1u;
}

__device__ __forceinline__ void ll_store(LLSlot* slot, const Part& p, uint32_t tag) {
  const unsigned long long t = static_cast<unsigned long long>(tag) << 32;
  const unsigned long long ib = static_cast<unsigned long long>(p.i);
  volatile unsigned long long* w = slot->w;
  w[0] = t | static_cast<uint32_t>(__double2loint(p.s));
  w[1] = t | static_cast<uint32_t>(__double2hiint(p.s));
  w[2] = t | __float_as_uint(p.m);
  w[3] = t;
  w[4] = t | (ib & 0xffffffffull);
  w[5] = t | (ib >> 32);
}

// A slot's six words as three 16-byte loads (each 8-byte element is read
// single-copy atomically, which is all the format needs).
__device__ __forceinline__ void ll_load_words(const LLSlot* slot, unsigned long long (&v)[6]) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v[0]), "=l"(v[1]) : "l"(slot->w) : "memory");
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v[2]), "=l"(v[3]) : "l"(slot->w + 2) : "memory");
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(v[4]), "=l"(v[5]) : "l"(slot->w + 4) : "memory");
}

__device__ __forceinline__ bool ll_decode(const unsigned long long (&v)[6], uint32_t tag, Part& p) {
  bool ok = true;
#pragma unroll
  for (int k = 0; k < 6; ++k) ok = ok && static_cast<uint32_t>(v[k] >> 32) == tag;
  if (!ok) return false;
  p.s = __hiloint2double(static_cast<int>(static_cast<uint32_t>(v[1])), static_cast<int>(static_cast<uint32_t>(v[0])));
  p.m = __uint_as_float(static_cast<uint32_t>(v[2]));
  p.reserved = 0;
  p.i = static_cast<long long>((v[5] << 32) | (v[4] & 0xffffffffull));
  return true;
}

// Bounded wait (kP2pWaitNs) until the non-null slots carry `tag`.  Both
// slots' words are requested before either is checked (one round trip per
// poll, not two).  After the first polls the waiter sleeps between polls so
// that it takes no issue slots from the CTAs still streaming on its SM.
__device__ __forceinline__ bool ll_wait(const LLSlot* s0, const LLSlot* s1, uint32_t tag, Part& p0, Part& p1) {
  bool d0 = s0 == nullptr, d1 = s1 == nullptr;
  unsigned long long t0 = 0;
  for (uint32_t it = 0;; ++it) {
    unsigned long long a[6], b[6];
    if (!d0) ll_load_words(s0, a);
    if (!d1) ll_load_words(s1, b);
    if (!d0) d0 = ll_decode(a, tag, p0);
    if (!d1) d1 = ll_decode(b, tag, p1);
    if (d0 && d1) return true;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (it == 0) t0 = t;
    else if (t - t0 > kP2pWaitNs) return false;
    if (it >= 8) __nanosleep(32);
  }
}

// Block-wide; `mine` is the same in every thread; `scratch` is shared memory
// for `world` Parts.  Thread r publishes to rank r and then collects rank r's
// slot of this rank's buffer, so the latencies of the ranks overlap; thread 0
// folds the collected slots in rank order.
__device__ void p2p_publish_and_combine(const Part& mine, const P2pArgs& a, Part* scratch) {
  __shared__ int all_ok;
  if (threadIdx.x == 0) all_ok = 1;
  __syncthreads();
  const int half = static_cast<int>(a.parity) * a.world;
  for (int r = threadIdx.x; r < a.world; r += blockDim.x) ll_store(a.peers[r] + half + a.rank, mine, a.tag);
  bool ok = true;
  for (int r = threadIdx.x; r < a.world; r += blockDim.x) {
    Part q, unused;
    if (ll_wait(a.peers[a.rank] + half + r, nullptr, a.tag, q, unused)) scratch[r] = q;
    else ok = false;
  }
  if (!ok) {
    all_ok = 0;
    atomicCAS(&g_reduce_watchdog, 0u, 2u);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    Part t = part_identity();
    if (all_ok)
      for (int r = 0; r < a.world; ++r) t = part_combine(t, scratch[r]);
    mcke_reduce_result res;
    res.sum = static_cast<float>(t.s);
    res.max = t.m;
    res.argmax = all_ok ? t.i : -1;
    *a.out = res;
    if (a.auto_epoch) *reinterpret_cast<volatile unsigned long long*>(epoch_counter(a)) = a.tag;
  }
}

// kEarly (MCKE_REDUCE_EARLY_READ): x is not written by the kernel launched just
// before on the stream, so the CTAs read it before waiting for that kernel and
// wait only before their first global write (the partial slots, the arrival
// count, the tag).  Every kernel of this library lets its successor start only
// after its own wait, and a kernel launched without programmatic serialization
// completes before its successor starts, so every earlier writer of x has
// completed by then.  Consecutive calls then overlap: the next call's CTAs
// stream while this call's last CTA folds and exchanges.
template <bool kP2p, bool kEarly = false>
__global__ void __launch_bounds__(kThreads, 3) reduce_full_stream_kernel(const float* __restrict__ x, int64_t n,
                                                                      int64_t head, long long base,
                                                                      Part* __restrict__ parts, P2pArgs p2p_in) {
  unsigned long long* const stamps = kP2p ? p2p_in.stamps : nullptr;
  if (kP2p && stamps && threadIdx.x == 0) atomicMin(stamps + kStampFirstEntry, global_ns());
  if constexpr (!kEarly) pdl_entry();
  if (kP2p && stamps && threadIdx.x == 0) {
    const unsigned long long t = global_ns();
    atomicMin(stamps + kStampFirstStart, t);
    atomicMax(stamps + kStampLastStart, t);
  }
  P2pArgs p2p = p2p_in;
  extern __shared__ __align__(16) uint8_t smem[];  // P2P: the ranks' collected partials
  __shared__ Part red[kWarps];
  const int tid = threadIdx.x;
  const float* xa = x + head;
  const int64_t nv = (n - head) / 4;
  const int64_t S = static_cast<int64_t>(gridDim.x) * kThreads;  // grid stride, in float4

  Part p = part_identity();
  if (blockIdx.x == 0 && tid == 0)
    for (int64_t i = 0; i < head; ++i) part_add(p, x[i], base + i);
  double s = p.s;
  float m = p.m;
  long long vbest = -1;
  int lbest = 0;
  float mbest = 0.f;
  const bool have_index = p.i >= 0;
  // Thread g reads float4 g, g + S, ... in increasing order, kLoads per
  // round, the next round's loads issued before this round's arithmetic.
  int64_t v0 = static_cast<int64_t>(blockIdx.x) * kThreads + tid;
  float4 q[kLoads], nxt[kLoads];
#pragma unroll
  for (int u = 0; u < kLoads; ++u)
    if (v0 + u * S < nv) q[u] = ld_stream_f4(xa + 4 * (v0 + u * S));
  for (; v0 < nv; v0 += kLoads * S) {
    const int64_t v1 = v0 + kLoads * S;
#pragma unroll
    for (int u = 0; u < kLoads; ++u)
      if (v1 + u * S < nv) nxt[u] = ld_stream_f4(xa + 4 * (v1 + u * S));
#pragma unroll
    for (int u = 0; u < kLoads; ++u) {
      const int64_t v = v0 + u * S;
      if (v >= nv) break;
      s += static_cast<double>(q[u].x);
      s += static_cast<double>(q[u].y);
      s += static_cast<double>(q[u].z);
      s += static_cast<double>(q[u].w);
      const float lm = fmaxf(fmaxf(q[u].x, q[u].y), fmaxf(q[u].z, q[u].w));
      if (lm > m || (vbest < 0 && !have_index && lm == m)) {
        m = lm;
        vbest = v;
        // the float4's first element equal to its maximum, with its own bits
        // (so a -0 ahead of a +0 wins)
        lbest = (q[u].x == lm) ? 0 : (q[u].y == lm) ? 1 : (q[u].z == lm) ? 2 : 3;
        mbest = lbest == 0 ? q[u].x : lbest == 1 ? q[u].y : lbest == 2 ? q[u].z : q[u].w;
      }
    }
#pragma unroll
    for (int u = 0; u < kLoads; ++u) q[u] = nxt[u];
  }
  p.s = s;
  if (vbest >= 0) {
    p.m = mbest;
    p.i = base + head + 4 * vbest + lbest;
  }
  if (blockIdx.x == 0 && tid == 0)
    for (int64_t e = head + 4 * nv; e < n; ++e) part_add(p, x[e], base + e);
  if constexpr (kEarly) pdl_entry();  // the previous grid has completed: writes may start
  p = block_combine(p, red);
  if (!kP2p && tid == 0) parts[blockIdx.x] = p;
  if constexpr (kP2p) {
    // Every CTA stores its partial in its slot of this rank's part area
    // (low-latency format) and counts itself in; the CTA that arrives last
    // collects the slots -- thread t the virtual lanes t and t+256 of
    // reduce_full_combine_kernel's 1024-thread fold (G <= kFullCtaCap < 512,
    // so the rest are the identity), which makes the shard partial
    // bit-identical to the two-launch path -- and runs the exchange.  No CTA
    // waits for another CTA of the grid.  No fence between a CTA's slot
    // stores and its arrival: the collector checks the epoch in every word of
    // every slot and polls until all have landed, so the counter may overtake
    // the stores (a fence there put one more round trip to L2 between the last
    // CTA's partial and the result).
    resolve_tag(p2p);
    LLSlot* local = p2p.peers[p2p.rank] + 2 * p2p.world;
    __shared__ int is_last;
    __shared__ int parts_ok;
    __shared__ Part own;  // this CTA's partial: the collector does not read its own slot back
    if (tid == 0) {
      own = p;
      if (stamps) {
        const unsigned long long t = global_ns();
        atomicMin(stamps + kStampFirstDone, t);
        atomicMax(stamps + kStampLastDone, t);
      }
      ll_store(local + blockIdx.x, p, p2p.tag);
      is_last = atomicAdd(arrival_count(p2p), 1u) == gridDim.x - 1u ? 1 : 0;
      if (stamps && is_last) stamps[kStampCounted] = global_ns();
      parts_ok = 1;
      if (is_last) *arrival_count(p2p) = 0u;  // the next call counts from 0
    }
    __syncthreads();
    if (!is_last) return;
    __shared__ Part red32[16];
    __shared__ Part shard;
    const int G = static_cast<int>(gridDim.x);
    // Every other CTA stored its slot before counting itself in, so all 256
    // threads read their two slots at once: one round trip (the epochs are
    // checked all the same, bounded wait).  This CTA's own partial comes from
    // shared memory: its slot store may still be on its way.  Measured at
    // 2^25 floats: 2.82 us from the count coming back to the shard partial
    // when each poll loaded one slot, checked it, then loaded the other.
    Part v0 = part_identity(), v1 = part_identity(), q0, q1;
    const int mine = static_cast<int>(blockIdx.x);
    const bool got = ll_wait(tid < G && tid != mine ? local + tid : nullptr,
                             tid + kThreads < G && tid + kThreads != mine ? local + tid + kThreads : nullptr,
                             p2p.tag, q0, q1);
    if (tid == mine) q0 = own;
    if (tid + kThreads == mine) q1 = own;
    if (!got) parts_ok = 0;
    if (got && tid < G) v0 = part_combine(v0, q0);
    if (got && tid + kThreads < G) v1 = part_combine(v1, q1);
    v0 = warp_butterfly(v0);
    v1 = warp_butterfly(v1);
    if ((tid & 31) == 0) {
      red32[tid >> 5] = v0;
      red32[(tid >> 5) + kWarps] = v1;
    }
    __syncthreads();
    if (tid < 32) {
      Part r = tid < 2 * kWarps ? red32[tid] : part_identity();
      r = warp_butterfly(r);
      if (tid == 0) {
        if (!parts_ok) {
          atomicCAS(&g_reduce_watchdog, 0u, 1u);
          r.i = -1;
        }
        shard = r;
        if (stamps) stamps[kStampFolded] = global_ns();
      }
    }
    __syncthreads();
    // dynamic shared memory: the ranks' results, collected in rank order
    p2p_publish_and_combine(shard, p2p, reinterpret_cast<Part*>(smem));
    if (stamps && tid == 0) stamps[kStampExchanged] = global_ns();
  }
}

// Pass 2 (and the cross-shard combine): one block folds `count` Parts in a
// fixed order and writes either a final result or one Part.
template <bool kFinal>
__global__ void __launch_bounds__(1024) reduce_full_combine_kernel(const Part* __restrict__ parts,
                                                                   int64_t count, void* out) {
  pdl_entry();
  __shared__ Part red[32];
  Part p = part_identity();
  for (int64_t j = threadIdx.x; j < count; j += blockDim.x) p = part_combine(p, parts[j]);
  p = block_combine(p, red);
  if (threadIdx.x == 0) {
    if (kFinal) {
      mcke_reduce_result r;
      r.sum = static_cast<float>(p.s);
      r.max = p.m;
      r.argmax = p.i;
      *static_cast<mcke_reduce_result*>(out) = r;
    } else {
      *static_cast<Part*>(out) = p;
    }
  }
}

// ---- row reduce ----------------------------------------------------------

// One warp per row.  Sum/mean accumulate in double, max is the std::max fold.
template <bool kMax, bool kVec>
__global__ void __launch_bounds__(kThreads) row_reduce_warp_kernel(const float* __restrict__ x,
                                                                   float* __restrict__ out,
                                                                   int64_t rows, int64_t cols,
                                                                   double divisor) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * cols;
  double s = 0.0;
  float m = -INFINITY;
  if (kVec) {
    const int64_t nv = cols / 4;
    for (int64_t v0 = lane; v0 < nv; v0 += 32 * kUnroll) {
      float4 q[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u)
        if (v0 + 32 * u < nv) q[u] = ld_stream_f4(xr + 4 * (v0 + 32 * u));
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (v0 + 32 * u >= nv) continue;
        if (kMax) {
          m = (m < q[u].x) ? q[u].x : m;
          m = (m < q[u].y) ? q[u].y : m;
          m = (m < q[u].z) ? q[u].z : m;
          m = (m < q[u].w) ? q[u].w : m;
        } else {
          s += static_cast<double>(q[u].x);
          s += static_cast<double>(q[u].y);
          s += static_cast<double>(q[u].z);
          s += static_cast<double>(q[u].w);
        }
      }
    }
  } else {
    for (int64_t c = lane; c < cols; c += 32) {
      const float v = xr[c];
      if (kMax) m = (m < v) ? v : m;
      else s += static_cast<double>(v);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    if (kMax) {
      const float t = __shfl_xor_sync(0xffffffffu, m, o);
      m = (m < t) ? t : m;
    } else {
      s += __shfl_xor_sync(0xffffffffu, s, o);
    }
  }
  if (lane == 0) out[row] = kMax ? m : static_cast<float>(s / divisor);
}

// Rows of at most 1024 floats (cols % 4 == 0, x 16-byte aligned; config 2's
// 32768 x 1024 is this shape): one warp per row with every load of the row
// issued before any arithmetic, NV float4 per lane (NV = cols / 128 rounded up
// to a power of two).  The warp kernel above issues four loads, adds, then
// issues the next four; here a row's 4 KB is in flight at once.  Each lane adds
// its float4s in the same order (lane, lane + 32, ...) and the warp folds the
// lanes with the same butterfly, so the two kernels give the same bits.
// Measured on B200 at 32768 x 1024, 40 launches back to back: 22.7 us per
// launch against 24.7 us.  The mean's double division is a subroutine call
// whose calling convention took the sum kernel to 80 registers (3 CTAs per SM
// instead of 8; 35 us instead of 23), so only the mean variant (kMean) carries
// it, with its registers bounded for six resident CTAs.
// Only for cols == 128 * NV (128, 256, 512, 1024), where every lane loads all NV
// float4 with no per-load guard: with guards (other widths) the compiler widened
// all 32 values to double at once, 80 registers and 3 CTAs per SM instead of 32
// and 8 (35 us instead of 23 at 32768 x 1024), so those widths keep the warp
// kernel above.
template <bool kMax, bool kMean, int NV>
__global__ void __launch_bounds__(kThreads) row_reduce_row_kernel(const float* __restrict__ x,
                                                                  float* __restrict__ out, int64_t rows,
                                                                  int64_t cols, double divisor) {
  pdl_entry();
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + row * cols;
  float4 q[NV];
#pragma unroll
  for (int u = 0; u < NV; ++u) q[u] = ld_stream_f4(xr + 4 * (lane + 32 * u));
  double s = 0.0;
  float m = -INFINITY;
#pragma unroll
  for (int u = 0; u < NV; ++u) {
    if (kMax) {
      m = (m < q[u].x) ? q[u].x : m;
      m = (m < q[u].y) ? q[u].y : m;
      m = (m < q[u].z) ? q[u].z : m;
      m = (m < q[u].w) ? q[u].w : m;
    } else {
      s += static_cast<double>(q[u].x);
      s += static_cast<double>(q[u].y);
      s += static_cast<double>(q[u].z);
      s += static_cast<double>(q[u].w);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    if (kMax) {
      const float t = __shfl_xor_sync(0xffffffffu, m, o);
      m = (m < t) ? t : m;
    } else {
      s += __shfl_xor_sync(0xffffffffu, s, o);
    }
  }
  if (lane == 0) {
    if constexpr (kMax) out[row] = m;
    else if constexpr (kMean) out[row] = static_cast<float>(s / divisor);
    else out[row] = static_cast<float>(s);
  }
}

template <bool kMax, bool kMean>
void launch_row_kernel(unsigned g, cudaStream_t s, const float* x, float* out, int64_t rows, int64_t cols,
                       double divisor) {
  if (cols == 128)
    launch_async(row_reduce_row_kernel<kMax, kMean, 1>, g, kThreads, 0, s, x, out, rows, cols, divisor);
  else if (cols == 256)
    launch_async(row_reduce_row_kernel<kMax, kMean, 2>, g, kThreads, 0, s, x, out, rows, cols, divisor);
  else if (cols == 512)
    launch_async(row_reduce_row_kernel<kMax, kMean, 4>, g, kThreads, 0, s, x, out, rows, cols, divisor);
  else
    launch_async(row_reduce_row_kernel<kMax, kMean, 8>, g, kThreads, 0, s, x, out, rows, cols, divisor);
}

// Two-pass for few long rows: pass 1 splits each row over `split` blocks and
// stores one double per (row, segment); pass 2 folds a row's segments in order.
template <bool kMax>
__global__ void __launch_bounds__(kThreads) row_reduce_split_kernel(const float* __restrict__ x,
                                                                    double* __restrict__ ws,
                                                                    int64_t cols, int64_t split) {
  pdl_entry();
  __shared__ double red[kWarps];
  const int64_t row = blockIdx.y;
  const int64_t seg = blockIdx.x;
  const int64_t len = (cols + split - 1) / split;
  const int64_t c0 = seg * len;
  const int64_t c1 = (c0 + len < cols) ? c0 + len : cols;
  const float* xr = x + row * cols;
  double s = 0.0;
  float m = -INFINITY;
  for (int64_t c = c0 + threadIdx.x; c < c1; c += kThreads) {
    const float v = xr[c];
    if (kMax) m = (m < v) ? v : m;
    else s += static_cast<double>(v);
  }
  double a = kMax ? static_cast<double>(m) : s;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const double t = __shfl_xor_sync(0xffffffffu, a, o);
    a = kMax ? ((a < t) ? t : a) : a + t;
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = red[0];
    for (int w = 1; w < kWarps; ++w) t = kMax ? ((t < red[w]) ? red[w] : t) : t + red[w];
    ws[row * split + seg] = t;
  }
}

template <bool kMax>
__global__ void __launch_bounds__(kThreads) row_reduce_fold_kernel(const double* __restrict__ ws,
                                                                   float* __restrict__ out,
                                                                   int64_t rows, int64_t split,
                                                                   double divisor) {
  pdl_entry();
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x;
  if (row >= rows) return;
  double t = kMax ? -INFINITY : 0.0;
  for (int64_t j = 0; j < split; ++j) {
    const double v = ws[row * split + j];
    t = kMax ? ((t < v) ? v : t) : t + v;
  }
  out[row] = kMax ? static_cast<float>(t) : static_cast<float>(t / divisor);
}

// Segments per row for the two-pass path: enough blocks to fill the machine
// (the reference's rule, kernels/reduce.cu:60-72, retargeted to 8 x 148), at
// most 64, and never segments shorter than one block's width.
int64_t two_pass_split(int64_t rows, int64_t cols) {
  if (rows <= 0) return 1;
  int64_t s = (kMaxBlocks + rows - 1) / rows;
  if (s > 64) s = 64;
  const int64_t by_len = (cols + kThreads - 1) / kThreads;
  if (s > by_len) s = by_len;
  return s < 1 ? 1 : s;
}

}  // namespace
}  // namespace mcke_sm100

using namespace mcke_sm100;

namespace mcke_sm100 {
namespace {
}  // namespace

// Reads and clears the streamed reduce's watchdog word on the current device.
int read_reduce_watchdog(uint32_t* site) {
  uint32_t v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_reduce_watchdog, sizeof(v));
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "reduce watchdog read: %s", cudaGetErrorString(e));
  if (v != 0) {
    const uint32_t zero = 0;
    e = cudaMemcpyToSymbol(g_reduce_watchdog, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "reduce watchdog clear: %s", cudaGetErrorString(e));
  }
  *site = v;
  return MCKE_OK;
}
}  // namespace mcke_sm100

extern "C" size_t mcke_sm100_reduce_full_workspace_bytes(int64_t n) {
  if (n <= 0) return 0;
  return static_cast<size_t>(full_blocks(n)) * sizeof(Part);
}

namespace {
int full_common(const char* who, const float* x, int64_t n, int64_t index_base, void* out,
                void* workspace, size_t workspace_bytes, bool final_result, mcke_stream_t stream,
                bool early = false) {
  if (!out) return fail(MCKE_INVALID_ARGUMENT, "%s: null output", who);
  if (n < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (n > 0 && !x) return fail(MCKE_INVALID_ARGUMENT, "%s: null input", who);
  if (index_base < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative index_base", who);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n == 0) {
    // The empty reduction still defines its output: sum 0, max -inf, argmax -1.
    if (final_result) launch_async(reduce_full_combine_kernel<true>, 1, 32, 0, s, nullptr, 0, out);
    else launch_async(reduce_full_combine_kernel<false>, 1, 32, 0, s, nullptr, 0, out);
    return check_launch(who);
  }
  if (!aligned(x, 4)) return fail(MCKE_INVALID_ARGUMENT, "%s: x not 4-byte aligned", who);
  const size_t need = mcke_sm100_reduce_full_workspace_bytes(n);
  if (!workspace || workspace_bytes < need)
    return fail(MCKE_INVALID_ARGUMENT,
                "%s: needs %zu bytes of workspace (got %zu); query "
                "mcke_sm100_reduce_full_workspace_bytes() first",
                who, need, workspace_bytes);
  if (!aligned(workspace, 16)) return fail(MCKE_INVALID_ARGUMENT, "%s: workspace not 16-byte aligned", who);
  const int64_t g = full_blocks(n);
  const uintptr_t addr = reinterpret_cast<uintptr_t>(x);
  int64_t head = static_cast<int64_t>(((16 - addr % 16) % 16) / 4);
  if (head > n) head = n;
  Part* parts = static_cast<Part*>(workspace);
  launch_async(early ? reduce_full_stream_kernel<false, true> : reduce_full_stream_kernel<false>,
               static_cast<unsigned>(g), kThreads, 0, s, x, n, head, index_base, parts, P2pArgs{});
  MCKE_RETURN_IF(check_launch(who));
  if (final_result) launch_async(reduce_full_combine_kernel<true>, 1, 1024, 0, s, parts, g, out);
  else launch_async(reduce_full_combine_kernel<false>, 1, 1024, 0, s, parts, g, out);
  return check_launch(who);
}
}  // namespace

extern "C" int mcke_sm100_reduce_full_f32(const float* x, int64_t n, mcke_reduce_result* out,
                                          void* workspace, size_t workspace_bytes,
                                          mcke_stream_t stream) {
  clear_error();
  return full_common("mcke_sm100_reduce_full_f32", x, n, 0, out, workspace, workspace_bytes, true,
                     stream);
}

extern "C" int mcke_sm100_reduce_full_f32_ex(const float* x, int64_t n, mcke_reduce_result* out,
                                             void* workspace, size_t workspace_bytes, unsigned flags,
                                             mcke_stream_t stream) {
  static const char* who = "mcke_sm100_reduce_full_f32_ex";
  clear_error();
  if (flags & ~static_cast<unsigned>(MCKE_REDUCE_EARLY_READ))
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown flags 0x%x", who, flags);
  return full_common(who, x, n, 0, out, workspace, workspace_bytes, true, stream,
                     (flags & MCKE_REDUCE_EARLY_READ) != 0);
}

extern "C" int mcke_sm100_reduce_full_partial_f32(const float* x, int64_t n, int64_t index_base,
                                                  mcke_reduce_partial* out, void* workspace,
                                                  size_t workspace_bytes, mcke_stream_t stream) {
  clear_error();
  return full_common("mcke_sm100_reduce_full_partial_f32", x, n, index_base, out, workspace,
                     workspace_bytes, false, stream);
}

extern "C" int mcke_sm100_reduce_combine(const mcke_reduce_partial* partials, int64_t count,
                                         mcke_reduce_result* out, mcke_stream_t stream) {
  static const char* who = "mcke_sm100_reduce_combine";
  clear_error();
  if (!out) return fail(MCKE_INVALID_ARGUMENT, "%s: null output", who);
  if (count < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative count", who);
  if (count > 0 && !partials) return fail(MCKE_INVALID_ARGUMENT, "%s: null partials", who);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  launch_async(reduce_full_combine_kernel<true>, 1, 1024, 0, s, reinterpret_cast<const Part*>(partials), count,
                                                      out);
  return check_launch(who);
}

extern "C" size_t mcke_sm100_reduce_row_workspace_bytes(int64_t rows, int64_t cols, int variant) {
  if (variant != MCKE_REDUCE_TWO_PASS || rows <= 0 || cols <= 0) return 0;
  return static_cast<size_t>(rows * two_pass_split(rows, cols)) * sizeof(double);
}

extern "C" int mcke_sm100_reduce_row_f32(const float* x, float* out, int64_t rows, int64_t cols,
                                         int kind, int variant, void* workspace,
                                         size_t workspace_bytes, mcke_stream_t stream) {
  static const char* who = "mcke_sm100_reduce_row_f32";
  clear_error();
  if (rows == 0 || cols == 0) return MCKE_OK;
  if (rows < 0 || cols < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (!x || !out) return fail(MCKE_INVALID_ARGUMENT, "%s: null pointer", who);
  if (kind < MCKE_REDUCE_SUM || kind > MCKE_REDUCE_MEAN)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown kind %d", who, kind);
  if (variant < MCKE_REDUCE_SMEM_TREE || variant > MCKE_REDUCE_TWO_PASS)
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown variant %d", who, variant);
  if (rows > 2147483647LL) return fail(MCKE_INVALID_ARGUMENT, "%s: rows exceeds the grid limit", who);
  const bool is_max = (kind == MCKE_REDUCE_MAX);
  const double divisor = (kind == MCKE_REDUCE_MEAN) ? static_cast<double>(cols) : 1.0;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (variant == MCKE_REDUCE_TWO_PASS) {
    if (workspace == nullptr && workspace_bytes == 0)
      return fail(MCKE_UNIMPLEMENTED,
                  "%s: the two-pass variant needs a workspace; query "
                  "mcke_sm100_reduce_row_workspace_bytes() and pass one",
                  who);
    const size_t need = mcke_sm100_reduce_row_workspace_bytes(rows, cols, variant);
    if (!workspace || workspace_bytes < need)
      return fail(MCKE_INVALID_ARGUMENT, "%s: two-pass needs %zu bytes of workspace (got %zu)", who,
                  need, workspace_bytes);
    if (!aligned(workspace, 8)) return fail(MCKE_INVALID_ARGUMENT, "%s: workspace not 8-byte aligned", who);
    if (rows > 65535) return fail(MCKE_INVALID_ARGUMENT, "%s: two-pass supports at most 65535 rows", who);
    const int64_t split = two_pass_split(rows, cols);
    double* ws = static_cast<double*>(workspace);
    const dim3 g1(static_cast<unsigned>(split), static_cast<unsigned>(rows), 1u);
    const unsigned g2 = static_cast<unsigned>((rows + kThreads - 1) / kThreads);
    if (is_max) {
      launch_async(row_reduce_split_kernel<true>, g1, kThreads, 0, s, x, ws, cols, split);
      MCKE_RETURN_IF(check_launch(who));
      launch_async(row_reduce_fold_kernel<true>, g2, kThreads, 0, s, ws, out, rows, split, divisor);
    } else {
      launch_async(row_reduce_split_kernel<false>, g1, kThreads, 0, s, x, ws, cols, split);
      MCKE_RETURN_IF(check_launch(who));
      launch_async(row_reduce_fold_kernel<false>, g2, kThreads, 0, s, ws, out, rows, split, divisor);
    }
    return check_launch(who);
  }
  const bool vec = (cols % 4 == 0) && aligned(x, 16);
  const unsigned g = static_cast<unsigned>((rows + kWarps - 1) / kWarps);
  if (vec && (cols == 128 || cols == 256 || cols == 512 || cols == 1024)) {
    if (is_max) launch_row_kernel<true, false>(g, s, x, out, rows, cols, divisor);
    else if (kind == MCKE_REDUCE_MEAN) launch_row_kernel<false, true>(g, s, x, out, rows, cols, divisor);
    else launch_row_kernel<false, false>(g, s, x, out, rows, cols, divisor);
    return check_launch(who);
  }
  if (is_max) {
    if (vec) launch_async(row_reduce_warp_kernel<true, true>, g, kThreads, 0, s, x, out, rows, cols, divisor);
    else launch_async(row_reduce_warp_kernel<true, false>, g, kThreads, 0, s, x, out, rows, cols, divisor);
  } else {
    if (vec) launch_async(row_reduce_warp_kernel<false, true>, g, kThreads, 0, s, x, out, rows, cols, divisor);
    else launch_async(row_reduce_warp_kernel<false, false>, g, kThreads, 0, s, x, out, rows, cols, divisor);
  }
  return check_launch(who);
}

// ---- full reduce with no caller scratch -------------------------------------
//
// Some callers cannot allocate device memory at all: a host runtime whose
// memory manager owns every device allocation and forbids side allocations, or
// a foreign-language binding that only ever holds the caller's own input and
// output buffers.  They cannot provide the workspace mcke_sm100_reduce_full_f32
// needs, so this variant keeps its pass-1 partials in a fixed array in device
// memory instead.  The array lives in this library's module: every GPU that
// loads the library holds these bytes until the process exits.
//
// Capacity: one partial per pass-1 block, and full_blocks() caps the pass-1
// grid at kFullCtaCap (444) blocks, so the array is 444 x 24 = 10,656 bytes and
// every n fits.  The capacity check below still rejects, with a clear error,
// any request that would need more, should the grid cap ever grow past the array.
namespace mcke_sm100 {
namespace {

constexpr int64_t kStaticParts = kFullCtaCap;
static_assert(kFullCtaCap <= kStaticParts, "the built-in scratch must hold one partial per pass-1 block");
static __device__ __align__(256) Part g_static_parts[kStaticParts];

// Device address of g_static_parts for each device, looked up once per device
// with that device current (the host-side name is only a stand-in; a kernel
// must be handed the device address).  The address belongs to the device's
// primary context: after cudaDeviceReset() (or any reset of that context) the
// library module is loaded again and the cached address is stale, so a process
// that resets a device must not call this entry point on it afterwards.
std::mutex g_static_mu;
void* g_static_addr[64] = {};

int static_parts_address(const char* who, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "%s: cudaGetDevice: %s", who, cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return fail(MCKE_INVALID_ARGUMENT, "%s: device index %d beyond 63", who, dev);
  std::lock_guard<std::mutex> lk(g_static_mu);
  if (!g_static_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_parts);
    if (e != cudaSuccess || !p)
      return fail(MCKE_CUDA_ERROR, "%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
    g_static_addr[dev] = p;
  }
  *out = g_static_addr[dev];
  return MCKE_OK;
}

}  // namespace
}  // namespace mcke_sm100

extern "C" int mcke_sm100_reduce_full_f32_noalloc(const float* x, int64_t n, mcke_reduce_result* out,
                                                  mcke_stream_t stream) {
  static const char* who = "mcke_sm100_reduce_full_f32_noalloc";
  clear_error();
  if (!out) return fail(MCKE_INVALID_ARGUMENT, "%s: null output", who);
  if (n < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative extent", who);
  if (n > 0 && !x) return fail(MCKE_INVALID_ARGUMENT, "%s: null input", who);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (n == 0) {
    launch_async(reduce_full_combine_kernel<true>, 1, 32, 0, s, nullptr, 0, out);
    return check_launch(who);
  }
  if (!aligned(x, 4)) return fail(MCKE_INVALID_ARGUMENT, "%s: x not 4-byte aligned", who);
  const int64_t g = full_blocks(n);
  if (g > kStaticParts)
    return fail(MCKE_INVALID_ARGUMENT,
                "%s: n = %lld needs %lld partials but the built-in scratch holds %lld (%lld bytes)", who,
                static_cast<long long>(n), static_cast<long long>(g), static_cast<long long>(kStaticParts),
                static_cast<long long>(kStaticParts * static_cast<int64_t>(sizeof(Part))));
  void* scratch = nullptr;
  MCKE_RETURN_IF(static_parts_address(who, &scratch));
  const uintptr_t addr = reinterpret_cast<uintptr_t>(x);
  int64_t head = static_cast<int64_t>(((16 - addr % 16) % 16) / 4);
  if (head > n) head = n;
  // Pass 1 writes partials [0, g) before pass 2 reads exactly those, so the
  // array's leftover contents from an earlier call are never read and nothing
  // needs clearing.
  Part* parts = static_cast<Part*>(scratch);
  launch_async(reduce_full_stream_kernel<false>, static_cast<unsigned>(g), kThreads, 0, s, x, n, head, 0, parts, P2pArgs{});
  MCKE_RETURN_IF(check_launch(who));
  launch_async(reduce_full_combine_kernel<true>, 1, 1024, 0, s, parts, g, out);
  return check_launch(who);
}

// ---- sharded full reduce with a peer-to-peer one-shot combine ----------------
namespace mcke_sm100 {
namespace {
// Only for an empty shard (no pass-1 CTA to run the exchange).
__global__ void __launch_bounds__(kThreads) reduce_p2p_empty_kernel(P2pArgs a_in) {
  pdl_entry();
  extern __shared__ __align__(16) uint8_t scratch[];
  P2pArgs a = a_in;
  resolve_tag(a);
  p2p_publish_and_combine(part_identity(), a, reinterpret_cast<Part*>(scratch));
}
}  // namespace
}  // namespace mcke_sm100

extern "C" size_t mcke_sm100_reduce_p2p_buffer_bytes(int world) {
  return world > 0 ? static_cast<size_t>(2 * world + kFullCtaCap + 1) * sizeof(LLSlot) : 0;
}

namespace {
int reduce_full_p2p(const char* who, const float* x, int64_t n, int64_t index_base, void* const* peer_buffers,
                    int world, int rank, uint64_t epoch, mcke_reduce_result* out, uint64_t* stamps,
                    mcke_stream_t stream, unsigned flags = 0) {
  clear_error();
  if (flags & ~static_cast<unsigned>(MCKE_REDUCE_EARLY_READ))
    return fail(MCKE_INVALID_ARGUMENT, "%s: unknown flags 0x%x", who, flags);
  if (!out || !peer_buffers) return fail(MCKE_INVALID_ARGUMENT, "%s: null output or peer table", who);
  if (world < 1 || world > 1024 || rank < 0 || rank >= world)
    return fail(MCKE_INVALID_ARGUMENT, "%s: bad world/rank %d/%d", who, world, rank);
  if (epoch > 0xffffffffull) return fail(MCKE_INVALID_ARGUMENT, "%s: epoch must be below 2^32", who);
  if (n < 0 || (n > 0 && !x)) return fail(MCKE_INVALID_ARGUMENT, "%s: bad input", who);
  if (index_base < 0) return fail(MCKE_INVALID_ARGUMENT, "%s: negative index_base", who);
  if (n > 0 && !aligned(x, 4)) return fail(MCKE_INVALID_ARGUMENT, "%s: x not 4-byte aligned", who);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  P2pArgs a;
  a.peers = reinterpret_cast<LLSlot* const*>(peer_buffers);
  a.out = out;
  a.tag = static_cast<uint32_t>(epoch);
  a.parity = static_cast<uint32_t>(epoch & 1);
  a.world = world;
  a.rank = rank;
  a.auto_epoch = epoch == 0 ? 1 : 0;
  a.stamps = reinterpret_cast<unsigned long long*>(stamps);
  if (n == 0) {
    launch_async(reduce_p2p_empty_kernel, 1, kThreads, static_cast<size_t>(world) * sizeof(Part), s, a);
    return check_launch(who);
  }
  const int64_t g = full_blocks(n);
  const uintptr_t addr = reinterpret_cast<uintptr_t>(x);
  int64_t head = static_cast<int64_t>(((16 - addr % 16) % 16) / 4);
  if (head > n) head = n;
  // dynamic shared memory: the ranks' collected partials (world <= 1024: 24 KB)
  // (the timeline entry point passes no flags: its stamps are written from entry on)
  launch_async((flags & MCKE_REDUCE_EARLY_READ) ? reduce_full_stream_kernel<true, true> : reduce_full_stream_kernel<true>,
               static_cast<unsigned>(g), kThreads, static_cast<size_t>(world) * sizeof(Part), s, x, n, head,
               index_base, nullptr, a);
  return check_launch(who);
}
}  // namespace

extern "C" int mcke_sm100_reduce_full_p2p_f32(const float* x, int64_t n, int64_t index_base,
                                              void* const* peer_buffers, int world, int rank, uint64_t epoch,
                                              mcke_reduce_result* out, mcke_stream_t stream) {
  return reduce_full_p2p("mcke_sm100_reduce_full_p2p_f32", x, n, index_base, peer_buffers, world, rank, epoch, out,
                         nullptr, stream);
}

extern "C" int mcke_sm100_reduce_full_p2p_f32_ex(const float* x, int64_t n, int64_t index_base,
                                                 void* const* peer_buffers, int world, int rank, uint64_t epoch,
                                                 mcke_reduce_result* out, unsigned flags, mcke_stream_t stream) {
  return reduce_full_p2p("mcke_sm100_reduce_full_p2p_f32_ex", x, n, index_base, peer_buffers, world, rank, epoch,
                         out, nullptr, stream, flags);
}

extern "C" int mcke_sm100_reduce_full_p2p_f32_timeline(const float* x, int64_t n, int64_t index_base,
                                                       void* const* peer_buffers, int world, int rank,
                                                       uint64_t epoch, mcke_reduce_result* out, uint64_t* stamps,
                                                       mcke_stream_t stream) {
  static const char* who = "mcke_sm100_reduce_full_p2p_f32_timeline";
  if (!stamps || !aligned(stamps, 8)) {
    clear_error();
    return fail(MCKE_INVALID_ARGUMENT, "%s: stamps must be 8-byte aligned device memory", who);
  }
  if (n == 0) {
    clear_error();
    return fail(MCKE_INVALID_ARGUMENT, "%s: an empty shard runs no streaming pass to time", who);
  }
  return reduce_full_p2p(who, x, n, index_base, peer_buffers, world, rank, epoch, out, stamps, stream);
}

// ---- CUDA IPC set-up helpers for the exchange buffers ---------------------------

extern "C" int mcke_sm100_ipc_buffer_create(size_t bytes, void** dev_ptr, void* handle_out) {
  static const char* who = "mcke_sm100_ipc_buffer_create";
  clear_error();
  if (!dev_ptr || !handle_out || bytes == 0) return fail(MCKE_INVALID_ARGUMENT, "%s: bad argument", who);
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return fail(MCKE_OUT_OF_MEMORY, "%s: cudaMalloc: %s", who, cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle_out), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return fail(MCKE_CUDA_ERROR, "%s: %s", who, cudaGetErrorString(e));
  }
  *dev_ptr = p;
  return MCKE_OK;
}

extern "C" int mcke_sm100_ipc_buffer_open(const void* handle, void** dev_ptr) {
  static const char* who = "mcke_sm100_ipc_buffer_open";
  clear_error();
  if (!handle || !dev_ptr) return fail(MCKE_INVALID_ARGUMENT, "%s: bad argument", who);
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "%s: %s", who, cudaGetErrorString(e));
  return MCKE_OK;
}

extern "C" int mcke_sm100_ipc_buffer_close(void* dev_ptr, int opened) {
  clear_error();
  const cudaError_t e = opened ? cudaIpcCloseMemHandle(dev_ptr) : cudaFree(dev_ptr);
  if (e != cudaSuccess) return fail(MCKE_CUDA_ERROR, "mcke_sm100_ipc_buffer_close: %s", cudaGetErrorString(e));
  return MCKE_OK;
}
