// GPU check of stream-ordered reuse in BuddyAllocator over device slabs (the
// reference's tests/test_stream_safety.cu asks the same of its pools: a block
// freed on one stream while that stream's work is still pending must not be
// handed to another stream).
//   1. X is allocated for stream A and filled with a pattern; a long FFMA
//      kernel runs on A, then a reader on A copies X (y = X + 0).  The host
//      frees X on A right away, while all of that is still queued.
//   2. Stream B asks for a block of X's size: it must get another block (X is
//      parked until A's work completes), and B overwrites that block.
//   3. Stream A asks for the same size: the slab holds only two such blocks,
//      so it gets X back at once (a block parked by the same stream is safe to
//      reuse in stream order) and zeroes it after the reader.
//   4. After both streams finish, A's reader must have seen X's pattern.
//   5. Everything freed and settled, the allocator's invariants hold.
// One GPU.  Prints "OK" and exits 0, or prints the failed check and exits 1.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdint>
#include <vector>

#include "mcke/memory/buddy_allocator.hpp"
#include "mcke_sm100.h"

#define CHECK(c)                                                   \
  do {                                                             \
    if (!(c)) {                                                    \
      std::printf("FAILED line %d: %s\n", __LINE__, #c);           \
      return 1;                                                    \
    }                                                              \
  } while (0)

int main() {
  using namespace mcke;
  CHECK(cudaSetDevice(0) == cudaSuccess);
  cudaStream_t sa = nullptr, sb = nullptr;
  CHECK(cudaStreamCreateWithFlags(&sa, cudaStreamNonBlocking) == cudaSuccess);
  CHECK(cudaStreamCreateWithFlags(&sb, cudaStreamNonBlocking) == cudaSuccess);

  BuddyConfig cfg;
  cfg.slab_bytes = std::size_t{8} << 20;  // two 4 MiB blocks per slab
  BuddyAllocator buddy(0, cfg);
  const std::size_t n = std::size_t{1} << 20;  // floats per block (4 MiB)
  const std::size_t bytes = n * sizeof(float);

  auto x = buddy.allocate(bytes, sa);
  CHECK(x.ok());
  float *zero = nullptr, *y = nullptr, *seed = nullptr, *sink = nullptr;
  CHECK(cudaMalloc(&zero, bytes) == cudaSuccess && cudaMalloc(&y, bytes) == cudaSuccess);
  CHECK(cudaMemset(zero, 0, bytes) == cudaSuccess);
  const std::int64_t threads = mcke_sm100_peak_fma_threads();
  CHECK(cudaMalloc(&seed, threads * sizeof(float)) == cudaSuccess);
  CHECK(cudaMalloc(&sink, threads * sizeof(float)) == cudaSuccess);
  CHECK(cudaMemset(seed, 0, threads * sizeof(float)) == cudaSuccess);
  // Load both kernels first: a kernel's first launch in a process loads its
  // module, which waits for the device and would drain stream A below.
  CHECK(mcke_sm100_peak_fma_f32(seed, sink, threads, 10, reinterpret_cast<mcke_stream_t>(sa)) == MCKE_OK);
  CHECK(mcke_sm100_vector_add_f32(zero, zero, y, n, reinterpret_cast<mcke_stream_t>(sa)) == MCKE_OK);
  CHECK(cudaDeviceSynchronize() == cudaSuccess);

  // 1. stream A: pattern, ~10 ms of FMA work, then the reader of X
  CHECK(cudaMemsetAsync(x->ptr, 0x3F, bytes, sa) == cudaSuccess);  // 0x3F3F3F3F = 0.747 as float
  CHECK(mcke_sm100_peak_fma_f32(seed, sink, threads, 150000, reinterpret_cast<mcke_stream_t>(sa)) == MCKE_OK);
  CHECK(mcke_sm100_vector_add_f32(static_cast<float*>(x->ptr), zero, y, n, reinterpret_cast<mcke_stream_t>(sa)) ==
        MCKE_OK);
  CHECK(buddy.deallocate(*x, sa).ok());
  const cudaError_t q = cudaStreamQuery(sa);
  if (q != cudaErrorNotReady) std::printf("stream A query: %d (%s)\n", static_cast<int>(q), cudaGetErrorString(q));
  CHECK(q == cudaErrorNotReady);  // A's work is still pending

  // 2. stream B wants the same size: not X
  auto z = buddy.allocate(bytes, sb);
  CHECK(z.ok());
  CHECK(z->ptr != x->ptr);
  CHECK(buddy.parked_blocks() >= 1);
  CHECK(cudaMemsetAsync(z->ptr, 0xFF, bytes, sb) == cudaSuccess);  // NaN pattern

  // 3. stream A again: X itself, queued behind A's reader
  auto w = buddy.allocate(bytes, sa);
  CHECK(w.ok());
  CHECK(w->ptr == x->ptr);
  CHECK(buddy.stats().deferred_reuses == 1);
  CHECK(cudaMemsetAsync(w->ptr, 0, bytes, sa) == cudaSuccess);

  // 4. the reader saw the pattern, not B's bytes nor A's later zeroes
  CHECK(cudaDeviceSynchronize() == cudaSuccess);
  std::vector<std::uint32_t> host(n);
  CHECK(cudaMemcpy(host.data(), y, bytes, cudaMemcpyDeviceToHost) == cudaSuccess);
  std::size_t bad = 0;
  for (std::uint32_t word : host) bad += (word != 0x3F3F3F3Fu);
  if (bad) std::printf("%zu of %zu words overwritten\n", bad, n);
  CHECK(bad == 0);

  // 5. free both, let the events complete, check the invariants
  CHECK(buddy.deallocate(*w, sa).ok());
  CHECK(buddy.deallocate(*z, sb).ok());
  CHECK(cudaDeviceSynchronize() == cudaSuccess);
  CHECK(buddy.settle_pending().ok());
  CHECK(buddy.parked_blocks() == 0);
  CHECK(buddy.validate().ok());
  const AllocatorStats st = buddy.stats();
  CHECK(st.raw_malloc_calls == 1);  // one slab, no cudaMalloc per request
  CHECK(st.bytes_in_use == 0);

  cudaFree(zero);
  cudaFree(y);
  cudaFree(seed);
  cudaFree(sink);
  cudaStreamDestroy(sa);
  cudaStreamDestroy(sb);
  std::printf("OK\n");
  return 0;
}
