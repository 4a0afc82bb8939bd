// mcke/graph/memory_plan.hpp -- how the executor places tensors in a device's arena.
//
// Mirrors mini-cuda-kernel-engine include/mcke/graph/memory_plan.hpp:67
// (MemoryPolicy, same values).  Graph inputs and outputs always own their
// bytes; the policy decides whether intermediates share.
#pragma once

#include <cstdint>

namespace mcke {

enum class MemoryPolicy : std::uint8_t {
  kAllocPerTensor,   // every tensor its own bytes (the numerics gate's golden arm)
  kReuseTopoNaive,   // the reference's deliberately unsafe arm; rejected here
  kReuseSameStream,  // an intermediate reuses a freed block of its own stream (stream order makes it safe)
  kReuseHappensBefore,  // here the same rule as kReuseSameStream: a block is reused only where
                        // stream order proves its last reader finished before the new writer
};

}  // namespace mcke
