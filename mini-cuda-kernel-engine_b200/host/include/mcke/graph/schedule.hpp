// mcke/graph/schedule.hpp -- how the executor spreads nodes over streams.
//
// Mirrors mini-cuda-kernel-engine include/mcke/graph/schedule.hpp:49
// (SchedulePolicy, same values).  On every device of a sharded executor the
// same node goes to the same stream index.
#pragma once

#include <cstdint>

namespace mcke {

enum class SchedulePolicy : std::uint8_t {
  kSequential,     // every node on stream 0, in topological order
  kLevelParallel,  // nodes of one topological level (longest path from an input) dealt round-robin over streams
  kChainGreedy,    // a node inherits its first producer's stream unless a sibling already did, else the least recently used
  // Added (no counterpart in the reference): every node on stream 0, level by
  // level (longest path from an input); the fp32 bias + activation nodes of a
  // level that the grouped kernel takes (same activation, vector width 4 or
  // automatic, cols % 512 == 0) go out as one launch of up to 16 jobs.  One
  // launch instead of one per node and no events: the host's cost per node of
  // an eager run falls with the group size.  Same bits as the other policies.
  kLevelGrouped,
};

}  // namespace mcke
