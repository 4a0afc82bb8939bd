"""Sharding helpers for one process per GPU (torch.distributed).

* ``bounds`` -- the contiguous range / row block a rank owns: [n*r//g, n*(r+1)//g),
  the split the C++ executor's sharding pass also uses;
* ``exchange_partials`` -- the one collective of a sharded full reduce: every
  rank contributes its 24-byte partial (mcke_reduce_partial) and receives all
  of them in rank order (NCCL all-gather on GPUs, gloo on CPU);
* ``combine_host`` -- the combine rule of the device kernel
  (mcke_sm100_reduce_combine), restated on the host so multi-rank tests can
  check the exchange without a GPU: sums add in double in rank order, the
  largest max wins, ties go to the lower global index, a shard with no
  element (index -1) never wins.
"""
from __future__ import annotations

import struct

import torch

PARTIAL_BYTES = 24


def bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    return n * rank // world, n * (rank + 1) // world


def pack_partial(s: float, m: float, idx: int) -> bytes:
    return struct.pack("<dfiq", s, m, 0, idx)


def unpack_partial(raw: bytes) -> tuple[float, float, int]:
    s, m, _, i = struct.unpack("<dfiq", raw[:PARTIAL_BYTES])
    return s, m, i


def exchange_partials(partial: torch.Tensor, world: int) -> torch.Tensor:
    """All-gather one uint8[24] partial per rank into uint8[world * 24], rank order."""
    import torch.distributed as td
    assert partial.dtype == torch.uint8 and partial.numel() == PARTIAL_BYTES
    out = torch.empty(world * PARTIAL_BYTES, dtype=torch.uint8, device=partial.device)
    if td.get_backend() == "nccl":
        td.all_gather_into_tensor(out, partial)
    else:
        parts = [torch.empty_like(partial) for _ in range(world)]
        td.all_gather(parts, partial)
        out.copy_(torch.cat(parts))
    return out


def combine_host(partials: list[tuple[float, float, int]]) -> tuple[float, float, int]:
    s, m, i = 0.0, float("-inf"), -1
    for ps, pm, pi in partials:
        s += ps
        if pi >= 0 and (i < 0 or pm > m or (pm == m and pi < i)):
            m, i = pm, pi
    return s, m, i
