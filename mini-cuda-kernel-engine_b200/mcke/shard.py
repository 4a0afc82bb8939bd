"""Sharding helpers for one process per GPU (torch.distributed).

* ``bounds`` -- the contiguous range / row block a rank owns: [n*r//g, n*(r+1)//g),
  the split the C++ executor's sharding pass also uses;
* ``exchange_partials`` -- the one collective of a sharded full reduce: every
  rank contributes its 24-byte partial (mcke_reduce_partial) and receives all
  of them in rank order (NCCL all-gather on GPUs, gloo on CPU);
* ``P2PExchange`` -- the same exchange without a collective library: the
  ranks' exchange buffers are shared with CUDA IPC once, and each step is one
  kernel pair (mcke_sm100_reduce_full_p2p_f32) that stores this rank's partial
  into every peer's buffer over NVLink and combines what arrived;
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


class P2PExchange:
    """Exchange buffers of a sharded full reduce, shared between the ranks of a
    torch.distributed group (one process per GPU, every rank on its own GPU).

    Collective to create and to close.  Each :meth:`reduce_full` call is one
    epoch; every rank must make the same calls in the same order on one
    stream, which keeps a rank at most one epoch ahead of a peer still reading
    (the device kernel double-buffers slots by epoch parity).
    """

    def __init__(self, device, group=None):
        import torch.distributed as td
        from . import ipc_buffer_close, ipc_buffer_create, ipc_buffer_open, lib
        self.world = td.get_world_size(group)
        self.rank = td.get_rank(group)
        self.device = torch.device(device)
        props = torch.cuda.get_device_properties(self.device)
        ident = (str(getattr(props, "uuid", "")), self.device.index)
        with torch.cuda.device(self.device):
            nbytes = lib().mcke_sm100_reduce_p2p_buffer_bytes(self.world)
            self._own, handle = ipc_buffer_create(nbytes)
            got = [None] * self.world
            td.all_gather_object(got, (ident, handle), group=group)
            if len({g[0] for g in got}) != self.world:
                ipc_buffer_close(self._own, False)
                raise ValueError("P2PExchange needs every rank on a distinct GPU "
                                 "(its combine kernels wait on one another)")
            self._opened = []
            ptrs = []
            for r, (_, h) in enumerate(got):
                if r == self.rank:
                    ptrs.append(self._own)
                else:
                    p = ipc_buffer_open(h)
                    self._opened.append(p)
                    ptrs.append(p)
            self.table = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.epoch = 0
        self._group = group

    def reduce_full(self, x, index_base: int, out=None, stream=None, early_read: bool = False):
        from . import reduce_full_p2p
        self.epoch += 1
        return reduce_full_p2p(x, index_base, self.table, self.world, self.rank, self.epoch, out=out,
                               stream=stream, early_read=early_read)

    def close(self) -> None:
        """Collective: every rank's kernels are done before any buffer goes."""
        import torch.distributed as td
        from . import ipc_buffer_close
        if self.table is None:
            return
        torch.cuda.synchronize(self.device)
        td.barrier(group=self._group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                ipc_buffer_close(p, True)
            td.barrier(group=self._group)
            ipc_buffer_close(self._own, False)
        self.table = None

