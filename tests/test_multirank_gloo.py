"""The N > 1 host path on CPU: two gloo ranks (127.0.0.1) shard a vector by
contiguous range, reduce their shards with the oracle (standing in for the
GPU partial kernel), exchange the 24-byte partials with the same helper the
bench uses at N GPUs, and combine them in rank order.  A second test makes one
rank leave before the exchange: the other rank's collective must end with an
error inside the short process-group timeout, not hang.
"""
from __future__ import annotations

import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mini-cuda-kernel-engine_b200")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    for p in (ROOT, PKG):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as td
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    td.init_process_group("gloo", rank=rank, world_size=world,
                          timeout=datetime.timedelta(seconds=timeout_s))
    return td


def _reduce_worker(rank, world, port, n, seed, q):
    td = _init(rank, world, port)
    try:
        import oracle
        from mcke import shard
        x = oracle.fill_random(n, seed)
        x[n - 3] = x[5] = np.float32(1.5)  # a tie across the two shards
        b0, b1 = shard.bounds(n, world, rank)
        s, m, i = oracle.full_reduce(x[b0:b1], index_base=b0)
        part = torch.frombuffer(bytearray(shard.pack_partial(s, float(m), i)), dtype=torch.uint8)
        gathered = shard.exchange_partials(part, world)
        raw = gathered.numpy().tobytes()
        parts = [shard.unpack_partial(raw[k * 24:(k + 1) * 24]) for k in range(world)]
        got = shard.combine_host(parts)
        want = oracle.full_reduce(x)
        q.put((rank, got, (want[0], float(want[1]), want[2])))
    finally:
        td.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_reduce_exchange_over_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    n = 100_003
    procs = [ctx.Process(target=_reduce_worker, args=(r, world, port, n, 7, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, want in results:
        assert got[1:] == want[1:] == (1.5, 5), (rank, got, want)
        assert np.float32(got[0]) == np.float32(want[0])


def _leaver_worker(rank, world, port, q):
    td = _init(rank, world, port, timeout_s=5)
    from mcke import shard
    if rank == 1:
        q.put((rank, "left"))
        q.close()
        q.join_thread()  # the message is out before the process goes
        os._exit(0)  # leaves between steps, before the exchange
    part = torch.zeros(24, dtype=torch.uint8)
    try:
        shard.exchange_partials(part, world)
        q.put((rank, "completed"))
    except Exception as e:  # gloo reports the missing peer
        q.put((rank, "error:" + type(e).__name__))


def test_a_rank_that_leaves_ends_the_exchange_with_an_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert got[1] == "left"
    assert got[0].startswith("error:"), got
