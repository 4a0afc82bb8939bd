"""Sharded full reduce with the peer-to-peer combine
(mcke_sm100_reduce_full_p2p_f32): bit-exact against the single-GPU entry point
at world 1, the bounded wait for a partial that never arrives, and two ranks on
two GPUs (one process each, exchange buffers shared with CUDA IPC) against the
oracle.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mcke  # noqa: E402
from mcke import shard as mshard  # noqa: E402


def _ll_slot(s, m, i, tag):
    """A 64-byte exchange slot: six 8-byte words, each 4 data bytes of the
    24-byte partial plus the 4-byte tag."""
    data = np.frombuffer(mshard.pack_partial(s, m, i), dtype=np.uint32).astype(np.uint64)
    words = np.zeros(8, dtype=np.uint64)
    words[:6] = data | (np.uint64(tag) << np.uint64(32))
    return words.view(np.uint8).copy()


def _table(*bufs):
    return torch.tensor([b.data_ptr() for b in bufs], dtype=torch.int64, device="cuda")


@pytest.mark.parametrize("n", [0, 1, 5, 3_000_007])
def test_world_one_matches_reduce_full_bitwise(n):
    v = oracle.fill_random(max(n, 1), 21)[:n]
    if n > 12:
        v[n - 3] = v[12] = np.float32(1.25)
    x = torch.from_numpy(v).cuda()
    buf = torch.zeros(mcke.lib().mcke_sm100_reduce_p2p_buffer_bytes(1), dtype=torch.uint8, device="cuda")
    table = _table(buf)
    want = mcke.reduce_full(x).cpu().numpy().tobytes()
    for epoch in (1, 2, 3):  # both slot halves, then the first again
        got = mcke.reduce_full_p2p(x, 0, table, 1, 0, epoch).cpu().numpy().tobytes()
        assert got == want, (epoch, mcke.decode_result(got), mcke.decode_result(want))
    mcke.check_device_errors()


def test_automatic_epochs_survive_graph_replay():
    # epoch 0: the kernel takes the epoch from the counter in its own buffer,
    # so a captured launch (whose arguments are fixed) can be replayed
    v = oracle.fill_random(1_000_003, 23)
    x = torch.from_numpy(v).cuda()
    buf = torch.zeros(mcke.lib().mcke_sm100_reduce_p2p_buffer_bytes(1), dtype=torch.uint8, device="cuda")
    table = _table(buf)
    out = torch.empty(16, dtype=torch.uint8, device="cuda")
    want = mcke.reduce_full(x).cpu().numpy().tobytes()
    for _ in range(3):
        assert mcke.reduce_full_p2p(x, 0, table, 1, 0, 0, out=out).cpu().numpy().tobytes() == want
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        mcke.reduce_full_p2p(x, 0, table, 1, 0, 0, out=out)
    for _ in range(4):
        out.zero_()
        g.replay()
        assert out.cpu().numpy().tobytes() == want
    counter = buf[-64:-56].cpu().numpy().view(np.uint64)[0]
    assert counter == 3 + 4  # three eager calls and four replays (the capture itself runs nothing)
    mcke.check_device_errors()


def test_index_base_and_rank_slot():
    # rank 1 of a world of 2 whose peer has already published: the combined
    # result covers both shards, indices offset by index_base
    v = oracle.fill_random(200_001, 4)
    v[150_000] = np.float32(1.5)
    lo, hi = v[:100_000], v[100_000:]
    x0, x1 = torch.from_numpy(lo).cuda(), torch.from_numpy(hi).cuda()
    nb = mcke.lib().mcke_sm100_reduce_p2p_buffer_bytes(2)
    b0 = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    b1 = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    table = _table(b0, b1)
    # Rank 0 has already published epoch 1 into rank 1's buffer: epoch 1 uses
    # the odd half (slots 2..3 of 64 bytes), rank 0's slot is 2.  Rank 1's call
    # stores its own slot 3 in both buffers and folds slots 2, 3 of b1.
    s0, m0, i0 = mcke.decode_partial(mcke.reduce_full_partial(x0, 0))
    b1[2 * 64:3 * 64].copy_(torch.from_numpy(_ll_slot(s0, m0, i0, 1)))
    got = mcke.decode_result(mcke.reduce_full_p2p(x1, 100_000, table, 2, 1, 1))
    want = oracle.full_reduce(v)
    assert got[1:] == (1.5, 150_000)
    assert abs(got[0] - np.float32(want[0])) <= np.spacing(np.float32(abs(want[0])))
    mcke.check_device_errors()
    # rank 1's partial reached rank 0's buffer too, every word tagged
    words = b0[3 * 64:4 * 64].cpu().numpy().view(np.uint64)
    assert all(int(w) >> 32 == 1 for w in words[:6])
    data = (words[:6] & np.uint64(0xFFFFFFFF)).astype(np.uint32).tobytes()
    assert mshard.unpack_partial(data)[1:] == (1.5, 150_000)


def test_missing_peer_expires_and_is_reported():
    # slot 1 of this rank's buffer is a flag nothing sets: the bounded wait
    # (1 s) gives up, the result says argmax -1, the error is reported on the
    # host and the context stays usable
    x = torch.ones(1000, device="cuda")
    nb = mcke.lib().mcke_sm100_reduce_p2p_buffer_bytes(2)
    b0 = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    b1 = torch.zeros(nb, dtype=torch.uint8, device="cuda")
    out = mcke.reduce_full_p2p(x, 0, _table(b0, b1), 2, 0, 1)
    assert mcke.decode_result(out)[2] == -1
    with pytest.raises(mcke.MckeError, match="did not arrive"):
        mcke.check_device_errors()
    mcke.check_device_errors()  # cleared
    assert mcke.decode_result(mcke.reduce_full(x))[:2] == (1000.0, 1.0)


def test_argument_checks():
    x = torch.ones(16, device="cuda")
    buf = torch.zeros(64, dtype=torch.uint8, device="cuda")
    t = _table(buf)
    for world, rank, epoch in ((0, 0, 1), (1, 1, 1), (1, 0, 1 << 32)):
        with pytest.raises(mcke.MckeError):
            mcke.reduce_full_p2p(x, 0, t, world, rank, epoch)
    with pytest.raises(mcke.MckeError):
        mcke.reduce_full_p2p(x, -1, t, 1, 0, 1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n, q):
    import torch.distributed as td
    from mcke import shard
    try:
        torch.cuda.set_device(rank)
        td.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                              timeout=__import__("datetime").timedelta(seconds=60))
        v = oracle.fill_random(n, 31)
        v[n - 5] = v[777] = np.float32(1.5)
        a, b = shard.bounds(n, world, rank)
        x = torch.from_numpy(v[a:b]).cuda()
        ex = shard.P2PExchange(torch.device("cuda", rank))
        res = []
        for i in range(5):  # the last three read x before waiting (MCKE_REDUCE_EARLY_READ)
            res.append(mcke.decode_result(ex.reduce_full(x, a, early_read=i >= 2)))
        torch.cuda.synchronize()
        mcke.check_device_errors()
        ex.close()
        td.destroy_process_group()
        q.put((rank, res))
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, repr(e)))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_ranks_on_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    n, world, port = 4_000_037, 2, _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    v = oracle.fill_random(n, 31)
    v[n - 5] = v[777] = np.float32(1.5)
    ws = np.float32(oracle.full_reduce(v)[0])
    for r in range(world):
        assert isinstance(got[r], list), got[r]
        for s, m, i in got[r]:
            assert (m, i) == (1.5, 777)
            assert abs(s - ws) <= np.spacing(np.float32(abs(ws)))
        assert got[r] == got[0]


def test_timeline_variant_same_bits_and_ordered_stamps():
    # the measuring aid gives the same result and stamps in phase order
    v = oracle.fill_random(5_000_011, 31)
    x = torch.from_numpy(v).cuda()
    buf = torch.zeros(mcke.lib().mcke_sm100_reduce_p2p_buffer_bytes(1), dtype=torch.uint8, device="cuda")
    table = _table(buf)
    want = mcke.reduce_full(x).cpu().numpy().tobytes()
    stamps = mcke.timeline_buffer(3, "cuda")
    for i in range(3):
        got = mcke.reduce_full_p2p_timeline(x, 0, table, 1, 0, 0, stamps[i]).cpu().numpy().tobytes()
        assert got == want
    mcke.check_device_errors()
    t = stamps.cpu().numpy().view(np.uint64)
    for row in t:
        entry, start, last_start, first_done, last_done, folded, exchanged, counted = (int(w) for w in row[:8])
        assert entry <= start <= last_start <= last_done <= counted <= folded <= exchanged, row
        assert start <= first_done <= last_done, row
        assert exchanged - start < 10_000_000  # well under 10 ms
    assert np.all(t[1:, 1] >= t[:-1, 6])  # a step starts after the previous one stored its result
