"""Grouped bias + activation (mcke_sm100_bias_act_f32_group) and the executor's
level-grouped schedule that issues it:
  * a group of jobs of different shapes gives, bit for bit, what one
    mcke_sm100_bias_act_f32 call per job gives (power-of-two and other
    chunks per row, an empty job, every activation);
  * a fan-out graph of bias + GELU nodes run level-grouped (eager and CUDA
    graph) gives the chain-greedy run's bits, with one launch per level.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mcke  # noqa: E402
from mcke import host as mhost  # noqa: E402


def _t(shape, seed):
    n = int(np.prod(shape))
    return torch.from_numpy(oracle.fill_random(max(n, 1), seed)[:n].reshape(shape) * 3).cuda()


@pytest.mark.parametrize("act", ["gelu_tanh", "gelu_erf", "relu", "none"])
def test_group_equals_one_call_per_job(act):
    shapes = [(64, 512), (33, 1536), (1, 512), (128, 1024), (0, 512), (7, 2560)]
    jobs, want = [], []
    for k, (r, c) in enumerate(shapes):
        x, b = _t((r, c), 10 + k), _t((c,), 40 + k)
        jobs.append((x, b, torch.full_like(x, float("nan"))))
        want.append(mcke.bias_act(x, b, act, vector_width=4))
    mcke.bias_act_group(jobs, act)
    torch.cuda.synchronize()
    mcke.check_device_errors()
    for k, ((_, _, y), w) in enumerate(zip(jobs, want)):
        assert torch.equal(y.view(torch.int32), w.view(torch.int32)), (act, shapes[k])


def test_group_of_sixteen_and_the_oracle():
    jobs = []
    for k in range(mcke.BIAS_ACT_GROUP_MAX):
        x, b = _t((16 + k, 512), 100 + k), _t((512,), 200 + k)
        jobs.append((x, b, torch.empty_like(x)))
    mcke.bias_act_group(jobs, "gelu_tanh")
    torch.cuda.synchronize()
    for x, b, y in jobs:
        ref = oracle.bias_act(x.cpu().numpy(), b.cpu().numpy(), "gelu_tanh")
        r = oracle.compare(y.cpu().numpy(), ref, 1e-5, 1e-6)
        assert r["mismatches"] == 0, r


def _fanout(cols=512, rows=256, branches=4, depth=4):
    g = mhost.Graph()
    x = g.input("x", (rows, cols))
    rng = np.random.default_rng(5)
    feeds = {x: rng.standard_normal((rows, cols)).astype(np.float32)}
    outs = []
    for br in range(branches):
        h = x
        for k in range(depth):
            b = g.input(f"b{br}_{k}", (cols,))
            feeds[b] = (rng.random(cols, dtype=np.float32) * 2 - 1)
            h = g.bias_act(h, b, "gelu_tanh", name=f"n{br}_{k}")
        g.output(h)
        outs.append(h)
    g.finalize()
    return g, feeds, outs


@pytest.mark.parametrize("cuda_graph", [False, True])
def test_level_grouped_run_equals_chain_greedy(cuda_graph):
    results = {}
    for sched in ("chain_greedy", "level_grouped"):
        g, feeds, outs = _fanout()
        ex = mhost.Executor(g, devices=[0], streams_per_device=4, cuda_graph=cuda_graph and sched != "chain_greedy",
                            schedule=sched)
        ex.plan()
        if sched == "level_grouped":
            assert ex.launch_items() == (4, 4)
        for t, arr in feeds.items():
            ex.set_input(t, arr)
        for _ in range(3):  # replays reuse the planned blocks
            ex.run()
        ex.synchronize()
        results[sched] = [ex.output(o) for o in outs]
        del ex, g
    mcke.check_device_errors()
    for a, b in zip(results["chain_greedy"], results["level_grouped"]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
