"""The executor's numerics gate and its allocator surface on the GPU.

* GraphExecutor::validate_numerics (the reference's gate,
  src/graph/executor.cpp:416-607): every {schedule} x {memory policy} x
  {eager, CUDA-graph replay} configuration, several runs each, bit for bit
  against a sequential, alloc-per-tensor, eager golden run -- on the config-5
  DAG (fused and unfused), the reference's fan-out and a range-sharded full
  reduce, on one GPU and on a device list that repeats it (two shards).
* Arenas from a per-device BuddyAllocator (the reference's DeviceAllocator
  interface): the DAG's outputs equal those of an executor that cudaMallocs its
  arena, and the allocator saw one allocation per executor and one slab.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

from mcke import host  # noqa: E402


def _dag(fused: bool, rows=256, d=128, f=256, branches=2):
    g = host.Graph()
    x = g.input("X", (rows, d), "bf16", "row_split")
    feeds = {x: oracle.to_bf16(oracle.fill_normal(rows * d, 1).reshape(rows, d))}
    outs = []
    for i in range(branches):
        w1 = g.input(f"W1_{i}", (d, f), "bf16")
        b1 = g.input(f"b1_{i}", (f,), "f32")
        w2 = g.input(f"W2_{i}", (f, d), "bf16")
        b2 = g.input(f"b2_{i}", (d,), "f32")
        feeds[w1] = oracle.to_bf16(oracle.fill_normal(d * f, 10 * i + 2, 0.0, 0.05).reshape(d, f))
        feeds[b1] = oracle.fill_random(f, 10 * i + 3)
        feeds[w2] = oracle.to_bf16(oracle.fill_normal(f * d, 10 * i + 4, 0.0, 0.05).reshape(f, d))
        feeds[b2] = oracle.fill_random(d, 10 * i + 5)
        if fused:
            hh = g.gemm(x, w1, bias=b1, act="gelu_tanh", out_dtype="bf16", name=f"gemm1_{i}")
            y = g.gemm(hh, w2, bias=b2, name=f"gemm2_{i}")
        else:
            hh = g.bias_act(g.gemm(x, w1, out_dtype="bf16", name=f"gemm1_{i}"), b1, "gelu_tanh", name=f"bg_{i}")
            y = g.bias_act(g.gemm(hh, w2, name=f"gemm2_{i}"), b2, "none", name=f"b2_{i}")
        p = g.softmax(y, name=f"softmax_{i}")
        g.output(p)
        outs.append(p)
    g.finalize()
    return g, feeds, outs


def _fanout():
    g = host.Graph()
    x = g.input("x", (512, 1024))
    feeds = {x: oracle.fill_normal(512 * 1024, 7).reshape(512, 1024)}
    for b in range(4):
        t = x
        for k in range(4):
            bias = g.input(f"b{b}_{k}", (1024,))
            feeds[bias] = oracle.fill_random(1024, 100 + 4 * b + k)
            t = g.bias_act(t, bias, "gelu_tanh", name=f"n{b}_{k}")
        g.output(t)
    g.finalize()
    return g, feeds


def _reduce():
    n = 3_000_007
    g = host.Graph()
    x = g.input("v", (n,))
    g.output(g.reduce_full(x))
    g.finalize()
    return g, {x: oracle.fill_random(n, 5)}


@pytest.mark.parametrize("devices", [[0], [0, 0]])
@pytest.mark.parametrize("case", ["dag_fused", "dag_unfused", "fanout", "reduce"])
def test_numerics_gate(case, devices):
    if case.startswith("dag"):
        g, feeds, _ = _dag(case == "dag_fused")
    elif case == "fanout":
        g, feeds = _fanout()
    else:
        g, feeds = _reduce()
    ex = host.Executor(g, devices=devices, streams_per_device=4, validate=True, buddy=True)
    ex.plan()
    for t, arr in feeds.items():
        ex.set_input(t, arr)
    r = ex.validate_numerics(repeats=3)
    assert r["passed"], r["detail"]
    assert r["configs"] == 24  # golden + 4 schedules x 3 memory policies x {eager, graph} - the golden's twin


def test_buddy_arena_matches_cudamalloc_arena():
    g, feeds, outs = _dag(True)
    runs = {}
    for buddy in (False, True):
        ex = host.Executor(g, devices=[0], streams_per_device=4, buddy=buddy, cuda_graph=buddy)
        ex.plan()
        for t, arr in feeds.items():
            ex.set_input(t, arr)
        ex.run()
        ex.run()
        ex.synchronize()
        runs[buddy] = [ex.output(p) for p in outs]
        if buddy:
            st = ex.alloc_stats(0)
            assert st["name"] == "buddy"
            assert st["alloc_calls"] == 1 and st["raw_malloc_calls"] == 1
            assert st["bytes_requested"] == ex.arena_bytes(0)
            assert st["bytes_in_use"] >= ex.arena_bytes(0)
        del ex
    for a, b in zip(runs[False], runs[True]):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_gate_fails_on_a_nondeterministic_op(tmp_path):
    # The gate's failure path, as the reference tests it: a C++ program defines
    # an op whose output changes on every launch and one that copies; the gate
    # must fail the first (naming the output and the word) and pass the second.
    import os
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    pkg = os.path.join(root, "mini-cuda-kernel-engine_b200")
    cuda = "/usr/local/cuda"
    exe = str(tmp_path / "gate_check")
    cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror",
           os.path.join(root, "tests", "cpp", "numerics_gate_check.cpp"), "-o", exe,
           "-I", os.path.join(pkg, "host", "include"), "-I", os.path.join(root, "include"),
           "-I", os.path.join(cuda, "include"), "-L", os.path.join(pkg, "lib"), "-lmcke_host",
           "-L", os.path.join(cuda, "lib64"), "-lcudart",
           "-Wl,-rpath," + os.path.join(pkg, "lib"), "-Wl,-rpath," + os.path.join(cuda, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout + r.stderr
    assert "nondeterministic op: [" in r.stdout and "word" in r.stdout, r.stdout


def test_buddy_allocator_keeps_a_block_from_another_stream_until_its_work_is_done(tmp_path):
    # The reference's stream-safety question for its pools, asked of this
    # repository's BuddyAllocator over device slabs (tests/cpp/stream_reuse_check.cpp):
    # a block freed on stream A while A still reads it goes to stream A again
    # at once but not to stream B, and A's reader sees its data intact.
    import os
    import subprocess
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    pkg = os.path.join(root, "mini-cuda-kernel-engine_b200")
    cuda = "/usr/local/cuda"
    exe = str(tmp_path / "stream_reuse_check")
    cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror",
           os.path.join(root, "tests", "cpp", "stream_reuse_check.cpp"), "-o", exe,
           "-I", os.path.join(pkg, "host", "include"), "-I", os.path.join(root, "include"),
           "-I", os.path.join(cuda, "include"), "-L", os.path.join(pkg, "lib"), "-lmcke_host", "-lmcke_sm100a",
           "-L", os.path.join(cuda, "lib64"), "-lcudart",
           "-Wl,-rpath," + os.path.join(pkg, "lib"), "-Wl,-rpath," + os.path.join(cuda, "lib64")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout + r.stderr
