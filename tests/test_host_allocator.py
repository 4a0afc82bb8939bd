"""The host layer's allocator surface and executor policies on the CPU (no GPU).

* tests/cpp/allocator_and_executor_check.cpp, compiled here against the host
  headers and libmcke_host.so: the BuddyAllocator over host slabs (sizes,
  alignment, splitting, buddy merging, the slab cap, bypass, trim, validate)
  and a GraphExecutor built through the reference's constructor
  GraphExecutor(Graph, DeviceAllocator&, DeviceInfo, ExecutorOptions)
  (include/mcke/graph/executor.hpp:285 of the reference), planned dry.
* The schedule and memory policies through plan_dry(): kSequential keeps every
  node on stream 0, kLevelParallel deals a level's nodes over the streams, and
  kAllocPerTensor needs more arena than the reusing policies.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mini-cuda-kernel-engine_b200")
CUDA = "/usr/local/cuda"


@pytest.fixture(scope="module")
def host():
    import mcke
    if not os.path.exists(mcke.LIB_PATH):
        subprocess.run([sys.executable, os.path.join(PKG, "build.py")], check=True)
    subprocess.run(["make", "-s", "-C", os.path.join(PKG, "host")], check=True)
    from mcke import host as h
    return h


def test_buddy_allocator_and_reference_constructor(host, tmp_path):
    exe = str(tmp_path / "check")
    src = os.path.join(ROOT, "tests", "cpp", "allocator_and_executor_check.cpp")
    cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", src, "-o", exe,
           "-I", os.path.join(PKG, "host", "include"), "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), "-L", os.path.join(PKG, "lib"), "-lmcke_host",
           "-Wl,-rpath," + os.path.join(PKG, "lib")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout + r.stderr


def _fanout(h, branches=4, depth=4):
    g = h.Graph()
    x = g.input("x", (256, 256))
    for b in range(branches):
        t = x
        for k in range(depth):
            t = g.bias_act(t, g.input(f"b{b}_{k}", (256,)), "gelu_tanh", name=f"n{b}_{k}")
        g.output(t)
    g.finalize()
    return g


def _streams(desc: str) -> dict:
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"node (\S+) \(\w+\) stream=(\d+)", desc)}


def test_schedule_policies(host):
    g = _fanout(host)
    seq = host.Executor(g, devices=[0], streams_per_device=4, schedule="sequential")
    seq.plan_dry()
    assert set(_streams(seq.describe()).values()) == {0}
    assert seq.num_events() == 0
    lvl = host.Executor(g, devices=[0], streams_per_device=4, schedule="level_parallel")
    lvl.plan_dry()
    st = _streams(lvl.describe())
    for k in range(4):  # the four nodes of one level sit on four different streams
        assert sorted(st[f"n{b}_{k}"] for b in range(4)) == [0, 1, 2, 3]
    chain = host.Executor(g, devices=[0], streams_per_device=4, schedule="chain_greedy")
    chain.plan_dry()
    st = _streams(chain.describe())
    for b in range(4):  # a chain keeps its stream
        assert len({st[f"n{b}_{k}"] for k in range(4)}) == 1
    assert chain.num_events() == 0


def test_memory_policies(host):
    g = _fanout(host, branches=2, depth=6)
    per_tensor = host.Executor(g, devices=[0], streams_per_device=2, memory="alloc_per_tensor")
    per_tensor.plan_dry()
    reuse = host.Executor(g, devices=[0], streams_per_device=2, memory="reuse_happens_before")
    reuse.plan_dry()
    same = host.Executor(g, devices=[0], streams_per_device=2, memory="reuse_same_stream")
    same.plan_dry()
    assert reuse.arena_bytes(0) == same.arena_bytes(0) < per_tensor.arena_bytes(0)


def test_memory_plan_fuzz_finds_no_unordered_reuse(host, tmp_path):
    # tests/cpp/memory_plan_fuzz.cpp: 150 random DAGs x 4 schedules (grouped
    # launches included) x 2 reuse policies x {1, 2, 4} streams, planned dry;
    # every two tensors that share arena bytes must have one's whole life in
    # earlier launch items than the other's producer, on one stream (the
    # reference's memory-plan race fuzz, run on this planner)
    exe = str(tmp_path / "fuzz")
    src = os.path.join(ROOT, "tests", "cpp", "memory_plan_fuzz.cpp")
    cmd = ["g++", "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", src, "-o", exe,
           "-I", os.path.join(PKG, "host", "include"), "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), "-L", os.path.join(PKG, "lib"), "-lmcke_host",
           "-Wl,-rpath," + os.path.join(PKG, "lib")]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("OK"), r.stdout + r.stderr
    assert "all ordered" in r.stdout and " 0 grouped" not in r.stdout
