"""The host layer's planning on the CPU (no GPU): graph build-time checks, the
sharding pass over 1/2/4/8 devices, stream assignment and the memory plan.
GraphExecutor.plan_dry() runs placement, streams and memory without CUDA.
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mini-cuda-kernel-engine_b200")


@pytest.fixture(scope="module")
def host():
    import mcke
    if not os.path.exists(mcke.LIB_PATH):
        subprocess.run([sys.executable, os.path.join(PKG, "build.py")], check=True)
    subprocess.run(["make", "-s", "-C", os.path.join(PKG, "host")], check=True)
    from mcke import host as h
    return h


def dag(h, branches=4, rows=8192, d=4096, f=16384, fused=True):
    """branches x (GEMM -> +b1 -> GELU -> GEMM -> +b2 -> softmax), bf16."""
    g = h.Graph()
    x = g.input("X", (rows, d), "bf16", "row_split")
    outs = []
    for i in range(branches):
        w1 = g.input(f"W1_{i}", (d, f), "bf16")
        b1 = g.input(f"b1_{i}", (f,), "f32")
        w2 = g.input(f"W2_{i}", (f, d), "bf16")
        b2 = g.input(f"b2_{i}", (d,), "f32")
        if fused:
            hh = g.gemm(x, w1, bias=b1, act="gelu_tanh", out_dtype="bf16", name=f"gemm1_{i}")
            y = g.gemm(hh, w2, bias=b2, name=f"gemm2_{i}")
        else:
            h0 = g.gemm(x, w1, out_dtype="bf16", name=f"gemm1_{i}")
            hh = g.bias_act(h0, b1, "gelu_tanh", name=f"bias_gelu_{i}")
            y0 = g.gemm(hh, w2, name=f"gemm2_{i}")
            y = g.bias_act(y0, b2, "none", name=f"bias2_{i}")
        p = g.softmax(y, name=f"softmax_{i}")
        g.output(p)
        outs.append(p)
    g.finalize()
    return g, x, outs


@pytest.mark.parametrize("ndev", [1, 2, 4, 8])
@pytest.mark.parametrize("fused", [True, False])
def test_dag_shards_rows_with_no_collective(host, ndev, fused):
    g, x, outs = dag(host, fused=fused)
    ex = host.Executor(g, devices=list(range(ndev)), streams_per_device=4)
    ex.plan_dry()
    want = "row_split" if ndev > 1 else "replicated"
    assert ex.placement(x) == want
    for p in outs:
        assert ex.placement(p) == want
    # weights stay whole on every device
    assert ex.placement(x + 1) == "replicated"
    # four independent branches -> four streams, nothing crosses streams
    assert ex.num_events() == 0
    d = ex.describe()
    streams = {ln.split("stream=")[1].split()[0] for ln in d.splitlines() if ln.startswith("node softmax")}
    assert streams == {"0", "1", "2", "3"}
    # per-device arena: inputs + outputs + intermediates, shrinking with the row split
    rows = 8192 // ndev
    io = 4 * (2 * (4096 * 16384 * 2) + 16384 * 4 + 4096 * 4) + rows * 4096 * 2 + 4 * rows * 4096 * 4
    assert ex.arena_bytes(0) >= io


def test_intermediates_reuse_memory_on_one_stream(host):
    g = host.Graph()
    x = g.input("x", (1024, 1024))
    b = g.input("b", (1024,))
    t = x
    for i in range(6):
        t = g.bias_act(t, b, "relu", name=f"ba{i}")
        t = g.softmax(t, name=f"sm{i}")
    g.output(t)
    g.finalize()
    ex = host.Executor(g, devices=[0], streams_per_device=4)
    ex.plan_dry()
    mb = 1024 * 1024 * 4
    # 12 intermediates of 4 MiB on one stream chain: two ping-pong blocks suffice
    assert ex.arena_bytes(0) <= 4 * mb + 4096 + 65536
    assert ex.num_events() == 0


def test_fanout_join_records_events(host):
    g = host.Graph()
    x = g.input("x", (256, 256))
    b = g.input("b", (256,))
    a1 = g.bias_act(x, b, "relu", name="left")
    a2 = g.bias_act(x, b, "gelu_erf", name="right")
    a3 = g.bias_act(a1, b, "none", name="left2")
    s = g.softmax(a2, name="right2")
    g.output(a3)
    g.output(s)
    g.finalize()
    ex = host.Executor(g, devices=[0], streams_per_device=2)
    ex.plan_dry()
    assert ex.num_events() == 0  # two chains on two streams
    g2 = host.Graph()
    x = g2.input("x", (256, 256))
    b = g2.input("b", (256,))
    y = g2.bias_act(x, b, "relu", name="p")
    z1 = g2.softmax(y, name="c1")
    z2 = g2.softmax(y, name="c2")  # second consumer of y lands on another stream
    g2.output(z1)
    g2.output(z2)
    g2.finalize()
    ex2 = host.Executor(g2, devices=[0], streams_per_device=2)
    ex2.plan_dry()
    assert ex2.num_events() == 1


def _fanout(host, cols, branches=4, depth=4, acts=("gelu_tanh",)):
    g = host.Graph()
    x = g.input("x", (64, cols))
    for br in range(branches):
        h = x
        for k in range(depth):
            b = g.input(f"b{br}_{k}", (cols,))
            h = g.bias_act(h, b, acts[br % len(acts)], name=f"n{br}_{k}")
        g.output(h)
    g.finalize()
    return g


def test_level_grouped_schedule_groups_a_level_of_bias_nodes(host):
    # 4 branches x 4 bias+GELU nodes: one grouped launch per level, no events
    ex = host.Executor(_fanout(host, 512), devices=[0], streams_per_device=4, schedule="level_grouped")
    ex.plan_dry()
    assert ex.launch_items() == (4, 4)
    assert ex.num_events() == 0
    # two activations: a level splits into one group per activation
    ex = host.Executor(_fanout(host, 1024, acts=("gelu_tanh", "relu")), devices=[0, 1], schedule="level_grouped")
    ex.plan_dry()
    assert ex.launch_items() == (8, 2)
    # 256 columns: the grouped kernel does not take them, one launch per node
    ex = host.Executor(_fanout(host, 256), devices=[0], schedule="level_grouped")
    ex.plan_dry()
    assert ex.launch_items() == (16, 1)
    # the other schedules never group
    for sched in ("sequential", "level_parallel", "chain_greedy"):
        ex = host.Executor(_fanout(host, 512), devices=[0], schedule=sched)
        ex.plan_dry()
        assert ex.launch_items() == (16, 1), sched


def test_column_split_gemm_and_range_split_reduce(host):
    g = host.Graph()
    a = g.input("A", (512, 256))
    b = g.input("B", (256, 1024))
    c = g.gemm(a, b, name="gemm")
    v = g.input("v", (1 << 20,))
    r = g.reduce_full(v, name="reduce")
    g.output(c)
    g.output(r)
    g.finalize()
    ex = host.Executor(g, devices=[0, 1, 2, 3])
    ex.plan_dry()
    assert ex.placement(a) == "replicated"
    assert ex.placement(b) == "col_split"
    assert ex.placement(c) == "col_split"
    assert ex.placement(v) == "row_split"
    assert ex.placement(r) == "replicated"


def test_tensor_core_f32_gemm_sizes_its_split_workspace(host):
    # kTcgen05Tf32x3 asks for the hi/lo split of A and of its B column block
    # (8 bytes per element of each), which the per-stream scratch must hold
    m, k, n, d = 512, 256, 1024, 2
    arenas = []
    for variant in (host.GEMM_VARIANT_TILED_REGBLOCK, host.GEMM_VARIANT_TCGEN05_TF32X3):
        g = host.Graph()
        a, b = g.input("A", (m, k)), g.input("B", (k, n))
        g.output(g.gemm(a, b, variant=variant))
        g.finalize()
        ex = host.Executor(g, devices=list(range(d)))
        ex.plan_dry()
        arenas.append(ex.arena_bytes(0))
    split = 8 * (m * k + k * n // d)
    assert arenas[1] - arenas[0] >= split - 4096  # (alignment slack)


def test_sharding_refuses_what_needs_a_collective(host):
    g = host.Graph()
    a = g.input("A", (64, 64))
    b = g.input("B", (64, 64))
    c = g.gemm(a, b, name="gemm")           # column-split output
    s = g.softmax(c, name="softmax")        # rows of a column-split tensor
    g.output(s)
    g.finalize()
    ex = host.Executor(g, devices=[0, 1])
    with pytest.raises(host.MckeError) as e:
        ex.plan_dry()
    assert e.value.code == 3 and "softmax" in e.value.message  # FailedPrecondition
    ex1 = host.Executor(g, devices=[0])
    ex1.plan_dry()  # one device: nothing to shard


def test_build_time_errors_name_the_node(host):
    g = host.Graph()
    x = g.input("x", (8, 16))
    bad_bias = g.input("b", (15,))
    with pytest.raises(host.MckeError) as e:
        g.bias_act(x, bad_bias, "relu", name="my_bias_act")
    assert e.value.code == 2 and "my_bias_act" in e.value.message
    w = g.input("w", (16, 4))
    with pytest.raises(host.MckeError) as e:  # epilogue fusion needs bf16 operands
        g.gemm(x, w, act="gelu_tanh", name="g1")
    assert "g1" in e.value.message
    w2 = g.input("w2", (17, 4))
    with pytest.raises(host.MckeError):
        g.gemm(x, w2, name="g2")  # inner dimensions disagree
    with pytest.raises(host.MckeError):
        g.gemm(x, w, name="g3", variant=1)  # kTiledSmem with the default tile: rejected, as in the reference
    with pytest.raises(host.MckeError) as e:
        g.gemm(x, w, name="g4", variant=4)  # the cuBLAS row is not part of the library
    assert e.value.code == 4


def test_too_few_rows_to_split(host):
    g = host.Graph()
    x = g.input("x", (3, 64), placement="row_split")
    s = g.softmax(x)
    g.output(s)
    g.finalize()
    ex = host.Executor(g, devices=[0, 1, 2, 3])
    with pytest.raises(host.MckeError):
        ex.plan_dry()


def test_graph_roofline_bound_is_the_reference_cost_model(host):
    # sum over nodes of max(flops / peak, bytes / bandwidth): a bf16 GEMM with a
    # fused epilogue (flop-bound here) and a softmax (byte-bound)
    m, k, n = 512, 256, 1024
    g = host.Graph()
    x = g.input("x", (m, k), "bf16")
    w = g.input("w", (k, n), "bf16")
    b = g.input("b", (n,), "f32")
    y = g.gemm(x, w, bias=b, name="gemm")  # f32 output
    g.output(g.softmax(y, name="softmax"))
    g.finalize()
    tf, gbs = 100.0, 1000.0
    gemm_flops = 2 * m * n * k
    gemm_bytes = (m * k + k * n) * 2 + m * n * 4 + n * 4
    soft_bytes = 2 * m * n * 4
    soft_flops = 5 * m * n
    want = (max(gemm_flops / (tf * 1e12), gemm_bytes / (gbs * 1e9)) +
            max(soft_flops / (tf * 1e12), soft_bytes / (gbs * 1e9))) * 1e3
    assert g.roofline_ms(tf, gbs) == pytest.approx(want, rel=1e-12)


def _flops_bytes(g):
    # the cost model's two terms of a one-node graph: with a huge bandwidth the
    # bound is flops / peak, with a huge peak it is bytes / bandwidth
    big = 1e30
    flops = g.roofline_ms(1.0, big) * 1e-3 * 1e12
    byts = g.roofline_ms(big, 1.0) * 1e-3 * 1e9
    return round(flops), round(byts)


@pytest.mark.parametrize("case", ["gemm_f32", "bias_none", "bias_relu", "bias_gelu_tanh", "bias_gelu_erf",
                                  "softmax", "reduce_sum", "reduce_max"])
def test_op_costs_match_the_reference_formulas(host, case):
    # The reference pins each op's cost (src/graph/ops_gemm.cpp:69-70,
    # ops_bias_act.cpp:51-97, ops_softmax.cpp:62-63, ops_reduce.cpp:91-92);
    # the same formulas here, through the graph-level bound.
    m, k, n = 96, 40, 72
    g = host.Graph()
    if case == "gemm_f32":
        a, b = g.input("a", (m, k)), g.input("b", (k, n))
        g.output(g.gemm(a, b, name="op"))
        want = (2 * m * n * k, (m * k + k * n + m * n) * 4)
    elif case.startswith("bias"):
        act = case[len("bias_"):]
        x, bias = g.input("x", (m, n)), g.input("bias", (n,))
        g.output(g.bias_act(x, bias, act, name="op"))
        per = {"none": 1, "relu": 2, "gelu_tanh": 10, "gelu_erf": 22}[act]
        want = (m * n * per, 2 * m * n * 4 + n * 4)
    elif case == "softmax":
        x = g.input("x", (m, n))
        g.output(g.softmax(x, name="op"))
        want = (5 * m * n, 2 * m * n * 4)
    else:
        kind = case[len("reduce_"):]
        x = g.input("x", (m, n))
        g.output(g.reduce_row(x, {"sum": 0, "max": 1}[kind], name="op"))  # ReduceParams::Kind
        want = (0 if kind == "max" else m * (n - 1), (m * n + m) * 4)
    g.finalize()
    assert _flops_bytes(g) == want
