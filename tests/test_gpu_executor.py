"""GraphExecutor on the GPU: the config-5 DAG (fused and unfused), a sharded
full reduce and a column-split GEMM, against the oracle composed op by op.

A device list may repeat a GPU ([0, 0] = two shards on GPU 0): the sharding
pass, per-shard arenas and streams, and the event-ordered peer-copy exchange
of partials then all run on one B200.
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


def _dag_inputs(rows, d, f, seed):
    x = oracle.to_bf16(oracle.fill_normal(rows * d, seed).reshape(rows, d))
    w1 = oracle.to_bf16(oracle.fill_normal(d * f, seed + 1, 0.0, 0.05).reshape(d, f))
    b1 = oracle.fill_random(f, seed + 2)
    w2 = oracle.to_bf16(oracle.fill_normal(f * d, seed + 3, 0.0, 0.05).reshape(f, d))
    b2 = oracle.fill_random(d, seed + 4)
    return x, w1, b1, w2, b2


def _dag_oracle(x, w1, b1, w2, b2, fused):
    f32 = oracle.bf16_to_f32
    lin1 = oracle.gemm(f32(x), f32(w1))
    if fused:
        hb = oracle.to_bf16(oracle.bias_act(lin1, b1, "gelu_tanh"))
    else:
        hb = oracle.to_bf16(oracle.bias_act(f32(oracle.to_bf16(lin1)), b1, "gelu_tanh"))
    y = oracle.bias_act(oracle.gemm(f32(hb), f32(w2)), b2, "none")
    return hb, oracle.row_softmax(y)


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("devices", [[0], [0, 0]])
def test_dag_matches_oracle(fused, devices):
    rows, d, f, branches = 256, 128, 256, 2
    g = host.Graph()
    x = g.input("X", (rows, d), "bf16", "row_split")
    data, outs, hs = {}, [], []
    for i in range(branches):
        xs = _dag_inputs(rows, d, f, 10 * i + 1)
        w1 = g.input(f"W1_{i}", (d, f), "bf16")
        b1 = g.input(f"b1_{i}", (f,), "f32")
        w2 = g.input(f"W2_{i}", (f, d), "bf16")
        b2 = g.input(f"b2_{i}", (d,), "f32")
        data.update({w1: xs[1], b1: xs[2], w2: xs[3], b2: xs[4]})
        data[x] = _dag_inputs(rows, d, f, 1)[0]
        if fused:
            hh = g.gemm(x, w1, bias=b1, act="gelu_tanh", out_dtype="bf16", name=f"gemm1_{i}")
            y = g.gemm(hh, w2, bias=b2, name=f"gemm2_{i}")
        else:
            h0 = g.gemm(x, w1, out_dtype="bf16", name=f"gemm1_{i}")
            hh = g.bias_act(h0, b1, "gelu_tanh", name=f"bias_gelu_{i}")
            y = g.bias_act(g.gemm(hh, w2, name=f"gemm2_{i}"), b2, "none", name=f"bias2_{i}")
        p = g.softmax(y, name=f"softmax_{i}")
        g.output(p)
        g.output(hh)
        outs.append((p, hh, xs))
    g.finalize()
    ex = host.Executor(g, devices=devices, streams_per_device=4)
    ex.plan()
    for t, arr in data.items():
        ex.set_input(t, arr)
    first = None
    for rep in range(2):
        ex.run()
        ex.synchronize()
        got = [(ex.output(p), ex.output(hh)) for p, hh, _ in outs]
        if first is None:
            first = got
        else:  # replay is bit-identical
            for (p0, h0), (p1, h1) in zip(first, got):
                assert np.array_equal(p0.view(np.uint32), p1.view(np.uint32))
                assert np.array_equal(h0, h1)
    for (p, hh, xs), (gp, gh) in zip(outs, first):
        want_h, want_p = _dag_oracle(data[x], xs[1], xs[2], xs[3], xs[4], fused)
        ulp = np.abs(gh.astype(np.int32) - want_h.astype(np.int32))
        assert (ulp <= 1).mean() > 0.999 and (ulp == 0).mean() > 0.98
        r = oracle.compare(gp, want_p, 1e-3, 1e-7)
        assert r["mismatches"] == 0 and abs(gp.sum(axis=1) - 1).max() < 1e-4, r


@pytest.mark.parametrize("devices", [[0], [0, 0, 0]])
def test_sharded_full_reduce(devices):
    n = 3_000_007
    v = oracle.fill_random(n, 5)
    v[2_999_999] = v[12] = np.float32(1.5)
    g = host.Graph()
    x = g.input("v", (n,))
    r = g.reduce_full(x)
    g.output(r)
    g.finalize()
    ex = host.Executor(g, devices=devices)
    ex.plan()
    ex.set_input(x, v)
    ex.run()
    import mcke
    s, m, i = mcke.decode_result(ex.output(r).tobytes())
    ws, wm, wi = oracle.full_reduce(v)
    assert (m, i) == (wm, wi) == (1.5, 12)
    assert abs(s - np.float32(ws)) <= np.spacing(np.float32(abs(ws)))


def test_column_split_gemm_f32():
    m, k, n = 96, 64, 260
    a = oracle.fill_random(m * k, 1).reshape(m, k)
    b = oracle.fill_random(k * n, 2).reshape(k, n)
    g = host.Graph()
    ta, tb = g.input("A", (m, k)), g.input("B", (k, n))
    c = g.gemm(ta, tb)
    g.output(c)
    g.finalize()
    ex = host.Executor(g, devices=[0, 0])
    ex.plan()
    assert ex.placement(c) == "col_split"
    ex.set_input(ta, a)
    ex.set_input(tb, b)
    ex.run()
    r = oracle.compare(ex.output(c), oracle.gemm(a, b), oracle.tol_gemm(k), oracle.abs_tol_gemm(k))
    assert r["mismatches"] == 0, r


two_gpus = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")


@two_gpus
def test_dag_on_two_gpus_matches_one():
    rows, d, f = 256, 128, 256
    outs = []
    for devices in ([0], [0, 1]):
        g = host.Graph()
        x = g.input("X", (rows, d), "bf16", "row_split")
        xs = _dag_inputs(rows, d, f, 3)
        w1, b1 = g.input("W1", (d, f), "bf16"), g.input("b1", (f,), "f32")
        w2, b2 = g.input("W2", (f, d), "bf16"), g.input("b2", (d,), "f32")
        hh = g.gemm(x, w1, bias=b1, act="gelu_tanh", out_dtype="bf16")
        p = g.softmax(g.gemm(hh, w2, bias=b2))
        g.output(p)
        g.finalize()
        ex = host.Executor(g, devices=devices)
        ex.plan()
        for t, arr in zip((x, w1, b1, w2, b2), xs):
            ex.set_input(t, arr)
        ex.run()
        outs.append(ex.output(p))
    # one GPU runs the 256 rows as one 2-CTA tile, two GPUs as 128-row tiles:
    # the same K-order accumulation, so agreement to a few fp32 ulp
    r = oracle.compare(outs[1], outs[0], 1e-5, 1e-9)
    assert r["mismatches"] == 0, r


@two_gpus
@pytest.mark.parametrize("nccl", [False, True])
def test_sharded_full_reduce_on_two_gpus(nccl):
    n = 2_000_003
    v = oracle.fill_random(n, 8)
    v[1_999_990] = v[40] = np.float32(1.75)
    g = host.Graph()
    x = g.input("v", (n,))
    r = g.reduce_full(x)
    g.output(r)
    g.finalize()
    ex = host.Executor(g, devices=[0, 1], nccl_exchange=nccl)
    ex.plan()
    ex.set_input(x, v)
    for _ in range(3):
        ex.run()
        import mcke
        s, m, i = mcke.decode_result(ex.output(r).tobytes())
        assert (m, i) == (1.75, 40)
        ws = oracle.full_reduce(v)[0]
        assert abs(s - np.float32(ws)) <= np.spacing(np.float32(abs(ws)))


# ---- CUDA-graph replay (ExecutorOptions::use_graph) --------------------------------

def _fanout_graph(branches, depth, rows, cols, seed):
    """The reference graph bench's fan-out shape: a shared input, `branches`
    chains of `depth` bias+GELU nodes each."""
    g = host.Graph()
    x = g.input("x", (rows, cols), "f32", "row_split")
    data = {x: oracle.fill_normal(rows * cols, seed).reshape(rows, cols)}
    outs = []
    for b in range(branches):
        h = x
        for k in range(depth):
            bias = g.input(f"b{b}_{k}", (cols,), "f32")
            data[bias] = oracle.fill_random(cols, seed + 10 * b + k + 1)
            h = g.bias_act(h, bias, "gelu_tanh", name=f"bias_gelu_{b}_{k}")
        g.output(h)
        outs.append(h)
    g.finalize()
    return g, x, data, outs


def _run(g, data, outs, devices, cuda_graph, reps=1, poison=False):
    ex = host.Executor(g, devices=devices, streams_per_device=4, cuda_graph=cuda_graph, poison=poison)
    ex.plan()
    for t, arr in data.items():
        ex.set_input(t, arr)
    for _ in range(reps):
        ex.run()
    ex.synchronize()
    return ex, [ex.output(o) for o in outs]


@pytest.mark.parametrize("devices", [[0], [0, 0]])
def test_graph_replay_matches_eager_bitwise(devices):
    g, x, data, outs = _fanout_graph(4, 4, 256, 384, 3)
    _, want = _run(g, data, outs, devices, cuda_graph=False)
    ex, got = _run(g, data, outs, devices, cuda_graph=True, reps=3, poison=True)
    for a, b in zip(got, want):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    assert ex.last_run_ms() > 0
    # a replay reads the current inputs: new data in, new (matching) results out
    data2 = dict(data)
    data2[x] = oracle.fill_normal(256 * 384, 99).reshape(256, 384)
    ex.set_input(x, data2[x])
    ex.run()
    got2 = [ex.output(o) for o in outs]
    _, want2 = _run(g, data2, outs, devices, cuda_graph=False)
    for a, b, c in zip(got2, want2, got):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
        assert not np.array_equal(a, c)
    # and against the oracle, op by op
    h = data2[x]
    for bias in list(data2)[1:5]:  # creation order: x, then b0_0 .. b0_3
        h = oracle.bias_act(h, data2[bias], "gelu_tanh")
    r = oracle.compare(got2[0], h, 1e-5, 1e-6)
    assert r["mismatches"] == 0, r


def test_graph_replay_of_dag_with_tcgen05_gemms():
    rows, d, f = 256, 128, 256
    gr = host.Graph()
    x = gr.input("X", (rows, d), "bf16", "row_split")
    xs = _dag_inputs(rows, d, f, 5)
    w1, b1 = gr.input("W1", (d, f), "bf16"), gr.input("b1", (f,), "f32")
    w2, b2 = gr.input("W2", (f, d), "bf16"), gr.input("b2", (d,), "f32")
    hh = gr.gemm(x, w1, bias=b1, act="gelu_tanh", out_dtype="bf16")
    p = gr.softmax(gr.gemm(hh, w2, bias=b2))
    gr.output(p)
    gr.finalize()
    data = dict(zip((x, w1, b1, w2, b2), xs))
    _, want = _run(gr, data, [p], [0], cuda_graph=False)
    _, got = _run(gr, data, [p], [0], cuda_graph=True, reps=2)
    assert np.array_equal(got[0].view(np.uint32), want[0].view(np.uint32))
    import mcke
    mcke.check_device_errors()


def test_graph_replay_of_sharded_reduce_on_one_gpu():
    n = 1_000_003
    v = oracle.fill_random(n, 6)
    v[999_000] = np.float32(1.5)
    g = host.Graph()
    x = g.input("v", (n,))
    r = g.reduce_full(x)
    g.output(r)
    g.finalize()
    import mcke
    _, want = _run(g, {x: v}, [r], [0, 0, 0], cuda_graph=False)
    _, got = _run(g, {x: v}, [r], [0, 0, 0], cuda_graph=True, reps=3)
    assert got[0].tobytes() == want[0].tobytes()
    assert mcke.decode_result(got[0].tobytes())[1:] == (1.5, 999_000)


@two_gpus
def test_graph_replay_with_nccl_exchange_on_two_gpus():
    n = 2_000_003
    v = oracle.fill_random(n, 9)
    v[1_500_000] = np.float32(1.5)
    g = host.Graph()
    x = g.input("v", (n,))
    r = g.reduce_full(x)
    g.output(r)
    g.finalize()
    import mcke
    _, want = _run(g, {x: v}, [r], [0, 1], cuda_graph=False)
    _, got = _run(g, {x: v}, [r], [0, 1], cuda_graph=True, reps=3)
    assert got[0].tobytes() == want[0].tobytes()
    assert mcke.decode_result(got[0].tobytes())[1:] == (1.5, 1_500_000)
    gf, xf, data, outs = _fanout_graph(2, 3, 512, 256, 4)
    _, want = _run(gf, data, outs, [0, 1], cuda_graph=False)
    _, got = _run(gf, data, outs, [0, 1], cuda_graph=True, reps=2)
    for a, b in zip(got, want):
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@two_gpus
def test_graph_mode_rejects_a_mixed_device_list():
    gr = host.Graph()
    xx = gr.input("v", (1000,))
    rr = gr.reduce_full(xx)
    gr.output(rr)
    gr.finalize()
    ex = host.Executor(gr, devices=[0, 0, 1], cuda_graph=True)
    ex.plan()
    ex.set_input(xx, oracle.fill_random(1000, 1))
    import mcke
    with pytest.raises(mcke.MckeError, match="distinct GPUs or one GPU repeated"):
        ex.run()


def test_graph_gemm_f32_on_the_tensor_cores_with_bias_and_gelu():
    # GemmOp with kTcgen05Tf32x3: the executor sizes the split workspace from
    # workspace_bytes(); column-split over two shards of one GPU as well
    m, k, n = 200, 96, 264
    a = oracle.fill_random(m * k, 21).reshape(m, k)
    b = oracle.fill_random(k * n, 22).reshape(k, n)
    bias = oracle.fill_random(n, 23)
    want = oracle.bias_act(oracle.gemm(a, b), bias, "gelu_tanh")
    for devices in ([0], [0, 0]):
        g = host.Graph()
        ta, tb, tbias = g.input("A", (m, k)), g.input("B", (k, n)), g.input("bias", (n,))
        c = g.gemm(ta, tb, bias=tbias, act="gelu_tanh", variant=host.GEMM_VARIANT_TCGEN05_TF32X3)
        g.output(c)
        g.finalize()
        ex = host.Executor(g, devices=devices)
        ex.plan()
        for t, arr in ((ta, a), (tb, b), (tbias, bias)):
            ex.set_input(t, arr)
        ex.run()
        r = oracle.compare(ex.output(c), want, oracle.tol_gemm(k), oracle.abs_tol_gemm(k))
        assert r["mismatches"] == 0, (devices, r)
