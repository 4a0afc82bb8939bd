"""Parity at every BASELINE configuration's full size (B200 only).

The smaller parity tests pin each kernel path on shapes the oracle finishes in
seconds; these run the exact shapes bench.py times, with BASELINE's input
distributions and seeds, so no benchmarked number rests on a kernel checked
only at a smaller shape:

* config 1, bias + GELU(tanh) fp32, all 4096 x 4096 elements against the
  oracle's reference_bias_act (tests/reference.hpp:143);
* config 2, row softmax fp32, all 32768 x 1024 elements against
  reference_row_softmax (:175);
* config 3, full reduce of 2^28 floats (fill_random seed 1): max and argmax
  bit for bit, the double-accumulated sum within one float ulp of the serial
  double sum (reference_row_reduce with rows = 1, :154), through the one-GPU
  entry point and through shard partials combined in order;
* config 4, GEMM 8192^3 (fill_random seeds 2 and 3): bf16 on the tensor cores
  with the schedule bench.py times (AUTO) and the column shard one rank runs
  at 8 GPUs, spot-checked at 2048 samples with the reference's
  spot_check_gemm (:401); fp32 through 3xTF32 on the tensor cores;
* config 5, one DAG branch at 8192 x 4096 x 16384 through the executor, with
  rows of H and of the softmax checked against the oracle composed op by op.

Tolerances are those of tests/test_gpu_parity.py and are written beside each
check.
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

DEV = torch.device("cuda:0")
N = 8192


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bf16_dev(a_bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a_bits.view(np.int16)).to(DEV).view(torch.bfloat16)


def check_close(got, want, rel, abs_, what, floor=None, max_rel=None):
    r = oracle.compare(got, want, rel, abs_)
    assert r["mismatches"] == 0 and not r["nan"] and not r["inf"], (what, r)
    if max_rel is not None:
        g = np.asarray(got, np.float64).ravel()
        w = np.asarray(want, np.float64).ravel()
        sel = np.abs(w) > floor
        worst = float(np.max(np.abs(g[sel] - w[sel]) / np.abs(w[sel])))
        assert worst <= max_rel, (what, worst)


# ------------------------------------------------------------ config 1

def test_config1_bias_gelu_all_rows():
    rows = cols = 4096
    x = oracle.fill_normal(rows * cols, 0).reshape(rows, cols)  # X ~ N(0, 1), drawn first
    b = oracle.fill_random(cols, 1000)                           # bias ~ U(-1, 1)
    want = oracle.bias_act(x, b, "gelu_tanh")
    got = host(mcke.bias_act(dev(x), dev(b), "gelu_tanh"))  # vector width 4: what bench.py times
    # north star: <= 1e-5 relative; 1e-6 absolute where GELU is near zero
    check_close(got, want, 1e-5, 1e-6, "config1", floor=1e-3, max_rel=1e-5)


# ------------------------------------------------------------ config 2

def test_config2_softmax_all_rows():
    x = oracle.softmax_config_input(32768, 1024, seed=2)  # N(0, 4^2), every 64th row +80
    want = oracle.row_softmax(x)
    got = host(mcke.softmax(dev(x)))
    check_close(got, want, 1e-5, 1e-8, "config2", floor=1e-30, max_rel=1e-5)
    assert np.abs(got.sum(axis=1, dtype=np.float64) - 1.0).max() < 1e-5


# ------------------------------------------------------------ config 3

@pytest.fixture(scope="module")
def reduce_input():
    v = oracle.fill_random(1 << 28, 1)  # U(-1, 1), seed 1
    return v, oracle.full_reduce(v)


def _same_result(got, want, what):
    s, m, i = got
    ws, wm, wi = want
    assert np.float32(m).view(np.uint32) == np.float32(wm).view(np.uint32), (what, m, wm)
    assert i == wi, (what, i, wi)
    assert abs(s - np.float32(ws)) <= np.spacing(np.float32(abs(ws))), (what, s, ws)


def test_config3_full_reduce_2pow28(reduce_input):
    v, want = reduce_input
    x = dev(v)
    _same_result(mcke.decode_result(mcke.reduce_full(x)), want, "one GPU")
    # the ranges a 2-, 4- and 8-GPU run reduces, folded in rank order
    n = v.size
    for g in (2, 4, 8):
        parts = torch.empty(g * mcke.PARTIAL_BYTES, dtype=torch.uint8, device=DEV)
        for r in range(g):
            lo, hi = n * r // g, n * (r + 1) // g
            mcke.reduce_full_partial(x[lo:hi], lo, out=parts[r * 24:(r + 1) * 24])
        _same_result(mcke.decode_result(mcke.reduce_combine(parts, g)), want, f"{g} shards")
    del x


def test_config3_full_reduce_2pow28_planted_maximum(reduce_input):
    # a unique maximum deep in the vector, and a tie later on: lowest index wins
    v, _ = reduce_input
    w = v.copy()
    w[200_000_003] = w[268_000_000] = np.float32(1.75)
    _same_result(mcke.decode_result(mcke.reduce_full(dev(w))), oracle.full_reduce(w), "planted")


# ------------------------------------------------------------ config 4

@pytest.fixture(scope="module")
def gemm_inputs():
    a = oracle.fill_random(N * N, 2).reshape(N, N)  # U(-1, 1), seeds 2 and 3
    b = oracle.fill_random(N * N, 3).reshape(N, N)
    return a, b


def test_config4_gemm_bf16_8192cubed(gemm_inputs):
    a, b = gemm_inputs
    ab, bb = oracle.to_bf16(a), oracle.to_bf16(b)
    ar, br = oracle.bf16_to_f32(ab).reshape(N, N), oracle.bf16_to_f32(bb).reshape(N, N)
    ta, tb = bf16_dev(ab), bf16_dev(bb)
    c = torch.empty(N, N, device=DEV)
    mcke.gemm(ta, tb, c, variant="tcgen05")  # the call bench.py times
    mcke.check_device_errors()
    got = host(c)
    # (1) against the oracle on the same bf16 inputs: fp32-accumulation
    # tolerance, 4x the reference's K-scaled bound (as the smaller tests)
    r = oracle.spot_check_gemm(ar, br, got, samples=2048, seed=41, rel_tol=4 * oracle.tol_gemm(N),
                               abs_tol=4 * oracle.abs_tol_gemm(N))
    assert r["mismatches"] == 0 and r["checked"] == 2048, r
    # (2) north star: <= 1e-2 against the fp32-input reference; absolute floor
    # ~10 sigma of the bf16 input-rounding error (4 sqrt(k) 2^-8 / 3)
    r = oracle.spot_check_gemm(a, b, got, samples=2048, seed=42, rel_tol=1e-2,
                               abs_tol=4 * np.sqrt(N) * 2.0 ** -8 / 3)
    assert r["mismatches"] == 0, r
    assert np.isfinite(got).all()


def test_config4_gemm_bf16_eighth_column_shard(gemm_inputs):
    # what one rank computes at 8 GPUs: C[:, j0:j1] = A B[:, j0:j1], 8192 x 1024 x 8192
    a, b = gemm_inputs
    j0, j1 = 3 * N // 8, 4 * N // 8
    ab = oracle.to_bf16(a)
    bs = np.ascontiguousarray(b[:, j0:j1])
    bsb = oracle.to_bf16(bs)
    got = host(mcke.gemm(bf16_dev(ab), bf16_dev(bsb), variant="tcgen05"))
    mcke.check_device_errors()
    r = oracle.spot_check_gemm(oracle.bf16_to_f32(ab).reshape(N, N), oracle.bf16_to_f32(bsb).reshape(N, j1 - j0),
                               got, samples=2048, seed=43, rel_tol=4 * oracle.tol_gemm(N),
                               abs_tol=4 * oracle.abs_tol_gemm(N))
    assert r["mismatches"] == 0, r


def test_config4_gemm_f32_tensor_cores_8192cubed(gemm_inputs):
    a, b = gemm_inputs
    ta, tb = dev(a), dev(b)
    c = torch.empty(N, N, device=DEV)
    ws = torch.empty(mcke.gemm_f32_tc_workspace_bytes(N, N, N), dtype=torch.uint8, device=DEV)
    mcke.gemm_f32_tc(ta, tb, c, workspace=ws)  # the call bench.py times
    mcke.check_device_errors()
    del ws
    got = host(c)
    # the reference's K-scaled fp32 tolerance (tests/reference.hpp:344, :370)
    r = oracle.spot_check_gemm(a, b, got, samples=2048, seed=44)
    assert r["mismatches"] == 0, r
    # north star: <= 1e-4 relative against the fp64-accumulated reference, on
    # outputs at least a quarter of their standard deviation sqrt(k / 9) from zero
    rng = np.random.default_rng(45)
    ii, jj = rng.integers(0, N, 2048), rng.integers(0, N, 2048)
    want = np.einsum("sk,ks->s", a[ii].astype(np.float64), b[:, jj].astype(np.float64))
    sel = np.abs(want) > 0.25 * np.sqrt(N / 9.0)
    worst = float(np.max(np.abs(got[ii, jj][sel] - want[sel]) / np.abs(want[sel])))
    assert worst <= 1e-4, worst


# ------------------------------------------------------------ config 5

def test_config5_dag_branch_full_size():
    from mcke import host as mhost
    rows, d, f = 8192, 4096, 16384
    x = oracle.to_bf16(oracle.fill_normal(rows * d, 50).reshape(rows, d))            # N(0, 1)
    w1 = oracle.to_bf16(oracle.fill_normal(d * f, 51, 0.0, 0.02).reshape(d, f))      # N(0, 0.02^2)
    b1 = oracle.fill_random(f, 52)                                                   # U(-1, 1)
    w2 = oracle.to_bf16(oracle.fill_normal(f * d, 53, 0.0, 0.02).reshape(f, d))
    b2 = oracle.fill_random(d, 54)
    g = mhost.Graph()
    tx = g.input("X", (rows, d), "bf16")
    tw1, tb1 = g.input("W1", (d, f), "bf16"), g.input("b1", (f,), "f32")
    tw2, tb2 = g.input("W2", (f, d), "bf16"), g.input("b2", (d,), "f32")
    th = g.gemm(tx, tw1, bias=tb1, act="gelu_tanh", out_dtype="bf16", name="gemm1")
    ty = g.gemm(th, tw2, bias=tb2, name="gemm2")
    tp = g.softmax(ty, name="softmax")
    for t in (th, ty, tp):
        g.output(t)
    g.finalize()
    ex = mhost.Executor(g, devices=[0], streams_per_device=4, cuda_graph=True)  # as bench.py runs it
    ex.plan()
    for t, arr in ((tx, x), (tw1, w1), (tb1, b1), (tw2, w2), (tb2, b2)):
        ex.set_input(t, arr)
    ex.run()
    ex.synchronize()
    h, y, p = ex.output(th), ex.output(ty), ex.output(tp)
    del ex, g
    f32 = oracle.bf16_to_f32
    # The oracle's gemm on transposed operands: H[r]^T = W1^T X[r]^T, the same
    # products summed in the same k order in double (and cache-friendly).
    w1t = torch.from_numpy(f32(w1).reshape(d, f)).t().contiguous().numpy()  # exact copies, blocked transpose
    w2t = torch.from_numpy(f32(w2).reshape(f, d)).t().contiguous().numpy()
    check_rows = [0, 1, 63, 64, 4095, 5000, 8190, 8191]
    for r in check_rows:
        lin1 = oracle.gemm(w1t, f32(x[r]).reshape(d, 1)).reshape(1, f)
        want_h = oracle.to_bf16(oracle.bias_act(lin1, b1, "gelu_tanh"))
        # One bf16 rounding of values that agree to fp32 accumulation error.
        # Within one bf16 ulp (2^-7 relative) or 1e-4 absolute: where x W1 + b1
        # cancels to near zero the GEMM's fp32 accumulation error (~sqrt(k)
        # eps |x W1| ~ 4e-6 here; GELU' <= 1.13) is a large fraction of the
        # output, as in the smaller fused-epilogue test's absolute floor.
        gh, wh = f32(h[r]).astype(np.float64), f32(want_h.ravel()).astype(np.float64)
        err = np.abs(gh - wh)
        assert np.all(err <= np.abs(wh) * 2.0 ** -7 + 1e-4), (r, float(err.max()))
        ulp = np.abs(h[r].astype(np.int32) - want_h.ravel().astype(np.int32))
        assert (ulp == 0).mean() > 0.99 and (ulp <= 1).mean() > 0.999, (r, float((ulp == 0).mean()))
        # GEMM2 + b2 from the kernel's own H (as stored), then the softmax of the kernel's own Y
        lin2 = oracle.gemm(w2t, f32(h[r]).reshape(f, 1)).reshape(1, d)
        want_y = oracle.bias_act(lin2, b2, "none")
        check_close(y[r:r + 1], want_y, 4 * oracle.tol_gemm(f), 4 * oracle.abs_tol_gemm(f), ("Y", r))
        check_close(p[r:r + 1], oracle.row_softmax(y[r:r + 1]), 1e-5, 1e-8, ("P", r))
    assert np.abs(p.sum(axis=1, dtype=np.float64) - 1.0).max() < 1e-5
    assert np.isfinite(y).all()
