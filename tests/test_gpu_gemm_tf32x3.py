"""fp32 GEMM on the tensor cores (mcke_sm100_gemm_f32_tc, 3xTF32) against the
oracle's fp64-accumulated reference GEMM (tests/reference.hpp:199 restated in
oracle/), with the reference's K-scaled tolerances (tests/reference.hpp:344,
:370) and the north star's 1e-4 relative bound for fp32 GEMM.
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

DEV = "cuda"


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def _check(got, want, k, ctx, amax=1.0):
    r = oracle.compare(got, want, oracle.tol_gemm(k), oracle.abs_tol_gemm(k, amax))
    assert r["mismatches"] == 0, (ctx, r)
    # 1e-4 relative on every output clear of zero (a quarter of the outputs'
    # standard deviation, sqrt(k/9) for U(-1,1) inputs)
    big = np.abs(want) > 0.25 * np.sqrt(k / 9.0) * amax * amax
    if big.any():
        rel = np.abs(got[big] - want[big]) / np.abs(want[big])
        assert rel.max() <= 1e-4, (ctx, float(rel.max()))


# single-CTA shape (m <= 128), the 2-CTA pair shape, ragged edges in every
# dimension, k not a multiple of the 32-deep k-block
# in_kernel: the GEMM kernel splits its raw fp32 tiles itself (no workspace)
SPLIT = pytest.mark.parametrize("in_kernel", [False, True], ids=["split_pass", "in_kernel_split"])


@SPLIT
@pytest.mark.parametrize("m,n,k", [(64, 64, 32), (128, 256, 64), (100, 260, 36), (300, 264, 516),
                                   (1024, 1024, 1024), (257, 1028, 2052), (512, 100, 64)])
def test_matches_oracle(m, n, k, in_kernel):
    a = oracle.fill_random(m * k, 2).reshape(m, k)
    b = oracle.fill_random(k * n, 3).reshape(k, n)
    got = host(mcke.gemm_f32_tc(dev(a), dev(b), in_kernel_split=in_kernel))
    mcke.check_device_errors()
    _check(got, oracle.gemm(a, b), k, (m, n, k))


@SPLIT
def test_large_k_spot_check(in_kernel):
    m, n, k = 512, 768, 8192
    a = oracle.fill_random(m * k, 4).reshape(m, k)
    b = oracle.fill_random(k * n, 5).reshape(k, n)
    got = host(mcke.gemm_f32_tc(dev(a), dev(b), in_kernel_split=in_kernel))
    r = oracle.spot_check_gemm(a, b, got, samples=1024, seed=3)
    assert r["mismatches"] == 0 and r["checked"] == 1024, r


def test_in_kernel_split_equals_the_split_pass():
    # the same hi/lo parts and the same MMA order: the same bits
    m, n, k = 1000, 1032, 1028
    a = dev(oracle.fill_random(m * k, 14).reshape(m, k))
    b = dev(oracle.fill_random(k * n, 15).reshape(k, n))
    u = mcke.gemm_f32_tc(a, b)
    v = mcke.gemm_f32_tc(a, b, in_kernel_split=True)
    torch.cuda.synchronize()
    mcke.check_device_errors()
    assert torch.equal(u, v)


def test_tensor_cores_beat_the_tf32_rounding():
    # One-pass TF32 would be off by ~1e-3 relative; the split must recover
    # fp32-level accuracy: compare the error against the FFMA kernel's.
    m, n, k = 256, 256, 2048
    a = oracle.fill_random(m * k, 6).reshape(m, k)
    b = oracle.fill_random(k * n, 7).reshape(k, n)
    want = oracle.gemm(a, b)
    tc = host(mcke.gemm_f32_tc(dev(a), dev(b)))
    simt = host(mcke.gemm(dev(a), dev(b), variant="simt"))
    err_tc = np.abs(tc - want).max()
    err_simt = np.abs(simt - want).max()
    assert err_tc <= 4 * err_simt + 1e-6, (err_tc, err_simt)


def test_epilogue_alpha_beta_bias_act():
    m, n, k = 200, 264, 96
    a = oracle.fill_random(m * k, 8).reshape(m, k)
    b = oracle.fill_random(k * n, 9).reshape(k, n)
    c0 = oracle.fill_random(m * n, 10).reshape(m, n)
    bias = oracle.fill_random(n, 11)
    got = host(mcke.gemm_f32_tc(dev(a), dev(b), dev(c0), alpha=0.5, beta=2.0))
    _check(got, oracle.gemm(a, b, c0, 0.5, 2.0), k, "alpha/beta", 2.0)
    got = host(mcke.gemm_f32_tc(dev(a), dev(b), bias=dev(bias), act="gelu_tanh"))
    want = oracle.bias_act(oracle.gemm(a, b), bias, "gelu_tanh")
    _check(got, want, k, "bias+gelu", 1.0)


def test_k_zero_writes_beta_c_and_bad_shapes_are_rejected():
    c0 = oracle.fill_random(8 * 8, 12).reshape(8, 8)
    c1 = dev(c0)
    z = torch.zeros(64, device=DEV)
    s = torch.cuda.current_stream().cuda_stream
    rc = mcke.lib().mcke_sm100_gemm_f32_tc(z.data_ptr(), z.data_ptr(), c1.data_ptr(), 8, 8, 0, 1.0, 0.5, None, 0,
                                           None, 0, s)
    assert rc == mcke.OK
    assert np.array_equal(host(c1), (c0 * np.float32(0.5)).astype(np.float32))
    a = torch.ones(16, 6, device=DEV)
    b = torch.ones(6, 16, device=DEV)
    with pytest.raises(mcke.MckeError, match="K % 4"):
        mcke.gemm_f32_tc(a, b)
    a = torch.ones(16, 8, device=DEV)
    b = torch.ones(8, 16, device=DEV)
    with pytest.raises(mcke.MckeError, match="workspace"):
        mcke.gemm_f32_tc(a, b, workspace=torch.empty(256, dtype=torch.uint8, device=DEV))
    mcke.check_device_errors()


def test_f32_auto_runs_the_in_kernel_split_where_the_shape_allows():
    # mcke_sm100_gemm_f32 with AUTO (the reference's launch_gemm_f32) takes the
    # tensor cores for K % 4 == 0, N % 4 == 0: the same bits as the in-kernel
    # split, alpha/beta included; other shapes stay on the FFMA kernel.
    m, n, k = 333, 516, 260
    a = dev(oracle.fill_random(m * k, 16).reshape(m, k))
    b = dev(oracle.fill_random(k * n, 17).reshape(k, n))
    c0 = dev(oracle.fill_random(m * n, 18).reshape(m, n))
    auto = mcke.gemm(a, b, c0.clone(), 0.75, 1.25)
    split = mcke.gemm_f32_tc(a, b, c0.clone(), 0.75, 1.25, in_kernel_split=True)
    simt = mcke.gemm(a, b, c0.clone(), 0.75, 1.25, variant="simt")
    torch.cuda.synchronize()
    assert torch.equal(auto, split)
    assert not torch.equal(auto, simt)  # FFMA sums in another order
    _check(host(auto), oracle.gemm(host(a), host(b), host(c0), 0.75, 1.25), k, "auto", 1.25)
    a3 = dev(oracle.fill_random(m * 258, 19).reshape(m, 258))  # K % 4 != 0
    b3 = dev(oracle.fill_random(258 * n, 20).reshape(258, n))
    assert torch.equal(mcke.gemm(a3, b3), mcke.gemm(a3, b3, variant="simt"))
    mcke.check_device_errors()


def test_f32_auto_8192_cube_spot_check():
    # the 8192^3 float32 GEMM of the reference's benchmark, through AUTO
    n = 8192
    g = torch.Generator(device="cpu").manual_seed(21)
    a = torch.rand((n, n), generator=g, dtype=torch.float32) * 2 - 1
    b = torch.rand((n, n), generator=g, dtype=torch.float32) * 2 - 1
    got = host(mcke.gemm(a.to(DEV), b.to(DEV)))
    r = oracle.spot_check_gemm(a.numpy(), b.numpy(), got, samples=512, seed=22)
    assert r["mismatches"] == 0 and r["checked"] == 512, r
