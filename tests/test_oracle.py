"""Pin the CPU oracle before trusting it (CPU only).

The C restatement (oracle/mcke_oracle.c) is checked three ways:
1. against the reference's own golden vectors (tests/golden/reference_vectors.json,
   converted from the reference's tests/data/reference_vectors.txt): exact cases
   bit for bit, approx cases at the reference's 1e-6 rel / 1e-7 abs
   (tests/test_host_core.cpp:2430-2450 in the reference);
2. against outputs of the reference's compiled oracle committed in
   tests/golden/ref_fixtures.npz: bit for bit;
3. live against oracle/_ref/libmcke_ref.so on fresh random shapes, when that
   library exists.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

import oracle

HEX = lambda h: np.array([int(t, 16) for t in h], dtype=np.uint32).view(np.float32)  # noqa: E731


@pytest.fixture(scope="module")
def vectors(golden_dir):
    with open(os.path.join(golden_dir, "reference_vectors.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="module")
def fixtures(golden_dir):
    return dict(np.load(os.path.join(golden_dir, "ref_fixtures.npz")))


def _run_case(c, impl):
    ints, arrs = c["ints"], {k: HEX(v) for k, v in c["arrays"].items()}
    fl = {k: HEX([v])[0] for k, v in c["floats"].items()}
    kind = c["kind"]
    if kind == "gemm":
        m, n, k = ints["m"], ints["n"], ints["k"]
        return oracle.gemm(arrs["a"].reshape(m, k), arrs["b"].reshape(k, n),
                           arrs["c"].reshape(m, n), float(fl["alpha"]), float(fl["beta"]),
                           impl=impl).ravel()
    rows, cols = ints["rows"], ints["cols"]
    x = arrs["x"].reshape(rows, cols)
    if kind == "bias_act":
        return oracle.bias_act(x, arrs["bias"], ints["act"], impl=impl).ravel()
    if kind == "row_reduce":
        return oracle.row_reduce(x, ints["kind"], impl=impl)
    if kind == "row_softmax":
        return oracle.row_softmax(x, impl=impl).ravel()
    raise AssertionError(f"unknown kind {kind}")


@pytest.mark.parametrize("impl", ["port", "reference"])
def test_golden_vectors(vectors, impl):
    if impl == "reference" and not oracle.have_reference():
        pytest.skip("oracle/_ref not built (reference tree absent when oracle/Makefile ran)")
    assert len(vectors) == 19
    exact = 0
    for c in vectors:
        want = HEX(c["arrays"]["expect"])
        got = _run_case(c, impl)
        if c["mode"] == "exact":
            exact += 1
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), c["name"]
        else:
            r = oracle.compare(got, want, 1e-6, 1e-7)
            assert r["mismatches"] == 0 and not r["nan"], (c["name"], r)
    assert exact >= 10


def test_mt19937_64_known_answer():
    # The C++ standard ([rand.predef]) fixes the 10000th output of a
    # default-constructed (seed 5489) std::mt19937_64.
    import ctypes
    state = ctypes.create_string_buffer(312 * 8 + 16)
    l = oracle.lib("port")
    l.oracle_mt64_seed(state, 5489)
    v = 0
    for _ in range(10000):
        v = l.oracle_mt64_next(state)
    assert v == 9981545732273789042


def test_fill_random_matches_reference(fixtures):
    for seed in (0, 1, 2, 3):
        got = oracle.fill_random(4096, seed)
        assert np.array_equal(got.view(np.uint32), fixtures[f"fill_random_seed{seed}"].view(np.uint32))
    got = oracle.fill_random(1000, 7, -4.0, 4.0)
    assert np.array_equal(got.view(np.uint32), fixtures["fill_random_lohi"].view(np.uint32))


def _bits_equal(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32),
                          np.asarray(b, np.float32).view(np.uint32))


def test_kernels_match_reference_fixtures(fixtures):
    fx = fixtures
    for name in ("none", "relu", "gelu_erf", "gelu_tanh"):
        assert _bits_equal(oracle.bias_act(fx["bias_act_x"], fx["bias_act_bias"], name),
                           fx[f"bias_act_{name}"]), name
    for kind in ("sum", "max", "mean"):
        assert _bits_equal(oracle.row_reduce(fx["row_reduce_x"], kind), fx[f"row_reduce_{kind}"])
    assert _bits_equal(oracle.row_softmax(fx["row_softmax_x"]), fx["row_softmax_y"])
    assert _bits_equal(oracle.gemm(fx["gemm_a"], fx["gemm_b"], fx["gemm_c"], 1.5, 0.5),
                       fx["gemm_out"])
    s, m, i = oracle.full_reduce(fx["full_x"])
    assert _bits_equal(np.float32(s), fx["full_sum"][0])
    assert _bits_equal(m, fx["full_max"][0])
    assert fx["full_x"][i] == m and np.all(fx["full_x"][:i] < m)


@pytest.mark.skipif(not oracle.have_reference(), reason="oracle/_ref not built")
def test_port_matches_reference_live():
    rng = np.random.default_rng(5)
    for rows, cols in [(1, 1), (3, 17), (64, 1024), (5, 4099)]:
        x = oracle.fill_random(rows * cols, int(rng.integers(1 << 30)), -6, 6).reshape(rows, cols)
        b = oracle.fill_random(cols, int(rng.integers(1 << 30)))
        for act in range(4):
            assert _bits_equal(oracle.bias_act(x, b, act), oracle.bias_act(x, b, act, impl="reference"))
        for kind in range(3):
            assert _bits_equal(oracle.row_reduce(x, kind), oracle.row_reduce(x, kind, impl="reference"))
        assert _bits_equal(oracle.row_softmax(x), oracle.row_softmax(x, impl="reference"))
    for m, n, k in [(1, 1, 1), (7, 9, 300), (17, 33, 5)]:
        a = oracle.fill_random(m * k, 21).reshape(m, k)
        b = oracle.fill_random(k * n, 22).reshape(k, n)
        c = oracle.fill_random(m * n, 23).reshape(m, n)
        assert _bits_equal(oracle.gemm(a, b, c, 0.75, -1.25), oracle.gemm(a, b, c, 0.75, -1.25, impl="reference"))
        got = oracle.gemm(a, b)
        assert oracle.spot_check_gemm(a, b, got, samples=64, seed=3) == \
            oracle.spot_check_gemm(a, b, got, samples=64, seed=3, impl="reference")
    for k in (1, 256, 8192):
        assert oracle.tol_gemm(k) == oracle.tol_gemm(k, impl="reference")
        assert oracle.abs_tol_gemm(k) == oracle.abs_tol_gemm(k, impl="reference")


def test_full_reduce_edge_cases():
    # Ties resolve to the lowest index; NaN never wins (std::max fold); all-NaN
    # and empty give max=-inf, argmax=-1; -inf alone is a valid maximum.
    x = np.array([1, 3, 3, -2, 3], np.float32)
    assert oracle.full_reduce(x)[1:] == (3.0, 1)
    x = np.array([np.nan, 2, np.nan, 2], np.float32)
    s, m, i = oracle.full_reduce(x)
    assert np.isnan(s) and m == 2 and i == 1
    s, m, i = oracle.full_reduce(np.array([np.nan, np.nan], np.float32))
    assert m == -np.inf and i == -1
    s, m, i = oracle.full_reduce(np.zeros(0, np.float32))
    assert s == 0 and m == -np.inf and i == -1
    s, m, i = oracle.full_reduce(np.array([-np.inf, -np.inf], np.float32))
    assert m == -np.inf and i == 0
    s, m, i = oracle.full_reduce(np.array([-0.0, 0.0], np.float32))
    assert i == 0 and np.signbit(m)
    assert oracle.full_reduce(np.array([5, 1], np.float32), index_base=100)[2] == 100


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    x = np.concatenate([oracle.fill_random(100000, 9, -1e3, 1e3),
                        np.array([0.0, -0.0, 1.0, 1.00390625, 1.01171875, 3.4e38, -3.4e38,
                                  np.inf, -np.inf, 1e-40, -1e-40], np.float32)])
    ours = oracle.to_bf16(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)
    assert _bits_equal(oracle.bf16_to_f32(ours), oracle.round_bf16(x))


def test_fill_normal_moments():
    z = oracle.fill_normal(1 << 20, 0, 0.0, 1.0)
    assert abs(float(z.mean())) < 5e-3 and abs(float(z.std()) - 1.0) < 5e-3
    z4 = oracle.fill_normal(1 << 16, 1, 0.0, 4.0)
    assert abs(float(z4.std()) - 4.0) < 0.05
    x = oracle.softmax_config_input(128, 64, seed=3)
    assert x[0].mean() > 70 and abs(float(x[1].mean())) < 3
