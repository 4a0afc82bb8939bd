"""Parity of the sm_100a kernels with the CPU oracle (B200 only).

Every test runs a CUDA kernel of libmcke_sm100a.so through its C-ABI (via the
ctypes binding in mini-cuda-kernel-engine_b200/mcke) and compares with the
oracle (oracle/, the restatement of the reference's tests/reference.hpp) on
the same seeded inputs:

* integer / index / max results: bit for bit;
* float results: the reference's mixed tolerance |got - want| <= abs + rel*|want|
  (tests/reference.hpp:249) with the tolerances written next to each check,
  plus the max relative error over |want| above a stated floor.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mcke  # noqa: E402

DEV = torch.device("cuda:0")
HEX = lambda h: np.array([int(t, 16) for t in h], dtype=np.uint32).view(np.float32)  # noqa: E731

# Tolerances (north star: <=1e-5 relative for fp32 softmax and bias-GELU,
# <=1e-4 for fp32 GEMM vs an fp64-accumulated reference, <=1e-2 for bf16 GEMM;
# bit-exact for max/argmax).  Absolute floors are the reference's
# (tests/reference.hpp:327-328, :370) for outputs that are near zero by chance.
REL_ELEMWISE, ABS_ELEMWISE = 1e-5, 1e-6
REL_SOFTMAX, ABS_SOFTMAX = 1e-5, 1e-8


def dev(a, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV, dtype)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def assert_close(got, want, rel, abs_, what="", floor=1e-3, max_rel=None):
    r = oracle.compare(got, want, rel, abs_)
    assert r["mismatches"] == 0 and not r["nan"] and not r["inf"], (what, r)
    if max_rel is not None:
        g = np.asarray(got, np.float64).ravel()
        w = np.asarray(want, np.float64).ravel()
        sel = np.abs(w) > floor
        if sel.any():
            worst = float(np.max(np.abs(g[sel] - w[sel]) / np.abs(w[sel])))
            assert worst <= max_rel, (what, worst)


@pytest.fixture(scope="module")
def vectors():
    with open(os.path.join(os.path.dirname(__file__), "golden", "reference_vectors.json")) as f:
        return json.load(f)["cases"]


@pytest.fixture(scope="module")
def fixtures():
    return dict(np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_fixtures.npz")))


# ----------------------------------------------------------------- vector add

@pytest.mark.parametrize("n", [1, 7, 4096, 1_000_003])
def test_vector_add_is_one_exact_add(n):
    a = oracle.fill_random(n + 1, 1, -9, 9)
    b = oracle.fill_random(n + 1, 2, -9, 9)
    for off in (0, 1):  # aligned and 4-byte-offset (scalar path) operands
        ta, tb = dev(a)[off:off + n], dev(b)[off:off + n]
        got = host(mcke.vector_add(ta, tb))
        assert np.array_equal(got.view(np.uint32), (a[off:off + n] + b[off:off + n]).view(np.uint32))


# ---------------------------------------------------------------- bias + act

def test_bias_act_golden_vectors(vectors):
    for c in vectors:
        if c["kind"] != "bias_act":
            continue
        rows, cols, act = c["ints"]["rows"], c["ints"]["cols"], c["ints"]["act"]
        x = HEX(c["arrays"]["x"]).reshape(rows, cols)
        b = HEX(c["arrays"]["bias"])
        want = HEX(c["arrays"]["expect"]).reshape(rows, cols)
        for vw in (1, 2):
            got = host(mcke.bias_act(dev(x), dev(b), act, vector_width=vw))
            # the reference's own bar for these vectors: 1e-6 rel, 1e-7 abs
            assert_close(got, want, 1e-6, 1e-7, c["name"])


def test_bias_act_reference_fixtures(fixtures):
    x, b = fixtures["bias_act_x"], fixtures["bias_act_bias"]
    for name in ("none", "relu", "gelu_erf", "gelu_tanh"):
        for vw in (1, 2, 4):
            got = host(mcke.bias_act(dev(x), dev(b), name, vector_width=vw))
            assert_close(got, fixtures[f"bias_act_{name}"], REL_ELEMWISE, ABS_ELEMWISE, name,
                         max_rel=REL_ELEMWISE)


def test_bias_gelu_config1_shape_slice():
    # Config 1 distribution (X ~ N(0,1), bias ~ U(-1,1)); 1024 of the 4096 rows.
    x = oracle.fill_normal(1024 * 4096, 0).reshape(1024, 4096)
    b = oracle.fill_random(4096, 1000)
    want = oracle.bias_act(x, b, "gelu_tanh")
    got = host(mcke.bias_act(dev(x), dev(b), "gelu_tanh"))
    assert_close(got, want, REL_ELEMWISE, ABS_ELEMWISE, "config1", max_rel=REL_ELEMWISE)
    # the starvation knob changes the launch geometry, never the result
    got2 = host(mcke.bias_act(dev(x), dev(b), "gelu_tanh", max_row_blocks=7))
    assert np.array_equal(got.view(np.uint32), got2.view(np.uint32))


@pytest.mark.parametrize("rows,cols,vw", [(1, 1, 1), (3, 17, 1), (5, 6, 2), (70000, 4, 4), (9, 4100, 4)])
def test_bias_act_odd_shapes(rows, cols, vw):
    x = oracle.fill_random(rows * cols, 3, -5, 5).reshape(rows, cols)
    b = oracle.fill_random(cols, 4)
    for act in range(4):
        got = host(mcke.bias_act(dev(x), dev(b), act, vector_width=vw))
        assert_close(got, oracle.bias_act(x, b, act), REL_ELEMWISE, ABS_ELEMWISE, (rows, cols, act))


def test_bias_add_and_activation_unfused():
    x = oracle.fill_random(64 * 256, 5, -4, 4).reshape(64, 256)
    b = oracle.fill_random(256, 6)
    t = mcke.bias_add(dev(x), dev(b))
    y = host(mcke.activation(t, "gelu_erf"))
    want_add = oracle.bias_act(x, b, "none")
    assert np.array_equal(host(t).view(np.uint32), want_add.view(np.uint32))  # one fp32 add: exact
    assert_close(y, oracle.bias_act(want_add, np.zeros(256, np.float32), "gelu_erf"), REL_ELEMWISE,
                 ABS_ELEMWISE)


def test_bias_act_bf16():
    rows, cols = 96, 1024
    xb = oracle.to_bf16(oracle.fill_normal(rows * cols, 7).reshape(rows, cols))
    b = oracle.fill_random(cols, 8)
    xt = torch.from_numpy(xb.view(np.int16)).to(DEV).view(torch.bfloat16)
    for act in ("gelu_tanh", "relu", "none"):
        got = host(mcke.bias_act(xt, dev(b), act).view(torch.int16)).view(np.uint16)
        want = oracle.to_bf16(oracle.bias_act(oracle.bf16_to_f32(xb), b, act))
        # one rounding to bf16 from a float that may differ by a few ulp: at most 1 bf16 ulp
        diff = np.abs(got.astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1, act
        assert (diff == 0).mean() > 0.99
    # scalar path (cols % 8 != 0)
    xb2 = oracle.to_bf16(oracle.fill_normal(7 * 13, 9).reshape(7, 13))
    b2 = oracle.fill_random(13, 10)
    xt2 = torch.from_numpy(xb2.view(np.int16)).to(DEV).view(torch.bfloat16)
    got = host(mcke.bias_act(xt2, dev(b2), "gelu_tanh").view(torch.int16)).view(np.uint16)
    want = oracle.to_bf16(oracle.bias_act(oracle.bf16_to_f32(xb2), b2, "gelu_tanh"))
    assert np.abs(got.astype(np.int32) - want.astype(np.int32)).max() <= 1


def test_bias_act_rejects_like_the_reference():
    x = torch.zeros(4, 6, device=DEV)
    b = torch.zeros(6, device=DEV)
    with pytest.raises(mcke.MckeError) as e:
        mcke.bias_act(x, b, vector_width=4)  # cols % 4 != 0
    assert e.value.code == mcke.INVALID_ARGUMENT
    with pytest.raises(mcke.MckeError):
        mcke.bias_act(x, b, vector_width=2, out=x)  # in place
    with pytest.raises(mcke.MckeError):
        mcke.bias_act(x[:, 1:].contiguous()[:, :4].contiguous(), b[1:5].contiguous(), vector_width=3)
    # empty extents: OK, no launch
    e0 = torch.zeros(0, 8, device=DEV)
    mcke.bias_act(e0, torch.zeros(8, device=DEV))


# -------------------------------------------------------------------- softmax

def test_softmax_golden_vector(vectors):
    for c in vectors:
        if c["kind"] != "row_softmax":
            continue
        rows, cols = c["ints"]["rows"], c["ints"]["cols"]
        x = HEX(c["arrays"]["x"]).reshape(rows, cols)
        want = HEX(c["arrays"]["expect"]).reshape(rows, cols)
        for variant in ("online", "three_pass"):
            got = host(mcke.softmax(dev(x), variant))
            assert_close(got, want, 1e-6, 1e-7, (c["name"], variant))


def test_softmax_reference_fixture(fixtures):
    x, want = fixtures["row_softmax_x"], fixtures["row_softmax_y"]
    for variant in ("online", "three_pass"):
        got = host(mcke.softmax(dev(x), variant))
        assert_close(got, want, REL_SOFTMAX, REL_SOFTMAX * 1e-3, variant, floor=1e-30, max_rel=REL_SOFTMAX)


def test_softmax_config2_slice():
    # Config 2: N(0, 4^2) logits, every 64th row shifted by +80; 2048 of 32768 rows.
    x = oracle.softmax_config_input(2048, 1024, seed=2)
    want = oracle.row_softmax(x)
    got = host(mcke.softmax(dev(x)))
    assert_close(got, want, REL_SOFTMAX, ABS_SOFTMAX, "config2", floor=1e-30, max_rel=REL_SOFTMAX)
    assert np.allclose(got.sum(axis=1), 1.0, atol=1e-5)


@pytest.mark.parametrize("rows,cols", [(1, 1), (5, 17), (33, 128), (9, 1000), (17, 1536), (4, 2048),
                                       (6, 3000), (3, 5000), (2, 16384), (2, 20000)])
def test_softmax_every_path(rows, cols):
    x = oracle.fill_random(rows * cols, 11, -30, 30).reshape(rows, cols)
    want = oracle.row_softmax(x)
    for variant in ("online", "three_pass"):
        got = host(mcke.softmax(dev(x), variant))
        assert_close(got, want, REL_SOFTMAX, 1e-12, (rows, cols, variant))


def test_softmax_unaligned_rows_take_the_generic_path():
    base = torch.from_numpy(oracle.fill_random(8 * 256 + 1, 12, -8, 8)).to(DEV)
    x = base[1:].view(8, 256)  # 4-byte offset: rows are not 16-byte aligned
    assert x.data_ptr() % 16 != 0
    got = host(mcke.softmax(x))
    want = oracle.row_softmax(host(x))
    assert_close(got, want, REL_SOFTMAX, 1e-12)


# ----------------------------------------------------------------- reductions

def test_reduce_full_matches_oracle_bitwise_for_max_and_argmax():
    n = (1 << 22) + 3
    x = oracle.fill_random(n, 1)
    x[123456] = x[3999999] = np.float32(1.5)  # a tie: the lower index must win
    s, m, i = mcke.decode_result(mcke.reduce_full(dev(x)))
    ws, wm, wi = oracle.full_reduce(x)
    assert np.float32(m).view(np.uint32) == np.float32(wm).view(np.uint32)
    assert i == wi == 123456
    # sum: double accumulation rounded once, like the oracle -> equal to 1 ulp
    assert abs(s - np.float32(ws)) <= np.spacing(np.float32(abs(ws)))


def test_reduce_full_is_deterministic_and_alignment_independent():
    n = 3_000_001
    base = dev(oracle.fill_random(n + 3, 2))
    r1 = host(mcke.reduce_full(base[:n]))
    r2 = host(mcke.reduce_full(base[:n]))
    assert r1.tobytes() == r2.tobytes()
    for off in (1, 2, 3):
        x = base[off:off + n]
        s, m, i = mcke.decode_result(mcke.reduce_full(x))
        ws, wm, wi = oracle.full_reduce(host(x))
        assert (m, i) == (wm, wi)
        assert abs(s - np.float32(ws)) <= np.spacing(np.float32(abs(ws)))


@pytest.mark.parametrize("vals,expect", [
    ([], (0.0, -np.inf, -1)),
    ([2.0], (2.0, 2.0, 0)),
    ([np.nan, 3.0, np.nan, 3.0, 1.0], (np.nan, 3.0, 1)),
    ([np.nan, np.nan], (np.nan, -np.inf, -1)),
    ([-np.inf, -np.inf, -np.inf], (-np.inf, -np.inf, 0)),
    ([-0.0, 0.0, -1.0], (-1.0, -0.0, 0)),
])
def test_reduce_full_edge_cases(vals, expect):
    x = torch.tensor(np.array(vals, np.float32), device=DEV)
    s, m, i = mcke.decode_result(mcke.reduce_full(x))
    es, em, ei = expect
    assert i == ei
    assert (np.isnan(s) and np.isnan(es)) or s == es
    assert np.float32(m).view(np.uint32) == np.float32(em).view(np.uint32)


def test_reduce_full_signed_zero_tie_in_the_vector_body():
    # all-negative data with a -0 then a +0 inside one float4: the first (-0) wins
    x = -np.abs(oracle.fill_random(1 << 16, 4)) - np.float32(1.0)
    x[4096 + 1] = np.float32(-0.0)
    x[4096 + 2] = np.float32(0.0)
    s, m, i = mcke.decode_result(mcke.reduce_full(dev(x)))
    ws, wm, wi = oracle.full_reduce(x)
    assert (i, np.float32(m).view(np.uint32)) == (wi, np.float32(wm).view(np.uint32)) == (4097, np.uint32(0x80000000))


def test_reduce_sharded_partials_combine_to_the_full_answer():
    n = 1 << 21
    x = oracle.fill_random(n, 3)
    x[n - 1] = np.float32(2.0)
    x[17] = np.float32(2.0)
    xt = dev(x)
    full = mcke.decode_result(mcke.reduce_full(xt))
    for g in (2, 3, 8):
        bounds = [n * r // g for r in range(g + 1)]
        parts = torch.empty(g * mcke.PARTIAL_BYTES, dtype=torch.uint8, device=DEV)
        for r in range(g):
            mcke.reduce_full_partial(xt[bounds[r]:bounds[r + 1]], bounds[r],
                                     out=parts[r * 24:(r + 1) * 24])
        s, m, i = mcke.decode_result(mcke.reduce_combine(parts, g))
        assert (m, i) == (full[1], full[2]) == (2.0, 17)
        ws = oracle.full_reduce(x)[0]
        assert abs(s - np.float32(ws)) <= np.spacing(np.float32(abs(ws)))


def test_reduce_row_golden_vectors(vectors):
    for c in vectors:
        if c["kind"] != "row_reduce":
            continue
        rows, cols, kind = c["ints"]["rows"], c["ints"]["cols"], c["ints"]["kind"]
        x = HEX(c["arrays"]["x"]).reshape(rows, cols)
        want = HEX(c["arrays"]["expect"])
        for variant in ("smem_tree", "warp_shuffle", "two_pass"):
            got = host(mcke.reduce_row(dev(x), kind, variant))
            if c["mode"] == "exact":
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (c["name"], variant)
            else:
                assert_close(got, want, 1e-6, 1e-7, (c["name"], variant))


@pytest.mark.parametrize("rows,cols", [(7, 333), (256, 4096), (64, 65536), (3, 1), (5, 17), (4099, 1024),
                                       (60001, 12), (9, 1020), (5000, 128), (333, 256), (71, 512), (3, 1024)])
def test_reduce_row_matches_oracle(rows, cols):
    x = oracle.fill_random(rows * cols, 13).reshape(rows, cols)
    for kind in ("sum", "max", "mean"):
        want = oracle.row_reduce(x, kind)
        for variant in ("warp_shuffle", "two_pass"):
            got = host(mcke.reduce_row(dev(x), kind, variant))
            if kind == "max":
                assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
            else:  # double accumulation: within one float ulp of the oracle
                assert np.all(np.abs(got - want) <= np.spacing(np.abs(want)) + 1e-30), (kind, variant)


def test_reduce_row_two_pass_needs_workspace():
    x = torch.zeros(4, 64, device=DEV)
    out = torch.zeros(4, device=DEV)
    rc = mcke.lib().mcke_sm100_reduce_row_f32(x.data_ptr(), out.data_ptr(), 4, 64, 0, 2, None, 0,
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == mcke.UNIMPLEMENTED


# ----------------------------------------------------------------------- GEMM

def test_gemm_f32_golden_vectors_bit_exact(vectors):
    n_exact = 0
    for c in vectors:
        if c["kind"] != "gemm":
            continue
        m, n, k = c["ints"]["m"], c["ints"]["n"], c["ints"]["k"]
        a = HEX(c["arrays"]["a"]).reshape(m, k)
        b = HEX(c["arrays"]["b"]).reshape(k, n)
        c0 = HEX(c["arrays"]["c"]).reshape(m, n)
        alpha = float(HEX([c["floats"]["alpha"]])[0])
        beta = float(HEX([c["floats"]["beta"]])[0])
        want = HEX(c["arrays"]["expect"]).reshape(m, n)
        got = host(mcke.gemm(dev(a), dev(b), dev(c0), alpha, beta))
        assert c["mode"] == "exact"
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), c["name"]
        n_exact += 1
    assert n_exact == 11


def test_gemm_f32_reference_fixture(fixtures):
    a, b, c0 = fixtures["gemm_a"], fixtures["gemm_b"], fixtures["gemm_c"]
    got = host(mcke.gemm(dev(a), dev(b), dev(c0), 1.5, 0.5))
    k = a.shape[1]
    assert_close(got, fixtures["gemm_out"], oracle.tol_gemm(k), oracle.abs_tol_gemm(k, 1.5))


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (3, 7, 5), (129, 131, 257), (512, 384, 1000), (300, 260, 3)])
def test_gemm_f32_matches_oracle(m, n, k):
    a = oracle.fill_random(m * k, 2).reshape(m, k)
    b = oracle.fill_random(k * n, 3).reshape(k, n)
    want = oracle.gemm(a, b)
    got = host(mcke.gemm(dev(a), dev(b)))
    # The reference's K-scaled mixed tolerance (tests/reference.hpp:344,:370)
    # on every element; the north star's <= 1e-4 relative on every output at
    # least a quarter of the outputs' standard deviation, sqrt(k/9), from zero
    # (closer to zero the error is set by the terms, not the result).
    assert_close(got, want, oracle.tol_gemm(k), oracle.abs_tol_gemm(k), (m, n, k), max_rel=1e-4,
                 floor=0.25 * np.sqrt(k / 9.0))


def test_gemm_f32_k_zero_and_beta():
    c0 = oracle.fill_random(6 * 5, 9).reshape(6, 5)
    ct = dev(c0)
    scratch = torch.zeros(64, device=DEV)  # k == 0 still needs non-null A and B, as in the reference
    for fn in (mcke.lib().mcke_sm100_gemm_f32, mcke.lib().mcke_sm100_gemm_bf16):
        c1 = ct.clone()
        assert fn(scratch.data_ptr(), scratch.data_ptr(), c1.data_ptr(), 6, 5, 0, 1.0, 0.5, 0,
                  torch.cuda.current_stream().cuda_stream) == mcke.OK
        assert np.array_equal(host(c1), (c0 * np.float32(0.5)).astype(np.float32))
    # beta == 0 never reads C: NaN in C must not leak
    cn = torch.full((4, 4), float("nan"), device=DEV)
    got = host(mcke.gemm(torch.ones(4, 2, device=DEV), torch.ones(2, 4, device=DEV), cn))
    assert np.all(got == 2.0)


def test_gemm_f32_spot_check_2048():
    m = n = k = 2048
    a = oracle.fill_random(m * k, 2).reshape(m, k)
    b = oracle.fill_random(k * n, 3).reshape(k, n)
    got = host(mcke.gemm(dev(a), dev(b)))
    r = oracle.spot_check_gemm(a, b, got, samples=1024, seed=7)
    assert r["mismatches"] == 0 and r["checked"] == 1024, r


def _bf16(a):
    return torch.from_numpy(oracle.to_bf16(a).view(np.int16)).to(DEV).view(torch.bfloat16)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 128), (1000, 712, 520), (129, 264, 8),
                                   (2048, 1024, 1024)])
def test_gemm_bf16_tcgen05_matches_oracle(m, n, k):
    a = oracle.fill_random(m * k, 2).reshape(m, k)
    b = oracle.fill_random(k * n, 3).reshape(k, n)
    ar, br = oracle.round_bf16(a), oracle.round_bf16(b)
    got = host(mcke.gemm(_bf16(a), _bf16(b), variant="tcgen05"))
    mcke.check_device_errors()
    # (1) against the oracle on the same bf16 inputs: fp32-accumulation tolerance
    if m * n * k <= 600 * 1000 * 1000:
        want = oracle.gemm(ar, br)
        assert_close(got, want, 4 * oracle.tol_gemm(k), 4 * oracle.abs_tol_gemm(k), (m, n, k))
        # (2) north star: <= 1e-2 against the fp32-input reference
        want32 = oracle.gemm(a, b)
        # abs floor ~10 sigma of the bf16 input-rounding error; max rel checked
        # over outputs above their RMS, sqrt(k/9)*3
        assert_close(got, want32, 1e-2, 4 * np.sqrt(k) * 2.0 ** -8 / 3, (m, n, k), max_rel=1e-2,
                     floor=float(np.sqrt(k / 3.0)))
    else:
        r = oracle.spot_check_gemm(ar, br, got, samples=512, seed=1, rel_tol=4 * oracle.tol_gemm(k),
                                   abs_tol=4 * oracle.abs_tol_gemm(k))
        assert r["mismatches"] == 0, r


@pytest.mark.parametrize("m,n,k", [(256, 512, 128), (1000, 712, 520), (300, 1544, 264), (2048, 2048, 1024)])
def test_gemm_bf16_wide_tile_matches_narrow_and_oracle(m, n, k):
    # the 256 x 512 pair tile (forced): same k order per output as the
    # 256 x 256 tile, so the results agree bit for bit
    a = oracle.fill_random(m * k, 4).reshape(m, k)
    b = oracle.fill_random(k * n, 5).reshape(k, n)
    ta, tb = _bf16(a), _bf16(b)
    wide = host(mcke.gemm(ta, tb, variant="tcgen05_wide"))
    narrow = host(mcke.gemm(ta, tb, variant="tcgen05_narrow"))
    mcke.check_device_errors()
    assert np.array_equal(wide.view(np.uint32), narrow.view(np.uint32))
    r = oracle.spot_check_gemm(oracle.round_bf16(a), oracle.round_bf16(b), wide, samples=1024, seed=2,
                               rel_tol=4 * oracle.tol_gemm(k), abs_tol=4 * oracle.abs_tol_gemm(k))
    assert r["mismatches"] == 0, r
    # fused epilogue and bf16 output on the wide tile
    bias = torch.from_numpy(oracle.fill_random(n, 6)).to(DEV)
    w2 = host(mcke.gemm(ta, tb, bias=bias, act="gelu_tanh", out_dtype=torch.bfloat16,
                        variant="tcgen05_wide").view(torch.int16))
    n2 = host(mcke.gemm(ta, tb, bias=bias, act="gelu_tanh", out_dtype=torch.bfloat16,
                        variant="tcgen05_narrow").view(torch.int16))
    assert np.array_equal(w2, n2)


@pytest.mark.parametrize("m,n,k", [(512, 1024, 4096), (2048, 1024, 8192), (8192, 1024, 2048), (8192, 4096, 1024),
                                   (768, 1536, 2056)])
def test_gemm_bf16_split_k_schedule(m, n, k):
    # Tiles cut between CTA pairs, 2 to 17 contributors per tile (k order
    # sums through C), after whole data-parallel waves for (8192, 4096, 1024).
    # Deterministic, within tolerance of the unsplit kernel and the oracle.
    a = oracle.fill_random(m * k, 7).reshape(m, k)
    b = oracle.fill_random(k * n, 8).reshape(k, n)
    ta, tb = _bf16(a), _bf16(b)
    dp = host(mcke.gemm(ta, tb, variant="tcgen05_wide"))
    s1 = host(mcke.gemm(ta, tb, variant="tcgen05_split"))
    s2 = host(mcke.gemm(ta, tb, variant="tcgen05_split"))
    mcke.check_device_errors()
    assert np.array_equal(s1.view(np.uint32), s2.view(np.uint32))
    tol, atol = 4 * oracle.tol_gemm(k), 4 * oracle.abs_tol_gemm(k)
    r = oracle.spot_check_gemm(oracle.round_bf16(a), oracle.round_bf16(b), s1, samples=2048, seed=3,
                               rel_tol=tol, abs_tol=atol)
    assert r["mismatches"] == 0, r
    assert np.all(np.abs(s1.astype(np.float64) - dp) <= 2 * (atol + tol * np.abs(dp)))
    # every element was written by the split schedule (no stale partial sums)
    assert np.isfinite(s1).all()
    # fused bias + GELU on the last contributor
    bias = torch.from_numpy(oracle.fill_random(n, 9)).to(DEV)
    e_dp = host(mcke.gemm(ta, tb, bias=bias, act="gelu_tanh", variant="tcgen05_wide"))
    e_sp = host(mcke.gemm(ta, tb, bias=bias, act="gelu_tanh", variant="tcgen05_split"))
    mcke.check_device_errors()
    assert np.all(np.abs(e_sp.astype(np.float64) - e_dp) <= 2 * (atol + tol * np.abs(e_dp)))


def test_gemm_bf16_split_k_chosen_and_concurrent():
    # 256 tiles of 256 x 512 for 74 CTA pairs: AUTO runs two data-parallel
    # waves and splits the rest (it differs from the unsplit result in the
    # last bits); two launches in flight on two streams use separate flag slots
    m, n, k = 8192, 4096, 4096
    gen = torch.Generator(device=DEV)
    gen.manual_seed(12)
    ta = (torch.rand(m, k, generator=gen, device=DEV) * 2 - 1).to(torch.bfloat16)
    tb = (torch.rand(k, n, generator=gen, device=DEV) * 2 - 1).to(torch.bfloat16)
    ref = mcke.gemm(ta, tb, variant="tcgen05_split")
    auto = mcke.gemm(ta, tb, variant="tcgen05")
    dp = mcke.gemm(ta, tb, variant="tcgen05_wide")
    torch.cuda.synchronize()
    assert torch.equal(auto, ref)
    assert not torch.equal(auto, dp)
    assert torch.allclose(ref, dp, rtol=4 * oracle.tol_gemm(k), atol=8 * oracle.abs_tol_gemm(k))
    s1, s2 = torch.cuda.Stream(DEV), torch.cuda.Stream(DEV)
    outs = []
    for _ in range(3):
        for st in (s1, s2):
            with torch.cuda.stream(st):
                outs.append(mcke.gemm(ta, tb, variant="tcgen05_split"))
    torch.cuda.synchronize()
    mcke.check_device_errors()
    for o in outs:
        assert torch.equal(o, ref)


def test_gemm_bf16_fused_epilogue():
    m, n, k = 256, 512, 192
    a = oracle.fill_normal(m * k, 4).reshape(m, k)
    b = oracle.fill_normal(k * n, 5, 0.0, 0.02 * 8).reshape(k, n)
    bias = oracle.fill_random(n, 6)
    ar, br = oracle.round_bf16(a), oracle.round_bf16(b)
    lin = oracle.gemm(ar, br)
    want = oracle.to_bf16(oracle.bias_act(lin, bias, "gelu_tanh"))
    wantf = oracle.bf16_to_f32(want).astype(np.float64)
    for variant in ("tcgen05", "simt"):
        out = mcke.gemm(_bf16(a), _bf16(b), bias=dev(bias), act="gelu_tanh",
                        out_dtype=torch.bfloat16, variant=variant)
        gotf = oracle.bf16_to_f32(host(out.view(torch.int16)).view(np.uint16)).astype(np.float64)
        # one bf16 rounding of values that agree to fp32 accuracy: within one
        # bf16 ulp (at most 2^-7 relative), or 1e-6 absolute where GELU is ~0 (there the
        # double oracle's 1 + tanh cancels to 0 while the kernel keeps the tiny value)
        err = np.abs(gotf - wantf)
        assert np.all(err <= np.abs(wantf) * 2.0 ** -7 + 1e-6), (variant, float(err.max()))
    # fp32 output with alpha/beta/bias
    c0 = oracle.fill_random(m * n, 7).reshape(m, n)
    got = host(mcke.gemm(_bf16(a), _bf16(b), dev(c0), 0.5, 2.0, bias=dev(bias), variant="tcgen05"))
    want = oracle.bias_act((np.float64(0.5) * lin + 2.0 * c0).astype(np.float32), bias, "none")
    assert_close(got, want, 1e-5, 1e-5)


def test_gemm_bf16_simt_fallback_for_tma_incompatible_shapes():
    m, n, k = 37, 5, 7  # K, N not multiples of 8: TMA cannot describe them
    a = oracle.fill_random(m * k, 2).reshape(m, k)
    b = oracle.fill_random(k * n, 3).reshape(k, n)
    got = host(mcke.gemm(_bf16(a), _bf16(b)))
    assert_close(got, oracle.gemm(oracle.round_bf16(a), oracle.round_bf16(b)), oracle.tol_gemm(k),
                 oracle.abs_tol_gemm(k))
    with pytest.raises(mcke.MckeError):
        mcke.gemm(_bf16(a), _bf16(b), variant="tcgen05")


def test_gemm_kernel_attrs_report_no_spills():
    for variant, dt in (("tcgen05", "bf16"), ("simt", "f32"), ("simt", "bf16")):
        at = mcke.gemm_kernel_attrs(variant, dt)
        assert at["local_bytes"] == 0 and at["regs_per_thread"] > 0, (variant, at)
        assert at["max_blocks_per_sm_api"] >= 1


# ------------------------------------------------------------ failure path

def test_bounded_wait_expiry_is_reported_and_the_context_survives():
    # A wait on a barrier nothing arrives on gives up after its 2 s limit; the
    # host reads the status, and the next kernels run normally.
    mcke.check_device_errors()  # start clean
    s = torch.cuda.current_stream().cuda_stream
    assert mcke.lib().mcke_sm100_watchdog_selftest(s) == mcke.OK
    with pytest.raises(mcke.MckeError) as e:
        mcke.check_device_errors()
    assert e.value.code == mcke.INTERNAL and "site 9" in e.value.message and "self-test" in e.value.message
    mcke.check_device_errors()  # the word was cleared
    x = dev(oracle.fill_random(4096, 3))
    assert mcke.decode_result(mcke.reduce_full(x))[2] == int(np.argmax(host(x)))


def test_peak_probes():
    # the roofline probes (triad, copy, FFMA) compute what they claim
    n = 1 << 20
    idx = torch.arange(n, device=DEV, dtype=torch.float32)
    b = idx % 97
    c = (idx % 13) * 0.5
    a = torch.empty(n, device=DEV)
    mcke.peak_triad(a, b, c, 3.0)
    assert torch.equal(a, b + 3.0 * c)  # small integers and halves: exact either way
    a2 = torch.empty(n, device=DEV)
    mcke.peak_copy(a2, b)
    assert torch.equal(a2, b)
    with pytest.raises(mcke.MckeError):
        mcke.peak_copy(a2[:7], b[:7])  # n % 4 != 0
    nt = mcke.peak_fma_threads()
    assert nt > 0 and nt % 256 == 0
    seed = (torch.arange(512, device=DEV, dtype=torch.float32) % 13)
    out = torch.empty(512, device=DEV)
    mcke.peak_fma(seed, out, 100)
    mcke.check_device_errors()
    s = seed.cpu().numpy().astype(np.float64)
    acc = np.stack([s + j for j in range(8)])
    for _ in range(100):  # fma(acc, m, 1): acc * m is exact in float64
        acc = (acc * np.float64(np.float32(0.999)) + 1.0).astype(np.float32).astype(np.float64)
    want = acc.astype(np.float32).sum(axis=0, dtype=np.float32)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5)


def test_tcgen05_peak_probe_runs_at_tensor_rate():
    # the bf16 probe completes (its bounded wait did not expire) and runs at a
    # tensor-core rate: between a third of and 10% above the nominal dense peak
    ctas = mcke.peak_mma_ctas()
    assert ctas == torch.cuda.get_device_properties(DEV).multi_processor_count
    mcke.peak_mma(ctas, 200)  # warm-up
    mcke.check_device_errors()
    iters = 4000
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    mcke.peak_mma(ctas, iters)
    e1.record()
    torch.cuda.synchronize()
    mcke.check_device_errors()
    tflops = mcke.peak_mma_flops(ctas, iters) / (e0.elapsed_time(e1) * 1e-3) / 1e12
    assert 750.0 < tflops < 2475.0, tflops


@pytest.mark.parametrize("m,n,k", [(8192, 4096, 4096), (4096, 8192, 2048), (2048, 4096, 1024), (8192, 1024, 2048),
                                   (300, 512, 256)])
def test_gemm_plan_matches_the_launch(m, n, k):
    # AUTO's result is bit-identical to the forced variant that
    # mcke_sm100_gemm_plan names (split and unsplit differ in the last bits)
    p = mcke.gemm_plan(m, n, k, "auto", "f32", torch.cuda.get_device_properties(DEV).multi_processor_count)
    gen = torch.Generator(device=DEV)
    gen.manual_seed(m + n + k)
    ta = (torch.rand(m, k, generator=gen, device=DEV) * 2 - 1).to(torch.bfloat16)
    tb = (torch.rand(k, n, generator=gen, device=DEV) * 2 - 1).to(torch.bfloat16)
    auto = mcke.gemm(ta, tb, variant="tcgen05")
    if p["split_kblocks"]:
        assert p["tile_n"] == 512
        forced = mcke.gemm(ta, tb, variant="tcgen05_split")
    else:
        forced = mcke.gemm(ta, tb, variant="tcgen05_wide" if p["tile_n"] == 512 else "tcgen05_narrow")
    torch.cuda.synchronize()
    mcke.check_device_errors()
    assert torch.equal(auto, forced), p
