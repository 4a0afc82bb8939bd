"""The bf16 GEMM's schedule choices, pinned on the CPU through
mcke_sm100_gemm_plan (host arithmetic only; the GPU parity tests run the
same shapes through the kernels).  The reference has no counterpart: its
GEMM launcher (kernels/gemm.cu:607 gemm_launch_spec) picks one fixed tile."""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "mini-cuda-kernel-engine_b200"))

import mcke  # noqa: E402

B200_SMS = 148


def plan(m, n, k, variant="auto", out_dtype="f32", sms=B200_SMS):
    return mcke.gemm_plan(m, n, k, variant, out_dtype, sms)


def test_one_gpu_8192_cubed_runs_the_wide_tile_in_whole_waves():
    p = plan(8192, 8192, 8192)
    assert (p["kernel"], p["tile_m"], p["tile_n"], p["tiles"], p["ctas"]) == (2, 256, 512, 512, 148)
    assert p["split_kblocks"] == 0  # 7 waves, 98.8% of the pairs busy


def test_column_shards_of_8192_cubed():
    # 2 GPUs: 256 tiles = 2 whole waves + 108 tiles split over the 74 pairs
    p = plan(8192, 4096, 8192)
    assert (p["tile_n"], p["tiles"], p["split_dp_tiles"]) == (512, 256, 148)
    assert p["split_kblocks"] == -(-(256 - 148) * 128 // 74)  # 187
    # 4 and 8 GPUs: one or two partial waves stay data-parallel (the split
    # measured slower there)
    for n, tiles, ctas in ((2048, 128, 148), (1024, 64, 128)):
        p = plan(8192, n, 8192)
        assert (p["tile_n"], p["tiles"], p["ctas"], p["split_kblocks"]) == (512, tiles, ctas, 0)


def test_dag_gemms():
    # GEMM1: bf16 output, no split; GEMM2: fp32 + bias, 256 tiles -> split
    g1 = plan(8192, 16384, 4096, out_dtype="bf16")
    assert (g1["tile_n"], g1["tiles"], g1["split_kblocks"]) == (512, 1024, 0)
    g2 = plan(8192, 4096, 16384)
    assert (g2["tile_n"], g2["split_dp_tiles"], g2["split_kblocks"]) == (512, 148, -(-108 * 256 // 74))


def test_short_k_prefers_the_overlapped_narrow_tile():
    p = plan(8192, 4096, 1024)
    assert (p["tile_n"], p["tiles"], p["split_kblocks"]) == (256, 512, 0)


def test_bf16_output_is_never_split():
    p = plan(8192, 4096, 8192, out_dtype="bf16")
    assert p["split_kblocks"] == 0 and p["ctas"] == 148


def test_forced_variants():
    assert plan(8192, 4096, 8192, "tcgen05_narrow")["tile_n"] == 256
    assert plan(8192, 4096, 8192, "tcgen05_narrow")["split_kblocks"] == 0
    assert plan(8192, 4096, 8192, "tcgen05_wide")["split_kblocks"] == 0
    s = plan(2048, 2048, 1024, "tcgen05_split")
    assert (s["tile_n"], s["tiles"], s["split_dp_tiles"], s["ctas"]) == (512, 32, 0, 148)
    assert s["split_kblocks"] == -(-32 * 16 // 74)
    # forced split on a shape it cannot take (N not a whole number of tiles)
    assert plan(2048, 2056, 1024, "tcgen05_split")["split_kblocks"] == 0


def test_single_cta_tiles_and_the_simt_fallback():
    p = plan(100, 512, 64)
    assert (p["kernel"], p["tile_m"], p["tile_n"], p["ctas"]) == (1, 128, 256, 2)
    s = plan(1000, 1001, 8)  # N % 8 != 0: CUDA-core kernel
    assert (s["kernel"], s["tile_m"], s["tiles"]) == (0, 128, 8 * 8)
    assert plan(8192, 8192, 8192, "simt")["kernel"] == 0
    with pytest.raises(mcke.MckeError):
        plan(1000, 1001, 8, "tcgen05")
    with pytest.raises(mcke.MckeError):
        plan(-1, 8, 8)
    with pytest.raises(mcke.MckeError):
        plan(8, 8, 8, 99)


@pytest.mark.parametrize("sms", [148, 132, 120])
def test_split_plans_cover_every_k_block(sms):
    pairs = sms // 2
    for m, n, k in ((8192, 4096, 8192), (4096, 4096, 4096), (8192, 8192, 2056), (2048, 4096, 16384)):
        for variant in ("auto", "tcgen05_split"):
            p = plan(m, n, k, variant, sms=sms)
            if p["kernel"] != 2 or p["split_kblocks"] == 0:
                continue
            kb = -(-k // 64)
            assert p["split_dp_tiles"] % pairs == 0 and p["split_dp_tiles"] < p["tiles"]
            assert p["split_kblocks"] * pairs >= (p["tiles"] - p["split_dp_tiles"]) * kb
            assert (p["split_kblocks"] - 1) * pairs < (p["tiles"] - p["split_dp_tiles"]) * kb
            assert p["ctas"] == 2 * pairs
