"""The C-ABI library on the CPU: it loads, exports every symbol include/mcke_sm100.h
declares, and rejects bad arguments before touching a device (no compute)."""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mini-cuda-kernel-engine_b200")


@pytest.fixture(scope="module")
def mcke():
    import mcke as m
    if not os.path.exists(m.LIB_PATH):
        subprocess.run([sys.executable, os.path.join(PKG, "build.py")], check=True)
    return m


def test_library_exports_every_declared_symbol(mcke):
    names = mcke.declared_symbols()
    assert len(names) >= 18
    l = ctypes.CDLL(mcke.LIB_PATH)
    missing = [n for n in names if not hasattr(l, n)]
    assert not missing, missing
    # and exports nothing under the prefix that the header does not declare
    out = subprocess.run(["nm", "-D", "--defined-only", mcke.LIB_PATH], capture_output=True, text=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T mcke_sm100_" in ln}
    assert exported == set(names)


def test_host_library_exports_every_declared_symbol(mcke):
    # include/mcke_host.h (graph / executor C-ABI over the C++ host layer)
    import re
    lib_path = os.path.join(PKG, "lib", "libmcke_host.so")
    if not os.path.exists(lib_path):
        subprocess.run(["make", "-s", "-C", os.path.join(PKG, "host")], check=True)
    with open(os.path.join(ROOT, "include", "mcke_host.h")) as f:
        names = sorted(set(re.findall(r"\b(mcke_(?:graph|executor|host)_\w+)\s*\(", f.read())))
    assert len(names) >= 20
    l = ctypes.CDLL(lib_path)
    missing = [n for n in names if not hasattr(l, n)]
    assert not missing, missing


def test_argument_validation_needs_no_device(mcke):
    l = mcke.lib()
    assert l.mcke_sm100_version() >= 100
    bogus = ctypes.c_void_p(0x1000)
    # null pointer / negative extent / bad width / aliasing -> INVALID_ARGUMENT, with a message
    assert l.mcke_sm100_bias_act_f32(None, bogus, bogus, 4, 4, 3, 4, 0, None) == mcke.INVALID_ARGUMENT
    assert b"null" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_bias_act_f32(bogus, bogus, ctypes.c_void_p(0x2000), 4, 6, 3, 4, 0, None) == mcke.INVALID_ARGUMENT
    assert b"multiple of vector_width" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_bias_act_f32(bogus, bogus, bogus, 4, 8, 3, 4, 0, None) == mcke.INVALID_ARGUMENT
    assert l.mcke_sm100_softmax_f32(bogus, bogus, 4, 4, 1, None) == mcke.INVALID_ARGUMENT
    assert l.mcke_sm100_softmax_f32(bogus, ctypes.c_void_p(0x2000), -1, 4, 1, None) == mcke.INVALID_ARGUMENT
    assert l.mcke_sm100_gemm_f32(bogus, ctypes.c_void_p(0x2000), bogus, 4, 4, 4, 1.0, 0.0, 0, None) == mcke.INVALID_ARGUMENT
    assert b"aliases" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_gemm_f32(bogus, bogus, ctypes.c_void_p(0x3000), 4, 4, 4, 1.0, 0.0, 2, None) == mcke.INVALID_ARGUMENT
    assert l.mcke_sm100_gemm_bf16(bogus, ctypes.c_void_p(0x2000), ctypes.c_void_p(0x3000), 4, 5, 7, 1.0, 0.0, 2, None) == mcke.INVALID_ARGUMENT
    assert b"no fallback" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_gemm_bf16_ex(bogus, ctypes.c_void_p(0x2000), ctypes.c_void_p(0x3000), 2, 8, 8, 8, 1.0, 1.0, None, 0, 0, None) == mcke.INVALID_ARGUMENT
    assert l.mcke_sm100_reduce_row_f32(bogus, ctypes.c_void_p(0x2000), 4, 64, 0, 2, None, 0, None) == mcke.UNIMPLEMENTED
    assert l.mcke_sm100_reduce_full_f32(bogus, 1000, ctypes.c_void_p(0x2000), None, 0, None) == mcke.INVALID_ARGUMENT
    assert b"workspace" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_reduce_full_p2p_f32_timeline(bogus, 1000, 0, bogus, 1, 0, 1, bogus, None,
                                                      None) == mcke.INVALID_ARGUMENT
    assert b"stamps" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_reduce_full_p2p_f32_timeline(bogus, 1000, 0, bogus, 1, 0, 1, bogus,
                                                      ctypes.c_void_p(0x1004), None) == mcke.INVALID_ARGUMENT
    # grouped bias + activation: count, shape, alignment and overlap checks
    J = mcke.BiasActJob
    jobs = (J * 17)()
    grp = lambda n: l.mcke_sm100_bias_act_f32_group(ctypes.cast(jobs, ctypes.c_void_p), n, 3, None)  # noqa: E731
    assert l.mcke_sm100_bias_act_f32_group(None, 1, 3, None) == mcke.INVALID_ARGUMENT
    assert grp(0) == mcke.INVALID_ARGUMENT and grp(17) == mcke.INVALID_ARGUMENT
    jobs[0] = J(0x100000, 0x200000, 0x300000, 4, 256)
    assert grp(1) == mcke.INVALID_ARGUMENT and b"multiple of 512" in l.mcke_sm100_last_error_string()
    jobs[0] = J(0x100004, 0x200000, 0x300000, 4, 512)
    assert grp(1) == mcke.INVALID_ARGUMENT and b"aligned" in l.mcke_sm100_last_error_string()
    jobs[0] = J(0x100000, 0x200000, 0x300000, 4, 512)  # x: 8 KB from 0x100000
    jobs[1] = J(0x400000, 0x200000, 0x100800, 4, 512)  # y inside job 0's x
    assert grp(2) == mcke.INVALID_ARGUMENT and b"overlaps" in l.mcke_sm100_last_error_string()
    jobs[1] = J(0x400000, 0x200000, 0x300000, 4, 512)  # same y as job 0
    assert grp(2) == mcke.INVALID_ARGUMENT and b"overlaps" in l.mcke_sm100_last_error_string()
    jobs[0] = J(0x100000, 0x200000, 0x100000, 4, 512)  # in place
    assert grp(1) == mcke.INVALID_ARGUMENT and b"overlaps" in l.mcke_sm100_last_error_string()
    jobs[0] = J(None, None, None, 0, 512)  # one empty job: nothing to launch
    assert grp(1) == mcke.OK
    # the _ex entry points take MCKE_REDUCE_EARLY_READ (1) and nothing else
    assert l.mcke_sm100_reduce_full_f32_ex(bogus, 1000, ctypes.c_void_p(0x2000), bogus, 1 << 20, 2,
                                           None) == mcke.INVALID_ARGUMENT
    assert b"unknown flags" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_reduce_full_f32_ex(bogus, 1000, ctypes.c_void_p(0x2000), None, 0, 1,
                                           None) == mcke.INVALID_ARGUMENT
    assert b"workspace" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_reduce_full_p2p_f32_ex(bogus, 1000, 0, bogus, 1, 0, 1, bogus, 0x80000000,
                                               None) == mcke.INVALID_ARGUMENT
    assert b"unknown flags" in l.mcke_sm100_last_error_string()
    assert l.mcke_sm100_reduce_full_p2p_f32_ex(bogus, 1000, 0, bogus, 0, 0, 1, bogus, 1,
                                               None) == mcke.INVALID_ARGUMENT
    assert b"world" in l.mcke_sm100_last_error_string()
    # empty extents are OK with no launch
    assert l.mcke_sm100_softmax_f32(None, None, 0, 16, 1, None) == mcke.OK
    assert l.mcke_sm100_bias_act_f32(None, None, None, 0, 0, 3, 4, 0, None) == mcke.OK
    assert l.mcke_sm100_gemm_f32(None, None, None, 0, 4, 4, 1.0, 0.0, 0, None) == mcke.OK


def test_workspace_queries(mcke):
    l = mcke.lib()
    assert l.mcke_sm100_reduce_full_workspace_bytes(0) == 0
    assert l.mcke_sm100_reduce_full_workspace_bytes(1) == 24
    # the combine grid is capped at 3 CTAs x 148 SMs, whatever the device
    assert l.mcke_sm100_reduce_full_workspace_bytes(1 << 28) == 3 * 148 * 24
    assert l.mcke_sm100_reduce_full_workspace_bytes(4096 * 5 + 1) == 6 * 24
    assert l.mcke_sm100_reduce_row_workspace_bytes(64, 1 << 19, 1) == 0
    assert l.mcke_sm100_reduce_row_workspace_bytes(64, 1 << 19, 2) == 64 * 19 * 8


def test_mma_probe_arguments_need_no_device(mcke):
    l = mcke.lib()
    assert l.mcke_sm100_peak_mma_flops(148, 10) == 148 * 10 * 4 * 2 * 128 * 256 * 16
    assert l.mcke_sm100_peak_mma_flops(0, 10) == 0.0
    assert l.mcke_sm100_peak_mma_bf16(-1, 10, None) == mcke.INVALID_ARGUMENT
    assert l.mcke_sm100_peak_mma_bf16(70000, 10, None) == mcke.INVALID_ARGUMENT
    assert l.mcke_sm100_peak_mma_bf16(0, 10, None) == mcke.OK  # nothing to launch
