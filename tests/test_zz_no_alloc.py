"""mcke_sm100_reduce_full_f32_noalloc: the full reduce for callers that cannot
allocate device memory (a runtime whose memory manager owns every device
allocation, or a foreign-language binding holding only its own input and
output buffers), so they cannot pass the workspace mcke_sm100_reduce_full_f32
needs.  It keeps its scratch in a fixed array inside the library instead.

Checked through the C-ABI against the existing entry point on the same inputs,
on three calls in a row of falling sizes (pass-1 grids of 444, 50 and 1
blocks).  The first input's unique maximum sits in a partial slot beyond the
later calls' grids, so a combine that folded leftover slots from the shared
array would report it.  Tolerances are those of
tests/test_gpu_parity.py: max and argmax bit for bit, the double-accumulated
sum within one float ulp.  This file sorts last so that a run stopping at the
first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover - CPU container
    pytest.skip("needs a CUDA device", allow_module_level=True)

import mcke  # noqa: E402


def _noalloc():
    fn = mcke.lib().mcke_sm100_reduce_full_f32_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
    return fn


def _with_workspace(x: torch.Tensor) -> tuple[float, float, int]:
    return mcke.decode_result(mcke.reduce_full(x))


def test_noalloc_matches_the_workspace_entry_point_on_two_calls_in_a_row():
    dev = torch.device("cuda:0")
    fn = _noalloc()
    stream = torch.cuda.current_stream(dev).cuda_stream
    big = oracle.fill_random((1 << 22) + 3, 11)
    big[777] = big[3_000_001] = np.float32(1.25)  # tie: lowest index wins
    # Thread t of pass-1 block j reads float4 j * 256 + t first, so element
    # 4 * (100 * 256 + 5) lands in partial slot 100: left in the array by this
    # call, never written by the next two (50 blocks, then 1 block).
    big[4 * (100 * 256 + 5)] = np.float32(7.0)
    middle = oracle.fill_random(50 * 4096, 13)  # 50 blocks of 4096 floats
    small = oracle.fill_random(1000, 12)
    for host in (big, middle, small):
        x = torch.from_numpy(host).to(dev)
        out = torch.zeros(16, dtype=torch.uint8, device=dev)
        rc = fn(x.data_ptr(), x.numel(), out.data_ptr(), stream)
        assert rc == mcke.OK, mcke.lib().mcke_sm100_last_error_string()
        torch.cuda.synchronize()
        s, m, i = mcke.decode_result(out)
        ws, wm, wi = _with_workspace(x)
        assert np.float32(m).view(np.uint32) == np.float32(wm).view(np.uint32)
        assert i == wi
        assert abs(s - ws) <= np.spacing(np.float32(abs(ws)))
        assert i == int(np.argmax(host)) and m == host.max()
    assert mcke.decode_result(out)[2] == int(np.argmax(small))


def test_noalloc_rejects_bad_arguments():
    fn = _noalloc()
    assert fn(None, 10, ctypes.c_void_p(0x1000), None) == mcke.INVALID_ARGUMENT
    assert fn(ctypes.c_void_p(0x1000), -1, ctypes.c_void_p(0x2000), None) == mcke.INVALID_ARGUMENT
