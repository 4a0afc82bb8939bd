"""MCKE_REDUCE_EARLY_READ (mcke_sm100_reduce_full_f32_ex,
mcke_sm100_reduce_full_p2p_f32_ex): the streaming kernel reads x before it
waits for the kernel enqueued just before it, and writes nothing until then.
Checked here:
  * back-to-back early calls (two inputs in turn, one shared workspace, one
    output per call) give the default path's bits, for the two-launch entry
    point and the one-kernel peer-to-peer entry point at world 1;
  * the caller's contract is enough: x rewritten by a torch kernel, then an
    unrelated kernel of this library, then the early-read reduce, which must
    see the new x (its writer ran two kernels earlier).
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


def _bytes(t) -> bytes:
    return t.cpu().numpy().tobytes()


def _input(n: int, seed: int) -> torch.Tensor:
    v = oracle.fill_random(max(n, 1), seed)[:n]
    if n > 40:
        v[n - 7] = v[31] = np.float32(2.5)  # tie: the lower index wins
    return torch.from_numpy(v).cuda()


@pytest.mark.parametrize("n", [1, 5, 3_000_007, (1 << 25) + 3])
def test_early_read_back_to_back_same_bits(n):
    xs = [_input(n, 41), _input(n, 42)]
    want = [_bytes(mcke.reduce_full(x)) for x in xs]
    ws = torch.empty(max(mcke.reduce_full_workspace_bytes(n), 16), dtype=torch.uint8, device="cuda")
    buf = torch.zeros(mcke.lib().mcke_sm100_reduce_p2p_buffer_bytes(1), dtype=torch.uint8, device="cuda")
    table = torch.tensor([buf.data_ptr()], dtype=torch.int64, device="cuda")
    steps = 8
    outs = [torch.empty(mcke.RESULT_BYTES, dtype=torch.uint8, device="cuda") for _ in range(2 * steps)]
    torch.cuda.synchronize()
    for i in range(steps):
        mcke.reduce_full(xs[i % 2], out=outs[i], workspace=ws, early_read=True)
    for i in range(steps):
        mcke.reduce_full_p2p(xs[i % 2], 0, table, 1, 0, i + 1, out=outs[steps + i], early_read=True)
    torch.cuda.synchronize()
    mcke.check_device_errors()
    for i in range(2 * steps):
        got = _bytes(outs[i])
        assert got == want[i % 2], (i, mcke.decode_result(got), mcke.decode_result(want[i % 2]))


def test_early_read_sees_a_writer_two_kernels_back():
    n = 1 << 24
    srcs = [_input(n, 50 + k) for k in range(3)]
    want = [_bytes(mcke.reduce_full(s)) for s in srcs]
    x = torch.empty(n, device="cuda")
    small = torch.randn(64, 256, device="cuda")
    small_out = torch.empty_like(small)
    ws = torch.empty(mcke.reduce_full_workspace_bytes(n), dtype=torch.uint8, device="cuda")
    outs = [torch.empty(mcke.RESULT_BYTES, dtype=torch.uint8, device="cuda") for _ in range(9)]
    torch.cuda.synchronize()
    for i in range(9):
        x.copy_(srcs[i % 3])                    # a torch kernel writes x
        mcke.softmax(small, out=small_out)      # this library's kernel, programmatic serialization
        mcke.reduce_full(x, out=outs[i], workspace=ws, early_read=True)
    torch.cuda.synchronize()
    mcke.check_device_errors()
    for i in range(9):
        assert _bytes(outs[i]) == want[i % 3], i
