"""Programmatic dependent launch (B200 only).

Every kernel of the library waits for the grid before it on the stream
(griddepcontrol.wait) before touching global memory, so launching it with
programmatic stream serialization may only move its start-up earlier, never
its reads or writes.  These tests run dependent chains back to back on one
stream with the attribute on and off and require the same bits, including a
write-after-read hazard: a kernel that overwrites the buffer the kernel before
it is reading.
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


@pytest.fixture
def restore_launch_mode():
    prev = mcke.set_programmatic_launch(True)
    yield
    mcke.set_programmatic_launch(prev)


def _chain(x, b, a16, b16, reps):
    outs = []
    for _ in range(reps):
        h = mcke.bias_act(x, b, "gelu_tanh")              # reads x
        p = mcke.softmax(h)                              # reads h as soon as bias_act is done
        m = mcke.reduce_row(p, "max")                    # reads p
        s = mcke.reduce_full(h)                          # reads h
        c = mcke.gemm(a16, b16, variant="tcgen05")       # tensor cores, independent inputs
        y = mcke.bias_act(c, b[: c.shape[1]], "relu")    # reads the GEMM's output
        outs.append((p, m, s, y))
    torch.cuda.synchronize()
    mcke.check_device_errors()
    return [tuple(t.cpu().numpy().copy() for t in o) for o in outs]


def test_dependent_chain_is_the_same_with_and_without_programmatic_launch(restore_launch_mode):
    x = torch.from_numpy(oracle.fill_normal(4096 * 1024, 1).reshape(4096, 1024)).to(DEV)
    b = torch.from_numpy(oracle.fill_random(1024, 2)).to(DEV)
    a16 = (torch.rand(512, 256, device=DEV) * 2 - 1).to(torch.bfloat16)
    b16 = (torch.rand(256, 1024, device=DEV) * 2 - 1).to(torch.bfloat16)
    results = {}
    for mode in (False, True):
        mcke.set_programmatic_launch(mode)
        results[mode] = _chain(x, b, a16, b16, reps=8)
    for plain, pdl in zip(results[False], results[True]):
        for u, v in zip(plain, pdl):
            assert np.array_equal(u.view(np.uint8), v.view(np.uint8))
    # and against the oracle for the softmax of the first step
    p0 = results[True][0][0]
    want = oracle.row_softmax(oracle.bias_act(x.cpu().numpy(), b.cpu().numpy(), "gelu_tanh"))
    r = oracle.compare(p0, want, 1e-5, 1e-8)
    assert r["mismatches"] == 0, r


def test_next_kernel_does_not_overwrite_an_input_still_being_read(restore_launch_mode):
    # per step: restore x, softmax reads x, then bias_act overwrites x.  A
    # kernel that wrote before the one ahead of it had finished reading would
    # leave some softmax row computed from the overwritten x.
    rows, cols = 32768, 1024
    x0 = torch.from_numpy(oracle.softmax_config_input(rows, cols, seed=3)).to(DEV)
    zero = torch.zeros_like(x0)
    other = torch.randn(rows, cols, device=DEV)
    bias = torch.zeros(cols, device=DEV)
    x = torch.empty_like(x0)
    ys = [torch.empty_like(x0) for _ in range(6)]
    mcke.set_programmatic_launch(True)
    for y in ys:
        mcke.vector_add(x0, zero, out=x)                 # x = x0
        mcke.softmax(x, out=y)                           # reads x
        mcke.bias_act(other, bias, "relu", out=x)        # overwrites x
    torch.cuda.synchronize()
    want = mcke.softmax(x0)
    torch.cuda.synchronize()
    for y in ys:
        assert torch.equal(y, want)
