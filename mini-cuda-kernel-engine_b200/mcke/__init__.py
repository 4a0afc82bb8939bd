"""Python binding of libmcke_sm100a.so (include/mcke_sm100.h) over ctypes.

Tensors are torch CUDA tensors: torch supplies device memory and streams, the
arithmetic is this library's CUDA kernels.  Every call enqueues on the current
torch stream of the tensor's device (or an explicit ``stream``) and never
synchronises.  A non-OK status raises :class:`MckeError` carrying the
library's message.  There is no CPU or library fallback: if the shared
library is missing the first call raises.
"""
from __future__ import annotations

import ctypes
import os
import re
import struct

import torch

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ROOT = os.path.dirname(PKG_DIR)
LIB_PATH = os.path.join(PKG_DIR, "lib", "libmcke_sm100a.so")
HEADER = os.path.join(ROOT, "include", "mcke_sm100.h")

OK, OUT_OF_MEMORY, INVALID_ARGUMENT, FAILED_PRECONDITION, UNIMPLEMENTED, INTERNAL, CUDA_ERROR = range(7)
ACT = {"none": 0, "relu": 1, "gelu_erf": 2, "gelu_tanh": 3}
REDUCE_KIND = {"sum": 0, "max": 1, "mean": 2}
REDUCE_VARIANT = {"smem_tree": 0, "warp_shuffle": 1, "two_pass": 2}
SOFTMAX_VARIANT = {"three_pass": 0, "online": 1}
GEMM_VARIANT = {"auto": 0, "simt": 1, "tcgen05": 2, "tcgen05_wide": 3, "tcgen05_narrow": 4, "tcgen05_split": 5}
DTYPE = {"f32": 0, "bf16": 2}
RESULT_BYTES = 16   # mcke_reduce_result
PARTIAL_BYTES = 24  # mcke_reduce_partial


class MckeError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[mcke status {code}] {message}")
        self.code = code
        self.message = message


_lib = None


def declared_symbols() -> list[str]:
    """Every mcke_sm100_* function declared in include/mcke_sm100.h."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(mcke_sm100_\w+)\s*\(", text)))


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build() "
                               "(there is no fallback path)")
        l = ctypes.CDLL(LIB_PATH)
        i64, i32, vp, f32, sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_float, ctypes.c_size_t
        sigs = {
            "mcke_sm100_version": (i32, []),
            "mcke_sm100_last_error_string": (ctypes.c_char_p, []),
            "mcke_sm100_check_device_errors": (i32, [vp]),
            "mcke_sm100_watchdog_selftest": (i32, [vp]),
            "mcke_sm100_set_programmatic_launch": (i32, [i32]),
            "mcke_sm100_vector_add_f32": (i32, [vp, vp, vp, sz, vp]),
            "mcke_sm100_peak_triad_f32": (i32, [vp, vp, vp, f32, i64, vp]),
            "mcke_sm100_peak_copy_f32": (i32, [vp, vp, i64, vp]),
            "mcke_sm100_peak_fma_threads": (i64, []),
            "mcke_sm100_peak_fma_f32": (i32, [vp, vp, i64, i32, vp]),
            "mcke_sm100_peak_mma_ctas": (i64, []),
            "mcke_sm100_peak_mma_flops": (ctypes.c_double, [i64, i32]),
            "mcke_sm100_peak_mma_bf16": (i32, [i64, i32, vp]),
            "mcke_sm100_bias_act_f32": (i32, [vp, vp, vp, i64, i64, i32, i32, i32, vp]),
            "mcke_sm100_bias_act_f32_group": (i32, [vp, i32, i32, vp]),
            "mcke_sm100_bias_add_f32": (i32, [vp, vp, vp, i64, i64, i32, vp]),
            "mcke_sm100_activation_f32": (i32, [vp, vp, i64, i32, i32, vp]),
            "mcke_sm100_bias_act_bf16": (i32, [vp, vp, vp, i64, i64, i32, vp]),
            "mcke_sm100_softmax_f32": (i32, [vp, vp, i64, i64, i32, vp]),
            "mcke_sm100_reduce_row_workspace_bytes": (sz, [i64, i64, i32]),
            "mcke_sm100_reduce_row_f32": (i32, [vp, vp, i64, i64, i32, i32, vp, sz, vp]),
            "mcke_sm100_reduce_full_workspace_bytes": (sz, [i64]),
            "mcke_sm100_reduce_full_f32": (i32, [vp, i64, vp, vp, sz, vp]),
            "mcke_sm100_reduce_full_f32_ex": (i32, [vp, i64, vp, vp, sz, ctypes.c_uint, vp]),
            "mcke_sm100_reduce_full_partial_f32": (i32, [vp, i64, i64, vp, vp, sz, vp]),
            "mcke_sm100_reduce_combine": (i32, [vp, i64, vp, vp]),
            "mcke_sm100_reduce_p2p_buffer_bytes": (sz, [i32]),
            "mcke_sm100_reduce_full_p2p_f32": (i32, [vp, i64, i64, vp, i32, i32, ctypes.c_uint64, vp, vp]),
            "mcke_sm100_reduce_full_p2p_f32_ex": (i32, [vp, i64, i64, vp, i32, i32, ctypes.c_uint64, vp,
                                                        ctypes.c_uint, vp]),
            "mcke_sm100_reduce_full_p2p_f32_timeline": (i32, [vp, i64, i64, vp, i32, i32, ctypes.c_uint64, vp, vp,
                                                              vp]),
            "mcke_sm100_ipc_buffer_create": (i32, [sz, ctypes.POINTER(vp), vp]),
            "mcke_sm100_ipc_buffer_open": (i32, [vp, ctypes.POINTER(vp)]),
            "mcke_sm100_ipc_buffer_close": (i32, [vp, i32]),
            "mcke_sm100_gemm_f32": (i32, [vp, vp, vp, i64, i64, i64, f32, f32, i32, vp]),
            "mcke_sm100_gemm_f32_tc_workspace_bytes": (sz, [i64, i64, i64]),
            "mcke_sm100_gemm_f32_tc": (i32, [vp, vp, vp, i64, i64, i64, f32, f32, vp, i32, vp, sz, vp]),
            "mcke_sm100_gemm_bf16": (i32, [vp, vp, vp, i64, i64, i64, f32, f32, i32, vp]),
            "mcke_sm100_gemm_bf16_ex": (i32, [vp, vp, vp, i32, i64, i64, i64, f32, f32, vp, i32, i32, vp]),
            "mcke_sm100_gemm_kernel_attrs": (i32, [i32, i32, vp]),
            "mcke_sm100_gemm_plan": (i32, [i64, i64, i64, i32, i32, i32, vp]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(l, name)
            fn.restype, fn.argtypes = res, args
        _lib = l
    return _lib


def set_programmatic_launch(enable: bool) -> bool:
    """Launch this library's kernels with programmatic dependent launch (the
    default) or plainly; returns the previous setting.  Results are the same."""
    return bool(lib().mcke_sm100_set_programmatic_launch(1 if enable else 0))


def _check(rc: int) -> None:
    if rc != OK:
        raise MckeError(rc, lib().mcke_sm100_last_error_string().decode())


def _ptr(t) -> int | None:
    if t is None:
        return None
    return t.data_ptr()


def _stream(t: torch.Tensor | None, stream) -> int | None:
    if stream is not None:
        return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)
    dev = t.device if t is not None else torch.device("cuda")
    return torch.cuda.current_stream(dev).cuda_stream


def _need(t: torch.Tensor, dtype, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _act(a) -> int:
    return ACT[a] if isinstance(a, str) else int(a)


# ---- vector add ------------------------------------------------------------------

def vector_add(a, b, out=None, stream=None):
    """out = a + b (float32), the toolchain smoke kernel."""
    _need(a, torch.float32, "a"); _need(b, torch.float32, "b")
    out = torch.empty_like(a) if out is None else out
    _check(lib().mcke_sm100_vector_add_f32(_ptr(a), _ptr(b), _ptr(out), a.numel(), _stream(a, stream)))
    return out


# ---- roofline denominators ---------------------------------------------------

PEAK_FMA_FLOP_PER_THREAD_STEP = 16  # 8 chains x (multiply + add)


def peak_triad(a, b, c, scalar: float = 3.0, stream=None):
    """a = b + scalar * c (float32, 12 bytes moved per element)."""
    for t, nm in ((a, "a"), (b, "b"), (c, "c")):
        _need(t, torch.float32, nm)
    _check(lib().mcke_sm100_peak_triad_f32(_ptr(a), _ptr(b), _ptr(c), float(scalar), a.numel(), _stream(a, stream)))
    return a


def peak_copy(a, b, stream=None):
    """a = b (float32, 8 bytes moved per element)."""
    _need(a, torch.float32, "a"); _need(b, torch.float32, "b")
    _check(lib().mcke_sm100_peak_copy_f32(_ptr(a), _ptr(b), a.numel(), _stream(a, stream)))
    return a


def peak_fma_threads() -> int:
    return int(lib().mcke_sm100_peak_fma_threads())


def peak_fma(seed, out, iters: int, stream=None):
    """FFMA probe: PEAK_FMA_FLOP_PER_THREAD_STEP * seed.numel() * iters flop."""
    _need(seed, torch.float32, "seed"); _need(out, torch.float32, "out")
    _check(lib().mcke_sm100_peak_fma_f32(_ptr(seed), _ptr(out), seed.numel(), int(iters), _stream(seed, stream)))
    return out


def peak_mma_ctas() -> int:
    return lib().mcke_sm100_peak_mma_ctas()


def peak_mma_flops(ctas: int, iters: int) -> float:
    return lib().mcke_sm100_peak_mma_flops(int(ctas), int(iters))


def peak_mma(ctas: int, iters: int, stream=None):
    """The tcgen05 bf16 probe (mcke_sm100_peak_mma_bf16) on the current stream."""
    _check(lib().mcke_sm100_peak_mma_bf16(int(ctas), int(iters), _stream(None, stream)))


# ---- bias + activation -------------------------------------------------------

class BiasActJob(ctypes.Structure):
    """mcke_bias_act_job: one job of mcke_sm100_bias_act_f32_group."""
    _fields_ = [("x", ctypes.c_void_p), ("bias", ctypes.c_void_p), ("y", ctypes.c_void_p),
                ("rows", ctypes.c_int64), ("cols", ctypes.c_int64)]


BIAS_ACT_GROUP_MAX = 16  # MCKE_BIAS_ACT_GROUP_MAX


def bias_act_group(jobs, act="gelu_tanh", stream=None):
    """Independent float32 y = act(x + bias) jobs in one launch
    (mcke_sm100_bias_act_f32_group); ``jobs``: (x [rows, cols], bias [cols],
    y [rows, cols]) triples with cols % 512 == 0.  Returns the outputs."""
    arr = (BiasActJob * max(len(jobs), 1))()
    for k, (x, b, y) in enumerate(jobs):
        _need(x, torch.float32, "x"); _need(b, torch.float32, "bias"); _need(y, torch.float32, "y")
        arr[k] = BiasActJob(_ptr(x), _ptr(b), _ptr(y), x.shape[0], x.shape[1])
    dev_t = jobs[0][0] if jobs else None
    _check(lib().mcke_sm100_bias_act_f32_group(ctypes.cast(arr, ctypes.c_void_p), len(jobs), _act(act),
                                               _stream(dev_t, stream) if dev_t is not None else None))
    return [y for _, _, y in jobs]


def bias_act(x, bias, act="gelu_tanh", vector_width: int = 4, out=None, max_row_blocks: int = 0,
             stream=None):
    """y = act(x + bias) over the last dim, x [rows, cols] float32 or bfloat16."""
    rows, cols = (x.shape[0], x.shape[1]) if x.dim() == 2 else (x.numel() // x.shape[-1], x.shape[-1])
    y = torch.empty_like(x) if out is None else out
    _need(bias, torch.float32, "bias")
    if x.dtype == torch.bfloat16:
        _need(x, torch.bfloat16, "x"); _need(y, torch.bfloat16, "out")
        _check(lib().mcke_sm100_bias_act_bf16(_ptr(x), _ptr(bias), _ptr(y), rows, cols, _act(act),
                                              _stream(x, stream)))
    else:
        _need(x, torch.float32, "x"); _need(y, torch.float32, "out")
        _check(lib().mcke_sm100_bias_act_f32(_ptr(x), _ptr(bias), _ptr(y), rows, cols, _act(act),
                                             vector_width, max_row_blocks, _stream(x, stream)))
    return y


def bias_add(x, bias, vector_width: int = 4, out=None, stream=None):
    rows, cols = x.shape
    y = torch.empty_like(x) if out is None else out
    _check(lib().mcke_sm100_bias_add_f32(_ptr(x), _ptr(bias), _ptr(y), rows, cols, vector_width,
                                         _stream(x, stream)))
    return y


def activation(x, act="gelu_tanh", vector_width: int = 4, out=None, stream=None):
    y = torch.empty_like(x) if out is None else out
    _need(x, torch.float32, "x")
    _check(lib().mcke_sm100_activation_f32(_ptr(x), _ptr(y), x.numel(), _act(act), vector_width,
                                           _stream(x, stream)))
    return y


# ---- softmax -------------------------------------------------------------------

def softmax(x, variant="online", out=None, stream=None):
    _need(x, torch.float32, "x")
    rows, cols = x.shape
    y = torch.empty_like(x) if out is None else out
    v = SOFTMAX_VARIANT[variant] if isinstance(variant, str) else int(variant)
    _check(lib().mcke_sm100_softmax_f32(_ptr(x), _ptr(y), rows, cols, v, _stream(x, stream)))
    return y


# ---- reductions ----------------------------------------------------------------

def reduce_full_workspace_bytes(n: int) -> int:
    return lib().mcke_sm100_reduce_full_workspace_bytes(n)


REDUCE_EARLY_READ = 1  # MCKE_REDUCE_EARLY_READ


def reduce_full(x, out=None, workspace=None, stream=None, early_read: bool = False):
    """sum/max/argmax of a float32 vector; returns a 16-byte uint8 device tensor
    holding one mcke_reduce_result (decode with :func:`decode_result`).
    ``early_read``: the caller guarantees that ``x`` is not written by the
    kernel enqueued just before on the stream (MCKE_REDUCE_EARLY_READ), so
    back-to-back calls overlap; same result."""
    _need(x, torch.float32, "x")
    n = x.numel()
    dev = x.device
    if out is None:
        out = torch.empty(RESULT_BYTES, dtype=torch.uint8, device=dev)
    need = reduce_full_workspace_bytes(n)
    if workspace is None:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=dev)
    if early_read:
        _check(lib().mcke_sm100_reduce_full_f32_ex(_ptr(x), n, _ptr(out), _ptr(workspace), workspace.numel(),
                                                   REDUCE_EARLY_READ, _stream(x, stream)))
    else:
        _check(lib().mcke_sm100_reduce_full_f32(_ptr(x), n, _ptr(out), _ptr(workspace),
                                                workspace.numel(), _stream(x, stream)))
    return out


def reduce_full_partial(x, index_base: int, out=None, workspace=None, stream=None):
    _need(x, torch.float32, "x")
    n = x.numel()
    if out is None:
        out = torch.empty(PARTIAL_BYTES, dtype=torch.uint8, device=x.device)
    need = reduce_full_workspace_bytes(n)
    if workspace is None:
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=x.device)
    _check(lib().mcke_sm100_reduce_full_partial_f32(_ptr(x), n, index_base, _ptr(out),
                                                    _ptr(workspace), workspace.numel(),
                                                    _stream(x, stream)))
    return out


def reduce_combine(partials, count: int, out=None, stream=None):
    if out is None:
        out = torch.empty(RESULT_BYTES, dtype=torch.uint8, device=partials.device)
    _check(lib().mcke_sm100_reduce_combine(_ptr(partials), count, _ptr(out), _stream(partials, stream)))
    return out


def reduce_full_p2p(x, index_base: int, peer_table, world: int, rank: int, epoch: int, out=None, stream=None,
                    early_read: bool = False):
    """One rank's step of a sharded full reduce with the peer-to-peer combine
    (mcke_sm100_reduce_full_p2p_f32).  ``peer_table``: int64 CUDA tensor of the
    ranks' exchange-buffer addresses as mapped in this process; see
    :class:`mcke.shard.P2PExchange`, which owns the buffers and the epochs.
    ``early_read`` as for :func:`reduce_full`."""
    _need(x, torch.float32, "x")
    if out is None:
        out = torch.empty(RESULT_BYTES, dtype=torch.uint8, device=x.device)
    if early_read:
        _check(lib().mcke_sm100_reduce_full_p2p_f32_ex(_ptr(x), x.numel(), index_base, _ptr(peer_table), world,
                                                       rank, epoch, _ptr(out), REDUCE_EARLY_READ,
                                                       _stream(x, stream)))
    else:
        _check(lib().mcke_sm100_reduce_full_p2p_f32(_ptr(x), x.numel(), index_base, _ptr(peer_table), world,
                                                    rank, epoch, _ptr(out), _stream(x, stream)))
    return out


TIMELINE_WORDS = 8
TIMELINE_PHASES = ("first_entry", "first_start", "last_start", "first_done", "last_done", "folded", "exchanged",
                   "counted")


def timeline_buffer(steps: int, device) -> "torch.Tensor":
    """int64 [steps, 8] stamps initialised as mcke_sm100_reduce_full_p2p_f32_timeline wants."""
    t = torch.zeros((steps, TIMELINE_WORDS), dtype=torch.int64, device=device)
    t[:, [0, 1, 3]] = -1  # UINT64_MAX
    return t


def reduce_full_p2p_timeline(x, index_base: int, peer_table, world: int, rank: int, epoch: int, stamps,
                             out=None, stream=None):
    """reduce_full_p2p that also records its phase times into ``stamps`` (one
    row of :func:`timeline_buffer`)."""
    _need(x, torch.float32, "x")
    if out is None:
        out = torch.empty(RESULT_BYTES, dtype=torch.uint8, device=x.device)
    _check(lib().mcke_sm100_reduce_full_p2p_f32_timeline(_ptr(x), x.numel(), index_base, _ptr(peer_table), world,
                                                         rank, epoch, _ptr(out), _ptr(stamps), _stream(x, stream)))
    return out


def ipc_buffer_create(nbytes: int) -> tuple[int, bytes]:
    """cudaMalloc + zero + CUDA IPC handle on the current device: (address, 64-byte handle)."""
    ptr = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(64)
    _check(lib().mcke_sm100_ipc_buffer_create(nbytes, ctypes.byref(ptr), handle))
    return ptr.value, handle.raw


def ipc_buffer_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    _check(lib().mcke_sm100_ipc_buffer_open(ctypes.create_string_buffer(bytes(handle), 64), ctypes.byref(ptr)))
    return ptr.value


def ipc_buffer_close(ptr: int, opened: bool) -> None:
    _check(lib().mcke_sm100_ipc_buffer_close(ptr, 1 if opened else 0))


def decode_result(buf) -> tuple[float, float, int]:
    """(sum, max, argmax) from an mcke_reduce_result (device or host bytes)."""
    raw = bytes(buf.cpu().numpy().tobytes()) if hasattr(buf, "cpu") else bytes(buf)
    s, m, i = struct.unpack("<ffq", raw[:16])
    return s, m, i


def decode_partial(buf) -> tuple[float, float, int]:
    raw = bytes(buf.cpu().numpy().tobytes()) if hasattr(buf, "cpu") else bytes(buf)
    s, m, _, i = struct.unpack("<dfiq", raw[:24])
    return s, m, i


def reduce_row_workspace_bytes(rows: int, cols: int, variant="warp_shuffle") -> int:
    v = REDUCE_VARIANT[variant] if isinstance(variant, str) else int(variant)
    return lib().mcke_sm100_reduce_row_workspace_bytes(rows, cols, v)


def reduce_row(x, kind="sum", variant="warp_shuffle", out=None, workspace=None, stream=None):
    _need(x, torch.float32, "x")
    rows, cols = x.shape
    if out is None:
        out = torch.empty(rows, dtype=torch.float32, device=x.device)
    v = REDUCE_VARIANT[variant] if isinstance(variant, str) else int(variant)
    k = REDUCE_KIND[kind] if isinstance(kind, str) else int(kind)
    if workspace is None and v == 2:
        need = reduce_row_workspace_bytes(rows, cols, v)
        workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=x.device)
    wsz = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib().mcke_sm100_reduce_row_f32(_ptr(x), _ptr(out), rows, cols, k, v, _ptr(workspace),
                                           wsz, _stream(x, stream)))
    return out


# ---- GEMM ------------------------------------------------------------------------

def gemm(a, b, c=None, alpha: float = 1.0, beta: float = 0.0, variant="auto", bias=None,
         act="none", out_dtype=None, stream=None):
    """C = act(alpha * A @ B + beta * C + bias); A, B float32 or bfloat16 (row-major)."""
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    v = GEMM_VARIANT[variant] if isinstance(variant, str) else int(variant)
    s = _stream(a, stream)
    if a.dtype == torch.float32:
        _need(a, torch.float32, "a"); _need(b, torch.float32, "b")
        if bias is not None or _act(act) != 0:
            raise ValueError("bias/activation epilogues are offered on the bf16 entry point")
        if c is None:
            c = torch.zeros((m, n), dtype=torch.float32, device=a.device)
        _need(c, torch.float32, "c")
        _check(lib().mcke_sm100_gemm_f32(_ptr(a), _ptr(b), _ptr(c), m, n, k, alpha, beta, v, s))
        return c
    _need(a, torch.bfloat16, "a"); _need(b, torch.bfloat16, "b")
    odt = out_dtype or (c.dtype if c is not None else torch.float32)
    if c is None:
        c = torch.zeros((m, n), dtype=odt, device=a.device)
    if bias is None and _act(act) == 0 and odt == torch.float32:
        _check(lib().mcke_sm100_gemm_bf16(_ptr(a), _ptr(b), _ptr(c), m, n, k, alpha, beta, v, s))
    else:
        if bias is not None:
            _need(bias, torch.float32, "bias")
        _check(lib().mcke_sm100_gemm_bf16_ex(_ptr(a), _ptr(b), _ptr(c),
                                             DTYPE["bf16" if odt == torch.bfloat16 else "f32"],
                                             m, n, k, alpha, beta, _ptr(bias), _act(act), v, s))
    return c


def gemm_f32_tc_workspace_bytes(m: int, n: int, k: int) -> int:
    return lib().mcke_sm100_gemm_f32_tc_workspace_bytes(m, n, k)


def gemm_f32_tc(a, b, c=None, alpha: float = 1.0, beta: float = 0.0, bias=None, act="none", workspace=None,
                stream=None, in_kernel_split: bool = False):
    """float32 C = act(alpha * A @ B + beta * C + bias) on the tensor cores
    (3xTF32, mcke_sm100_gemm_f32_tc); ``workspace`` holds the hi/lo split of A
    and B (allocated here when not given), or, with ``in_kernel_split``, no
    workspace is passed and the GEMM kernel splits its tiles itself."""
    _need(a, torch.float32, "a"); _need(b, torch.float32, "b")
    m, k = a.shape
    k2, n = b.shape
    if k != k2:
        raise ValueError("inner dimensions differ")
    if c is None:
        c = torch.zeros((m, n), dtype=torch.float32, device=a.device)
    _need(c, torch.float32, "c")
    if bias is not None:
        _need(bias, torch.float32, "bias")
    if in_kernel_split:
        _check(lib().mcke_sm100_gemm_f32_tc(_ptr(a), _ptr(b), _ptr(c), m, n, k, alpha, beta, _ptr(bias), _act(act),
                                            None, 0, _stream(a, stream)))
        return c
    need = gemm_f32_tc_workspace_bytes(m, n, k)
    if workspace is None:
        workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=a.device)
    _check(lib().mcke_sm100_gemm_f32_tc(_ptr(a), _ptr(b), _ptr(c), m, n, k, alpha, beta, _ptr(bias), _act(act),
                                        _ptr(workspace), workspace.numel(), _stream(a, stream)))
    return c


class GemmAttrs(ctypes.Structure):
    _fields_ = [("regs_per_thread", ctypes.c_int), ("static_smem_bytes", ctypes.c_size_t),
                ("dynamic_smem_bytes", ctypes.c_size_t), ("local_bytes", ctypes.c_size_t),
                ("threads_per_block", ctypes.c_int), ("max_blocks_per_sm_api", ctypes.c_int)]


def gemm_kernel_attrs(variant="auto", dtype="bf16") -> dict:
    out = GemmAttrs()
    v = GEMM_VARIANT[variant] if isinstance(variant, str) else int(variant)
    _check(lib().mcke_sm100_gemm_kernel_attrs(v, DTYPE[dtype], ctypes.byref(out)))
    return {f: getattr(out, f) for f, _ in GemmAttrs._fields_}


class GemmPlan(ctypes.Structure):
    _fields_ = [("kernel", ctypes.c_int), ("tile_m", ctypes.c_int), ("tile_n", ctypes.c_int),
                ("tiles", ctypes.c_int64), ("ctas", ctypes.c_int64), ("split_dp_tiles", ctypes.c_int),
                ("split_kblocks", ctypes.c_int)]


def gemm_plan(m: int, n: int, k: int, variant="auto", out_dtype="f32", sm_count: int = 148) -> dict:
    """The schedule mcke_sm100_gemm_bf16_ex takes for this shape (host arithmetic
    only: aligned operands and beta == 0 assumed; no GPU needed)."""
    out = GemmPlan()
    v = GEMM_VARIANT[variant] if isinstance(variant, str) else int(variant)
    _check(lib().mcke_sm100_gemm_plan(int(m), int(n), int(k), v, DTYPE[out_dtype], int(sm_count), ctypes.byref(out)))
    return {f: getattr(out, f) for f, _ in GemmPlan._fields_}


def check_device_errors(stream=None) -> None:
    _check(lib().mcke_sm100_check_device_errors(_stream(None, stream)))
