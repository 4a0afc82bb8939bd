"""numpy-facing wrappers over the two CPU checker libraries (test infrastructure).

Every function takes and returns numpy arrays and forwards to either the C
restatement (``impl="port"``, the default) or the compiled reference
(``impl="reference"``).  Function names follow the reference's
tests/reference.hpp; each C symbol cites the line it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np

__all__ = [
    "ACT", "REDUCE", "build", "have_reference", "lib", "fill_random", "fill_normal",
    "bias_act", "row_reduce", "row_softmax", "gemm", "full_reduce", "round_bf16", "to_bf16",
    "bf16_to_f32", "tol_gemm", "abs_tol_gemm", "compare", "spot_check_gemm", "gelu_tanh",
    "gelu_erf", "parallel_rows", "softmax_config_input", "ORACLE_DIR",
]

ORACLE_DIR = os.path.dirname(os.path.abspath(__file__))
_PORT_SO = os.path.join(ORACLE_DIR, "_build", "libmcke_oracle.so")
_REF_SO = os.path.join(ORACLE_DIR, "_ref", "libmcke_ref.so")

ACT = {"none": 0, "relu": 1, "gelu_erf": 2, "gelu_tanh": 3}
REDUCE = {"sum": 0, "max": 1, "mean": 2}

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_dblp = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_int64)
_szp = ctypes.POINTER(ctypes.c_size_t)
_intp = ctypes.POINTER(ctypes.c_int)
_i64 = ctypes.c_int64
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t

_lock = threading.Lock()
_libs: dict[str, ctypes.CDLL] = {}


def build(force: bool = False) -> None:
    """Run oracle/Makefile (the port always; the reference when its tree exists)."""
    if force or not os.path.exists(_PORT_SO) or not os.path.exists(_REF_SO):
        subprocess.run(["make", "-s", "-C", ORACLE_DIR], check=True)


def _declare(l: ctypes.CDLL, prefix: str) -> None:
    def sig(name, res, args):
        fn = getattr(l, prefix + name)
        fn.restype = res
        fn.argtypes = args

    sig("fill_random", None, [_f32p, _sz, _u64, ctypes.c_float, ctypes.c_float])
    sig("gelu_erf", ctypes.c_double, [ctypes.c_double])
    sig("gelu_tanh", ctypes.c_double, [ctypes.c_double])
    sig("bias_act", None, [_f32p, _f32p, _f32p, _i64, _i64, ctypes.c_int])
    sig("row_reduce", None, [_f32p, _f32p, _i64, _i64, ctypes.c_int])
    sig("row_softmax", None, [_f32p, _f32p, _i64, _i64])
    sig("gemm", None, [_f32p, _f32p, _f32p, _i64, _i64, _i64, ctypes.c_float, ctypes.c_float])
    sig("compare", _sz, [_f32p, _f32p, _sz, ctypes.c_double, ctypes.c_double, _dblp, _dblp,
                         _intp, _intp])
    sig("tol_gemm", ctypes.c_double, [_i64])
    sig("abs_tol_gemm", ctypes.c_double, [_i64, ctypes.c_double])
    sig("spot_check_gemm", _sz, [_f32p, _f32p, _f32p, _i64, _i64, _i64, ctypes.c_float, _sz,
                                 _u64, ctypes.c_double, ctypes.c_double, _szp, _dblp, _dblp])
    if prefix == "oracle_":
        sig("fill_normal", None, [_f32p, _sz, _u64, ctypes.c_float, ctypes.c_float])
        sig("full_reduce", None, [_f32p, _i64, _i64, _dblp, _f32p, _i64p])
        sig("round_bf16", None, [_f32p, _f32p, _sz])
        sig("to_bf16", None, [_f32p, _u16p, _sz])
        sig("mt64_next", _u64, [ctypes.c_void_p])
        sig("mt64_seed", None, [ctypes.c_void_p, _u64])


def have_reference() -> bool:
    return os.path.exists(_REF_SO)


def lib(impl: str = "port") -> ctypes.CDLL:
    """The loaded checker library: ``port`` (C restatement) or ``reference``."""
    with _lock:
        if impl not in _libs:
            path = _PORT_SO if impl == "port" else _REF_SO
            if not os.path.exists(path):
                if impl == "reference":
                    raise FileNotFoundError(
                        "oracle/_ref/libmcke_ref.so is absent: the reference tree was not "
                        "present when oracle/Makefile ran")
                subprocess.run(["make", "-s", "-C", ORACLE_DIR, "oracle"], check=True)
            l = ctypes.CDLL(path)
            _declare(l, "oracle_" if impl == "port" else "ref_")
            _libs[impl] = l
        return _libs[impl]


def _fn(impl: str, name: str):
    l = lib(impl)
    return getattr(l, ("oracle_" if impl == "port" else "ref_") + name)


def _p(a: np.ndarray, ptr=_f32p):
    return a.ctypes.data_as(ptr)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def fill_random(n: int, seed: int, lo: float = -1.0, hi: float = 1.0, impl: str = "port"):
    """tests/reference.hpp:101 -- mt19937_64, top 24 bits, scaled into [lo, hi]."""
    out = np.empty(int(n), dtype=np.float32)
    _fn(impl, "fill_random")(_p(out), out.size, seed, lo, hi)
    return out


def fill_normal(n: int, seed: int, mean: float = 0.0, stddev: float = 1.0):
    """Builder convention (no reference counterpart): Box-Muller over the same engine."""
    out = np.empty(int(n), dtype=np.float32)
    _fn("port", "fill_normal")(_p(out), out.size, seed, mean, stddev)
    return out


def softmax_config_input(rows: int, cols: int, seed: int, shift_every: int = 64,
                         shift: float = 80.0, stddev: float = 4.0):
    """Config-2 style logits: N(0, stddev^2), rows r % shift_every == 0 shifted by +shift."""
    x = fill_normal(rows * cols, seed, 0.0, stddev).reshape(rows, cols)
    x[::shift_every] += np.float32(shift)
    return x


def gelu_tanh(x: float, impl: str = "port") -> float:
    return _fn(impl, "gelu_tanh")(x)


def gelu_erf(x: float, impl: str = "port") -> float:
    return _fn(impl, "gelu_erf")(x)


def _into(out, shape) -> np.ndarray:
    """`out` if given (C-contiguous float32 of `shape`, written in place), else a new array."""
    if out is None:
        return np.empty(shape, dtype=np.float32)
    assert out.dtype == np.float32 and out.flags.c_contiguous and out.shape == tuple(shape)
    return out


def bias_act(x, bias, act: str | int = "gelu_tanh", impl: str = "port", out=None):
    """tests/reference.hpp:143 -- y = act(x + bias[col]) in double, stored float."""
    x = _f32(x)
    bias = _f32(bias)
    rows, cols = x.shape
    y = _into(out, x.shape)
    a = ACT[act] if isinstance(act, str) else int(act)
    _fn(impl, "bias_act")(_p(x), _p(bias), _p(y), rows, cols, a)
    return y


def row_reduce(x, kind: str | int = "sum", impl: str = "port", out=None):
    """tests/reference.hpp:154 -- per-row sum/max/mean in double, stored float."""
    x = _f32(x)
    rows, cols = x.shape
    out = _into(out, (rows,))
    k = REDUCE[kind] if isinstance(kind, str) else int(kind)
    _fn(impl, "row_reduce")(_p(x), _p(out), rows, cols, k)
    return out


def row_softmax(x, impl: str = "port", out=None):
    """tests/reference.hpp:175 -- max-subtracted softmax over the last dim."""
    x = _f32(x)
    rows, cols = x.shape
    y = _into(out, x.shape)
    _fn(impl, "row_softmax")(_p(x), _p(y), rows, cols)
    return y


def gemm(a, b, c=None, alpha: float = 1.0, beta: float = 0.0, impl: str = "port", out=None):
    """tests/reference.hpp:199 -- C = alpha*A@B + beta*C with double accumulation.
    With `out` (and no `c`) the product is written into `out`, whose current
    contents play C's role (the reference reads C even when beta is 0)."""
    a = _f32(a)
    b = _f32(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    if out is not None:
        assert c is None
        out = _into(out, (m, n))
    else:
        out = np.zeros((m, n), dtype=np.float32) if c is None else _f32(c).copy()
    _fn(impl, "gemm")(_p(a), _p(b), _p(out), m, n, k, alpha, beta)
    return out


def full_reduce(x, index_base: int = 0):
    """Full-vector (sum as double, max, argmax) -- the rows=1 case of
    tests/reference.hpp:154 plus an argmax (lowest index on ties; unpinned)."""
    x = _f32(x).ravel()
    s = ctypes.c_double()
    m = ctypes.c_float()
    i = ctypes.c_int64()
    _fn("port", "full_reduce")(_p(x), x.size, index_base, ctypes.byref(s), ctypes.byref(m),
                               ctypes.byref(i))
    return s.value, np.float32(m.value), i.value


def round_bf16(x):
    """Round-to-nearest-even to bfloat16, widened back to float32."""
    x = _f32(x)
    out = np.empty_like(x)
    _fn("port", "round_bf16")(_p(x), _p(out), x.size)
    return out


def to_bf16(x):
    """Round-to-nearest-even to bfloat16; returns the raw uint16 bit patterns."""
    x = _f32(x)
    out = np.empty(x.shape, dtype=np.uint16)
    _fn("port", "to_bf16")(_p(x), _p(out, _u16p), x.size)
    return out


def bf16_to_f32(h):
    h = np.ascontiguousarray(h, dtype=np.uint16)
    return (h.astype(np.uint32) << 16).view(np.float32)


def tol_gemm(k: int, impl: str = "port") -> float:
    return _fn(impl, "tol_gemm")(k)


def abs_tol_gemm(k: int, amax: float = 1.0, impl: str = "port") -> float:
    return _fn(impl, "abs_tol_gemm")(k, amax)


def compare(got, want, rel_tol: float, abs_tol: float = 1e-8, impl: str = "port"):
    """tests/reference.hpp:249 -- returns dict(mismatches, max_abs, max_rel, nan, inf)."""
    got = _f32(got).ravel()
    want = _f32(want).ravel()
    assert got.size == want.size
    ma, mr = ctypes.c_double(), ctypes.c_double()
    an, ai = ctypes.c_int(), ctypes.c_int()
    bad = _fn(impl, "compare")(_p(got), _p(want), got.size, rel_tol, abs_tol, ctypes.byref(ma),
                               ctypes.byref(mr), ctypes.byref(an), ctypes.byref(ai))
    return {"mismatches": int(bad), "max_abs": ma.value, "max_rel": mr.value,
            "nan": bool(an.value), "inf": bool(ai.value), "n": got.size}


def spot_check_gemm(a, b, got, alpha: float = 1.0, samples: int = 1024, seed: int = 0,
                    rel_tol: float | None = None, abs_tol: float | None = None,
                    impl: str = "port"):
    """tests/reference.hpp:401 -- recompute `samples` random C elements in double."""
    a = _f32(a)
    b = _f32(b)
    got = _f32(got)
    m, k = a.shape
    n = b.shape[1]
    rel = tol_gemm(k) if rel_tol is None else rel_tol
    ab = abs_tol_gemm(k) if abs_tol is None else abs_tol
    checked = ctypes.c_size_t()
    ma, mr = ctypes.c_double(), ctypes.c_double()
    bad = _fn(impl, "spot_check_gemm")(_p(a), _p(b), _p(got), m, n, k, alpha, samples, seed,
                                       rel, ab, ctypes.byref(checked), ctypes.byref(ma),
                                       ctypes.byref(mr))
    return {"mismatches": int(bad), "checked": checked.value, "max_abs": ma.value,
            "max_rel": mr.value}


def parallel_rows(fn, x: np.ndarray, y: np.ndarray, threads: int, *args):
    """Call a row-wise checker function on disjoint row blocks from `threads`
    threads (ctypes releases the GIL, so the calls run in parallel).  The
    arithmetic per row is unchanged; only the row ranges are split."""
    rows = x.shape[0]
    step = (rows + threads - 1) // threads
    chunks = [(r, min(rows, r + step)) for r in range(0, rows, step)]

    def work(rng):
        r0, r1 = rng
        fn(x[r0:r1], y[r0:r1], *args)

    with ThreadPoolExecutor(max_workers=threads) as ex:
        list(ex.map(work, chunks))
    return y
