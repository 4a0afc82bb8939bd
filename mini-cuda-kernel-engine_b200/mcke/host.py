"""Python binding of libmcke_host.so (include/mcke_host.h): Graph and
GraphExecutor of the C++ host layer.  Host arrays are numpy; the executor owns
its device memory (one arena per device) and its streams.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import MckeError, PKG_DIR  # noqa: F401

__all__ = ["Graph", "Executor", "MckeError", "lib"]

LIB_PATH = os.path.join(PKG_DIR, "lib", "libmcke_host.so")
DT = {"f32": 0, "bf16": 2, "u8": 4}
NP = {"f32": np.float32, "bf16": np.uint16, "u8": np.uint8}
PLACE = {"replicated": 0, "row_split": 1, "col_split": 2}
PLACE_NAME = {v: k for k, v in PLACE.items()}
ACT = {"none": 0, "relu": 1, "gelu_erf": 2, "gelu_tanh": 3}
GEMM_VARIANT_TILED_REGBLOCK = 2  # the reference's GemmParams default
GEMM_VARIANT_TCGEN05_TF32X3 = 9  # f32 operands on the tensor cores (3xTF32)
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is not built; run __graft_entry__.build()")
        l = ctypes.CDLL(LIB_PATH)
        vp, i32, u32, i64, sz, f32, cp = (ctypes.c_void_p, ctypes.c_int, ctypes.c_uint32, ctypes.c_int64,
                                          ctypes.c_size_t, ctypes.c_float, ctypes.c_char_p)
        u32p = ctypes.POINTER(ctypes.c_uint32)
        sigs = {
            "mcke_host_last_error_string": (cp, []),
            "mcke_graph_create": (vp, []),
            "mcke_graph_destroy": (None, [vp]),
            "mcke_graph_add_input": (i32, [vp, cp, ctypes.POINTER(ctypes.c_int64), i32, i32, i32, u32p]),
            "mcke_graph_add_gemm": (i32, [vp, cp, u32, u32, i64, f32, i32, i32, i32, u32p]),
            "mcke_graph_add_bias_act": (i32, [vp, cp, u32, u32, i32, i32, u32p]),
            "mcke_graph_add_softmax": (i32, [vp, cp, u32, i32, u32p]),
            "mcke_graph_add_reduce_row": (i32, [vp, cp, u32, i32, i32, u32p]),
            "mcke_graph_add_reduce_full": (i32, [vp, cp, u32, u32p]),
            "mcke_graph_mark_output": (i32, [vp, u32]),
            "mcke_graph_finalize": (i32, [vp]),
            "mcke_graph_roofline_ms": (i32, [vp, ctypes.c_double, ctypes.c_double, ctypes.POINTER(ctypes.c_double)]),
            "mcke_executor_create": (vp, [vp, ctypes.POINTER(ctypes.c_int), i32, i32]),
            "mcke_executor_create_ex": (vp, [vp, ctypes.POINTER(ctypes.c_int), i32, i32, ctypes.c_uint]),
            "mcke_executor_destroy": (None, [vp]),
            "mcke_executor_plan_dry": (i32, [vp]),
            "mcke_executor_plan": (i32, [vp]),
            "mcke_executor_set_input": (i32, [vp, u32, vp, sz]),
            "mcke_executor_run_async": (i32, [vp]),
            "mcke_executor_synchronize": (i32, [vp]),
            "mcke_executor_copy_output": (i32, [vp, u32, vp, sz]),
            "mcke_executor_describe": (i32, [vp, ctypes.c_char_p, sz]),
            "mcke_executor_placement": (i32, [vp, u32, ctypes.POINTER(ctypes.c_int)]),
            "mcke_executor_arena_bytes": (i32, [vp, i32, ctypes.POINTER(ctypes.c_size_t)]),
            "mcke_executor_num_events": (i32, [vp, ctypes.POINTER(ctypes.c_size_t)]),
            "mcke_executor_launch_items": (i32, [vp, ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_size_t)]),
            "mcke_executor_last_run_ms": (i32, [vp, ctypes.POINTER(ctypes.c_float)]),
            "mcke_executor_create_policy": (vp, [vp, ctypes.POINTER(ctypes.c_int), i32, i32, ctypes.c_uint, i32, i32]),
            "mcke_executor_validate_numerics": (i32, [vp, i32, ctypes.POINTER(ctypes.c_int),
                                                      ctypes.POINTER(ctypes.c_int), ctypes.c_char_p, sz]),
            "mcke_executor_alloc_stats": (i32, [vp, i32, ctypes.POINTER(AllocStats)]),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(l, name)
            fn.restype, fn.argtypes = res, args
        _lib = l
    return _lib


def _check(rc: int) -> None:
    if rc != 0:
        raise MckeError(rc, lib().mcke_host_last_error_string().decode())


class AllocStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint64) for n in ("alloc_calls", "free_calls", "raw_malloc_calls", "raw_free_calls",
                                               "bytes_reserved", "bytes_in_use", "bytes_requested",
                                               "peak_bytes_in_use")] + [("name", ctypes.c_char * 24)]


SCHEDULE = {"sequential": 0, "level_parallel": 1, "chain_greedy": 2, "level_grouped": 3}
MEMORY = {"alloc_per_tensor": 0, "reuse_same_stream": 2, "reuse_happens_before": 3}


class Graph:
    """mcke::Graph: add_input / ops / mark_output / finalize."""

    def __init__(self):
        self._h = lib().mcke_graph_create()
        self.desc: dict[int, tuple[tuple[int, ...], str]] = {}

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            try:
                _lib.mcke_graph_destroy(h)
            except Exception:  # interpreter teardown
                pass

    def _out(self, fn, *args) -> int:
        out = ctypes.c_uint32()
        _check(fn(self._h, *args, ctypes.byref(out)))
        return out.value

    def input(self, name: str, shape, dtype: str = "f32", placement: str = "replicated") -> int:
        dims = (ctypes.c_int64 * len(shape))(*shape)
        t = self._out(lib().mcke_graph_add_input, name.encode(), dims, len(shape), DT[dtype], PLACE[placement])
        self.desc[t] = (tuple(shape), dtype)
        return t

    def gemm(self, a: int, b: int, bias: int | None = None, alpha: float = 1.0, act: str = "none",
             out_dtype: str = "f32", name: str = "gemm", variant: int = GEMM_VARIANT_TILED_REGBLOCK) -> int:
        t = self._out(lib().mcke_graph_add_gemm, name.encode(), a, b, -1 if bias is None else bias, alpha,
                      ACT[act], DT[out_dtype], variant)
        m, n = self.desc[a][0][0], self.desc[b][0][1]
        self.desc[t] = ((m, n), out_dtype if self.desc[a][1] == "bf16" else "f32")
        return t

    def bias_act(self, x: int, bias: int, act: str = "gelu_tanh", vector_width: int = 0,
                 name: str = "bias_act") -> int:
        t = self._out(lib().mcke_graph_add_bias_act, name.encode(), x, bias, ACT[act], vector_width)
        self.desc[t] = self.desc[x]
        return t

    def softmax(self, x: int, variant: int = 1, name: str = "softmax") -> int:
        t = self._out(lib().mcke_graph_add_softmax, name.encode(), x, variant)
        self.desc[t] = self.desc[x]
        return t

    def reduce_row(self, x: int, kind: int = 0, variant: int = 1, name: str = "reduce") -> int:
        t = self._out(lib().mcke_graph_add_reduce_row, name.encode(), x, kind, variant)
        shp = self.desc[x][0]
        self.desc[t] = ((shp[0],) if len(shp) > 1 else (1,), "f32")
        return t

    def reduce_full(self, x: int, name: str = "reduce_full") -> int:
        t = self._out(lib().mcke_graph_add_reduce_full, name.encode(), x)
        self.desc[t] = ((16,), "u8")
        return t

    def output(self, t: int) -> None:
        _check(lib().mcke_graph_mark_output(self._h, t))

    def finalize(self) -> None:
        _check(lib().mcke_graph_finalize(self._h))

    def roofline_ms(self, peak_tflops: float, peak_gbs: float) -> float:
        """Sum over nodes of max(flops / peak, bytes / bandwidth), in ms (the
        reference's cost-model lower bound of one sequential run)."""
        ms = ctypes.c_double()
        _check(lib().mcke_graph_roofline_ms(self._h, float(peak_tflops), float(peak_gbs), ctypes.byref(ms)))
        return ms.value


class Executor:
    """mcke::GraphExecutor over the given CUDA device ordinals."""

    def __init__(self, graph: Graph, devices=(0,), streams_per_device: int = 4, cuda_graph: bool = False,
                 poison: bool = False, nccl_exchange: bool = False, buddy: bool = False, validate: bool = False,
                 schedule: str = "chain_greedy", memory: str = "reuse_happens_before"):
        """buddy: each device's arena comes from a BuddyAllocator of that device
        (the reference's DeviceAllocator interface); validate: keep host copies of
        the inputs for validate_numerics()."""
        self.graph = graph
        devs = (ctypes.c_int * len(devices))(*devices)
        flags = ((1 if cuda_graph else 0) | (2 if poison else 0) | (4 if nccl_exchange else 0) |
                 (8 if buddy else 0) | (16 if validate else 0))
        self._h = lib().mcke_executor_create_policy(graph._h, devs, len(devices), streams_per_device, flags,
                                                    SCHEDULE[schedule], MEMORY[memory])
        if not self._h:
            raise MckeError(2, "mcke_executor_create failed")

    def validate_numerics(self, repeats: int = 3) -> dict:
        ok, n = ctypes.c_int(), ctypes.c_int()
        buf = ctypes.create_string_buffer(4096)
        _check(lib().mcke_executor_validate_numerics(self._h, repeats, ctypes.byref(ok), ctypes.byref(n), buf,
                                                     len(buf)))
        return {"passed": bool(ok.value), "configs": n.value, "detail": buf.value.decode()}

    def alloc_stats(self, device_index: int = 0) -> dict:
        st = AllocStats()
        _check(lib().mcke_executor_alloc_stats(self._h, device_index, ctypes.byref(st)))
        d = {n: getattr(st, n) for n, _ in AllocStats._fields_ if n != "name"}
        d["name"] = st.name.decode()
        return d

    def __del__(self):
        h, self._h = getattr(self, "_h", None), None
        if h and _lib is not None:
            try:
                _lib.mcke_executor_destroy(h)
            except Exception:  # interpreter teardown
                pass

    def plan_dry(self) -> None:
        _check(lib().mcke_executor_plan_dry(self._h))

    def plan(self) -> None:
        _check(lib().mcke_executor_plan(self._h))

    def set_input(self, t: int, arr: np.ndarray) -> None:
        arr = np.ascontiguousarray(arr)
        _check(lib().mcke_executor_set_input(self._h, t, arr.ctypes.data, arr.nbytes))

    def run(self) -> None:
        _check(lib().mcke_executor_run_async(self._h))

    def synchronize(self) -> None:
        _check(lib().mcke_executor_synchronize(self._h))

    def output(self, t: int) -> np.ndarray:
        shape, dt = self.graph.desc[t]
        out = np.empty(shape, dtype=NP[dt])
        _check(lib().mcke_executor_copy_output(self._h, t, out.ctypes.data, out.nbytes))
        return out

    def last_run_ms(self) -> float:
        ms = ctypes.c_float()
        _check(lib().mcke_executor_last_run_ms(self._h, ctypes.byref(ms)))
        return ms.value

    def describe(self) -> str:
        buf = ctypes.create_string_buffer(1 << 16)
        _check(lib().mcke_executor_describe(self._h, buf, len(buf)))
        return buf.value.decode()

    def placement(self, t: int) -> str:
        p = ctypes.c_int()
        _check(lib().mcke_executor_placement(self._h, t, ctypes.byref(p)))
        return PLACE_NAME[p.value]

    def arena_bytes(self, device_index: int = 0) -> int:
        b = ctypes.c_size_t()
        _check(lib().mcke_executor_arena_bytes(self._h, device_index, ctypes.byref(b)))
        return b.value

    def num_events(self) -> int:
        b = ctypes.c_size_t()
        _check(lib().mcke_executor_num_events(self._h, ctypes.byref(b)))
        return b.value

    def launch_items(self) -> tuple[int, int]:
        """(number of launch items, nodes in the largest) of the plan."""
        n, big = ctypes.c_size_t(), ctypes.c_size_t()
        _check(lib().mcke_executor_launch_items(self._h, ctypes.byref(n), ctypes.byref(big)))
        return n.value, big.value
