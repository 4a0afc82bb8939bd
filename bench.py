#!/usr/bin/env python3
"""bench.py -- throughput of the mcke sm_100a kernel path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mcke|reference] [--ops LIST]

N > 1 is launched by torchrun (one process per GPU, NCCL); rank 0 prints ONE
JSON line.

Headline (``value``): BASELINE config 2, row softmax fp32 over logits
[32768 x 1024] ~ N(0, 4^2) with every 64th row shifted by +80.  A step is one
softmax pass over the whole batch, inputs already resident in HBM.  Bytes per
step are algorithmic, 2 * 32768 * 1024 * 4 = 268,435,456 (one read of x, one
write of y).  The K timed steps run back to back between one pair of CUDA
events on the launching stream, on inputs larger than L2 that rotate over
three buffer sets; ``cold_step_ms`` beside it is one step timed alone after an
L2 flush (a 256 MiB write, then a 256 MiB read), which also carries the
event's own cost.  At N GPUs every rank processes its own full batch (weak
scaling) and ``value`` = N * bytes * K / (max over ranks of the timed span).

``e2e``: the same step through the public API with HOST buffers: the pinned
host logits are copied in, softmax runs, the probabilities are copied back,
all inside the timed region.

``ops``: the other BASELINE configs at their full sizes (bias+GELU fp32,
full reduce fp32 sum/max/argmax, bf16 and fp32 GEMM 8192^3), each as an
absolute number and a roofline fraction; at N > 1 these are sharded across
ranks over a fixed total (strong scaling): rows, contiguous ranges with one
NCCL all-gather of 24-byte partials, and output columns respectively.

``--impl reference`` times the reference's own CPU implementation
(tests/reference.hpp compiled into oracle/_ref; the C restatement if that
library is absent) on the host cores, on bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "mini-cuda-kernel-engine_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "GEMM TFLOP/s; softmax/reduce/bias-GELU GB/s as % of B200 peak at 1/2/4/8 GPU"
TF32_NOMINAL_TFLOPS = 1100.0  # dense tf32 tensor peak per B200 (nominal; no measured tf32 peak exists)
ROWS, COLS = 32768, 1024
SOFTMAX_BYTES = 2 * ROWS * COLS * 4
BIAS_ROWS, BIAS_COLS = 4096, 4096
BIAS_BYTES = (2 * BIAS_ROWS * BIAS_COLS + BIAS_COLS) * 4
REDUCE_N = 1 << 28
REDUCE_BYTES = REDUCE_N * 4
GEMM_N = 8192
GEMM_FLOPS = 2 * GEMM_N ** 3
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic() -> dict:
    """kernel -> {"bytes", "read", "write", "algorithmic", "note"} from one ncu
    capture each (profiles/traffic.json)."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f).get("kernels", {})
    return {}


def traffic_of(traffic: dict, kernel: str):
    e = traffic.get(kernel)
    return None if e is None else e["bytes"]


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi samples (200 ms) of this GPU while the timed work runs."""

    FIELDS = ("uuid,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, uuid: str | None):
        self.uuid = uuid
        self.proc = None
        self.path = os.path.join("/tmp", f"mcke_clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "samples_under_load": 0}
        if self.proc is None or not os.path.exists(self.path):
            out["note"] = "nvidia-smi unavailable"
            return out
        rows = []
        with open(self.path) as f:
            for ln in f:
                parts = [p.strip() for p in ln.split(",")]
                if len(parts) < 10:
                    continue
                if self.uuid and self.uuid not in parts[0]:
                    continue
                rows.append(parts)
        out["samples"] = len(rows)
        load = [r for r in rows if r[4].replace(".", "").isdigit() and float(r[4]) >= 50.0]
        out["samples_under_load"] = len(load)
        use = load or rows
        try:
            if use:
                out["sm_mhz"] = statistics.median(float(r[1]) for r in use)
                out["sm_max_mhz"] = max(float(r[2]) for r in use)
                out["power_w_max"] = max(float(r[3]) for r in use)
        except ValueError:
            pass
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for k, name in enumerate(names):
            if any(r[6 + k].lower().startswith("active") for r in use):
                out["reasons"].append(name)
        out["window"] = ("one sampler over the headline's timed steps, the e2e pipeline and every ops entry "
                         "(the headline's steps alone last less than the 200 ms sampling period); the median "
                         "under load is set by the longest entries, the GEMMs, which run at the power cap")
        if not load:
            out["note"] = "no sample caught the GPU busy (timed region shorter than the 200 ms sampling period)"
        return out


# --------------------------------------------------------------- helpers

class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init(self, torch, backend="nccl"):
        if self.world > 1:
            import datetime
            import torch.distributed as td
            td.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                  device_id=torch.device("cuda", self.local) if backend == "nccl" else None)
            self.pg = td

    def barrier(self, torch):
        if self.pg is not None:
            t = torch.zeros(1, device="cuda")
            self.pg.all_reduce(t)
            torch.cuda.synchronize()

    def max(self, torch, v: float) -> float:
        if self.pg is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def min(self, torch, v: float) -> float:
        return -self.max(torch, -v)

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def timed_steps(torch, dist, launch, steps: int, warmup: int, flush=None, per_launch_kernels=1):
    """Warm up, then time exactly `steps` launches, each bracketed by CUDA events on
    the current stream, with an L2 flush between steps outside the events.
    Returns (total_ms max over ranks, list of per-step ms on this rank)."""
    stream = torch.cuda.current_stream()
    for _ in range(warmup):  # warm-up steps are timed steps without the events
        if flush is not None:
            flush()
        launch()
    torch.cuda.synchronize()
    dist.barrier(torch)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for i in range(steps):
        if flush is not None:
            flush()
        ev[i][0].record(stream)
        launch()
        ev[i][1].record(stream)
    torch.cuda.synchronize()
    dist.barrier(torch)
    torch.cuda.synchronize()
    per = [a.elapsed_time(b) for a, b in ev]
    return dist.max(torch, sum(per)), per


def timed_back_to_back(torch, dist, launch, steps: int, warmup: int) -> float:
    """`warmup` untimed steps, then EXACTLY `steps` steps launched back to back
    between one pair of CUDA events on the current stream, with a barrier and a
    synchronize on both sides; launch(i) runs step i.  Returns the total device
    time in ms, max over ranks.  Recording an event before every kernel costs
    the next kernel ~4 us of device time on B200 (an empty kernel measured 6.1 us
    between events, 2.2 us per launch back to back), so memory-bound steps of a
    few tens of microseconds are timed this way, on inputs larger than L2."""
    stream = torch.cuda.current_stream()
    for i in range(warmup):
        launch(i)
    torch.cuda.synchronize()
    dist.barrier(torch)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(steps):
        launch(warmup + i)
    e1.record(stream)
    torch.cuda.synchronize()
    dist.barrier(torch)
    torch.cuda.synchronize()
    return dist.max(torch, e0.elapsed_time(e1))


def cold_step_ms(torch, dist, launch, flush, steps: int = 5) -> float:
    """Mean time of one step with L2 flushed first and events around the step
    alone (launch latency and the event cost included), max over ranks."""
    total, _ = timed_steps(torch, dist, launch, steps, 2, flush)
    return total / steps


# Inputs rotate over this many buffer sets in the back-to-back timing, so a
# step's input was last touched ROTATE - 1 steps (>= 256 MiB of traffic) earlier.
ROTATE = 3


# ------------------------------------------------------------ CPU baselines
#
# The reference's own CPU implementation of each op (tests/reference.hpp,
# compiled into oracle/_ref; the C restatement in oracle/ if that library is
# absent) timed on this host's cores.  Each op's function runs on disjoint row
# (or range) blocks, one block per thread, into preallocated outputs; one
# untimed pass comes first (page faults, caches, the thread pool), then passes
# until a time budget is spent.  The same code serves the cpu_baseline entries
# of this arm and the whole --impl reference arm, so the two agree.  Inputs
# are synthetic with each config's shapes (values do not change the timing);
# GEMM-shaped work is timed on a row slice and extrapolated linearly.

class CpuBaselines:
    def __init__(self, budget_s: float = 2.0):
        from concurrent.futures import ThreadPoolExecutor
        import oracle
        self.oracle = oracle
        self.impl = "reference" if oracle.have_reference() else "port"
        self.threads = max(1, min(os.cpu_count() or 1, 64))
        self.budget = budget_s
        self.pool = ThreadPoolExecutor(max_workers=self.threads)
        self.rng = np.random.default_rng(1234)

    def close(self):
        self.pool.shutdown()

    def _blocks(self, n: int) -> list[tuple[int, int]]:
        step = -(-n // self.threads)
        return [(i, min(n, i + step)) for i in range(0, n, step)]

    def _time(self, work, items) -> tuple[float, int]:
        items = list(items)
        list(self.pool.map(work, items))  # untimed first pass
        reps, total = 0, 0.0
        while reps < 2 or (total < self.budget and reps < 50):
            t0 = time.perf_counter()
            list(self.pool.map(work, items))
            total += time.perf_counter() - t0
            reps += 1
        # the same function on one item (one thread's share, the items are equal
        # in size) on this thread alone, best of two: the single-thread figure
        single = float("inf")
        for _ in range(2):
            t0 = time.perf_counter()
            work(items[0])
            single = min(single, time.perf_counter() - t0)
        self._last = (total / reps, len(items), single)
        return total / reps, reps

    def _entry(self, value: float, unit: str, sample: str) -> dict:
        sec, n_items, single = self._last
        one = value * sec / (n_items * single)  # work of one item / its single-thread time
        sig = lambda v: float(f"{v:.4g}")  # noqa: E731  (4 significant figures: GEMM rates are ~1e-3 TFLOP/s)
        return {"value": sig(value), "unit": unit, "cores": self.threads, "kind": self.impl,
                "sample": sample,
                "single_thread": {"value": sig(one), "unit": unit, "cores": 1,
                                  "sample": "one thread's share of the same pass, run alone on one thread"}}

    def _uniform(self, *shape) -> np.ndarray:
        return self.rng.random(shape, dtype=np.float32) * np.float32(2) - np.float32(1)

    def softmax(self, rows: int = ROWS, cols: int = COLS) -> dict:
        o = self.oracle
        x = o.softmax_config_input(rows, cols, seed=2)
        y = np.empty_like(x)
        sec, reps = self._time(lambda b: o.row_softmax(x[b[0]:b[1]], self.impl, out=y[b[0]:b[1]]),
                               self._blocks(rows))
        return self._entry(2 * rows * cols * 4 / sec / 1e9, "GB/s",
                           f"full {rows}x{cols} batch per pass, {reps} timed passes; reference_row_softmax "
                           f"(tests/reference.hpp:175) over disjoint row blocks on {self.threads} threads")

    def bias_gelu(self) -> dict:
        o = self.oracle
        x = o.fill_normal(BIAS_ROWS * BIAS_COLS, 0).reshape(BIAS_ROWS, BIAS_COLS)
        b = o.fill_random(BIAS_COLS, 1000)
        y = np.empty_like(x)
        sec, reps = self._time(lambda r: o.bias_act(x[r[0]:r[1]], b, "gelu_tanh", self.impl, out=y[r[0]:r[1]]),
                               self._blocks(BIAS_ROWS))
        return self._entry(BIAS_BYTES / sec / 1e9, "GB/s",
                           f"full {BIAS_ROWS}x{BIAS_COLS} batch per pass, {reps} timed passes; reference_bias_act "
                           f"(tests/reference.hpp:143) over disjoint row blocks on {self.threads} threads")

    def reduce_full(self) -> dict:
        # sum and max: reference_row_reduce with rows = 1 on each thread's
        # contiguous range (two passes, as two of the reference's ReduceOp
        # nodes would run); the reference has no argmax, so none is timed
        o = self.oracle
        n = 1 << 26
        x = self._uniform(n)
        outs = np.empty((self.threads, 2), np.float32)
        blocks = list(enumerate(self._blocks(n)))

        def work(item):
            i, (lo, hi) = item
            seg = x[lo:hi].reshape(1, hi - lo)
            o.row_reduce(seg, "sum", self.impl, out=outs[i, 0:1])
            o.row_reduce(seg, "max", self.impl, out=outs[i, 1:2])

        sec, reps = self._time(work, blocks)
        return self._entry(n * 4 / sec / 1e9, "GB/s",
                           f"2^26 of config 3's 2^28 floats per pass, {reps} timed passes; reference_row_reduce "
                           f"(tests/reference.hpp:154, rows = 1) for sum and for max over contiguous ranges on "
                           f"{self.threads} threads (no argmax: the reference has none)")

    def row_reduce(self) -> dict:
        o = self.oracle
        x = self._uniform(ROWS, COLS)
        y = np.empty(ROWS, np.float32)
        sec, reps = self._time(lambda r: o.row_reduce(x[r[0]:r[1]], "sum", self.impl, out=y[r[0]:r[1]]),
                               self._blocks(ROWS))
        return self._entry((ROWS * COLS * 4 + ROWS * 4) / sec / 1e9, "GB/s",
                           f"full {ROWS}x{COLS} batch per pass, {reps} timed passes; reference_row_reduce sum "
                           f"(tests/reference.hpp:154) over disjoint row blocks on {self.threads} threads")

    def gemm(self) -> dict:
        # one row of C per thread: reference_gemm's i-j-k loop with double
        # accumulation (tests/reference.hpp:199); the bf16 path's oracle is the
        # same loop on bf16-rounded inputs, so the one figure serves both
        o = self.oracle
        rows = self.threads
        a = self._uniform(rows, GEMM_N)
        b = self._uniform(GEMM_N, GEMM_N)
        c = np.zeros((rows, GEMM_N), np.float32)
        sec, reps = self._time(lambda i: o.gemm(a[i:i + 1], b, impl=self.impl, out=c[i:i + 1]), range(rows))
        return self._entry(2 * rows * GEMM_N * GEMM_N / sec / 1e12, "TFLOP/s",
                           f"{rows} of 8192 rows of C per pass ({reps} timed passes), extrapolated linearly to "
                           f"8192^3; reference_gemm on {self.threads} threads, one row each")

    def dag_branch(self) -> dict:
        # one config-5 branch, one token row per thread: GEMM1 -> +b1, GELU ->
        # GEMM2 -> +b2 -> softmax with the reference's functions (fp32: the
        # reference has no bf16), extrapolated to 8192 rows x 4 branches
        o = self.oracle
        d, f = 4096, 16384
        rows = self.threads
        x = self._uniform(rows, d)
        w1, w2 = self._uniform(d, f) * np.float32(0.02), self._uniform(f, d) * np.float32(0.02)
        b1, b2 = self._uniform(f), self._uniform(d)
        lin1, h = np.zeros((rows, f), np.float32), np.zeros((rows, f), np.float32)
        lin2, y, p = (np.zeros((rows, d), np.float32) for _ in range(3))

        def work(i):
            s = slice(i, i + 1)
            o.gemm(x[s], w1, impl=self.impl, out=lin1[s])
            o.bias_act(lin1[s], b1, "gelu_tanh", self.impl, out=h[s])
            o.gemm(h[s], w2, impl=self.impl, out=lin2[s])
            o.bias_act(lin2[s], b2, "none", self.impl, out=y[s])
            o.row_softmax(y[s], self.impl, out=p[s])

        sec, reps = self._time(work, range(rows))
        return self._entry(2 * 2 * rows * d * f / sec / 1e12, "TFLOP/s",
                           f"{rows} of 8192 token rows of one branch per pass ({reps} timed passes), extrapolated "
                           f"linearly to 8192 rows x 4 branches; reference_gemm / reference_bias_act / "
                           f"reference_row_softmax on {self.threads} threads, one row each")

    def dag_fanout(self) -> dict:
        o = self.oracle
        fb, fd, fr, fc = 4, 4, 2048, 2048
        x = self._uniform(fr, fc)
        bias = [self._uniform(fc) for _ in range(fb * fd)]
        hs = [np.empty((fr, fc), np.float32) for _ in range(2)]

        def work(r):
            for bi in range(fb):
                src = x
                for k in range(fd):
                    dst = hs[k & 1]
                    o.bias_act(src[r[0]:r[1]], bias[bi * fd + k], "gelu_tanh", self.impl, out=dst[r[0]:r[1]])
                    src = dst

        sec, reps = self._time(work, self._blocks(fr))
        return self._entry(fb * fd * (2 * fr * fc + fc) * 4 / sec / 1e9, "GB/s",
                           f"all 16 bias+GELU nodes per pass, {reps} timed passes; reference_bias_act over "
                           f"disjoint row blocks on {self.threads} threads")


# keys of the ops entries -> the CpuBaselines method that times the same work
CPU_FOR_OP = {
    "bias_gelu_fp32_4096x4096": "bias_gelu",
    "reduce_full_fp32_2^28": "reduce_full",
    "row_reduce_sum_fp32_32768x1024": "row_reduce",
    "gemm_bf16_8192^3": "gemm",
    "gemm_f32_8192^3": "gemm",
    "dag_fused_config5": "dag_branch",
    "dag_unfused_config5": "dag_branch",
    "dag_fanout_4x4_2048x2048_f32": "dag_fanout",
}


def attach_cpu_baselines(ops: dict, cpu: CpuBaselines) -> None:
    memo: dict[str, dict] = {}
    for key, entry in ops.items():
        meth = CPU_FOR_OP.get(key)
        if meth is None or not isinstance(entry, dict):
            continue
        if meth not in memo:
            memo[meth] = getattr(cpu, meth)()
        entry["cpu_baseline"] = memo[meth]


def headline_config(g: int) -> dict:
    return {"workload": "row_softmax_fp32_32768x1024 (BASELINE config 2)", "rows_per_gpu": ROWS,
            "cols": COLS, "l2": (f"inputs larger than L2: steps run back to back between one event pair, the "
                                 f"128 MiB input and output rotating over {ROTATE} buffer sets (a step's buffers were "
                                 f"last touched {ROTATE - 1} steps earlier); cold_step_ms: L2 flushed before one step "
                                 f"timed alone"),
            "parallelism": f"rows, weak scaling, {g} x full batch"}


# ------------------------------------------------------------ reference arm

def run_reference(args, dist) -> None:
    """The reference's CPU implementation of the path on this host's cores,
    on the GPU arm's config, metric and unit: a step is one row softmax pass
    over the full config-2 batch.  The ops get the same CPU figures as the
    GPU arm's cpu_baseline entries."""
    if dist.rank != 0:
        return
    cpu = CpuBaselines(budget_s=0.0)
    o = cpu.oracle
    x = o.softmax_config_input(ROWS, COLS, seed=2)
    y = np.empty_like(x)
    blocks = cpu._blocks(ROWS)

    def step():
        list(cpu.pool.map(lambda b: o.row_softmax(x[b[0]:b[1]], cpu.impl, out=y[b[0]:b[1]]), blocks))

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = SOFTMAX_BYTES * args.steps / dt / 1e9
    ops = {}
    if args.ops:
        cpu.budget = 2.0
        for key, meth in CPU_FOR_OP.items():
            if any(w in key for w in args.ops.split(",")):
                ops[key] = {"cpu_baseline": getattr(cpu, meth)()}
    cpu.close()
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (N(0, 4^2) logits, every 64th row +80)",
        "config": headline_config(args.gpus),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cpu.threads, "kind": cpu.impl,
                         "sample": f"full {ROWS}x{COLS} batch per step; tests/reference.hpp reference_row_softmax "
                                   f"on {cpu.threads} host threads over disjoint row blocks"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "ops": ops,
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- output checks
#
# After each op's timed loop its last output is checked on sampled rows or
# elements against a float64 recomputation on the device (torch, used only as
# the checker): the reference's spot-check idea (tests/reference.hpp:401) with
# the tolerances of the parity tests.  The full parity gate is tests/; this
# records in the JSON line that the timed output itself is right.

def _gelu_tanh64(v):
    return 0.5 * v * (1.0 + (0.7978845608028654 * (v + 0.044715 * v * v * v)).tanh())


def check_softmax(torch, x, y, rows: int = 64) -> bool:
    n = x.shape[0]
    idx = torch.unique(torch.cat([torch.arange(0, n, max(1, n // rows)), torch.arange(0, min(n, 64 * 8), 64)])).to(x.device)
    ref = torch.softmax(x[idx].double(), dim=1)
    return bool(((y[idx].double() - ref).abs() <= 1e-8 + 1e-5 * ref.abs()).all())


def check_bias_gelu(torch, x, b, y, rows: int = 32) -> bool:
    idx = torch.arange(0, x.shape[0], max(1, x.shape[0] // rows), device=x.device)
    ref = _gelu_tanh64(x[idx].double() + b.double())
    return bool(((y[idx].double() - ref).abs() <= 1e-6 + 1e-5 * ref.abs()).all())


def check_row_reduce(torch, x, y, rows: int = 64) -> bool:
    idx = torch.arange(0, x.shape[0], max(1, x.shape[0] // rows), device=x.device)
    ref = x[idx].double().sum(dim=1)
    ulp = torch.finfo(torch.float32).eps * ref.abs()
    return bool(((y[idx].double() - ref).abs() <= ulp + 1e-30).all())


def check_gemm(torch, a, b, c, samples: int = 256, rel: float = 1e-5, seed: int = 0) -> bool:
    """c[i, j] against sum_k a[i, k] b[k, j] in float64, within `rel` of
    sum_k |a[i, k] b[k, j]| (the scale of the fp32 accumulation error)."""
    gen = torch.Generator(device=a.device)
    gen.manual_seed(seed)
    ii = torch.randint(0, a.shape[0], (samples,), generator=gen, device=a.device)
    jj = torch.randint(0, b.shape[1], (samples,), generator=gen, device=a.device)
    prod = a[ii].double() * b[:, jj].t().double()
    ref, scale = prod.sum(dim=1), prod.abs().sum(dim=1)
    got = c[ii, jj].double()
    return bool(torch.isfinite(got).all() and ((got - ref).abs() <= rel * scale).all())


def check_dag_branch(torch, dev, inputs, probs, fused: bool, rows: int = 4) -> bool:
    """Branch 0 of the config-5 DAG on sampled token rows, recomputed in float64
    on the device with H rounded to bf16 where the kernels store it (and, in the
    unfused graph, GEMM1's output too): the softmax rows within 5e-3 relative
    (a bf16 ulp of H moves the logits by ~1e-4) and summing to one."""
    x, w1, b1, w2, b2 = inputs
    idx = np.linspace(0, x.shape[0] - 1, rows).astype(np.int64)
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)  # noqa: E731
    xs = bf(x[idx]).double()
    lin1 = xs @ bf(w1).double()
    if not fused:
        lin1 = lin1.to(torch.bfloat16).double()
    h = _gelu_tanh64(lin1 + torch.from_numpy(b1).to(dev).double()).to(torch.bfloat16).double()
    y = h @ bf(w2).double() + torch.from_numpy(b2).to(dev).double()
    ref = torch.softmax(y, dim=1)
    got = torch.from_numpy(probs[idx]).to(dev).double()
    sums = torch.from_numpy(probs.sum(axis=1, dtype=np.float64))
    return bool(((got - ref).abs() <= 1e-9 + 5e-3 * ref.abs()).all() and (sums - 1.0).abs().max() < 1e-4)


def check_reduce(torch, dist, x, index_base: int, res_bytes) -> bool:
    """The combined {sum, max, argmax} against every rank's float64 sum, max and
    first index of the max, gathered and folded in rank order."""
    import mcke
    s, m, i = mcke.decode_result(res_bytes)
    local = torch.tensor([x.double().sum().item(), x.max().item(), float(int(x.argmax().item()) + index_base)],
                         dtype=torch.float64, device=x.device)
    if dist.pg is not None:
        parts = [torch.empty_like(local) for _ in range(dist.world)]
        dist.pg.all_gather(parts, local)
    else:
        parts = [local]
    rows = [p.tolist() for p in parts]
    ws = sum(r[0] for r in rows)
    wm = max(r[1] for r in rows)
    wi = int(min(r[2] for r in rows if r[1] == wm))
    return bool(m == np.float32(wm) and i == wi and abs(s - np.float32(ws)) <= np.spacing(np.float32(abs(ws))))


# ----------------------------------------------------------------- our arm

def run_mcke(args, dist) -> None:
    import torch
    torch.cuda.set_device(dist.local)
    dist.init(torch)
    import mcke
    mcke.lib()
    dev = torch.device("cuda", dist.local)
    peaks, peak_kind = load_peaks()
    traffic = load_traffic()
    g = dist.world
    uuid = None
    try:
        uuid = str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass

    # L2 flush between timed steps: write a 256 MiB buffer (twice the 126 MB
    # L2), then read a second one, so the next step starts with an L2 that
    # holds none of its data and no dirty lines waiting to be written back.
    flush_w = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    flush_r = torch.ones(64 << 20, dtype=torch.float32, device=dev)

    def flush():
        flush_w.fill_(1)
        flush_r.sum()

    gen = torch.Generator(device=dev)
    gen.manual_seed(2 + dist.rank)
    xs, ys = [], []
    for _ in range(ROTATE):
        xr = torch.randn(ROWS, COLS, generator=gen, device=dev) * 4.0
        xr[::64] += 80.0
        xs.append(xr)
        ys.append(torch.empty_like(xr))
    x, y = xs[0], ys[0]

    result: dict = {}
    with ClockSampler(uuid) as clocks:
        total_ms = timed_back_to_back(torch, dist, lambda i: mcke.softmax(xs[i % ROTATE], out=ys[i % ROTATE]),
                                      args.steps, args.warmup)
        last = (args.warmup + args.steps - 1) % ROTATE
        headline_checked = check_softmax(torch, xs[last], ys[last])
        kernel_ms = total_ms / args.steps
        achieved = SOFTMAX_BYTES / (kernel_ms * 1e-3) / 1e9
        value = g * SOFTMAX_BYTES * args.steps / (total_ms * 1e-3) / 1e9
        cold_ms = cold_step_ms(torch, dist, lambda: mcke.softmax(x, out=y), flush)
        del xs[1:], ys[1:]

        # e2e: host buffers, H2D + kernel + D2H inside the timed region.  The
        # batch moves in 8 row chunks over three streams so the copy in of
        # chunk c+1, the softmax of chunk c and the copy out of chunk c-1
        # overlap (PCIe is full duplex).  Measured with the steps serialised:
        # 8 chunks 86 GB/s, 16: 84, 32: 79, 64: 67 (per-copy cost), 4: 81
        # (pipeline fill and drain).  Consecutive steps also overlap: step i
        # uses device buffer set i % 2, so its first copies in run while step
        # i - 1's last chunks are still computed and copied out; a chunk's
        # buffers are reused only after step i - 2's softmax and copy out of
        # that chunk (events).  Every step still copies all of its input in
        # and all of its result out.
        xh = x.cpu().pin_memory()
        yh = torch.empty_like(xh).pin_memory()
        xd = [torch.empty_like(x) for _ in range(2)]
        yd = [torch.empty_like(x) for _ in range(2)]
        chunks = 8
        s_in, s_run, s_out = (torch.cuda.Stream(dev) for _ in range(3))
        ev_in = [[torch.cuda.Event() for _ in range(chunks)] for _ in range(2)]
        ev_run = [[torch.cuda.Event() for _ in range(chunks)] for _ in range(2)]
        ev_out = [[torch.cuda.Event() for _ in range(chunks)] for _ in range(2)]
        recorded = [[False] * chunks for _ in range(2)]
        e2e_steps = max(3, min(args.steps, 20))
        e2e_warm = 3

        def e2e_step(i):
            main = torch.cuda.current_stream(dev)
            if i == 0 or i == e2e_warm:  # after the idle point that opens each timed span
                for st in (s_in, s_run, s_out):
                    st.wait_stream(main)
            bs = i % 2
            step = ROWS // chunks
            for c in range(chunks):
                sl = slice(c * step, (c + 1) * step)
                if recorded[bs][c]:
                    s_in.wait_event(ev_run[bs][c])   # step i - 2's softmax has read xd[bs][c]
                    s_run.wait_event(ev_out[bs][c])  # step i - 2's copy out has read yd[bs][c]
                with torch.cuda.stream(s_in):
                    xd[bs][sl].copy_(xh[sl], non_blocking=True)
                    ev_in[bs][c].record(s_in)
                s_run.wait_event(ev_in[bs][c])
                mcke.softmax(xd[bs][sl], out=yd[bs][sl], stream=s_run)
                ev_run[bs][c].record(s_run)
                s_out.wait_event(ev_run[bs][c])
                with torch.cuda.stream(s_out):
                    yh[sl].copy_(yd[bs][sl], non_blocking=True)
                    ev_out[bs][c].record(s_out)
                recorded[bs][c] = True
            main.wait_stream(s_out)

        e2e_ms = timed_back_to_back(torch, dist, e2e_step, e2e_steps, e2e_warm)
        e2e_checked = check_softmax(torch, x, yh.to(dev))
        e2e_value = g * SOFTMAX_BYTES * e2e_steps / (e2e_ms * 1e-3) / 1e9
        del xd, yd

        ops = {}
        if args.ops:
            ops = run_ops(args, dist, torch, mcke, dev, flush, peaks, traffic)
    del flush_w, flush_r

    result = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": g, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (torch.randn * 4 on device, seed 2 + rank; every 64th row +80)",
        "config": headline_config(g),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks.get("hbm_gbs"),
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_kind": f"{peak_kind} hbm_gbs",
                     "traffic": traffic_of(traffic, "softmax_warp_row_kernel"),
                     "traffic_note": (traffic.get("softmax_warp_row_kernel") or {}).get("note"),
                     "algorithmic_bytes_per_launch": SOFTMAX_BYTES, "kernel_ms": round(kernel_ms, 5),
                     "cold_step_ms": round(cold_ms, 5)},
        "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": SOFTMAX_BYTES // 2,
                "d2h_bytes_per_step": SOFTMAX_BYTES // 2, "ms_per_step": round(e2e_ms / e2e_steps, 4),
                "path": "pinned host logits -> H2D -> mcke.softmax (C-ABI) -> D2H, 8 row chunks on 3 streams, "
                        "consecutive steps overlapping on two device buffer sets",
                "checked": e2e_checked,
                "pcie_ceiling_note": "H2D and D2H of 128 MiB each, concurrently: 2.715 ms (49.4 GB/s per direction) "
                                     "on this box, i.e. at most ~99 GB/s of this metric"},
        "checked": headline_checked,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
        "ops": ops,
    }
    dist.close()
    if dist.rank == 0 and g == 1 and not args.no_cpu_baseline:
        cpu = CpuBaselines()
        result["cpu_baseline"] = cpu.softmax()
        attach_cpu_baselines(ops, cpu)
        cpu.close()
    if dist.rank == 0:
        print(json.dumps(result), flush=True)


def run_ops(args, dist, torch, mcke, dev, flush, peaks, traffic) -> dict:
    g, r = dist.world, dist.rank
    want = set(args.ops.split(","))
    out = {}
    steps = max(3, min(args.steps, 50))
    warm = max(3, min(args.warmup, 5))
    ffma_peak = None  # set by the peaks op
    mma_peak = None   # the tcgen05 bf16 probe's rate, set by the peaks op

    from mcke import shard as mshard

    def shard(n):
        return mshard.bounds(n, g, r)

    if "peaks" in want:
        # The roofline denominators measured by the library's own probes on
        # this GPU in this run (the reference's bench/stream_triad.cu and
        # bench/fma_peak.cu), beside the driver's MEASURED_PEAKS.json figures
        # that the fractions in this line use.  Arrays of 1 GiB each (far
        # larger than L2), so no flush is needed.
        n = 1 << 28
        pa = torch.empty(n, device=dev)
        pb = torch.full((n,), 1.5, device=dev)
        pc = torch.full((n,), 0.25, device=dev)
        ps = max(3, min(steps, 10))
        ms_t, per_t = timed_steps(torch, dist, lambda: mcke.peak_triad(pa, pb, pc, 3.0), ps, warm, None)
        ms_c, per_c = timed_steps(torch, dist, lambda: mcke.peak_copy(pa, pb), ps, warm, None)
        del pa, pb, pc
        nt = mcke.peak_fma_threads()
        seed = (torch.arange(nt, device=dev, dtype=torch.float32) % 13)
        fo = torch.empty(nt, device=dev)
        iters = 40000
        ms_f, per_f = timed_steps(torch, dist, lambda: mcke.peak_fma(seed, fo, iters), max(3, min(steps, 5)), warm,
                                  None)
        del seed, fo
        # tcgen05 bf16: the GEMM's single-CTA MMA from shared memory, one CTA
        # per SM, ~5 ms per step
        mctas, miters = mcke.peak_mma_ctas(), 20000
        ms_m, per_m = timed_steps(torch, dist, lambda: mcke.peak_mma(mctas, miters), max(3, min(steps, 5)), warm,
                                  None)
        mcke.check_device_errors()
        sm = torch.cuda.get_device_properties(dev).multi_processor_count
        triad = 12 * n / (min(per_t) * 1e-3) / 1e9   # best step, as a peak is taken
        copy = 8 * n / (min(per_c) * 1e-3) / 1e9
        ffma = mcke.PEAK_FMA_FLOP_PER_THREAD_STEP * nt * iters / (min(per_f) * 1e-3) / 1e12
        nominal_ffma = sm * 128 * 2 * 1.965
        mma = mcke.peak_mma_flops(mctas, miters) / (min(per_m) * 1e-3) / 1e12
        triad, copy, ffma, mma = (dist.min(torch, v) for v in (triad, copy, ffma, mma))
        out["peaks"] = {
            "triad_gbs": round(triad, 1), "copy_gbs": round(copy, 1), "ffma_tflops": round(ffma, 2),
            "driver_hbm_copy_gbs": peaks["hbm_gbs"], "triad_over_driver_copy": round(triad / peaks["hbm_gbs"], 4),
            "copy_over_driver_copy": round(copy / peaks["hbm_gbs"], 4),
            "ffma_over_nominal": round(ffma / (nominal_ffma / 1000.0), 4),
            "tcgen05_bf16_tflops": round(mma, 1), "driver_bf16_burst_tflops": peaks["bf16_tflops"],
            "tcgen05_over_driver_bf16": round(mma / peaks["bf16_tflops"], 4),
            "tcgen05_over_nominal_dense": round(mma / 2250.0, 4),
            "note": "mcke_sm100_peak_{triad,copy,fma}_f32: a = b + 3c and a = b over 2^28 floats (12 and 8 B per "
                    "element), 8 FMA chains per thread x 40000 steps (16 flop per thread-step); best step, "
                    "minimum over ranks; nominal FFMA = SMs x 128 lanes x 2 x 1.965 GHz; "
                    "mcke_sm100_peak_mma_bf16: one CTA per SM, 20000 x 4 MMAs of 128 x 256 x 16 from shared "
                    "memory (no loads), against the driver's cuBLAS burst and the nominal dense 2250 TFLOP/s"}
        ffma_peak = ffma
        mma_peak = mma

    if "bias_gelu" in want:
        r0, r1 = shard(BIAS_ROWS)
        gen = torch.Generator(device=dev)
        gen.manual_seed(0)
        xfull = torch.randn(BIAS_ROWS, BIAS_COLS, generator=gen, device=dev)
        bb = torch.rand(BIAS_COLS, generator=gen, device=dev) * 2 - 1
        # 64 MiB in and out per step, less than L2: rotate over enough sets that
        # a step's buffers were last touched >= 384 MiB of traffic earlier
        nrot = 4
        xbs = [xfull[r0:r1].contiguous() for _ in range(nrot)]
        ybs = [torch.empty_like(xbs[0]) for _ in range(nrot)]
        del xfull
        ms = timed_back_to_back(torch, dist, lambda i: mcke.bias_act(xbs[i % nrot], bb, "gelu_tanh", out=ybs[i % nrot]),
                                steps, warm)
        lastb = (warm + steps - 1) % nrot
        checked = check_bias_gelu(torch, xbs[lastb], bb, ybs[lastb])
        kms = ms / steps
        xb, yb = xbs[0], ybs[0]
        cold = cold_step_ms(torch, dist, lambda: mcke.bias_act(xb, bb, "gelu_tanh", out=yb), flush)
        del xbs[1:], ybs[1:]
        loc = (2 * (r1 - r0) * BIAS_COLS + BIAS_COLS) * 4
        ach = loc / (kms * 1e-3) / 1e9
        out["bias_gelu_fp32_4096x4096"] = {
            "value": round(BIAS_BYTES * steps / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "scaling": "strong",
            "per_gpu_achieved": round(ach, 1), "frac_of_hbm": round(ach / peaks["hbm_gbs"], 4),
            "kernel_ms": round(kms, 5), "cold_step_ms": round(cold, 5), "algorithmic_bytes": BIAS_BYTES,
            "checked": checked, "timing": f"back to back over {nrot} rotating buffer sets",
            "traffic": traffic_of(traffic, "bias_act_f32_chunk_kernel"),
            "traffic_note": (traffic.get("bias_act_f32_chunk_kernel") or {}).get("note")}
        del xb, yb

    if "reduce" in want:
        r0, r1 = shard(REDUCE_N)
        gen = torch.Generator(device=dev)
        gen.manual_seed(1)
        xr = (torch.rand(r1 - r0, generator=gen, device=dev) * 2 - 1)
        ws = torch.empty(mcke.reduce_full_workspace_bytes(r1 - r0), dtype=torch.uint8, device=dev)
        res = torch.empty(16, dtype=torch.uint8, device=dev)
        part = torch.empty(24, dtype=torch.uint8, device=dev)
        nccl_ms = None
        p2p = None
        # Timed: MCKE_REDUCE_EARLY_READ (each step's kernel reads x before
        # waiting for the previous step's, which does not write x, so the
        # steps overlap); the default wait-first path is timed beside it.
        if g == 1:
            launch = lambda: mcke.reduce_full(xr, out=res, workspace=ws, early_read=True)  # noqa: E731
            launch_wait = lambda: mcke.reduce_full(xr, out=res, workspace=ws)  # noqa: E731
        else:
            # the NCCL all-gather of partials, timed for comparison; the
            # reported number uses the peer-to-peer combine kernel
            def launch_nccl():
                mcke.reduce_full_partial(xr, r0, out=part, workspace=ws)
                mcke.reduce_combine(mshard.exchange_partials(part, g), g, out=res)
            ms_n = timed_back_to_back(torch, dist, lambda i: launch_nccl(), steps, warm)
            nccl_ms = ms_n / steps
            nccl_result = mcke.decode_result(res)
            p2p = mshard.P2PExchange(dev)
            launch = lambda: p2p.reduce_full(xr, r0, out=res, early_read=True)  # noqa: E731
            launch_wait = lambda: p2p.reduce_full(xr, r0, out=res)  # noqa: E731
        ms_wait = timed_back_to_back(torch, dist, lambda i: launch_wait(), steps, warm)
        ms = timed_back_to_back(torch, dist, lambda i: launch(), steps, warm)
        torch.cuda.synchronize()
        checked = check_reduce(torch, dist, xr, r0, res.cpu().numpy().tobytes())
        kms = ms / steps
        cold = cold_step_ms(torch, dist, launch, flush)
        ach = (r1 - r0) * 4 / (kms * 1e-3) / 1e9
        p2p_matches = None
        if p2p is not None:
            torch.cuda.synchronize()
            mcke.check_device_errors()
            p2p.close()
            got = mcke.decode_result(res)
            # max and argmax bit for bit; the sums fold the same partials in
            # two fixed orders, so within a float ulp
            p2p_matches = bool(got[1:] == nccl_result[1:] and
                               abs(got[0] - nccl_result[0]) <= float(np.spacing(np.float32(abs(nccl_result[0])))))
        out["reduce_full_fp32_2^28"] = {
            "value": round(REDUCE_BYTES * steps / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "scaling": "strong",
            "per_gpu_achieved": round(ach, 1), "frac_of_hbm": round(ach / peaks["hbm_gbs"], 4),
            "step_ms": round(kms, 5), "cold_step_ms": round(cold, 5),
            "timing": "back to back (the 2^28 / N float input is >= 128 MiB per rank)",
            "input_read": "MCKE_REDUCE_EARLY_READ: a step's kernel streams x before waiting for the previous "
                          "step's kernel (which does not write x) and writes only after it",
            "wait_first_step_ms": round(ms_wait / steps, 5),
            "exchange": "peer stores of 24-byte partials over NVLink (one kernel)" if g > 1 else None,
            "nccl_allgather_step_ms": round(nccl_ms, 5) if nccl_ms is not None else None,
            "p2p_result_matches_nccl": p2p_matches, "checked": checked,
            "traffic": traffic_of(traffic, "reduce_full_stream_kernel")}
        del xr

    if "row_reduce" in want:
        # the reference's ReduceOp (row-wise sum over the last dim) on config
        # 2's shape: rows sharded, 128 MiB read per full batch
        r0, r1 = shard(ROWS)
        gen = torch.Generator(device=dev)
        gen.manual_seed(3)
        xrs = [torch.rand(r1 - r0, COLS, generator=gen, device=dev) * 2 - 1 for _ in range(ROTATE)]
        yrs = [torch.empty(r1 - r0, device=dev) for _ in range(ROTATE)]
        ms = timed_back_to_back(torch, dist, lambda i: mcke.reduce_row(xrs[i % ROTATE], "sum", out=yrs[i % ROTATE]),
                                steps, warm)
        lastb = (warm + steps - 1) % ROTATE
        checked = check_row_reduce(torch, xrs[lastb], yrs[lastb])
        kms = ms / steps
        xr, yr = xrs[0], yrs[0]
        cold = cold_step_ms(torch, dist, lambda: mcke.reduce_row(xr, "sum", out=yr), flush)
        del xrs[1:], yrs[1:]
        moved = ROWS * COLS * 4 + ROWS * 4
        ach = ((r1 - r0) * COLS * 4 + (r1 - r0) * 4) / (kms * 1e-3) / 1e9
        out["row_reduce_sum_fp32_32768x1024"] = {
            "value": round(moved * steps / (ms * 1e-3) / 1e9, 1), "unit": "GB/s", "scaling": "strong",
            "per_gpu_achieved": round(ach, 1), "frac_of_hbm": round(ach / peaks["hbm_gbs"], 4),
            "kernel_ms": round(kms, 5), "cold_step_ms": round(cold, 5), "algorithmic_bytes": moved,
            "checked": checked, "timing": f"back to back over {ROTATE} rotating buffer sets"}
        del xr, yr

    if "gemm_bf16" in want:
        n0, n1 = shard(GEMM_N)
        gen = torch.Generator(device=dev)
        gen.manual_seed(2)
        a = (torch.rand(GEMM_N, GEMM_N, generator=gen, device=dev) * 2 - 1).to(torch.bfloat16)
        gen.manual_seed(3)
        b = ((torch.rand(GEMM_N, GEMM_N, generator=gen, device=dev) * 2 - 1)[:, n0:n1]).to(torch.bfloat16).contiguous()
        c = torch.empty(GEMM_N, n1 - n0, dtype=torch.float32, device=dev)
        ms = timed_back_to_back(torch, dist, lambda i: mcke.gemm(a, b, c, variant="tcgen05"), steps, warm)
        mcke.check_device_errors()
        checked = check_gemm(torch, a, b, c, seed=r)
        kms = ms / steps
        loc_flops = 2 * GEMM_N * GEMM_N * (n1 - n0)
        ach = loc_flops / (kms * 1e-3) / 1e12
        out["gemm_bf16_8192^3"] = {
            "value": round(GEMM_FLOPS * steps / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "scaling": "strong",
            "per_gpu_achieved": round(ach, 1), "frac_of_bf16_peak": round(ach / peaks["bf16_tflops"], 4),
            "peak": peaks["bf16_tflops"], "kernel_ms": round(kms, 4), "parallelism": f"columns of B and C over {g}",
            "frac_of_tcgen05_probe": round(ach / mma_peak, 4) if mma_peak else None,
            "checked": checked}
        del a, b, c

    for fused in (True, False):
        key = "dag_fused" if fused else "dag_unfused"
        if key not in want:
            continue
        from mcke import host as mhost
        rows_total, dm, fm, branches = 8192, 4096, 16384, 4
        r0, r1 = shard(rows_total)
        rows = r1 - r0
        cpu = torch.Generator()
        cpu.manual_seed(5)
        bf = lambda t: t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)  # noqa: E731
        gr = mhost.Graph()
        x = gr.input("X", (rows, dm), "bf16")
        feeds = {x: bf(torch.randn(rows, dm, generator=cpu))}
        probs = []
        for i in range(branches):
            w1 = gr.input(f"W1_{i}", (dm, fm), "bf16")
            b1 = gr.input(f"b1_{i}", (fm,), "f32")
            w2 = gr.input(f"W2_{i}", (fm, dm), "bf16")
            b2 = gr.input(f"b2_{i}", (dm,), "f32")
            feeds[w1] = bf(torch.randn(dm, fm, generator=cpu) * 0.02)
            feeds[w2] = bf(torch.randn(fm, dm, generator=cpu) * 0.02)
            feeds[b1] = (torch.rand(fm, generator=cpu) * 2 - 1).numpy()
            feeds[b2] = (torch.rand(dm, generator=cpu) * 2 - 1).numpy()
            if fused:
                h = gr.gemm(x, w1, bias=b1, act="gelu_tanh", out_dtype="bf16", name=f"gemm1_{i}")
                y = gr.gemm(h, w2, bias=b2, name=f"gemm2_{i}")
            else:
                h = gr.bias_act(gr.gemm(x, w1, out_dtype="bf16", name=f"gemm1_{i}"), b1, "gelu_tanh",
                               name=f"bias_gelu_{i}")
                y = gr.bias_act(gr.gemm(h, w2, name=f"gemm2_{i}"), b2, "none", name=f"bias2_{i}")
            probs.append(gr.softmax(y, name=f"softmax_{i}"))
            gr.output(probs[-1])
            if i == 0:
                chk_in = (feeds[x], feeds[w1], feeds[b1], feeds[w2], feeds[b2])
        gr.finalize()
        # Config 5's memory: the arena comes from a BuddyAllocator of this GPU
        # (the reference's DeviceAllocator interface), and intermediates reuse
        # freed blocks where stream order proves the last reader done.
        # Replayed as a CUDA graph: the device time then excludes the host's
        # enqueue of 12-20 nodes and their events.
        ex = mhost.Executor(gr, devices=[dist.local], streams_per_device=4, cuda_graph=True, buddy=True,
                            memory="reuse_happens_before")
        ex.plan()
        no_reuse = mhost.Executor(gr, devices=[dist.local], streams_per_device=4, memory="alloc_per_tensor")
        no_reuse.plan_dry()
        mem = {"allocator": ex.alloc_stats(0), "arena_bytes": ex.arena_bytes(0),
               "arena_bytes_without_reuse": no_reuse.arena_bytes(0), "memory_policy": "reuse_happens_before"}
        del no_reuse
        for t, arr in feeds.items():
            ex.set_input(t, arr)
        del feeds
        for _ in range(warm):
            ex.run()
        ex.synchronize()
        dist.barrier(torch)
        ds = max(3, min(args.steps, 10))
        tot = 0.0
        for _ in range(ds):
            ex.run()
            tot += ex.last_run_ms()
        dist.barrier(torch)
        tot = dist.max(torch, tot)
        checked = check_dag_branch(torch, dev, chk_in, ex.output(probs[0]), fused)
        del chk_in
        flops = branches * 2 * 2 * rows_total * dm * fm
        out[key + "_config5"] = {
            "value": round(flops * ds / (tot * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "scaling": "strong",
            "ms_per_run": round(tot / ds, 3), "branches": branches, "rows_per_gpu": rows,
            "frac_of_bf16_peak": round(flops / g / (tot / ds * 1e-3) / 1e12 / peaks["bf16_tflops_sustained"], 4),
            "checked": checked, "memory": mem,
            # the reference's cost-model ratio: sum over this GPU's nodes of
            # max(flops / bf16 sustained, bytes / HBM copy) over the measured run
            "cost_model_ratio": round(gr.roofline_ms(peaks["bf16_tflops_sustained"], peaks["hbm_gbs"]) / (tot / ds), 4),
            "peak": peaks["bf16_tflops_sustained"], "peak_kind": "bf16_tflops_sustained (multi-kernel step)",
            "note": ("GEMM1 with fused bias+GELU (bf16 out) -> GEMM2 with fused +b2 -> softmax" if fused else
                     "GEMM1 -> bias+GELU -> GEMM2 -> +b2 -> softmax, one kernel each") +
                    "; 4 branches on 4 streams of the C++ GraphExecutor (CUDA-graph replay), timed by events "
                    "around each replay"}
        del ex, gr

    if "dag_fanout" in want:
        # The reference graph bench's fan-out (4 branches x 4 bias+GELU nodes,
        # 2048x2048 fp32, per GPU): eager enqueue against CUDA-graph replay.
        from mcke import host as mhost
        fb, fd, fr, fc = 4, 4, 2048, 2048
        cpu = torch.Generator()
        cpu.manual_seed(7)
        modes = {}
        # eager and graph: the reference's per-node launches (chain-greedy over
        # 4 streams); eager_level_grouped: one grouped launch per level
        for mode in ("eager", "graph", "eager_level_grouped"):
            gr = mhost.Graph()
            x = gr.input("x", (fr, fc))
            feeds = {x: torch.randn(fr, fc, generator=cpu).numpy()}
            chain, last = [], None
            for b in range(fb):
                h = x
                for k in range(fd):
                    bias = gr.input(f"b{b}_{k}", (fc,))
                    feeds[bias] = (torch.rand(fc, generator=cpu) * 2 - 1).numpy()
                    if b == 0:
                        chain.append(feeds[bias])
                    h = gr.bias_act(h, bias, "gelu_tanh", name=f"bias_gelu_{b}_{k}")
                gr.output(h)
                if b == 0:
                    last = h
            gr.finalize()
            ex = mhost.Executor(gr, devices=[dist.local], streams_per_device=4, cuda_graph=(mode == "graph"),
                                schedule="level_grouped" if mode == "eager_level_grouped" else "chain_greedy")
            ex.plan()
            for t, arr in feeds.items():
                ex.set_input(t, arr)
            for _ in range(warm):
                ex.run()
            ex.synchronize()
            dist.barrier(torch)
            runs = 50
            dev_ms, enq = 0.0, 0.0
            for _ in range(runs):  # one run at a time: device time and host enqueue time
                t0 = time.perf_counter()
                ex.run()
                enq += time.perf_counter() - t0
                dev_ms += ex.last_run_ms()
            ex.synchronize()
            t0 = time.perf_counter()
            for _ in range(runs):  # back to back: does the host keep up?
                ex.run()
            ex.synchronize()
            wall = (time.perf_counter() - t0) / runs * 1e3
            ref = torch.from_numpy(feeds[x][::64]).to(dev).double()
            for bias in chain:
                ref = _gelu_tanh64(ref + torch.from_numpy(bias).to(dev).double())
            got = torch.from_numpy(ex.output(last)[::64]).to(dev).double()
            fan_checked = bool(((got - ref).abs() <= 1e-6 + 4e-5 * ref.abs()).all())
            dist.barrier(torch)
            modes[mode] = {"checked": fan_checked, "device_ms_per_run": round(dist.max(torch, dev_ms / runs), 4),
                           "host_enqueue_us_per_run": round(enq / runs * 1e6, 1),
                           "back_to_back_ms_per_run": round(dist.max(torch, wall), 4)}
            del ex, gr
        moved = fb * fd * (2 * fr * fc + fc) * 4
        gms = modes["graph"]["device_ms_per_run"]
        out["dag_fanout_4x4_2048x2048_f32"] = {
            "value": round(moved * g / (gms * 1e-3) / 1e9, 1), "unit": "GB/s", "scaling": "weak",
            "checked": all(m["checked"] for m in modes.values()),
            "algorithmic_bytes_per_gpu": moved, "eager": modes["eager"], "graph": modes["graph"],
            "eager_level_grouped": modes["eager_level_grouped"],
            "host_enqueue_us_per_node": {k: round(m["host_enqueue_us_per_run"] / (fb * fd), 2) for k, m in modes.items()},
            "note": "16 bias+GELU nodes of the C++ GraphExecutor: eager and graph on 4 streams (chain-greedy, one "
                    "launch per node); eager_level_grouped on one stream with one grouped launch per level "
                    "(SchedulePolicy::kLevelGrouped, mcke_sm100_bias_act_f32_group); value from the CUDA-graph "
                    "replay's device time (events around each launch, max over ranks); back_to_back is host wall "
                    "clock"}

    if "gemm_f32" in want:
        # fp32 operands: the tensor-core 3xTF32 kernel (reported), and the
        # FFMA kernel of the reference's launch_gemm_f32 path for comparison
        n0, n1 = shard(GEMM_N)
        gen = torch.Generator(device=dev)
        gen.manual_seed(2)
        a = torch.rand(GEMM_N, GEMM_N, generator=gen, device=dev) * 2 - 1
        gen.manual_seed(3)
        b = (torch.rand(GEMM_N, GEMM_N, generator=gen, device=dev) * 2 - 1)[:, n0:n1].contiguous()
        c = torch.empty(GEMM_N, n1 - n0, dtype=torch.float32, device=dev)
        ws = torch.empty(mcke.gemm_f32_tc_workspace_bytes(GEMM_N, n1 - n0, GEMM_N), dtype=torch.uint8, device=dev)
        ms = timed_back_to_back(torch, dist, lambda i: mcke.gemm_f32_tc(a, b, c, workspace=ws), steps, warm)
        checked = check_gemm(torch, a, b, c, rel=1e-6, seed=r)
        kms = ms / steps
        loc_flops = 2 * GEMM_N * GEMM_N * (n1 - n0)
        ach = loc_flops / (kms * 1e-3) / 1e12
        # the reference's launch_gemm_f32 call (AUTO): the same 3xTF32 MMAs with
        # the hi/lo split inside the GEMM kernel, no workspace
        ms_auto = timed_back_to_back(torch, dist, lambda i: mcke.gemm(a, b, c), steps, warm)
        checked_auto = check_gemm(torch, a, b, c, rel=1e-6, seed=r + 100)
        fs = max(2, min(steps, 3))
        ms_s, per_s = timed_steps(torch, dist, lambda: mcke.gemm(a, b, c, variant="simt"), fs, 1, None)
        # Library ceilings on the same shard, measured here as denominators:
        # cuBLAS fp32 (FFMA) and cuBLAS with TF32 tensor cores (one pass).
        prev = torch.backends.cuda.matmul.allow_tf32
        try:
            torch.backends.cuda.matmul.allow_tf32 = False
            ms_cs, _ = timed_steps(torch, dist, lambda: torch.matmul(a, b, out=c), fs, 1, None)
            torch.backends.cuda.matmul.allow_tf32 = True
            ms_ct, _ = timed_steps(torch, dist, lambda: torch.matmul(a, b, out=c), fs, 1, None)
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev
        cublas_sgemm = loc_flops * fs / (ms_cs * 1e-3) / 1e12
        cublas_tf32 = loc_flops * fs / (ms_ct * 1e-3) / 1e12
        out["gemm_f32_8192^3"] = {
            "value": round(GEMM_FLOPS * steps / (ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "scaling": "strong",
            "per_gpu_achieved": round(ach, 1), "kernel_ms": round(kms, 3), "checked": checked,
            "path": "3xTF32 on tcgen05 (split pass + kind::tf32 MMAs, fp32 partial sums promoted every 128 k)",
            "launch_gemm_f32_auto": {"value": round(GEMM_FLOPS * steps / (ms_auto * 1e-3) / 1e12, 1),
                                     "unit": "TFLOP/s", "kernel_ms": round(ms_auto / steps, 3),
                                     "checked": checked_auto, "workspace_bytes": 0,
                                     "path": "mcke_sm100_gemm_f32 AUTO: hi/lo split of each smem tile by the "
                                             "epilogue warps inside the tcgen05 kernel"},
            "tf32_mma_tflops": round(3 * ach, 1),
            "frac_of_tf32_nominal": round(3 * ach / TF32_NOMINAL_TFLOPS, 4),
            "cublas_tf32_one_pass_tflops_per_gpu": round(cublas_tf32, 1),
            "frac_of_cublas_tf32_mma_rate": round(3 * ach / cublas_tf32, 4),
            "ffma_kernel_tflops": round(GEMM_FLOPS * fs / (ms_s * 1e-3) / 1e12, 2),
            "cublas_sgemm_tflops_per_gpu": round(cublas_sgemm, 2),
            "ffma_frac_of_cublas_sgemm": round(GEMM_FLOPS / g * fs / (ms_s * 1e-3) / 1e12 / cublas_sgemm, 4),
            "ffma_frac_of_measured_ffma_peak": (round(GEMM_FLOPS / g * fs / (ms_s * 1e-3) / 1e12 / ffma_peak, 4)
                                                if ffma_peak else None),
            "note": "tf32 MMA rate = 3 x fp32 flops, compared with nominal dense tf32 (1100 TFLOP/s) and with "
                    "cuBLAS's one-pass TF32 GEMM on the same shard (torch.matmul, allow_tf32); the FFMA kernel "
                    "compared with cuBLAS SGEMM (the reference's kCublasRef ceiling row)"}
        del a, b, c, ws
    return out


def reduce_timeline(torch, mcke, dev, n: int, steps: int = 60) -> dict:
    """Where a step of the one-kernel reduce (mcke_sm100_reduce_full_p2p_f32)
    spends its time on one GPU: median over `steps` back-to-back calls of the
    phases its %globaltimer stamps bound (ns -> us)."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    xs = [torch.rand(n, generator=gen, device=dev) * 2 - 1 for _ in range(3)]
    buf = torch.zeros(mcke.lib().mcke_sm100_reduce_p2p_buffer_bytes(1), dtype=torch.uint8, device=dev)
    table = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=dev)
    out = torch.empty(16, dtype=torch.uint8, device=dev)
    for i in range(5):
        mcke.reduce_full_p2p(xs[i % 3], 0, table, 1, 0, 0, out=out)
    stamps = mcke.timeline_buffer(steps, dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record()
    for i in range(steps):
        mcke.reduce_full_p2p_timeline(xs[i % 3], 0, table, 1, 0, 0, stamps[i], out=out)
    e1.record()
    torch.cuda.synchronize()
    mcke.check_device_errors()
    step_us = e0.elapsed_time(e1) * 1e3 / steps
    t = stamps.cpu().numpy().astype(np.int64)
    first_entry, first_start, last_start, first_done, last_done, folded, exchanged, counted = (t[:, k] for k in range(8))
    ph = {
        "gap_after_previous_step": first_start[1:] - exchanged[:-1],
        "dispatch_ramp": last_start - first_start,
        "streaming": last_done - first_start,
        "finish_spread": last_done - first_done,
        "fold": folded - last_done,
        "fold_arrival": counted - last_done,
        "fold_collect": folded - counted,
        "exchange": exchanged - folded,
        "kernel_first_start_to_result": exchanged - first_start,
        "early_entry_before_previous_grid_done": first_start - first_entry,
    }
    med = {k: round(float(np.median(v)) / 1e3, 2) for k, v in ph.items()}
    checks = bool(np.all(first_entry <= first_start) and np.all(first_start <= last_start) and
                  np.all(last_start <= last_done) and np.all(last_done <= counted) and
                  np.all(counted <= folded) and np.all(folded <= exchanged))
    stream_bytes = 4 * n
    return {"case": f"reduce_full_p2p world 1, n = {n} floats, {steps} steps back to back over 3 inputs",
            "step_us_cuda_events": round(step_us, 2),
            "phases_median_us": med,
            "streaming_gbs": round(stream_bytes / (med["streaming"] * 1e-6) / 1e9, 1),
            "step_gbs": round(stream_bytes / (step_us * 1e-6) / 1e9, 1),
            "stamps_ordered": checks}


def reduce_steps(torch, mcke, dev, lgs=(25, 28), steps: int = 60, reps: int = 2) -> dict:
    """Back-to-back step time of the full reduce, waiting first against
    MCKE_REDUCE_EARLY_READ, for the one-kernel peer-to-peer path at world 1
    and the two-launch path: CUDA events around `steps` calls on one input
    (which no call writes), the best of `reps` rounds that alternate the four
    cases; every output checked against the default path's bits."""
    gen = torch.Generator(device=dev)
    gen.manual_seed(12)
    buf = torch.zeros(mcke.lib().mcke_sm100_reduce_p2p_buffer_bytes(1), dtype=torch.uint8, device=dev)
    table = torch.tensor([buf.data_ptr()], dtype=torch.int64, device=dev)
    out = torch.empty(16, dtype=torch.uint8, device=dev)
    rows, same = {}, True
    for lg in lgs:
        x = torch.rand(1 << lg, generator=gen, device=dev) * 2 - 1
        ws = torch.empty(mcke.reduce_full_workspace_bytes(x.numel()), dtype=torch.uint8, device=dev)
        want = mcke.reduce_full(x).cpu().numpy().tobytes()
        cases = {
            "p2p_wait_first": lambda: mcke.reduce_full_p2p(x, 0, table, 1, 0, 0, out=out),
            "p2p_early_read": lambda: mcke.reduce_full_p2p(x, 0, table, 1, 0, 0, out=out, early_read=True),
            "two_launch_wait_first": lambda: mcke.reduce_full(x, out=out, workspace=ws),
            "two_launch_early_read": lambda: mcke.reduce_full(x, out=out, workspace=ws, early_read=True),
        }
        best = {}
        for _ in range(reps):
            for name, fn in cases.items():
                for _ in range(5):
                    fn()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record()
                for _ in range(steps):
                    fn()
                e1.record()
                torch.cuda.synchronize()
                same = same and out.cpu().numpy().tobytes() == want
                us = e0.elapsed_time(e1) * 1e3 / steps
                best[name] = min(best.get(name, us), us)
        rows[f"2^{lg}"] = {k: {"step_us": round(v, 2), "gbs": round(4 * x.numel() / (v * 1e-6) / 1e9, 1)}
                           for k, v in best.items()}
        del x, ws
    mcke.check_device_errors()
    return {"case": f"full reduce, {steps} steps back to back on one input, best of {reps}", "steps": rows,
            "same_bits_as_default": same}


def run_profile(args) -> None:
    """One full-size launch of each named kernel after two warm-ups, for ncu
    (`ncu -k regex:... -s 2 -c 1 python bench.py --profile NAME`).  Sizes are
    the BASELINE configs: at most ~1 GiB on the device, each launch < 2 ms."""
    import torch
    import mcke
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    names = args.profile.split(",")
    for name in names:
        if name == "softmax":
            x = torch.randn(ROWS, COLS, generator=gen, device=dev) * 4.0
            x[::64] += 80.0
            y = torch.empty_like(x)
            fn = lambda: mcke.softmax(x, out=y)  # noqa: E731
        elif name == "bias_gelu":
            x = torch.randn(BIAS_ROWS, BIAS_COLS, generator=gen, device=dev)
            b = torch.rand(BIAS_COLS, generator=gen, device=dev) * 2 - 1
            y = torch.empty_like(x)
            fn = lambda: mcke.bias_act(x, b, "gelu_tanh", out=y)  # noqa: E731
        elif name == "reduce":
            x = torch.rand(REDUCE_N, generator=gen, device=dev) * 2 - 1
            ws = torch.empty(mcke.reduce_full_workspace_bytes(REDUCE_N), dtype=torch.uint8, device=dev)
            res = torch.empty(16, dtype=torch.uint8, device=dev)
            fn = lambda: mcke.reduce_full(x, out=res, workspace=ws)  # noqa: E731
        elif name == "row_reduce":
            x = torch.rand(ROWS, COLS, generator=gen, device=dev) * 2 - 1
            y = torch.empty(ROWS, device=dev)
            fn = lambda: mcke.reduce_row(x, "sum", out=y)  # noqa: E731
        elif name == "bias_gelu_bf16":
            # the DAG's H (config 5): 8192 x 16384 bf16, bias over 16384 columns
            x = torch.randn(8192, 16384, generator=gen, device=dev).to(torch.bfloat16)
            b = torch.rand(16384, generator=gen, device=dev) * 2 - 1
            y = torch.empty_like(x)
            fn = lambda: mcke.bias_act(x, b, "gelu_tanh", out=y)  # noqa: E731
        elif name == "bias_group":
            # one level of the reference's fan-out as one grouped launch:
            # four 2048 x 2048 bias + GELU jobs (mcke_sm100_bias_act_f32_group)
            jobs = []
            for _ in range(4):
                xj = torch.randn(2048, 2048, generator=gen, device=dev)
                bj = torch.rand(2048, generator=gen, device=dev) * 2 - 1
                jobs.append((xj, bj, torch.empty_like(xj)))
            fn = lambda: mcke.bias_act_group(jobs, "gelu_tanh")  # noqa: E731
        elif name == "gemm_bf16":
            a = (torch.rand(GEMM_N, GEMM_N, generator=gen, device=dev) * 2 - 1).to(torch.bfloat16)
            b = (torch.rand(GEMM_N, GEMM_N, generator=gen, device=dev) * 2 - 1).to(torch.bfloat16)
            c = torch.empty(GEMM_N, GEMM_N, device=dev)
            fn = lambda: mcke.gemm(a, b, c, variant="tcgen05")  # noqa: E731
        elif name == "gemm_f32":
            n = 4096
            a = torch.rand(n, n, generator=gen, device=dev) * 2 - 1
            b = torch.rand(n, n, generator=gen, device=dev) * 2 - 1
            c = torch.empty(n, n, device=dev)
            ws = torch.empty(mcke.gemm_f32_tc_workspace_bytes(n, n, n), dtype=torch.uint8, device=dev)
            fn = lambda: mcke.gemm_f32_tc(a, b, c, workspace=ws)  # noqa: E731
        elif name == "gemm_f32_split":
            n = 4096
            a = torch.rand(n, n, generator=gen, device=dev) * 2 - 1
            b = torch.rand(n, n, generator=gen, device=dev) * 2 - 1
            c = torch.empty(n, n, device=dev)
            fn = lambda: mcke.gemm_f32_tc(a, b, c, in_kernel_split=True)  # noqa: E731
        elif name == "gemm_f32_ffma":
            n = 4096
            a = torch.rand(n, n, generator=gen, device=dev) * 2 - 1
            b = torch.rand(n, n, generator=gen, device=dev) * 2 - 1
            c = torch.empty(n, n, device=dev)
            fn = lambda: mcke.gemm(a, b, c, variant="simt")  # noqa: E731
        elif name.startswith("reduce_timeline"):
            # Phase breakdown of the one-kernel sharded reduce at world 1
            # (reduce_timeline or reduce_timeline:<log2 n>): K steps back to
            # back over three rotating inputs, each step's %globaltimer stamps.
            lg = int(name.split(":")[1]) if ":" in name else 25
            print(json.dumps(reduce_timeline(torch, mcke, dev, 1 << lg)))
            continue
        elif name == "reduce_steps":
            # waiting first against MCKE_REDUCE_EARLY_READ, back to back
            print(json.dumps(reduce_steps(torch, mcke, dev)))
            continue
        else:
            raise SystemExit(f"unknown profile case {name}")
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
    mcke.check_device_errors()
    print("profile cases done:", ",".join(names))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["mcke", "reference"], default="mcke")
    ap.add_argument("--ops", default="peaks,bias_gelu,reduce,row_reduce,gemm_bf16,dag_fused,dag_unfused,dag_fanout,gemm_f32",
                    help="comma list of extra configs to report under 'ops' ('' for none)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", default="", help="run one small case per named kernel for ncu and exit")
    args = ap.parse_args()
    if args.profile:
        run_profile(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
    else:
        run_mcke(args, dist)


if __name__ == "__main__":
    main()
