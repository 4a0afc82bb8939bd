"""Build libmcke_sm100a.so (the CUDA kernel library behind include/mcke_sm100.h).

    python mini-cuda-kernel-engine_b200/build.py [--force] [--verbose-ptxas]

Compiles every csrc/*.cu for sm_100a only (-gencode arch=compute_100a,code=sm_100a)
with -lineinfo, in parallel, into _build/, and links lib/libmcke_sm100a.so in
tree (static cudart, no -lcuda: the driver's tensor-map encoder is fetched at
run time through cudaGetDriverEntryPoint).  Re-running is incremental on
source and header timestamps.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "lib")
LIB = os.path.join(LIBDIR, "libmcke_sm100a.so")
INCLUDE = os.path.join(ROOT, "include")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _flags(verbose_ptxas: bool) -> list[str]:
    f = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE, "-I", CSRC,
                "--expt-relaxed-constexpr"]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))
    cc = nvcc()
    flags = _flags(verbose_ptxas)
    objs, jobs = [], []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, [src] + headers):
            jobs.append([cc] + flags + ["-c", src, "-o", obj])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for cmd, r in ex.map(run, jobs):
            out = (r.stdout + r.stderr).strip()
            if r.returncode != 0:
                failed.append((cmd[-3], out))
            elif out and (verbose_ptxas or not quiet):
                print(out, file=sys.stderr)
    if failed:
        msg = "\n\n".join(f"{src}:\n{out}" for src, out in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    if force or jobs or _stale(LIB, objs):
        cmd = [cc] + ARCH + ["-shared", "-o", LIB] + objs + ["-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas))
