"""The drop-in proof on the CPU: the reference-side binding
(mini-cuda-kernel-engine_b200/integration/kernels_sm100.cpp) compiles against
the reference's own headers and links against libmcke_sm100a.so with every
launcher of the reference's include/mcke/kernels/kernels.hpp defined.

Runs only where the reference tree exists (the build container); the GPU box
has no reference tree and skips it.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mini-cuda-kernel-engine_b200")
# the reference source tree: MCKE_REFERENCE_TREE, else a checkout named
# `reference` beside this repository
REF = os.environ.get("MCKE_REFERENCE_TREE", os.path.join(os.path.dirname(ROOT), "reference"))
SHIM = os.path.join(PKG, "integration", "kernels_sm100.cpp")

pytestmark = pytest.mark.skipif(not os.path.exists(os.path.join(REF, "include", "mcke", "kernels", "kernels.hpp")),
                                reason="reference tree absent")


def test_shim_compiles_against_the_reference_headers_and_links(tmp_path):
    lib = os.path.join(PKG, "lib", "libmcke_sm100a.so")
    if not os.path.exists(lib):
        subprocess.run([sys.executable, os.path.join(PKG, "build.py")], check=True)
    obj = tmp_path / "shim.o"
    so = tmp_path / "libshim.so"
    cc = ["g++", "-std=c++20", "-O2", "-fPIC", "-Wall", "-DMCKE_WITH_CUDA=1", f"-I{REF}/include",
          f"-I{ROOT}/include", "-I/usr/local/cuda/include", "-c", SHIM, "-o", str(obj)]
    r = subprocess.run(cc, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run(["g++", "-shared", "-o", str(so), str(obj), f"-L{PKG}/lib", "-lmcke_sm100a",
                        "-Wl,--no-undefined", "-L/usr/local/cuda/lib64", "-lcudart"],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    # every launcher the reference header declares is defined by the shim
    with open(os.path.join(REF, "include", "mcke", "kernels", "kernels.hpp")) as f:
        code = "\n".join(ln.split("//", 1)[0] for ln in f)  # declarations, not comments
    declared = set(re.findall(r"\b(launch_\w+|row_reduce_workspace_bytes|gemm_kernel_attrs)\s*\(", code))
    assert len(declared) >= 8
    nm = subprocess.run(["nm", "-C", "--defined-only", str(so)], capture_output=True, text=True).stdout
    defined = {name for name in declared if f"mcke::kernels::{name}(" in nm}
    assert defined == declared, declared - defined
