#!/usr/bin/env python3
"""Regenerate the committed golden fixtures under tests/golden/.

Run where the reference tree exists (its path with --ref; the default is the
build container's checkout):

    python tests/golden/make_golden.py [--ref PATH_TO_REFERENCE_TREE]

It writes two files, both consumed by tests/test_oracle.py and the GPU parity
tests, none of which read the reference tree at run time:

* reference_vectors.json -- the reference's own golden vectors
  (tests/data/reference_vectors.txt, 19 cases written by its independent Python
  generator tools/gen_reference.py) converted case by case to JSON.  Floats
  stay 8-hex-digit IEEE-754 bit patterns so nothing is re-rounded.
* ref_fixtures.npz -- outputs of the reference's compiled CPU oracle
  (tests/reference.hpp, built into oracle/_ref/libmcke_ref.so by
  oracle/Makefile) on small seeded inputs: fill_random streams, every
  activation of reference_bias_act, reference_row_reduce, reference_row_softmax
  (with +80-shifted rows), reference_gemm with alpha/beta, and the rows=1
  full-vector sum and max.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402


def parse_vectors(path: str) -> list[dict]:
    """Token reader for the reference's vector format (case ... end blocks)."""
    toks = []
    with open(path) as f:
        for line in f:
            line = line.split("#", 1)[0]
            toks.extend(line.split())
    cases, i = [], 0
    while i < len(toks):
        if toks[i] != "case":
            i += 1
            continue
        c = {"name": toks[i + 1], "ints": {}, "floats": {}, "arrays": {}}
        i += 2
        while toks[i] != "end":
            t = toks[i]
            if t in ("kind", "mode"):
                c[t] = toks[i + 1]
                i += 2
            elif t == "int":
                c["ints"][toks[i + 1]] = int(toks[i + 2])
                i += 3
            elif t == "float":
                c["floats"][toks[i + 1]] = toks[i + 2]
                i += 3
            elif t == "array":
                key, n = toks[i + 1], int(toks[i + 2])
                c["arrays"][key] = toks[i + 3:i + 3 + n]
                i += 3 + n
            else:
                raise ValueError(f"unknown token {t!r} in case {c['name']}")
        cases.append(c)
        i += 1
    return cases


def make_ref_fixtures() -> dict[str, np.ndarray]:
    R = "reference"
    fx: dict[str, np.ndarray] = {}
    for seed in (0, 1, 2, 3):
        fx[f"fill_random_seed{seed}"] = oracle.fill_random(4096, seed, impl=R)
    fx["fill_random_lohi"] = oracle.fill_random(1000, 7, -4.0, 4.0, impl=R)

    x = oracle.fill_random(48 * 96, 10, -4.0, 4.0, impl=R).reshape(48, 96)
    bias = oracle.fill_random(96, 11, -1.0, 1.0, impl=R)
    fx["bias_act_x"], fx["bias_act_bias"] = x, bias
    for name in ("none", "relu", "gelu_erf", "gelu_tanh"):
        fx[f"bias_act_{name}"] = oracle.bias_act(x, bias, name, impl=R)

    xr = oracle.fill_random(7 * 333, 12, -1.0, 1.0, impl=R).reshape(7, 333)
    fx["row_reduce_x"] = xr
    for kind in ("sum", "max", "mean"):
        fx[f"row_reduce_{kind}"] = oracle.row_reduce(xr, kind, impl=R)

    xs = oracle.fill_random(16 * 1024, 13, -16.0, 16.0, impl=R).reshape(16, 1024)
    xs[::4] += np.float32(80.0)
    fx["row_softmax_x"] = xs
    fx["row_softmax_y"] = oracle.row_softmax(xs, impl=R)

    a = oracle.fill_random(33 * 47, 14, impl=R).reshape(33, 47)
    b = oracle.fill_random(47 * 65, 15, impl=R).reshape(47, 65)
    c = oracle.fill_random(33 * 65, 16, impl=R).reshape(33, 65)
    fx["gemm_a"], fx["gemm_b"], fx["gemm_c"] = a, b, c
    fx["gemm_out"] = oracle.gemm(a, b, c, 1.5, 0.5, impl=R)

    v = oracle.fill_random(20011, 1, impl=R)
    fx["full_x"] = v
    fx["full_sum"] = oracle.row_reduce(v.reshape(1, -1), "sum", impl=R)
    fx["full_max"] = oracle.row_reduce(v.reshape(1, -1), "max", impl=R)
    return fx


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get(
        "MCKE_REFERENCE_TREE", os.path.join(os.path.dirname(os.path.dirname(HERE)), "..", "reference")),
        help="the reference source tree (default: MCKE_REFERENCE_TREE, else `reference` beside this repository)")
    args = ap.parse_args()
    src = os.path.join(args.ref, "tests", "data", "reference_vectors.txt")
    cases = parse_vectors(src)
    with open(os.path.join(HERE, "reference_vectors.json"), "w") as f:
        json.dump({"source": "mini-cuda-kernel-engine tests/data/reference_vectors.txt "
                             "(generated there by tools/gen_reference.py)",
                   "cases": cases}, f, indent=1)
    oracle.build()
    if not oracle.have_reference():
        raise SystemExit("oracle/_ref/libmcke_ref.so missing: cannot make ref_fixtures.npz")
    np.savez_compressed(os.path.join(HERE, "ref_fixtures.npz"), **make_ref_fixtures())
    print(f"wrote {len(cases)} vector cases and ref_fixtures.npz")


if __name__ == "__main__":
    main()
