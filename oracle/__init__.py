"""CPU checker for the mcke sm_100a kernel library.  TEST INFRASTRUCTURE ONLY.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's cpu_baseline leg (and
its ``--impl reference`` arm) may import this package.  The product library
never loads it, and nothing here is a fallback for a missing CUDA extension.

Two implementations sit behind one numpy-facing API:

* ``port``      -- oracle/mcke_oracle.c, a C restatement of the reference's
                   CPU oracle (mini-cuda-kernel-engine tests/reference.hpp),
                   built into oracle/_build/libmcke_oracle.so;
* ``reference`` -- the reference's tests/reference.hpp itself, compiled from
                   the reference tree by oracle/Makefile into
                   oracle/_ref/libmcke_ref.so (absent when it could not be
                   built; tests that need it skip with that reason).

tests/test_oracle.py pins the port against the reference's golden vectors and
against the reference library, bit for bit.
"""
from .oracle import *  # noqa: F401,F403
from .oracle import __all__  # noqa: F401
