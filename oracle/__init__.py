"""CPU checkers for the parity tests (test infrastructure, never product code).

* :mod:`oracle.oracle` — ctypes wrappers over ``liboracle.so`` (our plain-C
  restatement of the reference's Q8_0 path, ``q8_oracle.c``) and over
  ``_ref/libaxion_ref.so`` (the reference's own C++ sources compiled by
  ``oracle/Makefile`` + ``ref_shim.cpp``).

Only ``tests/``, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline
leg use this package.
"""
