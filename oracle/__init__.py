"""CPU oracle for LMPool's KV data path.

TEST INFRASTRUCTURE ONLY: the checker the CUDA path is compared against, and
the timed CPU baseline of bench.py. The product (``lmpool_b200``) never
imports this package. Two restatements of the reference live here:

* ``kv_oracle.c`` (threaded C, built by :mod:`oracle.build`), fast enough for
  full-geometry parity cases and the CPU baseline;
* ``numpy_ref`` (plain numpy on uint8/uint16 views), small cases only.

Both are pinned against golden vectors produced by the reference itself
(``tests/golden/``).
"""
