"""CPU oracle for the trnblas_b200 hot path -- TEST INFRASTRUCTURE ONLY.

A plain numpy restatement of the reference trnblas algorithms on the hot path
(GEMM / batched GEMM / SYRK semantics, the Ozaki fp64 split and recombination,
the DF-MP2 pair energy), each function citing the reference file:line it
follows. Only `tests/`, `__graft_entry__.smoke()` and `bench.py`'s CPU
baseline / reference arm may import it, and only as the checker or the timed
CPU baseline: the product path (`trnblas_b200`) never calls it.

Pinned: `tests/test_oracle_golden.py` checks every function here against golden
vectors produced by the reference itself (`tests/golden/make_golden.py`, which
imports trnsci/trnblas 0.13.0 in a subprocess) and against the reference's own
known-answer tests restated.
"""
