"""ORACLE -- test infrastructure, not product code.

CPU restatement of the reference examples' own correctness checks (the
PyTorch CPU expressions each ``examples/*/*.py`` compares its kernel against),
plus a plain-C restatement of the integer GEMMs (``int_gemm.c``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import or run anything here,
and only as the checker or the timed CPU baseline.  The xb200 product path
never calls it.

Pinning: ``tests/golden/make_golden.py`` runs the reference examples' own
``bench_*`` functions (from the reference source tree) with their kernel
launch swapped for a recorder, and stores each example's inputs and its own
expected output; ``tests/test_oracle_golden.py`` checks these functions
against those fixtures.  int16 GEMM has no reference test (the reference
claims int16 support, README.md:21, but ships no example): its semantics
(int32 accumulation, wraparound mod 2^32) follow the reference's accumulator
choice ``accum_type="i32"`` (amd_triton_npu/backend/matmul_transform.py:62-64)
and are pinned only against int64 arithmetic -- parity unpinned by the
reference for that one dtype.
"""
