"""CPU oracle for the segmented-operator path -- TEST INFRASTRUCTURE ONLY.

Nothing in ``bysj_b200`` imports this package.  Only ``tests/``,
``__graft_entry__.smoke()`` (as the checker) and ``bench.py``'s CPU-baseline /
``--impl reference`` leg (as the timed CPU implementation) may use it.

Contents
--------
``oracle.reference``
    The restatement, in PyTorch fp32, of the reference project's
    ``python/reference`` package (lipengfei1409/bysj): same function names,
    arguments, validation and results (``segment_sum_reference``,
    ``segment_softmax_reference``, ``force_assembly_reference``, ``rmsnorm``,
    ``zonal_scatter_reference``).  Its one copy ships as
    ``bysj_b200.reference``; this package re-exports it.  Plus the two
    compositions the reference has no
    single function for (fused softmax + weighted sum, per-degree RMSNorm).
``oracle.truth``
    float64 NumPy ground truth of every operator, and the integer CSR helpers
    (``segment_offsets``, ``group_by_source``) in NumPy, exact.
``oracle.loops``
    Pure-Python loops for tiny inputs, used to check the two above.

Pinning: ``tests/golden/make_golden.py`` ran the reference's own code in the
build container and stored inputs and outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this oracle against those fixtures and
against the reference test suite's known-answer values.
"""
