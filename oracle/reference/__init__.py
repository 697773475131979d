"""The fp32 restatement of the reference project's ``reference`` package.

Test infrastructure only (see ``oracle/__init__.py``).  The restatement has
one copy, shipped as :mod:`bysj_b200.reference` (the ``reference.*`` API that
users of lipengfei1409/bysj compare against, ``python/reference/__init__.py:3-18``);
this package re-exports it under the reference's own package name so parity
tests read like the reference's own tests (``from reference import ...``).
That module is plain PyTorch with the reference's ATen operation sequence
(zero-init + ``index_add_`` over ``dst``, per-segment ``amax``), so on CPU it
reproduces the reference's fp32 results bit for bit; ``tests/test_oracle_golden.py``
pins it to fixtures made by running the reference's own code.  The
dependency only runs this way: nothing under ``bysj_b200`` imports ``oracle``.
"""

from bysj_b200.reference import (
    force_assembly_reference,
    gie_zonal_scatter_reference,
    rmsnorm,
    rmsnorm_per_degree,
    rotate_back_aggregate_reference,
    segment_attention_reference,
    segment_softmax_reference,
    segment_sum_reference,
    zonal_scatter_reference,
)

__all__ = [
    "force_assembly_reference",
    "gie_zonal_scatter_reference",
    "rmsnorm",
    "rmsnorm_per_degree",
    "rotate_back_aggregate_reference",
    "segment_attention_reference",
    "segment_softmax_reference",
    "segment_sum_reference",
    "zonal_scatter_reference",
]
