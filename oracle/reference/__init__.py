"""PyTorch fp32 restatement of the reference project's ``reference`` package.

Test infrastructure only (see ``oracle/__init__.py``).  Function names and
signatures are those of lipengfei1409/bysj ``python/reference/__init__.py:3-18``
so parity tests read like the reference's own tests.
"""

from .gie import gie_zonal_scatter_reference, zonal_scatter_reference
from .rmsnorm import rmsnorm, rmsnorm_per_degree
from .segment import (
    force_assembly_reference,
    segment_attention_reference,
    segment_softmax_reference,
    segment_sum_reference,
)

__all__ = [
    "force_assembly_reference",
    "gie_zonal_scatter_reference",
    "rmsnorm",
    "rmsnorm_per_degree",
    "segment_attention_reference",
    "segment_softmax_reference",
    "segment_sum_reference",
    "zonal_scatter_reference",
]
