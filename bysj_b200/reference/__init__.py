"""PyTorch reference implementations for explicit testing and comparison.

The ``reference`` package of lipengfei1409/bysj
(``python/reference/__init__.py:3-18``): the same functions, signatures and
validation messages, plus ``segment_attention_reference`` (the fused
operator's composition) and ``rmsnorm_per_degree`` (the per-degree weights).
They run on any device with plain PyTorch and are never called by
:mod:`bysj_b200.kernels`.
"""

from .gie import gie_zonal_scatter_reference, zonal_scatter_reference
from .rmsnorm import rmsnorm, rmsnorm_per_degree
from .segment import (
    force_assembly_reference,
    rotate_back_aggregate_reference,
    segment_attention_reference,
    segment_softmax_reference,
    segment_sum_reference,
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
