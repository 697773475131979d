"""B200 (sm_100a) native operators with the reference's ``kernels`` API.

Same public names as the reference's ``python/kernels/__init__.py:14-26``,
plus ``segment_attention`` (the fused softmax + weighted sum).
"""

from .attention import segment_attention
from .gie import gie_available, gie_zonal_scatter, zonal_scatter
from .rmsnorm import rmsnorm, rmsnorm_available
from .segment import (
    force_assembly,
    group_by_source,
    segment_available,
    segment_offsets,
    segment_softmax,
    segment_sum,
)

__all__ = [
    "force_assembly",
    "gie_available",
    "gie_zonal_scatter",
    "group_by_source",
    "rmsnorm",
    "rmsnorm_available",
    "segment_attention",
    "segment_available",
    "segment_offsets",
    "segment_softmax",
    "segment_sum",
    "zonal_scatter",
]
