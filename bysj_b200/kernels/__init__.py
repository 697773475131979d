"""B200 (sm_100a) native operators with the reference's ``kernels`` API.

Same public names as the reference's ``python/kernels/__init__.py:14-26``,
plus ``segment_attention`` (the fused softmax + weighted sum),
``rotate_back_aggregate`` (the fused rotate-back aggregation of the flash
seam) and ``edge_chain`` (an elementwise chain over the edge stream in one
pass).
"""

from .attention import segment_attention
from .chain import edge_chain
from .gie import gie_available, gie_zonal_scatter, zonal_scatter
from .rmsnorm import rmsnorm, rmsnorm_available
from .rotate import rotate_back_aggregate
from .segment import destination_csr  # noqa: F401  (used by the DeepMD seam; not in __all__)
from .segment import (
    force_assembly,
    group_by_source,
    segment_available,
    segment_offsets,
    segment_softmax,
    segment_sum,
)

__all__ = [
    "edge_chain",
    "force_assembly",
    "gie_available",
    "gie_zonal_scatter",
    "group_by_source",
    "rmsnorm",
    "rmsnorm_available",
    "rotate_back_aggregate",
    "segment_attention",
    "segment_available",
    "segment_offsets",
    "segment_softmax",
    "segment_sum",
    "zonal_scatter",
]
