"""bysj_b200: B200-native (sm_100a) segmented operators for DeepMD DPA4/SeZM.

Subpackages mirror the reference project's Python API:

* :mod:`bysj_b200.kernels` -- the ``kernels.*`` operator wrappers
  (segment_offsets, segment_sum, segment_softmax, segment_attention,
  force_assembly, rmsnorm, zonal_scatter).
* :mod:`bysj_b200.reference` -- the ``reference.*`` PyTorch implementations
  for explicit testing and comparison (never called by the kernels).
* :mod:`bysj_b200.model` -- ``DPA4Model(fused=...)`` and the DeepMD seam.
* :mod:`bysj_b200.sharding` -- multi-GPU frame sharding and the
  destination-range partition of one large frame.

The kernels live in ``libbysj_b200.so`` (C ABI: ``include/bysj_b200.h``),
reached from Python through the ``bysj_b200._C`` torch shim.
"""

__version__ = "1.0.0"
