"""The shipped ``bysj_b200.reference`` API (no GPU needed).

``reference.*`` is part of the reference project's public Python API
(``python/reference/__init__.py:3-18``).  The package ships its own
implementation of it; this file runs the golden-fixture checks of
``test_oracle_golden.py`` against that implementation (the same assertions,
with the shipped functions swapped in) and checks that it is not the test
oracle re-exported.
"""
from __future__ import annotations

import pytest

import test_oracle_golden as G
import bysj_b200.reference as R

REFERENCE_ALL = {
    "force_assembly_reference", "gie_zonal_scatter_reference", "rmsnorm",
    "segment_softmax_reference", "segment_sum_reference", "zonal_scatter_reference",
}
SWAPPED = ("force_assembly_reference", "rmsnorm", "rmsnorm_per_degree",
           "segment_attention_reference", "segment_softmax_reference", "segment_sum_reference",
           "zonal_scatter_reference")
GOLDEN_CHECKS = [
    ("test_segment_sum_matches_reference_and_gradients", None),
    ("test_segment_softmax_matches_reference_and_gradients", None),
    ("test_attention_composition_matches_reference", None),
    ("test_force_assembly_matches_reference", None),
    ("test_rmsnorm_matches_reference_and_gradients", "w17"),
    ("test_rmsnorm_matches_reference_and_gradients", "w128"),
    ("test_rmsnorm_matches_reference_and_gradients", "w257"),
    ("test_rmsnorm_per_degree_matches_reference_slices", None),
    ("test_gie_matches_reference_and_gradients", None),
]


def test_exports_the_reference_names():
    assert REFERENCE_ALL <= set(R.__all__)
    for name in R.__all__:
        fn = getattr(R, name)
        assert fn.__module__.startswith("bysj_b200.reference"), name


@pytest.mark.parametrize("check,arg", GOLDEN_CHECKS)
def test_shipped_reference_reproduces_golden_outputs(monkeypatch, check, arg):
    for name in SWAPPED:
        monkeypatch.setattr(G, name, getattr(R, name))
    fn = getattr(G, check)
    fn() if arg is None else fn(arg)


def test_shipped_reference_validation_matches():
    import torch

    with pytest.raises(TypeError):
        R.rmsnorm(torch.zeros(4, dtype=torch.float64))
    with pytest.raises(ValueError):
        R.segment_sum_reference(torch.zeros(3, 2), torch.tensor([0, 0, 1]),
                                torch.tensor([0, 3]))
