"""The opt-in device index guard (B200).

The operators trust their index inputs, as the reference's native paths do
(``python/kernels/gie.py:80-81`` documents the trust); ``check_indices``
checks those invariants on the device -- offsets an exclusive prefix sum from
0 to ``n_edges``, ``order`` a permutation, slot / destination tables inside
their range -- and the operators run it first when grouping validation is
asked for.  Every bad input here is stopped by the guard before any operator
kernel sees it: the guard itself only reads inside the given tensors and
range-checks a value before it uses it as a bitmap index.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

from bysj_b200 import kernels as K  # noqa: E402
from bysj_b200.kernels import segment as S  # noqa: E402


def csr(sizes, device="cuda"):
    sizes = torch.as_tensor(sizes, dtype=torch.int64)
    off = torch.zeros(sizes.numel() + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(sizes, 0)
    return off.to(device)


def test_valid_indices_pass():
    off = csr([3, 0, 5, 1])
    order = torch.randperm(9, generator=torch.Generator().manual_seed(1)).cuda()
    values = torch.tensor([0, 4, 6, 6], device="cuda")
    S.check_indices(off, 9, order=order, values=values, value_limit=7)
    S.check_indices(csr([]), 0)                       # no segments, no edges
    S.check_indices(csr([0, 0]), 0, order=torch.empty(0, dtype=torch.int64, device="cuda"))


@pytest.mark.parametrize("bad", ["first", "last", "decreasing", "negative", "past_end"])
def test_bad_offsets_are_named(bad):
    off = csr([2, 3, 1, 4])
    n_edges = 10
    if bad == "first":
        off[0] = 1
    elif bad == "last":
        n_edges = 11
    elif bad == "decreasing":
        off[2] = 1
    elif bad == "negative":
        off[1] = -1
    else:
        off[3] = 12
    with pytest.raises(ValueError, match="prefix sum"):
        S.check_indices(off, n_edges)


@pytest.mark.parametrize("bad", ["repeat", "past_end", "negative"])
def test_bad_order_is_named(bad):
    order = torch.arange(1000, device="cuda").flip(0).contiguous()
    if bad == "repeat":
        order[17] = order[900]
    elif bad == "past_end":
        order[3] = 1000
    else:
        order[999] = -5
    with pytest.raises(ValueError, match="permutation"):
        S.check_indices(None, 1000, order=order)


def test_large_permutation_with_one_repeat():
    n = 5_000_000
    order = torch.randperm(n, device="cuda")
    S.check_indices(None, n, order=order)
    order[n - 1] = order[0]
    with pytest.raises(ValueError, match="permutation"):
        S.check_indices(None, n, order=order)


def test_every_violation_is_listed():
    off = csr([2, 2])
    off[1] = 5
    order = torch.tensor([0, 0, 1, 2], device="cuda")
    values = torch.tensor([3], device="cuda")
    with pytest.raises(ValueError) as info:
        S.check_indices(off, 4, order=order, values=values, value_limit=3, name="probe")
    text = str(info.value)
    assert text.startswith("probe:")
    assert "prefix sum" in text and "permutation" in text and "within range" in text


def test_argument_errors():
    off = csr([1, 1])
    with pytest.raises(RuntimeError, match="order must have n_edges"):
        S.check_indices(off, 2, order=torch.arange(3, device="cuda"))
    with pytest.raises(RuntimeError, match="int64"):
        S.check_indices(off.int(), 2)


def test_segment_operators_stop_before_the_kernel():
    gen = torch.Generator().manual_seed(2)
    off = csr([4, 0, 3, 5])
    src = torch.randn(12, 16, generator=gen).cuda()
    dst = torch.repeat_interleave(torch.arange(4), torch.tensor([4, 0, 3, 5])).cuda()
    good = K.segment_sum(src, dst, off, check_grouping=True)
    assert torch.equal(good, K.segment_sum(src, dst, off))
    bad = off.clone()
    bad[2] = 13
    with pytest.raises(ValueError, match="segment sum: offsets"):
        K.segment_sum(src, dst, bad, check_grouping=True)
    order = torch.arange(12, device="cuda")
    order[5] = 4
    with pytest.raises(ValueError, match="segment sum: order"):
        K.segment_sum(src, dst, off, order=order, check_grouping=True)
    logit = torch.randn(12, 2, generator=gen).cuda()
    env = torch.rand(12, generator=gen).cuda()
    with pytest.raises(ValueError, match="segment softmax: order"):
        K.segment_softmax(logit, env, off, order=order, check_grouping=True)
    with pytest.raises(ValueError, match="segment softmax: offsets"):
        K.segment_softmax(logit, env, bad, check_grouping=True)


def test_env_switch_guards_attention_and_gie(monkeypatch):
    monkeypatch.setattr(S, "_CHECK_GROUPING", True)
    gen = torch.Generator().manual_seed(3)
    off = csr([2, 3])
    logit = torch.randn(5, 2, generator=gen).cuda()
    value = torch.randn(5, 4, 8, generator=gen).cuda()
    K.segment_attention(logit, value, off)            # valid: runs
    bad = off.clone()
    bad[-1] = 4
    with pytest.raises(ValueError, match="segment attention: offsets"):
        K.segment_attention(logit, value, bad)

    e, rows, n_radial, c, nodes = 6, 3, 2, 8, 3
    zonal = torch.randn(e, rows, generator=gen).cuda()
    radial = torch.randn(e, n_radial, c, generator=gen).cuda()
    dst = torch.tensor([0, 0, 1, 2, 2, 2], device="cuda")
    inv = torch.rand(nodes, generator=gen).cuda()
    slot = torch.tensor([0, 1, 1], device="cuda")
    K.zonal_scatter(zonal, radial, dst, slot, inv)   # valid: runs
    with pytest.raises(ValueError, match="GIE radial_slot"):
        K.zonal_scatter(zonal, radial, dst, torch.tensor([0, 1, 2], device="cuda"), inv)
    with pytest.raises(ValueError, match="GIE dst"):
        K.zonal_scatter(zonal, radial, torch.tensor([0, 0, 1, 2, 2, 3], device="cuda"), slot, inv)
