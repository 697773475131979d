"""Pin the CPU oracle before trusting it (no GPU needed).

1. Against the golden fixtures produced by running the reference's own code
   (``tests/golden/make_golden.py``): the fp32 oracle reproduces the reference
   outputs, and its autograd gradients reproduce the reference's.
2. Against the known-answer values in the reference's host tests
   (``tests/python/test_segment_ops_reference.py:30-46,63-69,147-158``,
   ``tests/python/test_gie.py:180-189``).
3. Against independent pure-Python loops and the float64 NumPy truth.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import loops, truth
from reference import (
    force_assembly_reference,
    rmsnorm,
    rmsnorm_per_degree,
    segment_attention_reference,
    segment_softmax_reference,
    segment_sum_reference,
    zonal_scatter_reference,
)


def t(a, grad=False):
    out = torch.from_numpy(np.ascontiguousarray(a))
    return out.requires_grad_(True) if grad else out


# ---- golden fixtures ---------------------------------------------------------

def test_csr_helpers_match_reference():
    g = golden("csr")
    n = g["offsets"].size - 1
    np.testing.assert_array_equal(truth.segment_offsets(g["dst"], n), g["offsets"])
    order, offsets = truth.group_by_source(g["src"], n)
    np.testing.assert_array_equal(order, g["src_order"])
    np.testing.assert_array_equal(offsets, g["src_offsets"])


def test_segment_sum_matches_reference_and_gradients():
    g = golden("segment_sum")
    src = t(g["src"], grad=True)
    nscale = t(g["node_scale"], grad=True)
    out = segment_sum_reference(src, t(g["dst"]), t(g["offsets"]), t(g["edge_scale"]), nscale)
    np.testing.assert_array_equal(out.detach().numpy(), g["out"])
    gs, gn = torch.autograd.grad(out, (src, nscale), t(g["upstream"]))
    np.testing.assert_allclose(gs.numpy(), g["grad_src"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(gn.numpy(), g["grad_node_scale"], rtol=1e-6, atol=1e-6)


def test_segment_softmax_matches_reference_and_gradients():
    g = golden("segment_softmax")
    logit, env, null = t(g["logit"], True), t(g["env"], True), t(g["null_logit"], True)
    alpha, null_alpha = segment_softmax_reference(logit, env, t(g["dst"]), t(g["offsets"]), null)
    np.testing.assert_array_equal(alpha.detach().numpy(), g["alpha"])
    np.testing.assert_array_equal(null_alpha.detach().numpy(), g["null_alpha"])
    grads = torch.autograd.grad((alpha, null_alpha), (logit, env, null),
                                (t(g["grad_alpha"]), t(g["grad_null_alpha"])))
    for got, key in zip(grads, ("grad_logit", "grad_env", "grad_null_logit")):
        np.testing.assert_allclose(got.numpy(), g[key], rtol=1e-6, atol=1e-6)
    plain, none = segment_softmax_reference(t(g["logit"]), t(g["env"]), t(g["dst"]),
                                            t(g["offsets"]))
    assert none is None
    np.testing.assert_array_equal(plain.numpy(), g["alpha_nonull"])


def test_attention_composition_matches_reference():
    g = golden("segment_attention")
    out = segment_attention_reference(t(g["logit"]), t(g["value"]), t(g["dst"]), t(g["offsets"]))
    np.testing.assert_allclose(out.numpy(), g["out"], rtol=1e-6, atol=1e-7)
    deep = truth.segment_attention(g["logit"], g["value"], g["dst"], g["offsets"].size - 1)
    np.testing.assert_allclose(g["out"], deep, rtol=1e-5, atol=1e-6)


def test_force_assembly_matches_reference():
    g = golden("force_assembly")
    force, virial = force_assembly_reference(
        t(g["grad_edge"]), t(g["edge_vec"]), t(g["src"]), t(g["dst"]),
        t(g["dst_offsets"]), t(g["src_offsets"]))
    np.testing.assert_array_equal(force.numpy(), g["force"])
    np.testing.assert_array_equal(virial.numpy(), g["virial"])
    n = g["dst_offsets"].size - 1
    f64, w64 = truth.force_assembly(g["grad_edge"], g["edge_vec"], g["src"], g["dst"], n)
    np.testing.assert_allclose(g["force"], f64, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(g["virial"], w64, rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("tag", ["w17", "w128", "w257"])
def test_rmsnorm_matches_reference_and_gradients(tag):
    g = golden("rmsnorm")
    x, s = t(g[f"{tag}_x"], True), t(g[f"{tag}_scale"], True)
    y = rmsnorm(x, s, eps=1e-5)
    np.testing.assert_array_equal(y.detach().numpy(), g[f"{tag}_y"])
    gx, gs = torch.autograd.grad(y, (x, s), t(g[f"{tag}_upstream"]))
    np.testing.assert_allclose(gx.numpy(), g[f"{tag}_grad_x"], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(gs.numpy(), g[f"{tag}_grad_scale"], rtol=1e-6, atol=1e-5)


def test_rmsnorm_per_degree_matches_reference_slices():
    g = golden("rmsnorm")
    y = rmsnorm_per_degree(t(g["deg_x"]), t(g["deg_w"]))
    np.testing.assert_array_equal(y.numpy(), g["deg_y"])
    deep, _ = truth.rmsnorm(g["deg_x"], g["deg_w"], 1e-6, per_degree=True)
    np.testing.assert_allclose(g["deg_y"], deep, rtol=1e-5, atol=1e-6)


def test_gie_matches_reference_and_gradients():
    g = golden("gie")
    z, r, inv = t(g["zonal"], True), t(g["radial"], True), t(g["inv"], True)
    out = zonal_scatter_reference(z, r, t(g["dst"]), t(g["slot"]), inv)
    np.testing.assert_array_equal(out.detach().numpy(), g["out"])
    grads = torch.autograd.grad(out, (z, r, inv), t(g["upstream"]))
    for got, key in zip(grads, ("grad_zonal", "grad_radial", "grad_inv")):
        np.testing.assert_allclose(got.numpy(), g[key], rtol=1e-6, atol=1e-6)


# ---- the reference tests' known answers --------------------------------------

def _graph(sizes):
    dst = np.repeat(np.arange(len(sizes)), sizes).astype(np.int64)
    return dst, np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)


def test_known_answer_offsets_and_source_grouping():
    dst, offsets = _graph([2, 0, 3])
    np.testing.assert_array_equal(truth.segment_offsets(dst, 3), offsets)
    order, off = truth.group_by_source(np.array([2, 0, 2, 1, 0]), 3)
    np.testing.assert_array_equal(off, [0, 2, 3, 5])
    assert order.tolist()[:2] == [1, 4]
    with pytest.raises(ValueError):
        truth.segment_offsets(np.array([0, 3]), 3)


def test_known_answer_empty_segments_stay_zero():
    dst, offsets = _graph([0, 2, 0])
    out = segment_sum_reference(torch.ones(2, 3), t(dst), t(offsets))
    assert out[0].count_nonzero() == 0 and out[2].count_nonzero() == 0
    torch.testing.assert_close(out[1], torch.full((3,), 2.0))


def test_known_answer_masked_edges_carry_no_mass():
    dst, offsets = _graph([2, 1, 3])
    gen = torch.Generator().manual_seed(0)
    logit = torch.randn(6, 3, generator=gen)
    env = torch.tensor([0.9, -0.2, 0.7, 0.0, 1.1, 0.3])
    null = torch.randn(3, 3, generator=gen)
    alpha, null_alpha = segment_softmax_reference(logit, env, t(dst), t(offsets), null)
    assert alpha[1].count_nonzero() == 0 and alpha[3].count_nonzero() == 0
    mass = torch.zeros(3, 3).index_add_(0, t(dst), alpha) + null_alpha
    torch.testing.assert_close(mass, torch.ones(3, 3), rtol=1e-5, atol=1e-6)


def test_known_answer_normalise_after_destination_sum():
    zonal = torch.tensor([[1e8], [-1e8 + 8], [1.0]])
    out = zonal_scatter_reference(zonal, torch.ones(3, 1, 1), torch.zeros(3, dtype=torch.int64),
                                  torch.zeros(1, dtype=torch.int64), torch.tensor([0.3]))
    torch.testing.assert_close(out[0, 1], zonal.sum(0) * 0.3, rtol=0, atol=0)


# ---- independent loops and the float64 truth -----------------------------------

def test_oracles_agree_with_loops_on_small_inputs():
    rng = np.random.default_rng(5)
    dst, offsets = _graph([3, 0, 4, 1, 6])
    e = dst.size
    src = rng.standard_normal((e, 5)).astype(np.float32)
    ws, ns = rng.random(e).astype(np.float32) + 0.5, rng.random(5).astype(np.float32) + 0.5
    want = np.array(loops.segment_sum(src.tolist(), offsets.tolist(), ws.tolist(), ns.tolist()))
    got = segment_sum_reference(t(src), t(dst), t(offsets), t(ws), t(ns)).numpy()
    np.testing.assert_allclose(got, want, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(truth.segment_sum(src, dst, 5, ws, ns), want, rtol=1e-12)

    logit = rng.standard_normal((e, 3)).astype(np.float32)
    env = np.where(rng.random(e) < 0.3, -0.5, rng.random(e) + 0.1).astype(np.float32)
    null = rng.standard_normal((5, 3)).astype(np.float32)
    la, ln = loops.segment_softmax(logit.tolist(), env.tolist(), offsets.tolist(), null.tolist())
    a, n0 = segment_softmax_reference(t(logit), t(env), t(dst), t(offsets), t(null))
    np.testing.assert_allclose(a.numpy(), la, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n0.numpy(), ln, rtol=1e-5, atol=1e-6)
    ta, tn = truth.segment_softmax(logit, env, dst, 5, null)
    np.testing.assert_allclose(ta, la, rtol=1e-12, atol=1e-15)

    srcn = rng.integers(0, 5, e)
    g3, v3 = rng.standard_normal((e, 3)), rng.standard_normal((e, 3))
    lf, lw = loops.force_assembly(g3.tolist(), v3.tolist(), srcn.tolist(), dst.tolist(), 5)
    tf, tw = truth.force_assembly(g3, v3, srcn, dst, 5)
    np.testing.assert_allclose(tf, lf, rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(tw, lw, rtol=1e-12, atol=1e-14)
