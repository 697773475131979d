"""Size-independent properties of the oracle on generated graphs (CPU).

The golden fixtures pin the oracle at fixed points; these properties hold for
every input, so they check it between the fixtures: the float64 truth
(``oracle/truth.py``) against the mathematics of each operator -- integer
CSR invariants, conservation, invariance under per-segment shifts, envelope
scaling and edge order, linearity, an independent dense formulation -- and
the fp32 restatement of the reference (``reference.*``) against the truth
within fp32 rounding.  Graphs include empty edge lists, nodes without edges,
all-masked segments and null logits.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch
from hypothesis import HealthCheck, example, given, settings
from hypothesis import strategies as st

from oracle import truth
from reference import (
    force_assembly_reference,
    rmsnorm,
    rotate_back_aggregate_reference,
    rmsnorm_per_degree,
    segment_attention_reference,
    segment_softmax_reference,
    segment_sum_reference,
    zonal_scatter_reference,
)

# Derandomised: the same examples every run, so the CPU suite is deterministic.
PROPS = settings(max_examples=60, deadline=None, derandomize=True, database=None,
                 suppress_health_check=[HealthCheck.too_slow])

# Fixed cases beside the generated ones: no edges at all, and a node (1) that
# no edge reaches.
NO_EDGES = (3, np.zeros(0, np.int64), np.zeros(0, np.int64), 1)
LONE_NODE = (3, np.array([0, 2, 2, 0], np.int64), np.array([2, 0, 1, 1], np.int64), 2)


@st.composite
def graphs(draw, max_nodes=9, max_edges=40):
    """(n_nodes, dst, src, seed): destinations in any order, sources independent;
    the seed draws the values."""
    n = draw(st.integers(1, max_nodes))
    e = draw(st.integers(0, max_edges))
    ids = st.lists(st.integers(0, n - 1), min_size=e, max_size=e)
    dst = np.array(draw(ids), dtype=np.int64)
    src = np.array(draw(ids), dtype=np.int64)
    return n, dst, src, draw(st.integers(0, 2**32 - 1))


def _t(a):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a))


def _envelope(rng, e, kind):
    if kind == "ones":
        return np.ones(e, np.float32)
    env = rng.uniform(0.05, 1.0, e).astype(np.float32)
    if kind == "some_zero":
        env[rng.uniform(size=e) < 0.4] = 0.0
    return env


@PROPS
@given(graphs())
@example(NO_EDGES)
@example(LONE_NODE)
def test_offsets_and_source_grouping_invariants(g):
    n, dst, src, _ = g
    off = truth.segment_offsets(dst, n)
    assert off[0] == 0 and off[-1] == dst.size and np.all(np.diff(off) >= 0)
    assert np.array_equal(np.diff(off), np.bincount(dst, minlength=n))
    assert np.array_equal(truth.dst_from_offsets(off), np.sort(dst))
    order, soff = truth.group_by_source(src, n)
    assert np.array_equal(np.sort(order), np.arange(src.size))  # a permutation
    keys = src[order]
    assert np.all(np.diff(keys) >= 0)  # grouped by source
    assert np.all(np.diff(order)[np.diff(keys) == 0] > 0)  # stable inside a group
    assert np.array_equal(truth.dst_from_offsets(soff), keys)
    with pytest.raises(ValueError, match="within the node range"):
        truth.segment_offsets(np.append(dst, n), n)


@PROPS
@given(graphs(), st.integers(1, 4), st.booleans(), st.sampled_from(["ones", "random", "some_zero"]))
@example(NO_EDGES, 2, True, "ones")
@example(LONE_NODE, 3, True, "some_zero")
@example(LONE_NODE, 1, False, "random")
def test_softmax_normalises_and_is_free_of_per_segment_factors(g, heads, with_null, env_kind):
    n, dst, _, seed = g
    rng = np.random.default_rng(seed)
    e = dst.size
    logit = rng.normal(size=(e, heads)) * 3
    env = _envelope(rng, e, env_kind).astype(np.float64)
    null = rng.normal(size=(n, heads)) if with_null else None
    alpha, null_alpha = truth.segment_softmax(logit, env, dst, n, null)
    assert np.all(alpha >= 0) and np.all(alpha[env == 0] == 0)
    # each segment's mass is one, or zero when every edge is masked and there
    # is no null logit
    mass = truth.segment_sum(alpha, dst, n) + (null_alpha if with_null else 0.0)
    live = (np.bincount(dst[env > 0], minlength=n) > 0)[:, None] | with_null
    np.testing.assert_allclose(mass, np.where(live, 1.0, 0.0) + 0 * mass, rtol=0, atol=1e-12)
    # a per-segment shift of every logit (and the null logit) changes nothing
    shift = rng.normal(size=(n, 1)) * 50
    shifted, shifted_null = truth.segment_softmax(
        logit + shift[dst], env, dst, n, None if null is None else null + shift)
    np.testing.assert_allclose(shifted, alpha, rtol=1e-9, atol=1e-12)
    if with_null:
        np.testing.assert_allclose(shifted_null, null_alpha, rtol=1e-9, atol=1e-12)
    else:
        # the envelope weighs by env^2: a per-segment factor on it cancels
        k = rng.uniform(0.2, 3.0, size=n)
        scaled, _ = truth.segment_softmax(logit, env * k[dst], dst, n, None)
        np.testing.assert_allclose(scaled, alpha, rtol=1e-9, atol=1e-12)


@PROPS
@given(graphs(), st.integers(1, 4), st.booleans(), st.sampled_from(["ones", "random", "some_zero"]))
@example(NO_EDGES, 2, True, "ones")
@example(LONE_NODE, 2, True, "some_zero")
def test_reference_softmax_and_attention_match_truth(g, heads, with_null, env_kind):
    n, dst, _, seed = g
    rng = np.random.default_rng(seed)
    e, dh = dst.size, 2
    logit = (rng.normal(size=(e, heads)) * 3).astype(np.float32)
    env = _envelope(rng, e, env_kind)
    null = rng.normal(size=(n, heads)).astype(np.float32) if with_null else None
    value = rng.normal(size=(e, 3, heads * dh)).astype(np.float32)
    off = _t(truth.segment_offsets(dst, n))
    alpha, null_alpha = segment_softmax_reference(_t(logit), _t(env), _t(dst), off, _t(null))
    want, want_null = truth.segment_softmax(logit, env, dst, n, null)
    np.testing.assert_allclose(alpha.numpy(), want, rtol=1e-5, atol=1e-6)
    if with_null:
        np.testing.assert_allclose(null_alpha.numpy(), want_null, rtol=1e-5, atol=1e-6)
    out = segment_attention_reference(_t(logit), _t(value), _t(dst), off, _t(env), _t(null))
    truth_out = truth.segment_attention(logit, value, dst, n, env, null)
    np.testing.assert_allclose(out.numpy(), truth_out, rtol=1e-5, atol=1e-5)
    # the weighted sum is linear in the values
    other = rng.normal(size=value.shape)
    mixed = truth.segment_attention(logit, 2.0 * value - 3.0 * other, dst, n, env, null)
    np.testing.assert_allclose(
        mixed, 2.0 * truth_out - 3.0 * truth.segment_attention(logit, other, dst, n, env, null),
        rtol=1e-9, atol=1e-9)


@PROPS
@given(graphs(), st.integers(1, 6), st.booleans(), st.booleans())
@example(NO_EDGES, 2, True, True)
@example(LONE_NODE, 3, True, True)
def test_segment_sum_is_the_incidence_product(g, channels, edge_scaled, node_scaled):
    n, dst, _, seed = g
    rng = np.random.default_rng(seed)
    e = dst.size
    src = rng.normal(size=(e, channels)).astype(np.float32)
    es = rng.uniform(-2, 2, size=e).astype(np.float32) if edge_scaled else None
    ns = rng.uniform(-2, 2, size=n).astype(np.float32) if node_scaled else None
    want = truth.segment_sum(src, dst, n, es, ns)
    incidence = np.zeros((n, e))
    incidence[dst, np.arange(e)] = 1.0
    terms = src.astype(np.float64) * (1.0 if es is None else es.astype(np.float64)[:, None])
    dense = (incidence @ terms) * (1.0 if ns is None else ns.astype(np.float64)[:, None])
    np.testing.assert_allclose(want, dense, rtol=1e-12, atol=1e-12)
    got = segment_sum_reference(_t(src), _t(dst), _t(truth.segment_offsets(dst, n)), _t(es), _t(ns))
    np.testing.assert_allclose(got.numpy(), want, rtol=1e-5, atol=1e-5)


@PROPS
@given(graphs())
@example(NO_EDGES)
@example(LONE_NODE)
def test_force_assembly_conserves_momentum(g):
    n, dst, src, seed = g
    rng = np.random.default_rng(seed)
    e = dst.size
    grad = rng.normal(size=(e, 3)).astype(np.float32)
    vec = rng.normal(size=(e, 3)).astype(np.float32)
    force, virial = truth.force_assembly(grad, vec, src, dst, n)
    size = 1.0 + float(np.abs(grad).sum())
    # every edge adds g to its destination and takes it from its source
    np.testing.assert_allclose(force.sum(axis=0), np.zeros(3), rtol=0, atol=1e-12 * size)
    outer = -(grad.astype(np.float64)[:, :, None] * vec.astype(np.float64)[:, None, :])
    np.testing.assert_allclose(virial.sum(axis=0), outer.reshape(e, 9).sum(axis=0),
                               rtol=1e-12, atol=1e-12 * size * 10)
    f32, v32 = force_assembly_reference(_t(grad), _t(vec), _t(src), _t(dst),
                                        _t(truth.segment_offsets(dst, n)),
                                        _t(truth.segment_offsets(src, n)))
    np.testing.assert_allclose(f32.numpy(), force, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(v32.numpy(), virial, rtol=1e-5, atol=1e-5)


@PROPS
@given(graphs(), st.integers(1, 5), st.integers(1, 3), st.integers(1, 4))
@example(NO_EDGES, 3, 2, 4)
@example(LONE_NODE, 3, 2, 4)
def test_zonal_scatter_ignores_edge_order_and_is_linear(g, rows, n_radial, channels):
    n, dst, _, seed = g
    rng = np.random.default_rng(seed)
    e = dst.size
    zonal = rng.normal(size=(e, rows)).astype(np.float32)
    radial = rng.normal(size=(e, n_radial, channels)).astype(np.float32)
    slot = rng.integers(0, n_radial, size=rows).astype(np.int64)
    inv = rng.uniform(0.1, 1.0, size=n).astype(np.float32)
    out = truth.zonal_scatter(zonal, radial, dst, slot, inv)
    assert np.all(out[:, 0, :] == 0)  # row zero is reserved
    perm = rng.permutation(e)
    np.testing.assert_allclose(truth.zonal_scatter(zonal[perm], radial[perm], dst[perm], slot, inv),
                               out, rtol=1e-12, atol=1e-12)
    other = rng.normal(size=radial.shape)
    np.testing.assert_allclose(
        truth.zonal_scatter(zonal, 2.0 * radial - other, dst, slot, inv),
        2.0 * out - truth.zonal_scatter(zonal, other, dst, slot, inv), rtol=1e-9, atol=1e-9)
    ref = zonal_scatter_reference(_t(zonal), _t(radial), _t(dst), _t(slot), _t(inv))
    np.testing.assert_allclose(ref.numpy(), out, rtol=1e-5, atol=1e-5)


@PROPS
@given(st.integers(1, 4), st.integers(0, 3), st.integers(1, 24), st.floats(0.01, 100.0),
       st.integers(0, 2**32 - 1))
def test_rmsnorm_has_unit_rms_and_no_scale(rows, degree, width, factor, seed):
    rng = np.random.default_rng(seed)
    comps = (degree + 1) ** 2
    x = rng.normal(size=(rows, comps, width))
    y, _ = truth.rmsnorm(x, eps=1e-30)
    np.testing.assert_allclose(np.sqrt((y * y).mean(axis=-1)), 1.0, rtol=1e-9)
    np.testing.assert_allclose(truth.rmsnorm(factor * x, eps=1e-30)[0], y, rtol=1e-9, atol=1e-12)
    x32 = x.astype(np.float32)
    scale = rng.uniform(0.5, 1.5, size=width).astype(np.float32)
    np.testing.assert_allclose(rmsnorm(_t(x32), _t(scale)).numpy(),
                               truth.rmsnorm(x32, scale, 1e-6)[0], rtol=1e-5, atol=1e-6)
    weight = rng.uniform(0.5, 1.5, size=(degree + 1, width)).astype(np.float32)
    np.testing.assert_allclose(rmsnorm_per_degree(_t(x32), _t(weight)).numpy(),
                               truth.rmsnorm(x32, weight, 1e-6, per_degree=True)[0],
                               rtol=1e-5, atol=1e-6)


def _orthogonal(rng, e, m):
    """e random orthogonal m x m matrices (QR with the signs fixed)."""
    q, r = np.linalg.qr(rng.normal(size=(e, m, m)))
    return q * np.sign(np.diagonal(r, axis1=1, axis2=2))[:, None, :]


@PROPS
@given(graphs(max_edges=24), st.integers(0, 3), st.integers(1, 3), st.integers(1, 3), st.booleans())
@example(NO_EDGES, 2, 2, 2, True)
@example(LONE_NODE, 3, 2, 1, False)
def test_rotate_back_undoes_orthogonal_rotations(g, lmax, heads, dh, rescaled):
    # x_local = D x_global per degree block with D orthogonal: the rotate-back
    # returns the weighted destination sum of x_global itself.
    n, dst, _, seed = g
    rng = np.random.default_rng(seed)
    e, comps, channels = dst.size, (lmax + 1) ** 2, heads * dh
    x_global = rng.normal(size=(e, comps, channels))
    x_local = np.empty_like(x_global)
    packed = []
    for l in range(lmax + 1):
        m = 2 * l + 1
        d = _orthogonal(rng, e, m)
        x_local[:, l * l:(l + 1) ** 2, :] = d @ x_global[:, l * l:(l + 1) ** 2, :]
        packed.append(d.reshape(e, m * m))
    rotation = np.concatenate(packed, axis=1) if e else np.zeros((0, truth.rotation_block_offsets(lmax)[-1]))
    alpha = rng.uniform(0.0, 1.0, size=(e, heads))
    rescale = rng.uniform(0.5, 2.0, size=e) if rescaled else None
    weight = np.repeat(alpha, dh, axis=1)[:, None, :] * (1.0 if rescale is None else rescale[:, None, None])
    want = truth.segment_sum((x_global * weight).reshape(e, comps * channels), dst, n)
    want = want.reshape(n, comps, channels)
    got = truth.rotate_back_aggregate(x_local, rotation, rescale, alpha, dst, n, lmax, heads)
    np.testing.assert_allclose(got, want, rtol=1e-9, atol=1e-9)
    f32 = [a.astype(np.float32) for a in (x_local, rotation, alpha)]
    r32 = None if rescale is None else rescale.astype(np.float32)
    ref = rotate_back_aggregate_reference(_t(f32[0]), _t(f32[1]), _t(r32), _t(f32[2]), None,
                                          _t(truth.segment_offsets(dst, n)), _t(dst), lmax, heads)
    np.testing.assert_allclose(ref.numpy(),
                               truth.rotate_back_aggregate(*f32[:2], r32, f32[2], dst, n, lmax, heads),
                               rtol=1e-5, atol=1e-5)


@PROPS
@given(st.integers(0, 6), st.integers(1, 4), st.integers(1, 5), st.integers(1, 4),
       st.integers(0, 2**32 - 1))
def test_edge_chain_adds_terms_and_applies_the_activation_last(e, comps, channels, n_terms, seed):
    rng = np.random.default_rng(seed)
    shape = (e, comps, channels)
    kinds = [shape, (e, 1, channels), (1, comps, 1), (e, comps, 1)]
    terms = []
    for t in range(n_terms):
        a = rng.normal(size=kinds[t % 4])
        coef = float(rng.uniform(-2, 2))
        terms.append((coef, a) if t % 2 else (coef, a, rng.normal(size=kinds[(t + 1) % 4])))
    lin = truth.edge_chain(terms, shape)
    np.testing.assert_allclose(lin, sum(truth.edge_chain([t], shape) for t in terms) + 0 * lin,
                               rtol=1e-12, atol=1e-12)
    doubled = [(2.0 * t[0],) + tuple(t[1:]) for t in terms]
    np.testing.assert_allclose(truth.edge_chain(doubled, shape), 2.0 * lin, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(truth.edge_chain(terms, shape, "silu"),
                               lin * truth.edge_chain(terms, shape, "sigmoid"), rtol=1e-12, atol=1e-12)
