"""GPU parity of segment_offsets, segment_sum and segment_softmax (B200).

Each kernel is compared with the CPU oracle on the same seeded inputs
(rtol 1e-5 / atol 1e-6 for fp32, as the reference's device tests use
2e-5 / 2e-6), with the golden fixtures made from the reference's own code,
and at larger sizes with the float64 truth and an fp32 error budget
(``atol = 1e-5 * max|y|``, the reference's own large-graph criterion).
Integer outputs must be bit-exact; repeated runs bit-identical.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import truth
from reference import segment_softmax_reference, segment_sum_reference

pytestmark = pytest.mark.gpu

from bysj_b200 import _C  # noqa: E402
from bysj_b200 import kernels as K  # noqa: E402
from bysj_b200 import workloads as W  # noqa: E402


def graph(sizes, device="cuda"):
    sizes = torch.as_tensor(sizes, dtype=torch.int64)
    dst = torch.repeat_interleave(torch.arange(sizes.numel()), sizes)
    off = torch.zeros(sizes.numel() + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(sizes, 0)
    return dst.to(device), off.to(device)


def skewed_sizes(seed, nodes=300, giant=5000):
    gen = torch.Generator().manual_seed(seed)
    sizes = torch.randint(0, 12, (nodes,), generator=gen)
    sizes[nodes // 3] = giant
    sizes[nodes // 2] = 0
    sizes[-1] = giant // 2
    return sizes


def budget(expected):
    return 1e-5 * float(np.abs(expected).max()) + 1e-7


# ---- segment_offsets -----------------------------------------------------------

def test_offsets_bit_exact_sorted_and_unsorted(cuda):
    g = W.c1_box(device="cuda")
    got = K.segment_offsets(g.dst, g.n_atoms)
    want = truth.segment_offsets(g.dst.cpu().numpy(), g.n_atoms)
    np.testing.assert_array_equal(got.cpu().numpy(), want)
    gen = torch.Generator().manual_seed(1)
    src = torch.randint(0, 777, (50000,), generator=gen)
    got = K.segment_offsets(src.cuda(), 777)
    np.testing.assert_array_equal(got.cpu().numpy(), truth.segment_offsets(src.numpy(), 777))
    order, off = K.group_by_source(src.cuda(), 777)
    want_order, want_off = truth.group_by_source(src.numpy(), 777)
    np.testing.assert_array_equal(order.cpu().numpy(), want_order)
    np.testing.assert_array_equal(off.cpu().numpy(), want_off)


def test_offsets_edge_cases(cuda):
    dst, off = graph([2, 0, 3])
    assert torch.equal(K.segment_offsets(dst, 3), off)
    empty = torch.empty(0, dtype=torch.int64, device="cuda")
    assert K.segment_offsets(empty, 4).tolist() == [0, 0, 0, 0, 0]
    with pytest.raises(ValueError):
        K.segment_offsets(torch.tensor([0, 3], device="cuda"), 3)
    with pytest.raises(ValueError):
        K.segment_offsets(torch.tensor([2, -1], device="cuda"), 3)
    # many empty nodes between two edges (long boundary runs)
    dst = torch.tensor([0, 0, 9999], device="cuda")
    want = truth.segment_offsets(dst.cpu().numpy(), 10000)
    np.testing.assert_array_equal(K.segment_offsets(dst, 10000).cpu().numpy(), want)


def test_offsets_golden(cuda):
    g = golden("csr")
    n = g["offsets"].size - 1
    got = K.segment_offsets(torch.from_numpy(g["dst"]).cuda(), n)
    np.testing.assert_array_equal(got.cpu().numpy(), g["offsets"])
    order, off = K.group_by_source(torch.from_numpy(g["src"]).cuda(), n)
    np.testing.assert_array_equal(order.cpu().numpy(), g["src_order"])
    np.testing.assert_array_equal(off.cpu().numpy(), g["src_offsets"])


@pytest.mark.parametrize("case", ["small", "block", "scan", "mixed", "dense_tiles",
                                  "many_keys"])
def test_group_by_source_every_sort_regime(cuda, case):
    # groups of <= 256 edges (warp sort), 257..4096 (CTA sort), > 4096 (scan);
    # 65536 and 300000 random keys put more distinct keys in a 4096-edge tile
    # than the counting pass's shared-memory table holds (its direct-atomic path)
    gen = torch.Generator().manual_seed(len(case))
    n = {"small": 3000, "block": 40, "scan": 6, "mixed": 500, "dense_tiles": 65536,
         "many_keys": 300000}[case]
    e = {"small": 200000, "block": 60000, "scan": 60000, "mixed": 120000,
         "dense_tiles": 500000, "many_keys": 400000}[case]
    src = torch.randint(0, n, (e,), generator=gen)
    if case == "mixed":  # one giant, a few medium, many small and some empty keys
        src[: e // 3] = 7
        src[e // 3: e // 2] = torch.randint(100, 110, (e // 2 - e // 3,), generator=gen)
        src[src == 42] = 43
        src = src[torch.randperm(e, generator=gen)]
    order, off = K.group_by_source(src.cuda(), n)
    want_order, want_off = truth.group_by_source(src.numpy(), n)
    np.testing.assert_array_equal(off.cpu().numpy(), want_off)
    np.testing.assert_array_equal(order.cpu().numpy(), want_order)
    again, _ = K.group_by_source(src.cuda(), n)
    assert torch.equal(order, again)


def test_group_by_source_edge_cases(cuda):
    empty = torch.empty(0, dtype=torch.int64, device="cuda")
    order, off = K.group_by_source(empty, 3)
    assert order.numel() == 0 and off.tolist() == [0, 0, 0, 0]
    order, off = K.group_by_source(torch.tensor([2, 0, 2, 1, 0], device="cuda"), 3)
    assert order.tolist() == [1, 4, 3, 0, 2] and off.tolist() == [0, 2, 3, 5]
    with pytest.raises(ValueError):
        K.group_by_source(torch.tensor([0, 3], device="cuda"), 3)
    with pytest.raises(ValueError):
        K.group_by_source(torch.tensor([-1, 0], device="cuda"), 3)
    one = torch.zeros(5000, dtype=torch.int64, device="cuda")
    order, off = K.group_by_source(one, 1)
    assert torch.equal(order.cpu(), torch.arange(5000)) and off.tolist() == [0, 5000]


# ---- segment_sum -----------------------------------------------------------------

@pytest.mark.parametrize("channels", [1, 3, 8, 17, 64, 640, 1024, 1500])
def test_segment_sum_matches_oracle(cuda, channels):
    dst, off = graph([2, 0, 3, 7, 1, 0, 11, 4])
    e = dst.numel()
    gen = torch.Generator().manual_seed(channels)
    src = torch.randn(e, channels, generator=gen)
    ws, ns = torch.rand(e, generator=gen) + 0.5, torch.rand(8, generator=gen) + 0.5
    got = K.segment_sum(src.cuda(), dst, off, ws.cuda(), ns.cuda())
    want = segment_sum_reference(src, dst.cpu(), off.cpu(), ws, ns)
    torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=1e-6)
    assert got[1].count_nonzero() == 0 and got[5].count_nonzero() == 0


def test_segment_sum_golden_forward_and_backward(cuda):
    g = golden("segment_sum")
    src = torch.from_numpy(g["src"]).cuda().requires_grad_(True)
    ns = torch.from_numpy(g["node_scale"]).cuda().requires_grad_(True)
    dst, off = torch.from_numpy(g["dst"]).cuda(), torch.from_numpy(g["offsets"]).cuda()
    out = K.segment_sum(src, dst, off, torch.from_numpy(g["edge_scale"]).cuda(), ns)
    np.testing.assert_allclose(out.detach().cpu().numpy(), g["out"], rtol=1e-5, atol=1e-6)
    gs, gn = torch.autograd.grad(out, (src, ns), torch.from_numpy(g["upstream"]).cuda())
    np.testing.assert_allclose(gs.cpu().numpy(), g["grad_src"], rtol=2e-5, atol=2e-6)
    np.testing.assert_allclose(gn.cpu().numpy(), g["grad_node_scale"], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("channels", [4, 48, 1024])
def test_segment_sum_skewed_degrees_split_segments(cuda, channels):
    sizes = skewed_sizes(channels)
    dst, off = graph(sizes)
    e = dst.numel()
    gen = torch.Generator().manual_seed(7)
    src = torch.randn(e, channels, generator=gen)
    ns = torch.rand(sizes.numel(), generator=gen) + 0.5
    got = K.segment_sum(src.cuda(), dst, off, None, ns.cuda())
    want = truth.segment_sum(src.numpy(), dst.cpu().numpy(), sizes.numel(), None, ns.numpy())
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=budget(want))
    again = K.segment_sum(src.cuda(), dst, off, None, ns.cuda())
    assert torch.equal(got, again), "repeated runs must be bit-identical"


@pytest.mark.parametrize("channels,permuted", [(4, False), (64, True), (256, False), (512, True), (1024, True)])
def test_segment_sum_backward_both_gradients(cuda, channels, permuted):
    # grad_src[e] = upstream[dst e] w[e] s[dst e];  grad_s[n] = sum_e w[e] <upstream[n], src[e]>
    # on skewed degrees (split segments), rows in storage order or permuted.
    sizes = skewed_sizes(channels, nodes=200, giant=3000)
    dst, off = graph(sizes)
    e, n = dst.numel(), sizes.numel()
    gen = torch.Generator().manual_seed(channels)
    src = torch.randn(e, channels, generator=gen)
    w, s = torch.rand(e, generator=gen) + 0.5, torch.rand(n, generator=gen) + 0.5
    up = torch.randn(n, channels, generator=gen)
    order = torch.randperm(e, generator=gen) if permuted else None
    stored, stored_w = src, w
    if permuted:  # logical edge i lives at storage row order[i], with its scale
        stored, stored_w = torch.empty_like(src), torch.empty_like(w)
        stored[order], stored_w[order] = src, w
    args = (up.cuda(), stored.cuda(), dst, off, stored_w.cuda(), s.cuda(), True,
            order.cuda() if permuted else None)
    gs, gn = _C.segment_sum_backward(*args)
    d = dst.cpu().numpy()
    u64, x64, w64, s64 = (t.double().numpy() for t in (up, src, w, s))
    want_gs = u64[d] * (w64 * s64[d])[:, None]
    want_gn = np.zeros(n)
    np.add.at(want_gn, d, w64 * np.einsum("ec,ec->e", u64[d], x64))
    got_gs = gs.cpu().numpy()[order.numpy()] if permuted else gs.cpu().numpy()
    np.testing.assert_allclose(got_gs, want_gs, rtol=1e-5, atol=budget(want_gs))
    np.testing.assert_allclose(gn.cpu().numpy(), want_gn, rtol=1e-4, atol=budget(want_gn))
    gs2, gn2 = _C.segment_sum_backward(*args)
    assert torch.equal(gs, gs2) and torch.equal(gn, gn2), "repeated runs must be bit-identical"


def test_segment_sum_order_permutation_and_bf16(cuda):
    g = W.c1_box(device="cuda")
    off = K.segment_offsets(g.dst, g.n_atoms)
    gen = torch.Generator(device="cuda").manual_seed(3)
    src = torch.randn(g.n_edges, 64, device="cuda", generator=gen)
    perm = torch.randperm(g.n_edges, device="cuda", generator=gen)
    shuffled = torch.empty_like(src)
    shuffled[perm] = src  # edge e of the grouped list lives at row perm[e]
    got = K.segment_sum(shuffled, g.dst, off, order=perm)
    want = truth.segment_sum(src.cpu().numpy(), g.dst.cpu().numpy(), g.n_atoms)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=budget(want))
    bf = src.to(torch.bfloat16)
    got16 = K.segment_sum(bf, g.dst, off)
    want16 = truth.segment_sum(bf.float().cpu().numpy(), g.dst.cpu().numpy(), g.n_atoms)
    np.testing.assert_allclose(got16.cpu().numpy(), want16, rtol=1e-2, atol=1e-2)


def test_segment_sum_large_graph_matches_float64(cuda):
    torch.manual_seed(11)
    atoms, edges, channels = 64, 4096, 32
    dst = torch.sort(torch.randint(0, atoms, (edges,), device="cuda")).values
    off = K.segment_offsets(dst, atoms)
    src = torch.randn(edges, channels, device="cuda")
    ns = torch.rand(atoms, device="cuda") + 0.5
    got = K.segment_sum(src, dst, off, None, ns)
    want = truth.segment_sum(src.cpu().numpy(), dst.cpu().numpy(), atoms, None, ns.cpu().numpy())
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=budget(want))


def test_segment_sum_empty_edges(cuda):
    off = torch.zeros(4, dtype=torch.int64, device="cuda")
    src = torch.empty(0, 5, device="cuda")
    out = K.segment_sum(src, torch.empty(0, dtype=torch.int64, device="cuda"), off)
    assert out.shape == (3, 5) and out.count_nonzero() == 0


# ---- segment_softmax -------------------------------------------------------------

def test_segment_softmax_golden_forward_and_backward(cuda):
    g = golden("segment_softmax")
    logit = torch.from_numpy(g["logit"]).cuda().requires_grad_(True)
    env = torch.from_numpy(g["env"]).cuda().requires_grad_(True)
    null = torch.from_numpy(g["null_logit"]).cuda().requires_grad_(True)
    off = torch.from_numpy(g["offsets"]).cuda()
    alpha, null_alpha = K.segment_softmax(logit, env, off, null)
    np.testing.assert_allclose(alpha.detach().cpu().numpy(), g["alpha"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(null_alpha.detach().cpu().numpy(), g["null_alpha"], rtol=1e-5,
                               atol=1e-6)
    grads = torch.autograd.grad(
        (alpha, null_alpha), (logit, env, null),
        (torch.from_numpy(g["grad_alpha"]).cuda(), torch.from_numpy(g["grad_null_alpha"]).cuda()))
    for got, key in zip(grads, ("grad_logit", "grad_env", "grad_null_logit")):
        np.testing.assert_allclose(got.cpu().numpy(), g[key], rtol=2e-4, atol=2e-5)
    plain = K.segment_softmax(logit.detach(), env.detach(), off)
    np.testing.assert_allclose(plain.cpu().numpy(), g["alpha_nonull"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("channels", [1, 3, 8, 16, 64, 256, 300])
def test_segment_softmax_matches_oracle(cuda, channels):
    sizes = [2, 0, 3, 1, 9, 4]
    dst, off = graph(sizes)
    e = dst.numel()
    gen = torch.Generator().manual_seed(channels)
    logit = torch.randn(e, channels, generator=gen)
    env = torch.where(torch.rand(e, generator=gen) < 0.25, torch.tensor(-0.3),
                      torch.rand(e, generator=gen) + 0.1)
    null = torch.randn(len(sizes), channels, generator=gen)
    a, n0 = K.segment_softmax(logit.cuda(), env.cuda(), off, null.cuda())
    wa, wn = segment_softmax_reference(logit, env, dst.cpu(), off.cpu(), null)
    torch.testing.assert_close(a.cpu(), wa, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(n0.cpu(), wn, rtol=1e-5, atol=1e-6)
    # gradients through the closed-form backward kernels
    lg = logit.cuda().requires_grad_(True)
    ev = env.abs().cuda().requires_grad_(True)
    nl = null.cuda().requires_grad_(True)
    a, n0 = K.segment_softmax(lg, ev, off, nl)
    ua, un = torch.randn_like(a), torch.randn_like(n0)
    got = torch.autograd.grad((a, n0), (lg, ev, nl), (ua, un))
    rl, re, rn = (x.detach().cpu().requires_grad_(True) for x in (lg, ev, nl))
    ra, rnull = segment_softmax_reference(rl, re, dst.cpu(), off.cpu(), rn)
    want = torch.autograd.grad((ra, rnull), (rl, re, rn), (ua.cpu(), un.cpu()))
    for x, y in zip(got, want):
        torch.testing.assert_close(x.cpu(), y, rtol=2e-4, atol=2e-5)


def test_segment_softmax_skewed_split_segments(cuda):
    sizes = skewed_sizes(5, nodes=200, giant=6000)
    dst, off = graph(sizes)
    e = dst.numel()
    gen = torch.Generator().manual_seed(9)
    logit = torch.randn(e, 8, generator=gen) * 2
    env = torch.rand(e, generator=gen) + 0.05
    null = torch.randn(sizes.numel(), 8, generator=gen)
    a, n0 = K.segment_softmax(logit.cuda(), env.cuda(), off, null.cuda())
    wa, wn = truth.segment_softmax(logit.numpy(), env.numpy(), dst.cpu().numpy(), sizes.numel(),
                                   null.numpy())
    np.testing.assert_allclose(a.cpu().numpy(), wa, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n0.cpu().numpy(), wn, rtol=1e-5, atol=1e-6)
    a2, _ = K.segment_softmax(logit.cuda(), env.cuda(), off, null.cuda())
    assert torch.equal(a, a2)
    # backward on the split path
    ga, gn = torch.randn_like(a), torch.randn_like(n0)
    ext = __import__("bysj_b200._C", fromlist=["_C"])
    gl, gnl, genv = ext.segment_softmax_backward(a, ga, env.cuda(), off, n0, gn)
    S = torch.zeros(sizes.numel(), 8, dtype=torch.float64).index_add_(
        0, dst.cpu(), (a * ga).double().cpu()) + (n0 * gn).double().cpu()
    want_gl = a.double().cpu() * (ga.double().cpu() - S[dst.cpu()])
    np.testing.assert_allclose(gl.cpu().numpy(), want_gl.numpy(), rtol=1e-4, atol=1e-6)
    want_env = want_gl.sum(1) * 2.0 / env.double()
    np.testing.assert_allclose(genv.cpu().numpy(), want_env.numpy(), rtol=1e-4, atol=1e-5)
    want_gnl = n0.double().cpu() * (gn.double().cpu() - S)
    np.testing.assert_allclose(gnl.cpu().numpy(), want_gnl.numpy(), rtol=1e-4, atol=1e-6)
    # the same rows stored in a permuted order and addressed through `order`
    perm = torch.randperm(e, generator=gen)
    ap, gp, ep = (torch.empty_like(t) for t in (a, ga, env.cuda()))
    ap[perm.cuda()], gp[perm.cuda()], ep[perm.cuda()] = a, ga, env.cuda()
    glp, _, genvp = ext.segment_softmax_backward(ap, gp, ep, off, n0, gn, order=perm.cuda())
    np.testing.assert_allclose(glp[perm.cuda()].cpu().numpy(), want_gl.numpy(), rtol=1e-4,
                               atol=1e-6)
    np.testing.assert_allclose(genvp[perm.cuda()].cpu().numpy(), want_env.numpy(), rtol=1e-4,
                               atol=1e-5)


@pytest.mark.parametrize("heads", [4, 8, 16])
def test_segment_softmax_forward_permuted_storage(cuda, heads):
    # rows stored in a permuted order and addressed through `order` (the layout
    # of an edge list that is not grouped by destination), with envelopes,
    # masked edges, a null logit and one segment longer than a chunk
    sizes = skewed_sizes(heads, nodes=300, giant=700)
    dst, off = graph(sizes)
    e, n = dst.numel(), sizes.numel()
    gen = torch.Generator().manual_seed(heads)
    logit = torch.randn(e, heads, generator=gen) * 2
    env = torch.where(torch.rand(e, generator=gen) < 0.1, torch.tensor(-1.0),
                      torch.rand(e, generator=gen) + 0.05)
    null = torch.randn(n, heads, generator=gen)
    perm = torch.randperm(e, generator=gen)
    lp, ep = torch.empty_like(logit), torch.empty_like(env)
    lp[perm], ep[perm] = logit, env
    a, n0 = K.segment_softmax(lp.cuda(), ep.cuda(), off, null.cuda(), order=perm.cuda())
    wa, wn = truth.segment_softmax(logit.numpy(), env.numpy(), dst.cpu().numpy(), n, null.numpy())
    np.testing.assert_allclose(a[perm.cuda()].cpu().numpy(), wa, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n0.cpu().numpy(), wn, rtol=1e-5, atol=1e-6)
    a2, _ = K.segment_softmax(lp.cuda(), ep.cuda(), off, null.cuda(), order=perm.cuda())
    assert torch.equal(a, a2), "repeated runs must be bit-identical"


# Segment lengths at the edges of the per-lane row-slot forms: the whole-
# segment kernels take a shorter unrolled form for segments within 3/4 (H =
# 4, 16: 96 rows) or 7/8 (H = 8: 112 rows) of a 128-row chunk, the staged
# backward within 96 rows, the permuted-storage forward within 112 (H = 8) or
# 96 (H = 4, chunk 256) rows; longer segments take the full form or the
# multi-chunk path.
BOUNDARY_SIZES = [1, 95, 96, 97, 111, 112, 113, 127, 128, 129, 255, 256, 257, 40, 0, 3]


@pytest.mark.parametrize("heads", [4, 8, 16])
def test_segment_softmax_row_slot_boundaries(cuda, heads):
    dst, off = graph(BOUNDARY_SIZES)
    e, n = dst.numel(), len(BOUNDARY_SIZES)
    gen = torch.Generator().manual_seed(100 + heads)
    logit = torch.randn(e, heads, generator=gen) * 2
    env = torch.where(torch.rand(e, generator=gen) < 0.1, torch.tensor(-1.0),
                      torch.rand(e, generator=gen) + 0.05)
    null = torch.randn(n, heads, generator=gen)
    a, n0 = K.segment_softmax(logit.cuda(), env.cuda(), off, null.cuda())
    wa, wn = segment_softmax_reference(logit, env, dst.cpu(), off.cpu(), null)
    torch.testing.assert_close(a.cpu(), wa, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(n0.cpu(), wn, rtol=1e-5, atol=1e-6)
    # backward through the closed-form kernels
    lg = logit.cuda().requires_grad_(True)
    ev = env.abs().cuda().requires_grad_(True)
    nl = null.cuda().requires_grad_(True)
    a, n0 = K.segment_softmax(lg, ev, off, nl)
    ua, un = torch.randn_like(a), torch.randn_like(n0)
    got = torch.autograd.grad((a, n0), (lg, ev, nl), (ua, un))
    rl, re, rn = (x.detach().cpu().requires_grad_(True) for x in (lg, ev, nl))
    ra, rnull = segment_softmax_reference(rl, re, dst.cpu(), off.cpu(), rn)
    want = torch.autograd.grad((ra, rnull), (rl, re, rn), (ua.cpu(), un.cpu()))
    for x, y in zip(got, want):
        torch.testing.assert_close(x.cpu(), y, rtol=2e-4, atol=2e-5)
    # the same rows in a permuted storage order
    perm = torch.randperm(e, generator=gen)
    lp, ep = torch.empty_like(logit), torch.empty_like(env)
    lp[perm], ep[perm] = logit, env
    ap, np0 = K.segment_softmax(lp.cuda(), ep.cuda(), off, null.cuda(), order=perm.cuda())
    torch.testing.assert_close(ap[perm.cuda()].cpu(), wa, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(np0.cpu(), wn, rtol=1e-5, atol=1e-6)
    # and the backward in that order (the gather kernel at H = 8) against the
    # storage-order backward of the same rows
    ext = __import__("bysj_b200._C", fromlist=["_C"])
    a, n0 = a.detach(), n0.detach()
    plain = ext.segment_softmax_backward(a, ua, ev.detach(), off, n0, un)
    pa, pu, pe = (torch.empty_like(t) for t in (a, ua, ev))
    pa[perm.cuda()], pu[perm.cuda()], pe[perm.cuda()] = a, ua, ev.detach()
    gl_p, gnl_p, genv_p = ext.segment_softmax_backward(pa, pu, pe, off, n0, un,
                                                       order=perm.cuda())
    torch.testing.assert_close(gl_p[perm.cuda()], plain[0], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(gnl_p, plain[1], rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(genv_p[perm.cuda()], plain[2], rtol=1e-5, atol=1e-5)


def test_segment_softmax_all_masked_segment_is_zero(cuda):
    dst, off = graph([3, 2])
    logit = torch.randn(5, 4, device="cuda")
    env = torch.tensor([-1.0, 0.0, -2.0, 0.5, 0.7], device="cuda")
    a = K.segment_softmax(logit, env, off)
    assert a[:3].count_nonzero() == 0
    torch.testing.assert_close(a[3:].sum(0), torch.ones(4, device="cuda"))


@pytest.mark.parametrize("heads", [8, 4, 16])
def test_segment_softmax_hub_segments(cuda, heads):
    # Hubs (100k, 30k, 20k, 12k and 5k edges) among 3000 short segments: the
    # whole-segment kernel shares them among the partitions they span and the
    # dependent hub pass writes their weights.  Every weight, with env and null
    # logit, against the float64 truth at rtol 1e-5 / atol 1e-6; the short
    # segments also against the fp32 oracle.  (The fp32 oracle's own
    # normalisation sum over a 100k-edge segment carries relative errors of a
    # few 1e-5, so the hubs are held to the exact values.)  Repeats
    # bit-identical.
    gen = torch.Generator().manual_seed(heads)
    sizes = torch.randint(20, 120, (3000,), generator=gen)
    sizes[1234], sizes[2999], sizes[0] = 100_000, 20_000, 5000
    sizes[1500], sizes[1501] = 30_000, 12_000  # adjacent hubs: a partition ends one, starts one
    dst, off = graph(sizes)
    e = dst.numel()
    logit = torch.randn(e, heads, generator=gen) * 2
    env = torch.where(torch.rand(e, generator=gen) < 0.1, torch.tensor(0.0),
                      torch.rand(e, generator=gen) + 0.05)
    null = torch.randn(sizes.numel(), heads, generator=gen)
    a, n0 = K.segment_softmax(logit.cuda(), env.cuda(), off, null.cuda())
    ta, tn = truth.segment_softmax(logit.numpy(), env.numpy(), dst.cpu().numpy(),
                                   sizes.numel(), null.numpy())
    np.testing.assert_allclose(a.cpu().numpy(), ta, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n0.cpu().numpy(), tn, rtol=1e-5, atol=1e-6)
    wa, wn = segment_softmax_reference(logit, env, dst.cpu(), off.cpu(), null)
    short = (sizes < 4096)[dst.cpu()]
    torch.testing.assert_close(a.cpu()[short], wa[short], rtol=1e-5, atol=1e-6)
    a2, n2 = K.segment_softmax(logit.cuda(), env.cuda(), off, null.cuda())
    assert torch.equal(a, a2) and torch.equal(n0, n2)
    # plain (no null, all-ones env) takes the same path
    ones = torch.ones(e)
    got = K.segment_softmax(logit.cuda(), ones.cuda(), off)
    want, _ = truth.segment_softmax(logit.numpy(), ones.numpy(), dst.cpu().numpy(), sizes.numel())
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-6)


def test_segment_softmax_single_hub_frame(cuda):
    # One 50,000-edge segment is the whole frame: every partition but the first
    # holds only a slice of it.
    gen = torch.Generator().manual_seed(11)
    dst, off = graph([50_000])
    logit = torch.randn(50_000, 8, generator=gen) * 3
    env = torch.rand(50_000, generator=gen) + 0.01
    null = torch.randn(1, 8, generator=gen)
    a, n0 = K.segment_softmax(logit.cuda(), env.cuda(), off, null.cuda())
    ta, tn = truth.segment_softmax(logit.numpy(), env.numpy(), dst.cpu().numpy(), 1, null.numpy())
    np.testing.assert_allclose(a.cpu().numpy(), ta, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(n0.cpu().numpy(), tn, rtol=1e-5, atol=1e-6)
