"""Seeded randomised parity of every operator against the float64 oracle (B200).

Each case draws a segment-size mix (empty segments, tiny ones, ~90-edge ones
and a few giants that get split across warps), an operator width, optional
envelope / null logits and a permuted storage order, then compares the CUDA
path with ``oracle.truth``.  Tolerances: rtol 1e-5 with an absolute floor of
1e-5 of the largest magnitude (the reference's large-graph criterion).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import truth

pytestmark = pytest.mark.gpu

from bysj_b200 import _C  # noqa: E402
from bysj_b200 import kernels as K  # noqa: E402
from bysj_b200 import workloads as W  # noqa: E402


def close(got, want, rtol=1e-5):
    want = np.asarray(want)
    atol = 1e-5 * float(np.abs(want).max()) + 1e-6 if want.size else 1e-6
    np.testing.assert_allclose(np.asarray(got), want, rtol=rtol, atol=atol)


def draw_graph(rng):
    n = int(rng.integers(1, 400))
    kind = rng.random(n)
    sizes = np.where(kind < 0.15, 0, np.where(kind < 0.4, rng.integers(1, 8, n),
                                                rng.integers(60, 130, n)))
    for _ in range(int(rng.integers(0, 3))):
        sizes[rng.integers(0, n)] = int(rng.integers(2000, 6000))
    dst = np.repeat(np.arange(n), sizes).astype(np.int64)
    return n, sizes, dst


@pytest.mark.parametrize("seed", range(12))
def test_segmented_operators_fuzz(cuda, seed):
    rng = np.random.default_rng(seed)
    n, sizes, dst_np = draw_graph(rng)
    e = dst_np.size
    if e == 0:
        return
    dst = torch.from_numpy(dst_np).cuda()
    off = K.segment_offsets(dst, n)
    heads = int(rng.choice([1, 2, 4, 8, 16]))
    channels = heads * int(rng.choice([1, 2, 4, 8]))
    comps = int(rng.choice([1, 3, 16]))
    logit = rng.normal(0, 1.5, (e, heads)).astype(np.float32)
    env = np.where(rng.random(e) < 0.1, -0.5, rng.random(e) + 0.05).astype(np.float32)
    null = rng.normal(0, 1, (n, heads)).astype(np.float32)
    use_env, use_null = bool(rng.random() < 0.7), bool(rng.random() < 0.5)
    perm = rng.permutation(e) if rng.random() < 0.4 else None

    def stored(a):  # rows of `a` in storage order (slot s -> row perm[s])
        if perm is None:
            return torch.from_numpy(np.ascontiguousarray(a)).cuda()
        out = np.empty_like(a)
        out[perm] = a
        return torch.from_numpy(out).cuda()

    order = torch.from_numpy(perm).cuda() if perm is not None else None
    env_t = stored(env) if use_env else None
    null_t = torch.from_numpy(null).cuda() if use_null else None

    # softmax forward / backward
    env_for = env_t if env_t is not None else torch.ones(e, device="cuda")
    alpha, null_alpha = _C.segment_softmax_forward(stored(logit), env_for, off, null_t, order)
    wa, wn = truth.segment_softmax(logit, env if use_env else None, dst_np, n,
                                   null if use_null else None)
    got_alpha = alpha.cpu().numpy()[perm] if perm is not None else alpha.cpu().numpy()
    close(got_alpha, wa)
    if use_null:
        close(null_alpha.cpu().numpy(), wn)
    ga = rng.normal(0, 1, (e, heads)).astype(np.float32)
    gn = rng.normal(0, 1, (n, heads)).astype(np.float32) if use_null else None
    a64 = wa.astype(np.float64)
    S = np.zeros((n, heads))
    np.add.at(S, dst_np, a64 * ga)
    if use_null:
        S += wn * gn
    want_gl = a64 * (ga - S[dst_np])
    gl, gnl, genv = _C.segment_softmax_backward(
        stored(wa.astype(np.float32)), stored(ga), env_for, off,
        torch.from_numpy(wn.astype(np.float32)).cuda() if use_null else None,
        torch.from_numpy(gn).cuda() if use_null else None, order)
    got_gl = gl.cpu().numpy()[perm] if perm is not None else gl.cpu().numpy()
    close(got_gl, want_gl, rtol=1e-4)

    # segment sum with both scales
    src = rng.normal(0, 1, (e, channels)).astype(np.float32)
    ws = (rng.random(e) + 0.5).astype(np.float32)
    ns = (rng.random(n) + 0.5).astype(np.float32)
    out = _C.segment_sum_forward(stored(src), off, stored(ws), torch.from_numpy(ns).cuda(), order)
    close(out.cpu().numpy(), truth.segment_sum(src, dst_np, n, ws, ns))

    # fused attention
    value = rng.normal(0, 1, (e, comps, channels)).astype(np.float32)
    att = K.segment_attention(stored(logit), stored(value), off, env_t, null_t, order=order)
    close(att.cpu().numpy(), truth.segment_attention(logit, value, dst_np, n,
                                                     env if use_env else None,
                                                     null if use_null else None))


@pytest.mark.parametrize("seed", range(6))
def test_force_grouping_and_gie_fuzz(cuda, seed):
    rng = np.random.default_rng(100 + seed)
    n, sizes, dst_np = draw_graph(rng)
    e = dst_np.size
    if e == 0:
        return
    src_np = rng.integers(0, n, e).astype(np.int64)
    if rng.random() < 0.3:  # a hub atom that many edges leave
        src_np[rng.random(e) < 0.3] = int(rng.integers(0, n))
    dst, src = torch.from_numpy(dst_np).cuda(), torch.from_numpy(src_np).cuda()
    off = K.segment_offsets(dst, n)
    order, soff = K.group_by_source(src, n)
    wo, woff = truth.group_by_source(src_np, n)
    np.testing.assert_array_equal(order.cpu().numpy(), wo)
    np.testing.assert_array_equal(soff.cpu().numpy(), woff)
    g = rng.normal(0, 0.1, (e, 3)).astype(np.float32)
    v = rng.normal(0, 1, (e, 3)).astype(np.float32)
    force, virial = K.force_assembly(torch.from_numpy(g).cuda(), torch.from_numpy(v).cuda(),
                                     src, dst, off, soff, order)
    tf, tv = truth.force_assembly(g, v, src_np, dst_np, n)
    close(force.cpu().numpy(), tf)
    close(virial.cpu().numpy(), tv)

    lmax = int(rng.choice([1, 2, 3]))
    rows = (lmax + 1) ** 2 - 1
    channels = int(rng.choice([4, 16, 64]))
    zonal = rng.normal(0, 1, (e, rows)).astype(np.float32)
    radial = rng.normal(0, 1, (e, lmax + 1, channels)).astype(np.float32)
    slot = W.degree_slots(lmax, zero_based=bool(rng.random() < 0.5)).numpy()
    inv = (rng.random(n) + 0.2).astype(np.float32)
    shuffled = rng.permutation(e)
    zt = torch.from_numpy(zonal[shuffled]).cuda().requires_grad_(True)
    rt = torch.from_numpy(radial[shuffled]).cuda().requires_grad_(True)
    it = torch.from_numpy(inv).cuda().requires_grad_(True)
    dsh = torch.from_numpy(dst_np[shuffled]).cuda()
    out = K.zonal_scatter(zt, rt, dsh, torch.from_numpy(slot).cuda(), it)
    close(out.detach().cpu().numpy(),
          truth.zonal_scatter(zonal[shuffled], radial[shuffled], dst_np[shuffled], slot, inv))
    up = rng.normal(0, 1, (n, rows + 1, channels)).astype(np.float32)
    gz, gr, gi = torch.autograd.grad(out, (zt, rt, it), torch.from_numpy(up).cuda())
    # float64 gradients of out[n, r+1, c] = inv[n] sum_e z[e, r] radial[e, slot r, c]
    z64, r64, u64 = zonal[shuffled].astype(np.float64), radial[shuffled].astype(np.float64), \
        up.astype(np.float64)
    d = dst_np[shuffled]
    gi_up = u64[d, 1:, :] * inv.astype(np.float64)[d, None, None]
    want_gz = np.einsum("erc,erc->er", gi_up, r64[:, slot, :])
    want_gr = np.zeros_like(r64)
    for r_ in range(rows):
        want_gr[:, slot[r_], :] += gi_up[:, r_, :] * z64[:, r_:r_ + 1]
    pre = np.zeros((n, rows, channels))
    np.add.at(pre, d, z64[:, :, None] * r64[:, slot, :])
    want_gi = np.einsum("nrc,nrc->n", u64[:, 1:, :], pre)
    close(gz.cpu().numpy(), want_gz, rtol=2e-4)
    close(gr.cpu().numpy(), want_gr, rtol=2e-4)
    close(gi.cpu().numpy(), want_gi, rtol=2e-4)
