"""GPU parity of the fused rotate-back aggregation (B200).

``kernels.rotate_back_aggregate`` against the fp32 oracle
``reference.rotate_back_aggregate_reference`` at rtol 1e-5 / atol 1e-6 and
against the float64 ``oracle.truth``: every degree 0..3, channel widths that
select each lane layout (1, 2 or 4 channels per lane, one or several column
tiles), per-edge rescale or none, empty segments, segments split over many
warps (a 5000-edge hub), permuted storage (``order``), bit-identical repeats,
the reduction to ``segment_attention`` for identity rotations, and the
24576-atom C3 geometry at its full size (every output against a float64
evaluation on the GPU, a segment sample against the fp32 oracle).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import truth
from reference import rotate_back_aggregate_reference

pytestmark = pytest.mark.gpu

from bysj_b200 import kernels as K  # noqa: E402
from bysj_b200 import workloads as W  # noqa: E402
from test_gpu_segment import graph, skewed_sizes  # noqa: E402


def orthogonal_pool(count, lmax, gen, device="cpu"):
    """``count`` packed rows of random orthogonal degree blocks."""
    blocks = []
    for l in range(lmax + 1):
        m = 2 * l + 1
        a = torch.randn(count, m, m, generator=gen, dtype=torch.float64)
        q, _ = torch.linalg.qr(a)
        blocks.append(q.reshape(count, m * m))
    return torch.cat(blocks, dim=1).float().to(device)


def segment_softmax_weights(logit, dst, n):
    """Per-head attention weights normalised over each destination segment."""
    peak = torch.full((n, logit.shape[1]), -float("inf"), device=logit.device)
    peak = peak.scatter_reduce(0, dst[:, None].expand(-1, logit.shape[1]), logit, "amax")
    w = torch.exp(logit - peak[dst])
    total = torch.zeros_like(peak).index_add_(0, dst, w)
    return (w / total[dst]).contiguous()


def make_case(sizes, lmax, heads, channels, seed, rescale=True):
    gen = torch.Generator().manual_seed(seed)
    dst, off = graph(sizes, device="cpu")
    e, n = dst.numel(), off.numel() - 1
    x = torch.randn(e, (lmax + 1) ** 2, channels, generator=gen)
    rot = orthogonal_pool(e, lmax, gen)
    alpha = segment_softmax_weights(torch.randn(e, heads, generator=gen) * 2, dst, n)
    scale = (torch.rand(e, generator=gen) + 0.5) if rescale else None
    return x, rot, scale, alpha, off, dst


def run(x, rot, scale, alpha, off, dst, lmax, heads, order=None):
    cuda = lambda t: None if t is None else t.cuda()  # noqa: E731
    return K.rotate_back_aggregate(cuda(x), cuda(rot), cuda(scale), cuda(alpha), cuda(order),
                                   cuda(off), cuda(dst), lmax, heads)


@pytest.mark.parametrize("lmax,heads,channels,rescale", [
    (3, 8, 64, True), (3, 8, 64, False), (3, 4, 32, True), (3, 8, 128, True),
    (2, 2, 12, True), (2, 4, 16, False), (1, 1, 3, True), (0, 2, 8, True), (3, 3, 48, True),
    (1, 4, 256, False)])
def test_rotate_back_matches_oracles(cuda, lmax, heads, channels, rescale):
    sizes = [3, 0, 7, 1, 12, 0, 5, 40, 2]
    x, rot, scale, alpha, off, dst = make_case(sizes, lmax, heads, channels,
                                               seed=lmax * 100 + channels, rescale=rescale)
    got = run(x, rot, scale, alpha, off, dst, lmax, heads)
    assert tuple(got.shape) == (len(sizes), (lmax + 1) ** 2, channels)
    want = rotate_back_aggregate_reference(x, rot, scale, alpha, None, off, dst, lmax, heads)
    torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=1e-6)
    want64 = truth.rotate_back_aggregate(x.numpy(), rot.numpy(),
                                         None if scale is None else scale.numpy(),
                                         alpha.numpy(), dst.numpy(), len(sizes), lmax, heads)
    np.testing.assert_allclose(got.cpu().numpy(), want64, rtol=1e-5, atol=1e-6)
    assert got[1].abs().max() == 0 and got[5].abs().max() == 0  # empty segments


def test_rotate_back_split_hub_order_and_determinism(cuda):
    sizes = skewed_sizes(8, nodes=300, giant=5000)
    x, rot, scale, alpha, off, dst = make_case(sizes, 3, 8, 64, seed=8)
    got = run(x, rot, scale, alpha, off, dst, 3, 8)
    want = truth.rotate_back_aggregate(x.numpy(), rot.numpy(), scale.numpy(), alpha.numpy(),
                                       dst.numpy(), sizes.numel(), 3, 8)
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=1e-6)
    assert torch.equal(got, run(x, rot, scale, alpha, off, dst, 3, 8))
    # permuted storage: slot s holds edge perm[s]
    gen = torch.Generator().manual_seed(9)
    e = dst.numel()
    perm = torch.randperm(e, generator=gen)
    xp, rp, sp, ap = (torch.empty_like(t) for t in (x, rot, scale, alpha))
    xp[perm], rp[perm], sp[perm], ap[perm] = x, rot, scale, alpha
    dp = torch.empty_like(dst)
    dp[perm] = dst
    got_p = run(xp, rp, sp, ap, off, dp, 3, 8, order=perm)
    np.testing.assert_allclose(got_p.cpu().numpy(), want, rtol=1e-5, atol=1e-6)


def test_identity_rotations_reduce_to_segment_attention(cuda):
    g = W.c1_box(device="cuda")
    off = K.segment_offsets(g.dst, g.n_atoms)
    gen = torch.Generator(device="cuda").manual_seed(10)
    logit = torch.randn(g.n_edges, 8, device="cuda", generator=gen) * 2
    value = torch.randn(g.n_edges, 16, 64, device="cuda", generator=gen)
    alpha = segment_softmax_weights(logit, g.dst, g.n_atoms)
    eye = torch.cat([torch.eye(2 * l + 1, device="cuda").reshape(1, -1) for l in range(4)], 1)
    rot = eye.expand(g.n_edges, -1).contiguous()
    got = K.rotate_back_aggregate(value, rot, None, alpha, None, off, g.dst, 3, 8)
    att = K.segment_attention(logit, value, off)          # [N, H, S, dh]
    want = att.permute(0, 2, 1, 3).reshape(g.n_atoms, 16, 64)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)


def test_rotate_back_validation(cuda):
    x, rot, scale, alpha, off, dst = make_case([2, 1], 1, 2, 4, seed=1)
    args = [t.cuda() for t in (x, rot, scale, alpha)]
    with pytest.raises(ValueError):
        K.rotate_back_aggregate(args[0], args[1][:, :9], args[2], args[3], None, off.cuda(),
                                dst.cuda(), 1, 2)
    with pytest.raises(ValueError):
        K.rotate_back_aggregate(*args, None, off.cuda(), dst.cuda(), 2, 2)
    with pytest.raises(TypeError):
        K.rotate_back_aggregate(args[0].double(), *args[1:], None, off.cuda(), dst.cuda(), 1, 2)
    with pytest.raises(RuntimeError):
        K.rotate_back_aggregate(args[0].requires_grad_(True), *args[1:], None, off.cuda(),
                                dst.cuda(), 1, 2)


def test_rotate_back_c3_full_frame(cuda):
    g = W.c3_box(device="cuda", seed=0)
    e, n = g.n_edges, g.n_atoms
    off = K.segment_offsets(g.dst, n)
    gen = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(e, 16, 64, device="cuda", generator=gen)
    pool = orthogonal_pool(4096, 3, torch.Generator().manual_seed(12), device="cuda")
    rot = pool[torch.arange(e, device="cuda") % 4096].contiguous()
    alpha = segment_softmax_weights(torch.randn(e, 8, device="cuda", generator=gen) * 2 ** 0.5,
                                    g.dst, n)
    scale = torch.rand(e, device="cuda", generator=gen) + 0.5
    got = K.rotate_back_aggregate(x, rot, scale, alpha, None, off, g.dst, 3, 8)
    # float64 on the GPU, chunked over edges
    want = torch.zeros(n, 16, 64, dtype=torch.float64, device="cuda")
    offs = truth.rotation_block_offsets(3)
    for a in range(0, e, 1 << 18):
        b = min(e, a + (1 << 18))
        xs = x[a:b].double()
        y = torch.empty_like(xs)
        for l in range(4):
            m = 2 * l + 1
            d = rot[a:b, offs[l]:offs[l + 1]].double().reshape(b - a, m, m)
            y[:, l * l:(l + 1) ** 2] = torch.bmm(d.transpose(1, 2), xs[:, l * l:(l + 1) ** 2])
        w = alpha[a:b].double().repeat_interleave(8, dim=1)[:, None, :] * scale[a:b, None, None]
        want.index_add_(0, g.dst[a:b], y * w)
    diff = (got.double() - want).abs()
    bound = 1e-6 + 1e-5 * want.abs()
    assert int((diff > bound).sum()) == 0, float((diff / bound).max())
    # a seeded sample of segments against the fp32 oracle on the CPU
    off_cpu = off.cpu()
    segs = torch.unique(torch.randperm(n, generator=torch.Generator().manual_seed(13))[:1024])
    idx = torch.cat([torch.arange(int(off_cpu[s]), int(off_cpu[s + 1])) for s in segs])
    sizes = off_cpu[segs + 1] - off_cpu[segs]
    sub_dst = torch.repeat_interleave(torch.arange(segs.numel()), sizes)
    sub_off = torch.zeros(segs.numel() + 1, dtype=torch.int64)
    sub_off[1:] = torch.cumsum(sizes, 0)
    ic = idx.cuda()
    ref = rotate_back_aggregate_reference(x[ic].cpu(), rot[ic].cpu(), scale[ic].cpu(),
                                          alpha[ic].cpu(), None, sub_off, sub_dst, 3, 8)
    torch.testing.assert_close(got[segs.cuda()].cpu(), ref, rtol=1e-5, atol=1e-6)
    assert torch.equal(got, K.rotate_back_aggregate(x, rot, scale, alpha, None, off, g.dst, 3, 8))
