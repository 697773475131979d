"""Pin the rotate-back aggregation oracle before trusting it (no GPU needed).

The reference records DeepMD's flash aggregation seam ``_flash_atten_fn`` only
by its argument list (``docs/deepmd-fused-dispatch.md:127-128``: a
block-diagonal rotate-back of the edge messages, weighted by the attention
coefficients and summed into the destination); DeepMD is not installed here,
so no fixture of DeepMD's own function exists.  The three restatements --
the fp32 ``reference.rotate_back_aggregate_reference``, the float64
``oracle.truth`` and the loop form ``oracle.loops`` -- are pinned to each
other and to known answers: a hand-computed quarter turn, identity blocks
(the operator must reduce to an alpha-weighted segment sum) and a round trip
through random orthogonal blocks.  The float64 truth of the one-pass edge
chain (``oracle.truth.edge_chain``) is pinned to hand-computed values here too.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import loops, truth
from reference import rotate_back_aggregate_reference, segment_sum_reference


def csr(sizes):
    sizes = torch.as_tensor(sizes, dtype=torch.int64)
    dst = torch.repeat_interleave(torch.arange(sizes.numel()), sizes)
    off = torch.zeros(sizes.numel() + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(sizes, 0)
    return dst, off


def random_orthogonal_rotation(e, lmax, gen):
    """Packed rows of random orthogonal blocks (QR of Gaussian matrices)."""
    blocks = []
    for l in range(lmax + 1):
        m = 2 * l + 1
        q, _ = torch.linalg.qr(torch.randn(e, m, m, generator=gen, dtype=torch.float64))
        blocks.append(q.reshape(e, m * m))
    return torch.cat(blocks, dim=1)


def test_quarter_turn_known_answer():
    # lmax 1, one edge, one channel: l = 0 passes through, the l = 1 block is a
    # quarter turn D = [[0,-1,0],[1,0,0],[0,0,1]]; rotate-back is D^T x.
    x = torch.tensor([[[2.0], [1.0], [0.0], [3.0]]])
    rot = torch.tensor([[1.0, 0.0, -1.0, 0.0, 1.0, 0.0, 0.0, 0.0, 0.0, 1.0]])
    alpha, scale = torch.tensor([[0.5]]), torch.tensor([2.0])
    dst, off = csr([1])
    want = [[[2.0], [0.0], [-1.0], [3.0]]]
    got = rotate_back_aggregate_reference(x, rot, scale, alpha, None, off, dst, 1, 1)
    assert got.tolist() == want
    np.testing.assert_array_equal(truth.rotate_back_aggregate(x, rot, scale, alpha, dst, 1, 1, 1),
                                  np.asarray(want))
    assert loops.rotate_back_aggregate(x.tolist(), rot.tolist(), scale.tolist(), alpha.tolist(),
                                       dst.tolist(), 1, 1, 1) == want


def test_identity_blocks_reduce_to_a_weighted_segment_sum():
    gen = torch.Generator().manual_seed(3)
    lmax, heads, c = 2, 2, 6
    dst, off = csr([3, 0, 2, 4])
    e = dst.numel()
    x = torch.randn(e, 9, c, generator=gen)
    rot = torch.cat([torch.eye(2 * l + 1).reshape(1, -1).expand(e, -1)
                     for l in range(lmax + 1)], dim=1).contiguous()
    alpha = torch.rand(e, heads, generator=gen)
    got = rotate_back_aggregate_reference(x, rot, None, alpha, None, off, dst, lmax, heads)
    weighted = x * alpha.repeat_interleave(c // heads, dim=1).unsqueeze(1)
    want = segment_sum_reference(weighted.reshape(e, -1), dst, off).reshape(4, 9, c)
    torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)
    assert got[1].abs().max() == 0  # empty segment


def test_round_trip_through_orthogonal_blocks():
    gen = torch.Generator().manual_seed(4)
    lmax, e, c = 3, 7, 5
    rot = random_orthogonal_rotation(e, lmax, gen)
    x_global = torch.randn(e, 16, c, generator=gen, dtype=torch.float64)
    offs = truth.rotation_block_offsets(lmax)
    x_local = torch.empty_like(x_global)
    for l in range(lmax + 1):
        m = 2 * l + 1
        d = rot[:, offs[l]:offs[l + 1]].reshape(e, m, m)
        x_local[:, l * l:(l + 1) ** 2] = torch.bmm(d, x_global[:, l * l:(l + 1) ** 2])
    dst, off = csr([1] * e)
    got = truth.rotate_back_aggregate(x_local.numpy(), rot.numpy(), None, np.ones((e, 1)),
                                      dst.numpy(), e, lmax, 1)
    np.testing.assert_allclose(got, x_global.numpy(), rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("lmax,heads,channels,rescale", [(1, 1, 4, False), (2, 2, 6, True),
                                                         (3, 4, 8, True), (3, 1, 3, False)])
def test_three_restatements_agree(lmax, heads, channels, rescale):
    gen = torch.Generator().manual_seed(lmax * 10 + heads)
    dst, off = csr([2, 0, 5, 1, 3])
    e = dst.numel()
    comps = (lmax + 1) ** 2
    x = torch.randn(e, comps, channels, generator=gen)
    rot = random_orthogonal_rotation(e, lmax, gen).float()
    alpha = torch.rand(e, heads, generator=gen)
    scale = torch.rand(e, generator=gen) + 0.5 if rescale else None
    ref = rotate_back_aggregate_reference(x, rot, scale, alpha, None, off, dst, lmax, heads)
    t = truth.rotate_back_aggregate(x.numpy(), rot.numpy(), None if scale is None else
                                    scale.numpy(), alpha.numpy(), dst.numpy(), 5, lmax, heads)
    lp = loops.rotate_back_aggregate(x.tolist(), rot.tolist(),
                                     None if scale is None else scale.tolist(), alpha.tolist(),
                                     dst.tolist(), 5, lmax, heads)
    np.testing.assert_allclose(ref.numpy(), t, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(np.asarray(lp), t, rtol=1e-12, atol=1e-12)


def test_reference_validation():
    dst, off = csr([2])
    x = torch.randn(2, 4, 4)
    rot = torch.randn(2, 10)
    alpha = torch.rand(2, 2)
    with pytest.raises(ValueError):
        rotate_back_aggregate_reference(x, rot, None, alpha, None, off, dst, 2, 2)  # comps
    with pytest.raises(ValueError):
        rotate_back_aggregate_reference(x, rot[:, :9], None, alpha, None, off, dst, 1, 2)
    with pytest.raises(ValueError):
        rotate_back_aggregate_reference(x, rot, None, alpha, None, off, dst, 1, 3)  # heads
    with pytest.raises(ValueError):
        rotate_back_aggregate_reference(x, rot, None, alpha[:, :1], None, off, dst, 1, 2)


def test_edge_chain_truth_known_answers():
    # x + y * g with a [E, 1, C] gate, then the two activations
    x = np.array([[[1.0, -2.0]], [[0.5, 0.0]]])            # [2, 1, 2]
    y = np.array([[[3.0, 1.0]], [[-1.0, 2.0]]])
    g = np.array([[[0.5, 2.0]], [[1.0, 1.0]]])             # gate, same shape here
    z = truth.edge_chain([(1.0, x), (1.0, y, g)], (2, 1, 2))
    np.testing.assert_array_equal(z, [[[2.5, 0.0]], [[-0.5, 2.0]]])
    sig = truth.edge_chain([(1.0, x), (1.0, y, g)], (2, 1, 2), "sigmoid")
    np.testing.assert_allclose(sig, 1.0 / (1.0 + np.exp(-z)))
    silu = truth.edge_chain([(1.0, x), (1.0, y, g)], (2, 1, 2), "silu")
    np.testing.assert_allclose(silu, z / (1.0 + np.exp(-z)))
    # broadcasting: a per-channel vector and a per-edge scale
    w = np.array([1.0, 10.0])
    s = np.array([[[2.0]], [[3.0]]])
    got = truth.edge_chain([(-1.0, w, s)], (2, 3, 2))
    assert got.shape == (2, 3, 2)
    np.testing.assert_array_equal(got[1, 2], [-3.0, -30.0])
