"""GPU parity of RMSNorm and the GIE zonal scatter (B200)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import truth
from reference import rmsnorm as reference_rmsnorm
from reference import rmsnorm_per_degree, zonal_scatter_reference

pytestmark = pytest.mark.gpu

from bysj_b200 import kernels as K  # noqa: E402
from bysj_b200 import workloads as W  # noqa: E402


# ---- RMSNorm ---------------------------------------------------------------------------

@pytest.mark.parametrize("shape", [(1, 1), (7, 127), (2, 3, 257), (0, 65), (33, 128),
                                   (5, 16, 128), (3, 4096), (9, 8), (4, 2, 2000)])
def test_rmsnorm_forward_shapes(cuda, shape):
    gen = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(*shape, generator=gen)
    scale = torch.randn(shape[-1], generator=gen)
    got = K.rmsnorm(x.cuda(), scale.cuda(), eps=1e-5)
    want = reference_rmsnorm(x, scale, eps=1e-5)
    torch.testing.assert_close(got.cpu(), want, rtol=2e-5, atol=2e-5)
    assert tuple(got.shape) == shape
    plain = K.rmsnorm(x.cuda())
    torch.testing.assert_close(plain.cpu(), reference_rmsnorm(x), rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("tag", ["w17", "w128", "w257"])
def test_rmsnorm_golden_with_gradients(cuda, tag):
    g = golden("rmsnorm")
    x = torch.from_numpy(g[f"{tag}_x"]).cuda().requires_grad_(True)
    s = torch.from_numpy(g[f"{tag}_scale"]).cuda().requires_grad_(True)
    y = K.rmsnorm(x, s, eps=1e-5)
    np.testing.assert_allclose(y.detach().cpu().numpy(), g[f"{tag}_y"], rtol=2e-5, atol=2e-5)
    gx, gs = torch.autograd.grad(y, (x, s), torch.from_numpy(g[f"{tag}_upstream"]).cuda())
    np.testing.assert_allclose(gx.cpu().numpy(), g[f"{tag}_grad_x"], rtol=3e-5, atol=3e-5)
    np.testing.assert_allclose(gs.cpu().numpy(), g[f"{tag}_grad_scale"], rtol=3e-5, atol=3e-4)


def test_rmsnorm_per_degree_fp32_bf16_and_scale_grad(cuda):
    g = golden("rmsnorm")
    x, w = torch.from_numpy(g["deg_x"]), torch.from_numpy(g["deg_w"])
    got = K.rmsnorm(x.cuda(), w.cuda())
    np.testing.assert_allclose(got.cpu().numpy(), g["deg_y"], rtol=1e-5, atol=1e-6)
    xb = x.to(torch.bfloat16)
    got16 = K.rmsnorm(xb.cuda(), w.cuda())
    assert got16.dtype == torch.bfloat16
    want16 = rmsnorm_per_degree(xb.float(), w)
    torch.testing.assert_close(got16.float().cpu(), want16, rtol=1e-2, atol=1e-2)
    xg = x.cuda().requires_grad_(True)
    wg = w.cuda().requires_grad_(True)
    up = torch.randn(x.shape).cuda()
    gx, gw = torch.autograd.grad(K.rmsnorm(xg, wg), (xg, wg), up)
    rx, rw = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    ex, ew = torch.autograd.grad(rmsnorm_per_degree(rx, rw), (rx, rw), up.cpu())
    torch.testing.assert_close(gx.cpu(), ex, rtol=3e-5, atol=3e-5)
    torch.testing.assert_close(gw.cpu(), ew, rtol=3e-5, atol=3e-4)


def test_rmsnorm_deterministic_scale_gradient_and_stream(cuda):
    x = torch.randn(4096, 128, device="cuda", requires_grad=True)
    s = torch.randn(128, device="cuda", requires_grad=True)
    up = torch.randn(4096, 128, device="cuda")
    g1 = torch.autograd.grad(K.rmsnorm(x, s), (x, s), up)
    g2 = torch.autograd.grad(K.rmsnorm(x, s), (x, s), up)
    assert torch.equal(g1[0], g2[0]) and torch.equal(g1[1], g2[1])
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        xs = torch.randn(9, 131, device="cuda")
        sc = torch.randn(131, device="cuda")
        got = K.rmsnorm(xs, sc)
    torch.cuda.current_stream().wait_stream(stream)
    torch.testing.assert_close(got.cpu(), reference_rmsnorm(xs.cpu(), sc.cpu()), rtol=2e-5,
                               atol=2e-5)


# ---- GIE zonal scatter -----------------------------------------------------------------

def test_gie_golden_forward_and_backward(cuda):
    g = golden("gie")
    z = torch.from_numpy(g["zonal"]).cuda().requires_grad_(True)
    r = torch.from_numpy(g["radial"]).cuda().requires_grad_(True)
    inv = torch.from_numpy(g["inv"]).cuda().requires_grad_(True)
    dst, slot = torch.from_numpy(g["dst"]).cuda(), torch.from_numpy(g["slot"]).cuda()
    out = K.zonal_scatter(z, r, dst, slot, inv)
    np.testing.assert_allclose(out.detach().cpu().numpy(), g["out"], rtol=2e-5, atol=2e-6)
    assert out[:, 0, :].count_nonzero() == 0
    grads = torch.autograd.grad(out, (z, r, inv), torch.from_numpy(g["upstream"]).cuda())
    for got, key in zip(grads, ("grad_zonal", "grad_radial", "grad_inv")):
        np.testing.assert_allclose(got.cpu().numpy(), g[key], rtol=4e-4, atol=2e-5)


def _small(device="cuda", degree_shape=(2,), requires_grad=False):
    zonal = torch.tensor([[0.2, -0.1, 0.3], [0.4, 0.5, -0.2], [-0.3, 0.6, 0.1], [0.7, -0.2, 0.4]],
                         device=device, requires_grad=requires_grad)
    radial = (torch.arange(24, dtype=torch.float32, device=device).reshape(4, 2, 3) / 10)
    radial.requires_grad_(requires_grad)
    dst = torch.tensor([1, 0, 1, 1], device=device)
    slot = torch.tensor([0, 0, 1], device=device)
    inv = torch.tensor([0.7, 0.5], device=device).reshape(degree_shape)
    inv.requires_grad_(requires_grad)
    return zonal, radial, dst, slot, inv


def test_gie_colliding_unsorted_destinations_and_3d_inverse(cuda):
    inputs = _small(requires_grad=True)
    up = torch.randn(2, 4, 3, device="cuda")
    got = K.zonal_scatter(*inputs)
    gg = torch.autograd.grad(got, (inputs[0], inputs[1], inputs[4]), up)
    ref_in = tuple(v.detach().cpu().requires_grad_(v.requires_grad) if v.dtype.is_floating_point
                   else v.cpu() for v in inputs)
    want = zonal_scatter_reference(*ref_in)
    wg = torch.autograd.grad(want, (ref_in[0], ref_in[1], ref_in[4]), up.cpu())
    torch.testing.assert_close(got.detach().cpu(), want.detach(), rtol=2e-5, atol=2e-6)
    for a, b in zip(gg, wg):
        torch.testing.assert_close(a.cpu(), b, rtol=4e-4, atol=2e-5)
    three = K.zonal_scatter(*_small(degree_shape=(2, 1, 1)))
    torch.testing.assert_close(three.cpu(), want.detach(), rtol=2e-5, atol=2e-6)


def test_gie_inverse_gradient_normalises_after_sum(cuda):
    zonal = torch.tensor([[1e8], [-1e8 + 8], [1.0]], device="cuda")
    radial = torch.ones(3, 1, 1, device="cuda")
    dst = torch.zeros(3, dtype=torch.int64, device="cuda")
    slots = torch.zeros(1, dtype=torch.int64, device="cuda")
    inverse = torch.ones(1, device="cuda", requires_grad=True)
    out = K.zonal_scatter(zonal, radial, dst, slots, inverse)
    (grad,) = torch.autograd.grad(out, (inverse,), torch.tensor([[[0.0], [0.3]]], device="cuda"))
    assert 2.39 <= grad.item() <= 2.71
    # In edge order: (1e8 + (-1e8 + 8)) + 1 = 9 exactly in fp32, then * inv.
    assert out[0, 1].item() == 9.0


def test_gie_empty_edges_and_stream(cuda):
    out = K.zonal_scatter(torch.empty(0, 3, device="cuda"), torch.empty(0, 2, 4, device="cuda"),
                          torch.empty(0, dtype=torch.int64, device="cuda"),
                          torch.tensor([0, 0, 1], device="cuda"), torch.ones(2, device="cuda"))
    assert tuple(out.shape) == (2, 4, 4) and out.count_nonzero() == 0
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        inputs = _small()
        got = K.zonal_scatter(*inputs)
    torch.cuda.current_stream().wait_stream(stream)
    want = zonal_scatter_reference(*(v.cpu() for v in _small()))
    torch.testing.assert_close(got.cpu(), want, rtol=2e-5, atol=2e-6)


def test_gie_c1_geometry_matches_float64(cuda):
    g = W.c1_box(device="cuda")
    zonal = W.real_sph_zonal(g.unit)
    gen = torch.Generator(device="cuda").manual_seed(12)
    radial = torch.randn(g.n_edges, 4, 64, device="cuda", generator=gen)
    slot = W.degree_slots().cuda()
    deg = torch.bincount(g.dst, minlength=g.n_atoms).float()
    inv = torch.rsqrt(deg + 1.0)
    out = K.zonal_scatter(zonal, radial, g.dst, slot, inv)
    want = truth.zonal_scatter(zonal.cpu().numpy(), radial.cpu().numpy(), g.dst.cpu().numpy(),
                               slot.cpu().numpy(), inv.cpu().numpy())
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5,
                               atol=1e-5 * float(np.abs(want).max()))
    assert torch.equal(out, K.zonal_scatter(zonal, radial, g.dst, slot, inv))


@pytest.mark.parametrize("zero_based,channels", [(True, 64), (False, 16), (True, 128), (False, 4)])
def test_gie_degree_layout_with_split_segments(cuda, zero_based, channels):
    # Rows grouped by degree (the DPA4 layout) take the degree-specialised
    # kernel; a skewed graph forces segments split across partitions.
    gen = torch.Generator().manual_seed(channels)
    sizes = torch.randint(0, 10, (300,), generator=gen)
    sizes[50], sizes[-1] = 3000, 1200
    dst = torch.repeat_interleave(torch.arange(300), sizes)
    e = dst.numel()
    zonal = torch.randn(e, 15, generator=gen)
    radial = torch.randn(e, 4, channels, generator=gen)
    slot = W.degree_slots(zero_based=zero_based)
    inv = torch.rand(300, generator=gen) + 0.2
    out = K.zonal_scatter(zonal.cuda(), radial.cuda(), dst.cuda(), slot.cuda(), inv.cuda())
    want = truth.zonal_scatter(zonal.numpy(), radial.numpy(), dst.numpy(), slot.numpy(),
                               inv.numpy())
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5,
                               atol=1e-5 * float(np.abs(want).max()))
    assert out[:, 0, :].count_nonzero() == 0


def test_rmsnorm_misaligned_scale_view(cuda):
    x = torch.randn(64, 128, device="cuda")
    big = torch.randn(129, device="cuda")
    scale = big[1:]  # contiguous view whose data pointer is 4 bytes past alignment
    got = K.rmsnorm(x, scale)
    torch.testing.assert_close(got.cpu(), reference_rmsnorm(x.cpu(), scale.cpu()), rtol=2e-5,
                               atol=2e-5)


@pytest.mark.parametrize("zero_based,channels,shuffled",
                         [(True, 64, False), (False, 16, True), (False, 64, True), (True, 4, False)])
def test_gie_degree_layout_backward(cuda, zero_based, channels, shuffled):
    # The degree-specialised backward: skewed segments (split across
    # partitions), optionally unsorted destinations (CSR view with an order).
    gen = torch.Generator().manual_seed(3 * channels + shuffled)
    sizes = torch.randint(0, 12, (200,), generator=gen)
    sizes[30], sizes[-1] = 2500, 900
    dst = torch.repeat_interleave(torch.arange(200), sizes)
    if shuffled:
        dst = dst[torch.randperm(dst.numel(), generator=gen)]
    e = dst.numel()
    z = torch.randn(e, 15, generator=gen)
    r = torch.randn(e, 4, channels, generator=gen)
    inv = torch.rand(200, generator=gen) + 0.2
    slot = W.degree_slots(zero_based=zero_based)
    up = torch.randn(200, 16, channels, generator=gen)
    zc, rc, ic = (t.cuda().requires_grad_(True) for t in (z, r, inv))
    out = K.zonal_scatter(zc, rc, dst.cuda(), slot.cuda(), ic)
    got = torch.autograd.grad(out, (zc, rc, ic), up.cuda())
    zr, rr, ir = (t.clone().requires_grad_(True) for t in (z, r, inv))
    want = zonal_scatter_reference(zr, rr, dst, slot, ir)
    wg = torch.autograd.grad(want, (zr, rr, ir), up)
    for a, b in zip(got, wg):
        torch.testing.assert_close(a.cpu(), b, rtol=4e-4, atol=2e-5 * float(b.abs().max()) + 2e-5)
    unused = 0 if not zero_based else 3  # the radial slot no row reads
    assert got[1][:, unused, :].count_nonzero() == 0
    again = torch.autograd.grad(K.zonal_scatter(zc, rc, dst.cuda(), slot.cuda(), ic),
                                (zc, rc, ic), up.cuda())
    assert all(torch.equal(a, b) for a, b in zip(got, again))


@pytest.mark.parametrize("table", ["degree", "shuffled", "base1"])
def test_gie_degree_shape_slot_table_checked_on_device(cuda, table):
    # 15 rows and 64 channels: the shape of DPA4's degree layout, so the
    # library launches both the degree kernel and the generic one and each
    # decides on the device from the slot table.  The degree table (base 0,
    # or base 1 over five radial slots) must be taken by the degree kernel
    # with that base, a shuffled table by the generic kernel.
    gen = torch.Generator().manual_seed({"degree": 1, "shuffled": 2, "base1": 3}[table])
    sizes = torch.randint(0, 40, (300,), generator=gen)
    sizes[7] = 900
    dst = torch.repeat_interleave(torch.arange(300), sizes)
    e = dst.numel()
    n_radial = 4
    slot = W.degree_slots()
    if table == "shuffled":
        slot = slot[torch.randperm(15, generator=gen)]
    elif table == "base1":
        slot = slot + 1  # degrees 1..3 read radial slots 2..4
        n_radial = 5
    z = torch.randn(e, 15, generator=gen)
    r = torch.randn(e, n_radial, 64, generator=gen)
    inv = torch.rand(300, generator=gen) + 0.2
    up = torch.randn(300, 16, 64, generator=gen)
    zc, rc, ic = (t.cuda().requires_grad_(True) for t in (z, r, inv))
    out = K.zonal_scatter(zc, rc, dst.cuda(), slot.cuda(), ic)
    zr, rr, ir = (t.clone().requires_grad_(True) for t in (z, r, inv))
    want = zonal_scatter_reference(zr, rr, dst, slot, ir)
    torch.testing.assert_close(out.detach().cpu(), want.detach(), rtol=1e-5,
                               atol=1e-5 * float(want.detach().abs().max()))
    got = torch.autograd.grad(out, (zc, rc, ic), up.cuda())
    wg = torch.autograd.grad(want, (zr, rr, ir), up)
    for a, b in zip(got, wg):
        torch.testing.assert_close(a.cpu(), b, rtol=4e-4, atol=2e-5 * float(b.abs().max()) + 2e-5)


def test_gie_degree_backward_inverse_gradient_sums_first(cuda):
    # Degree layout with L = 1 (rows 0..2 read radial slot 1): the three
    # edges' unnormalised sums cancel exactly before the dot with g.
    zonal = torch.zeros(3, 3, device="cuda")
    zonal[:, 0] = torch.tensor([1e8, -1e8 + 8, 1.0], device="cuda")
    radial = torch.ones(3, 2, 4, device="cuda")
    dst = torch.zeros(3, dtype=torch.int64, device="cuda")
    slot = torch.tensor([1, 1, 1], device="cuda")
    inverse = torch.ones(1, device="cuda", requires_grad=True)
    out = K.zonal_scatter(zonal, radial, dst, slot, inverse)
    up = torch.zeros(1, 4, 4, device="cuda")
    up[0, 1, :] = 0.3
    (grad,) = torch.autograd.grad(out, (inverse,), up)
    assert abs(grad.item() - 4 * 0.3 * 9.0) < 1e-4


@pytest.mark.parametrize("rows,n_radial,channels,slot_kind",
                         [(15, 4, 64, "degree"), (15, 4, 32, "degree"), (3, 2, 8, "generic")])
def test_gie_dst_offsets_takes_the_given_csr(cuda, rows, n_radial, channels, slot_kind):
    # With the CSR of a grouped dst passed in, the operator skips its own
    # derivation and read-back: the same kernels, so the same bits as the
    # dst-only call, forward and backward (empty nodes and a split hub in).
    gen = torch.Generator().manual_seed(rows * channels)
    sizes = torch.randint(0, 9, (400,), generator=gen)
    sizes[::7] = 0
    sizes[123] = 4000
    dst = torch.repeat_interleave(torch.arange(400), sizes).cuda()
    e = dst.numel()
    off = K.segment_offsets(dst, 400)
    zonal = torch.randn(e, rows, generator=gen).cuda().requires_grad_(True)
    radial = torch.randn(e, n_radial, channels, generator=gen).cuda().requires_grad_(True)
    inv = (torch.rand(400, generator=gen) + 0.2).cuda().requires_grad_(True)
    slot = (W.degree_slots() if slot_kind == "degree" else torch.tensor([0, 1, 1])).cuda()
    up = torch.randn(400, rows + 1, channels, generator=gen).cuda()
    base = K.zonal_scatter(zonal, radial, dst, slot, inv)
    given = K.zonal_scatter(zonal, radial, dst, slot, inv, dst_offsets=off)
    assert torch.equal(base, given)
    gb = torch.autograd.grad(base, (zonal, radial, inv), up)
    gg = torch.autograd.grad(given, (zonal, radial, inv), up)
    assert all(torch.equal(a, b) for a, b in zip(gb, gg))
    empty = K.zonal_scatter(zonal[:0], radial[:0], dst[:0], slot, inv,
                            dst_offsets=torch.zeros(401, dtype=torch.int64, device="cuda"))
    assert empty.count_nonzero() == 0


def test_gie_dst_offsets_arguments_and_grouping_check(cuda, monkeypatch):
    from bysj_b200.kernels import segment as S

    zonal, radial, dst, slot, inv = _small()
    dst = torch.tensor([0, 1, 1, 1], device="cuda")
    off = torch.tensor([0, 1, 4], device="cuda")
    want = K.zonal_scatter(zonal, radial, dst, slot, inv)
    assert torch.equal(K.zonal_scatter(zonal, radial, dst, slot, inv, dst_offsets=off), want)
    with pytest.raises(TypeError, match="dst_offsets must be int64"):
        K.zonal_scatter(zonal, radial, dst, slot, inv, dst_offsets=off.int())
    with pytest.raises(ValueError, match=r"shape \(n_nodes \+ 1,\)"):
        K.zonal_scatter(zonal, radial, dst, slot, inv, dst_offsets=off[:2])
    monkeypatch.setattr(S, "_CHECK_GROUPING", True)
    assert torch.equal(K.zonal_scatter(zonal, radial, dst, slot, inv, dst_offsets=off), want)
    with pytest.raises(ValueError, match="GIE dst_offsets: offsets"):
        K.zonal_scatter(zonal, radial, dst, slot, inv,
                        dst_offsets=torch.tensor([0, 1, 5], device="cuda"))
    with pytest.raises(ValueError, match="not the CSR of a grouped dst"):
        K.zonal_scatter(zonal, radial, dst, slot, inv,
                        dst_offsets=torch.tensor([0, 2, 4], device="cuda"))
    unsorted = torch.tensor([1, 0, 1, 1], device="cuda")
    with pytest.raises(ValueError, match="not the CSR of a grouped dst"):
        K.zonal_scatter(zonal, radial, unsorted, slot, inv, dst_offsets=off)
