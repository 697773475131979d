"""GPU parity at the benchmark configurations' full sizes (B200).

The small-graph tests pin every operator against the oracle where almost every
segment is split across warps; the benchmarked frames exercise the other code
paths (whole segments walked by one warp, capped partition plans, 2.2 M
edges).  Here each benchmarked configuration is run at its full size and
checked two ways:

* every output against a float64 evaluation of the same formula on the GPU
  (written in the test with plain torch ops, independent of the kernels), and
* a seeded sample of 2,048 whole segments (plus the heaviest ones and both
  ends of the frame) against the fp32 CPU oracle, ``reference.*`` restated
  from the reference project's ``python/reference``, and ``oracle.truth``.

Tolerances are the spec's: fp32 rtol 1e-5 / atol 1e-6; bf16 value inputs
rtol 1e-2 against the fp32-valued result; integers bit-exact; the fp64-summed
force assembly within 2 ulp of the float64 truth.  Plain sums of unnormalised
terms (segment_sum, the zonal scatter) are the exception: any fp32 summation of
n terms, the reference's ``index_add_`` included, can be off by up to
n * 2^-24 * sum|terms| (Higham's bound), so where a ~90-term sum of N(0, 1)
terms cancels to ~0.06 two fp32 sums in different orders differ by ~1e-5.
Those outputs are held to rtol 1e-5 / atol 1e-6 plus 2^-20 * sum|terms|
(16 units of roundoff of the absolute sum, far inside the n u bound).

Configurations (BASELINE): C2 RMSNorm [24576, 16, 128] fp32 and bf16 with
per-degree weights [4, 128]; C3 the 24576-atom, ~2.22 M-edge box with logits
[E, 8] ~ N(0, 2) and values [E, 16, 64] fp32 and bf16 (fused attention,
standalone softmax at H = 8, segment_sum at C = 1024); C4 the same geometry
with zonal [E, 15], radial [E, 4, 64] and dE/dr [E, 3] ~ N(0, 0.1).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import truth
from reference import (
    force_assembly_reference,
    rmsnorm_per_degree,
    segment_attention_reference,
    segment_softmax_reference,
    segment_sum_reference,
    zonal_scatter_reference,
)

pytestmark = pytest.mark.gpu

from bysj_b200 import kernels as K  # noqa: E402
from bysj_b200 import workloads as W  # noqa: E402

RTOL, ATOL = 1e-5, 1e-6
CHUNK = 1 << 18  # edges per float64 chunk (2 GB at 1024 channels)


@pytest.fixture(scope="module")
def c3():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    g = W.c3_box(device="cuda", seed=0)
    off = K.segment_offsets(g.dst, g.n_atoms)
    return g, off


def sample_segments(off_cpu: torch.Tensor, count: int = 2048, seed: int = 5) -> torch.Tensor:
    """A seeded sample of segments plus the 16 heaviest and both ends."""
    n = off_cpu.numel() - 1
    gen = torch.Generator().manual_seed(seed)
    pick = torch.randperm(n, generator=gen)[:count]
    heavy = torch.topk(off_cpu[1:] - off_cpu[:-1], 16).indices
    ends = torch.tensor([0, 1, n - 2, n - 1])
    return torch.unique(torch.cat([pick, heavy, ends]))


def subset(off_cpu: torch.Tensor, segs: torch.Tensor):
    """Edge indices, renumbered dst and offsets of the chosen segments."""
    starts, ends = off_cpu[segs], off_cpu[segs + 1]
    sizes = ends - starts
    idx = torch.cat([torch.arange(int(s), int(e)) for s, e in zip(starts, ends)])
    dst = torch.repeat_interleave(torch.arange(segs.numel()), sizes)
    sub_off = torch.zeros(segs.numel() + 1, dtype=torch.int64)
    sub_off[1:] = torch.cumsum(sizes, 0)
    return idx, dst, sub_off


def softmax_f64(logit, dst, n, env=None, null=None):
    """(alpha, null_alpha) in float64 on the GPU: the gated segment softmax."""
    lg = logit.double()
    if env is not None:
        keep = env > 0
        lg = torch.where(keep[:, None], lg + 2.0 * torch.log(torch.where(keep, env, 1.0)
                                                              .double())[:, None],
                         torch.full_like(lg, -float("inf")))
    h = lg.shape[1]
    peak = torch.full((n, h), -float("inf"), dtype=torch.float64, device=lg.device)
    peak = peak.scatter_reduce(0, dst[:, None].expand(-1, h), lg, "amax", include_self=True)
    if null is not None:
        peak = torch.maximum(peak, null.double())
    finite = torch.isfinite(peak)
    base = torch.where(finite, peak, torch.zeros_like(peak))
    w = torch.where(torch.isfinite(lg) & finite[dst], torch.exp(lg - base[dst]),
                    torch.zeros_like(lg))
    total = torch.zeros_like(peak).index_add_(0, dst, w)
    w0 = None
    if null is not None:
        w0 = torch.where(finite, torch.exp(null.double() - base), torch.zeros_like(peak))
        total = total + w0
    safe = torch.where(total > 0, total, torch.ones_like(total))
    return w / safe[dst], (w0 / safe if w0 is not None else None)


def attention_f64(logit, value, dst, n, env=None, null=None):
    alpha, _ = softmax_f64(logit, dst, n, env, null)
    e, s, c = value.shape
    h = logit.shape[1]
    out = torch.zeros(n, s, h, c // h, dtype=torch.float64, device=value.device)
    for a in range(0, e, CHUNK):
        b = min(e, a + CHUNK)
        rows = value[a:b].double().reshape(b - a, s, h, c // h) * alpha[a:b, None, :, None]
        out.index_add_(0, dst[a:b], rows)
    return out.permute(0, 2, 1, 3)


def assert_close_f64(got: torch.Tensor, want: torch.Tensor, rtol=RTOL, atol=ATOL, what=""):
    """|got - want| <= atol + rtol |want| elementwise (want in float64), on the GPU."""
    diff = (got.double() - want).abs()
    bound = atol + rtol * want.abs()
    bad = diff > bound
    if bool(bad.any()):
        i = int(torch.argmax((diff - bound).reshape(-1)))
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {bad.numel()} elements outside rtol {rtol} / atol "
            f"{atol}; worst got {float(got.reshape(-1)[i])} want {float(want.reshape(-1)[i])}")


def assert_sum_close(got: torch.Tensor, want: torch.Tensor, magnitude: torch.Tensor,
                     what: str, ulps: float = 16.0):
    """A sum against its float64 value: within atol + rtol |want| + ulps u sum|terms|."""
    diff = (got.double() - want).abs()
    bound = ATOL + RTOL * want.abs() + ulps * 2.0 ** -24 * magnitude
    bad = diff > bound
    if bool(bad.any()):
        i = int(torch.argmax((diff - bound).reshape(-1)))
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {bad.numel()} elements outside the summation bound; "
            f"worst got {float(got.reshape(-1)[i])} want {float(want.reshape(-1)[i])} "
            f"sum|terms| {float(magnitude.reshape(-1)[i])}")


# ---- C3: integer CSR ---------------------------------------------------------------------

def test_c3_offsets_and_grouping_bit_exact(c3):
    g, off = c3
    np.testing.assert_array_equal(off.cpu().numpy(),
                                  truth.segment_offsets(g.dst.cpu().numpy(), g.n_atoms))
    order, soff = K.group_by_source(g.src, g.n_atoms)
    want_order, want_off = truth.group_by_source(g.src.cpu().numpy(), g.n_atoms)
    np.testing.assert_array_equal(order.cpu().numpy(), want_order)
    np.testing.assert_array_equal(soff.cpu().numpy(), want_off)


# ---- C3: fused attention -------------------------------------------------------------------

def _c3_attention_inputs(g, seed=17):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    logit = torch.randn(g.n_edges, 8, device="cuda", generator=gen) * (2.0 ** 0.5)
    value = torch.randn(g.n_edges, 16, 64, device="cuda", generator=gen)
    return logit, value


def _check_attention_sample(out, logit, value, off, env=None, null=None):
    off_cpu = off.cpu()
    segs = sample_segments(off_cpu)
    idx, dst, sub_off = subset(off_cpu, segs)
    lg, val = logit[idx.cuda()].cpu(), value[idx.cuda()].float().cpu()
    ev = env[idx.cuda()].cpu() if env is not None else None
    nl = null[segs.cuda()].cpu() if null is not None else None
    want = segment_attention_reference(lg, val, dst, sub_off, ev, nl)
    torch.testing.assert_close(out[segs.cuda()].cpu(), want, rtol=RTOL, atol=ATOL)
    # the float64 NumPy truth on the first 256 sampled segments
    k = 256
    m = int(sub_off[k])
    want64 = truth.segment_attention(lg[:m].numpy(), val[:m].numpy(), dst[:m].numpy(), k,
                                     None if ev is None else ev[:m].numpy(),
                                     None if nl is None else nl[:k].numpy())
    np.testing.assert_allclose(out[segs[:k].cuda()].cpu().numpy(), want64, rtol=RTOL, atol=ATOL)


def test_c3_attention_fp32_full_frame(c3):
    g, off = c3
    logit, value = _c3_attention_inputs(g)
    out = K.segment_attention(logit, value, off)
    assert tuple(out.shape) == (g.n_atoms, 8, 16, 8)
    assert_close_f64(out, attention_f64(logit, value, g.dst, g.n_atoms), what="C3 fp32")
    _check_attention_sample(out, logit, value, off)
    assert torch.equal(out, K.segment_attention(logit, value, off))


def test_c3_attention_env_and_null_full_frame(c3):
    g, off = c3
    logit, value = _c3_attention_inputs(g, seed=18)
    gen = torch.Generator(device="cuda").manual_seed(19)
    env = torch.rand(g.n_edges, device="cuda", generator=gen) * 0.95 + 0.05
    env[torch.rand(g.n_edges, device="cuda", generator=gen) < 0.05] = 0.0
    null = torch.randn(g.n_atoms, 8, device="cuda", generator=gen)
    out = K.segment_attention(logit, value, off, env, null)
    assert_close_f64(out, attention_f64(logit, value, g.dst, g.n_atoms, env, null),
                     what="C3 env + null")
    _check_attention_sample(out, logit, value, off, env, null)


def test_c3_attention_bf16_values_full_frame(c3):
    g, off = c3
    logit, value = _c3_attention_inputs(g)
    vb = value.to(torch.bfloat16)
    out16 = K.segment_attention(logit, vb, off)
    # the arithmetic is fp32 on exactly widened inputs: strict against the
    # float64 result of the same bf16 values ...
    assert_close_f64(out16, attention_f64(logit, vb, g.dst, g.n_atoms), what="C3 bf16 strict")
    _check_attention_sample(out16, logit, vb, off)
    # ... and within the bf16 input rounding of the fp32-valued result: each
    # value moved by at most 2^-9 of itself, so the output by at most
    # 2^-9 sum_e alpha_e |v_e| (bounded here with 2^-8 for the fp32 arithmetic)
    out32 = K.segment_attention(logit, value, off)
    spread = attention_f64(logit, value.abs(), g.dst, g.n_atoms)
    excess = (out16.double() - out32.double()).abs() - (2.0 ** -8 * spread + ATOL)
    assert float(excess.max()) <= 0.0
    torch.testing.assert_close(out16, out32, rtol=1e-2, atol=1e-2)
    assert torch.equal(out16, K.segment_attention(logit, vb, off))


# ---- C3: standalone softmax (H = 8) and segment_sum (C = 1024) -------------------------------

@pytest.mark.parametrize("gated", [False, True])
def test_c3_softmax_h8_full_frame(c3, gated):
    g, off = c3
    gen = torch.Generator(device="cuda").manual_seed(23)
    logit = torch.randn(g.n_edges, 8, device="cuda", generator=gen) * (2.0 ** 0.5)
    if gated:
        env = torch.rand(g.n_edges, device="cuda", generator=gen) * 0.95 + 0.05
        env[torch.rand(g.n_edges, device="cuda", generator=gen) < 0.05] = 0.0
        null = torch.randn(g.n_atoms, 8, device="cuda", generator=gen)
        alpha, null_alpha = K.segment_softmax(logit, env, off, null)
    else:
        env = torch.ones(g.n_edges, device="cuda")
        null = None
        alpha = K.segment_softmax(logit, env, off)
    want = segment_softmax_reference(logit.cpu(), env.cpu(), g.dst.cpu(), off.cpu(),
                                     None if null is None else null.cpu())
    torch.testing.assert_close(alpha.cpu(), want[0], rtol=RTOL, atol=ATOL)
    a64, n64 = softmax_f64(logit, g.dst, g.n_atoms, env, null)
    assert_close_f64(alpha, a64, what="C3 softmax")
    if gated:
        torch.testing.assert_close(null_alpha.cpu(), want[1], rtol=RTOL, atol=ATOL)
        assert_close_f64(null_alpha, n64, what="C3 null alpha")


def test_c3_segment_sum_c1024_full_frame(c3):
    g, off = c3
    e, n = g.n_edges, g.n_atoms
    gen = torch.Generator(device="cuda").manual_seed(29)
    src = torch.randn(e, 1024, device="cuda", generator=gen)
    ws = torch.rand(e, device="cuda", generator=gen) + 0.5
    ns = torch.rand(n, device="cuda", generator=gen) + 0.5
    out = K.segment_sum(src, g.dst, off, ws, ns)
    want = torch.zeros(n, 1024, dtype=torch.float64, device="cuda")
    mag = torch.zeros_like(want)
    for a in range(0, e, CHUNK):
        b = min(e, a + CHUNK)
        terms = src[a:b].double() * ws[a:b, None].double()
        want.index_add_(0, g.dst[a:b], terms)
        mag.index_add_(0, g.dst[a:b], terms.abs())
    want *= ns[:, None].double()
    mag *= ns[:, None].double()
    assert_sum_close(out, want, mag, "C3 segment_sum")
    off_cpu = off.cpu()
    segs = sample_segments(off_cpu)
    idx, dst, sub_off = subset(off_cpu, segs)
    ref = segment_sum_reference(src[idx.cuda()].cpu(), dst, sub_off, ws[idx.cuda()].cpu(),
                                ns[segs.cuda()].cpu())
    # two fp32 sums in different orders: twice the single-sum bound
    assert_sum_close(out[segs.cuda()].cpu(), ref.double(), mag[segs.cuda()].cpu(),
                     "C3 segment_sum vs the fp32 oracle", ulps=32.0)
    del src
    # bf16 rows against the float64 sum of the same values
    vb = torch.randn(e, 1024, device="cuda", generator=gen).to(torch.bfloat16)
    out16 = K.segment_sum(vb, g.dst, off)
    want16 = torch.zeros(n, 1024, dtype=torch.float64, device="cuda")
    mag16 = torch.zeros_like(want16)
    for a in range(0, e, CHUNK):
        b = min(e, a + CHUNK)
        want16.index_add_(0, g.dst[a:b], vb[a:b].double())
        mag16.index_add_(0, g.dst[a:b], vb[a:b].double().abs())
    assert_sum_close(out16, want16, mag16, "C3 segment_sum bf16")


# ---- C2: RMSNorm --------------------------------------------------------------------------

def test_c2_rmsnorm_fp32_and_bf16_per_degree():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gen = torch.Generator().manual_seed(31)
    x = torch.randn(24576, 16, 128, generator=gen)
    w = torch.rand(4, 128, generator=gen) + 0.5
    y = K.rmsnorm(x.cuda(), w.cuda(), 1e-6)
    want = rmsnorm_per_degree(x, w, 1e-6)
    torch.testing.assert_close(y.cpu(), want, rtol=RTOL, atol=ATOL)
    y64, _ = truth.rmsnorm(x.numpy(), w.numpy(), 1e-6, per_degree=True)
    np.testing.assert_allclose(y.cpu().numpy(), y64, rtol=RTOL, atol=ATOL)
    # the reference API's [C] scale on the same frame
    y1 = K.rmsnorm(x.cuda(), w[2].cuda(), 1e-6)
    from reference import rmsnorm as reference_rmsnorm

    torch.testing.assert_close(y1.cpu(), reference_rmsnorm(x, w[2], 1e-6), rtol=RTOL, atol=ATOL)
    xb = x.to(torch.bfloat16)
    yb = K.rmsnorm(xb.cuda(), w.cuda(), 1e-6)
    assert yb.dtype == torch.bfloat16
    torch.testing.assert_close(yb.float().cpu(), want, rtol=1e-2, atol=1e-2)
    # against the same bf16 inputs: only the output rounding to bf16 differs
    wantb = rmsnorm_per_degree(xb.float(), w, 1e-6)
    torch.testing.assert_close(yb.float().cpu(), wantb, rtol=2 ** -8, atol=1e-6)


# ---- C4: zonal scatter and force assembly -----------------------------------------------------

def test_c4_zonal_scatter_full_frame(c3):
    g, off = c3
    e, n = g.n_edges, g.n_atoms
    gen = torch.Generator(device="cuda").manual_seed(37)
    zonal = W.real_sph_zonal(g.unit)
    radial = torch.randn(e, 4, 64, device="cuda", generator=gen)
    slot = W.degree_slots().to("cuda")
    inv = torch.rsqrt(torch.bincount(g.dst, minlength=n).float() + 1.0)
    out = K.zonal_scatter(zonal, radial, g.dst, slot, inv)
    rows = torch.zeros(n, 15, 64, dtype=torch.float64, device="cuda")
    absrows = torch.zeros_like(rows)
    for a in range(0, e, CHUNK):
        b = min(e, a + CHUNK)
        msg = zonal[a:b].double()[:, :, None] * radial[a:b][:, slot, :].double()
        rows.index_add_(0, g.dst[a:b], msg)
        absrows.index_add_(0, g.dst[a:b], msg.abs())
    want = torch.zeros(n, 16, 64, dtype=torch.float64, device="cuda")
    mag = torch.zeros_like(want)
    want[:, 1:, :] = rows * inv.double()[:, None, None]
    mag[:, 1:, :] = absrows * inv.double()[:, None, None]
    assert_sum_close(out, want, mag, "C4 zonal scatter")
    off_cpu = off.cpu()
    segs = sample_segments(off_cpu)
    idx, dst, _ = subset(off_cpu, segs)
    ref = zonal_scatter_reference(zonal[idx.cuda()].cpu(), radial[idx.cuda()].cpu(), dst,
                                  slot.cpu(), inv[segs.cuda()].cpu())
    assert_sum_close(out[segs.cuda()].cpu(), ref.double(), mag[segs.cuda()].cpu(),
                     "C4 zonal scatter vs the fp32 oracle", ulps=32.0)


@pytest.mark.parametrize("atom_order", ["morton", "random"])
def test_c4_force_assembly_full_frame(c3, atom_order):
    g, off = c3
    e, n = g.n_edges, g.n_atoms
    gen = torch.Generator(device="cuda").manual_seed(41)
    grad = torch.randn(e, 3, device="cuda", generator=gen) * 0.1
    src, dst, vec = g.src, g.dst, g.unit
    if atom_order == "random":
        label = torch.randperm(n, device="cuda", generator=gen)
        dst, src = label[dst], label[src]
        perm = torch.argsort(dst * n + src)
        dst, src, vec = dst[perm].contiguous(), src[perm].contiguous(), vec[perm].contiguous()
        grad = grad[perm].contiguous()
        off = K.segment_offsets(dst, n)
    force, virial = K.force_assembly(grad, vec, src, dst, off)
    order, soff = K.group_by_source(src, n)
    wf, wv = force_assembly_reference(grad.cpu(), vec.cpu(), src.cpu(), dst.cpu(), off.cpu(),
                                      soff.cpu())
    torch.testing.assert_close(force.cpu(), wf, rtol=RTOL, atol=ATOL)
    torch.testing.assert_close(virial.cpu(), wv, rtol=RTOL, atol=ATOL)
    tf, tv = truth.force_assembly(grad.cpu().numpy(), vec.cpu().numpy(), src.cpu().numpy(),
                                  dst.cpu().numpy(), n)
    # one fp32 rounding of an fp64 sum: within 2 ulp (2^-22 relative) of the truth
    np.testing.assert_allclose(force.cpu().numpy(), tf, rtol=2.0 ** -22, atol=5e-8)
    np.testing.assert_allclose(virial.cpu().numpy(), tv, rtol=2.0 ** -22, atol=5e-8)
    f2, v2 = K.force_assembly(grad, vec, src, dst, off, soff, order)
    assert torch.equal(force, f2) and torch.equal(virial, v2)
