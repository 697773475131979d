"""GPU parity of the fused segment attention and of force_assembly (B200)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden
from oracle import truth
from reference import force_assembly_reference, segment_attention_reference

pytestmark = pytest.mark.gpu

from bysj_b200 import kernels as K  # noqa: E402
from bysj_b200 import workloads as W  # noqa: E402
from test_gpu_segment import budget, graph, skewed_sizes  # noqa: E402


# ---- segment_attention -------------------------------------------------------------

def test_attention_golden(cuda):
    g = golden("segment_attention")
    out = K.segment_attention(torch.from_numpy(g["logit"]).cuda(),
                              torch.from_numpy(g["value"]).cuda(),
                              torch.from_numpy(g["offsets"]).cuda())
    np.testing.assert_allclose(out.cpu().numpy(), g["out"], rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("heads,comps,channels", [(8, 16, 64), (8, 4, 16), (4, 3, 12),
                                                  (2, 5, 6), (1, 2, 3), (16, 2, 32)])
def test_attention_matches_oracle_with_env_and_null(cuda, heads, comps, channels):
    sizes = [3, 0, 5, 1, 12, 2, 7]
    dst, off = graph(sizes)
    e = dst.numel()
    gen = torch.Generator().manual_seed(heads * 100 + channels)
    logit = torch.randn(e, heads, generator=gen) * 2
    value = torch.randn(e, comps, channels, generator=gen)
    env = torch.where(torch.rand(e, generator=gen) < 0.2, torch.tensor(0.0),
                      torch.rand(e, generator=gen) + 0.05)
    null = torch.randn(len(sizes), heads, generator=gen)
    got = K.segment_attention(logit.cuda(), value.cuda(), off, env.cuda(), null.cuda())
    want = segment_attention_reference(logit, value, dst.cpu(), off.cpu(), env, null)
    torch.testing.assert_close(got.cpu(), want, rtol=1e-5, atol=1e-6)
    plain = K.segment_attention(logit.cuda(), value.cuda(), off)
    want_plain = segment_attention_reference(logit, value, dst.cpu(), off.cpu())
    torch.testing.assert_close(plain.cpu(), want_plain, rtol=1e-5, atol=1e-6)


def test_attention_c1_fp32_bf16_and_determinism(cuda):
    g = W.c1_box(device="cuda")
    off = K.segment_offsets(g.dst, g.n_atoms)
    gen = torch.Generator(device="cuda").manual_seed(2)
    logit = torch.randn(g.n_edges, 8, device="cuda", generator=gen) * 2
    value = torch.randn(g.n_edges, 16, 64, device="cuda", generator=gen)
    out = K.segment_attention(logit, value, off)
    want = truth.segment_attention(logit.cpu().numpy(), value.cpu().numpy(),
                                   g.dst.cpu().numpy(), g.n_atoms)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5, atol=budget(want))
    fp32_oracle = segment_attention_reference(logit.cpu(), value.cpu(), g.dst.cpu(), off.cpu())
    torch.testing.assert_close(out.cpu(), fp32_oracle, rtol=1e-5, atol=1e-6)
    assert torch.equal(out, K.segment_attention(logit, value, off))
    vb = value.to(torch.bfloat16)
    out16 = K.segment_attention(logit, vb, off)
    want16 = truth.segment_attention(logit.cpu().numpy(), vb.float().cpu().numpy(),
                                     g.dst.cpu().numpy(), g.n_atoms)
    np.testing.assert_allclose(out16.cpu().numpy(), want16, rtol=1e-2, atol=1e-3)


def test_attention_skewed_split_segments_and_order(cuda):
    sizes = skewed_sizes(3, nodes=150, giant=4000)
    dst, off = graph(sizes)
    e = dst.numel()
    gen = torch.Generator().manual_seed(4)
    logit = torch.randn(e, 8, generator=gen) * 2
    value = torch.randn(e, 4, 32, generator=gen)
    env = torch.rand(e, generator=gen) + 0.05
    null = torch.randn(sizes.numel(), 8, generator=gen)
    got = K.segment_attention(logit.cuda(), value.cuda(), off, env.cuda(), null.cuda())
    want = truth.segment_attention(logit.numpy(), value.numpy(), dst.cpu().numpy(),
                                   sizes.numel(), env.numpy(), null.numpy())
    np.testing.assert_allclose(got.cpu().numpy(), want, rtol=1e-5, atol=budget(want))
    assert torch.equal(got, K.segment_attention(logit.cuda(), value.cuda(), off, env.cuda(),
                                                null.cuda()))
    perm = torch.randperm(e, generator=gen)
    lp, vp, ep = torch.empty_like(logit), torch.empty_like(value), torch.empty_like(env)
    lp[perm], vp[perm], ep[perm] = logit, value, env
    got_p = K.segment_attention(lp.cuda(), vp.cuda(), off, ep.cuda(), null.cuda(),
                                order=perm.cuda())
    np.testing.assert_allclose(got_p.cpu().numpy(), want, rtol=1e-5, atol=budget(want))


def test_attention_all_masked_segment_is_zero(cuda):
    dst, off = graph([2, 3])
    logit = torch.randn(5, 2, device="cuda")
    value = torch.randn(5, 2, 4, device="cuda")
    env = torch.tensor([0.0, -1.0, 0.5, 0.2, 0.9], device="cuda")
    out = K.segment_attention(logit, value, off, env)
    assert out[0].count_nonzero() == 0


# ---- force_assembly --------------------------------------------------------------------

def test_force_golden(cuda):
    g = golden("force_assembly")
    to = lambda k: torch.from_numpy(g[k]).cuda()  # noqa: E731
    force, virial = K.force_assembly(to("grad_edge"), to("edge_vec"), to("src"), to("dst"),
                                     to("dst_offsets"), to("src_offsets"), to("src_order"))
    np.testing.assert_allclose(force.cpu().numpy(), g["force"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(virial.cpu().numpy(), g["virial"], rtol=1e-5, atol=1e-6)


def test_force_c1_matches_oracle_and_conserves_momentum(cuda):
    g = W.c1_box(device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(8)
    grad = torch.randn(g.n_edges, 3, device="cuda", generator=gen) * 0.1
    off = K.segment_offsets(g.dst, g.n_atoms)
    force, virial = K.force_assembly(grad, g.unit, g.src, g.dst, off)
    order, soff = K.group_by_source(g.src, g.n_atoms)
    wf, wv = force_assembly_reference(grad.cpu(), g.unit.cpu(), g.src.cpu(), g.dst.cpu(),
                                      off.cpu(), soff.cpu())
    torch.testing.assert_close(force.cpu(), wf, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(virial.cpu(), wv, rtol=1e-5, atol=1e-6)
    tf, tv = truth.force_assembly(grad.cpu().numpy(), g.unit.cpu().numpy(), g.src.cpu().numpy(),
                                  g.dst.cpu().numpy(), g.n_atoms)
    np.testing.assert_allclose(force.cpu().numpy(), tf, rtol=1e-6, atol=1e-6)
    torch.testing.assert_close(force.double().sum(0).cpu(), torch.zeros(3, dtype=torch.float64),
                               atol=1e-4, rtol=0)
    f2, v2 = K.force_assembly(grad, g.unit, g.src, g.dst, off, soff, order)
    assert torch.equal(force, f2) and torch.equal(virial, v2)


def test_force_heavy_atoms_use_several_slot_rounds(cuda):
    # 64 atoms of 80-400 edges per side: every atom runs several 60-slot
    # chunks of its triplet loop
    gen = torch.Generator().manual_seed(21)
    sizes = torch.randint(80, 400, (64,), generator=gen)
    dst = torch.repeat_interleave(torch.arange(64), sizes)
    off = torch.zeros(65, dtype=torch.int64)
    off[1:] = torch.cumsum(sizes, 0)
    e = dst.numel()
    src = torch.randint(0, 64, (e,), generator=gen)
    grad, vec = torch.randn(e, 3, generator=gen), torch.randn(e, 3, generator=gen)
    force, virial = K.force_assembly(grad.cuda(), vec.cuda(), src.cuda(), dst.cuda(), off.cuda())
    tf, tv = truth.force_assembly(grad.numpy(), vec.numpy(), src.numpy(), dst.numpy(), 64)
    # fp64 sums rounded once to fp32: within 2 ulp of the float64 truth
    np.testing.assert_allclose(force.cpu().numpy(), tf, rtol=2.0 ** -22, atol=1e-7)
    np.testing.assert_allclose(virial.cpu().numpy(), tv, rtol=2.0 ** -22, atol=1e-7)


def test_force_skewed_and_empty_atom(cuda):
    sizes = skewed_sizes(6, nodes=120, giant=3000)
    dst, off = graph(sizes)
    e = dst.numel()
    gen = torch.Generator().manual_seed(6)
    src = torch.randint(0, sizes.numel(), (e,), generator=gen)
    src[src == 7] = 8  # atom 7 has no source edges
    grad, vec = torch.randn(e, 3, generator=gen), torch.randn(e, 3, generator=gen)
    force, virial = K.force_assembly(grad.cuda(), vec.cuda(), src.cuda(), dst, off)
    tf, tv = truth.force_assembly(grad.numpy(), vec.numpy(), src.numpy(), dst.cpu().numpy(),
                                  sizes.numel())
    np.testing.assert_allclose(force.cpu().numpy(), tf, rtol=2.0 ** -22, atol=1e-7)
    np.testing.assert_allclose(virial.cpu().numpy(), tv, rtol=2.0 ** -22, atol=1e-7)


def test_force_hub_source_atom_and_unsorted_sources(cuda):
    # Atom 37 is the source of 4000 extra edges (a hub on the gathered side),
    # sources are in random order inside each destination segment, and edge
    # vectors are long (|v| ~ 5): forces and virials stay within 2 ulp of the
    # float64 truth, repeats are bit-identical, and the source-side partial
    # used by the multi-GPU partition agrees with the truth in fp64.
    gen = torch.Generator().manual_seed(33)
    n = 200
    sizes = torch.randint(50, 120, (n,), generator=gen)
    dst = torch.repeat_interleave(torch.arange(n), sizes)
    off = torch.zeros(n + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(sizes, 0)
    e = dst.numel()
    src = torch.randint(0, n, (e,), generator=gen)
    src[torch.randperm(e, generator=gen)[:4000]] = 37
    grad = torch.randn(e, 3, generator=gen) * 0.1
    vec = torch.randn(e, 3, generator=gen) * 3.0
    force, virial = K.force_assembly(grad.cuda(), vec.cuda(), src.cuda(), dst.cuda(), off.cuda())
    tf, tv = truth.force_assembly(grad.numpy(), vec.numpy(), src.numpy(), dst.numpy(), n)
    np.testing.assert_allclose(force.cpu().numpy(), tf, rtol=2.0 ** -22, atol=1e-7)
    np.testing.assert_allclose(virial.cpu().numpy(), tv, rtol=2.0 ** -22, atol=1e-7)
    f2, v2 = K.force_assembly(grad.cuda(), vec.cuda(), src.cuda(), dst.cuda(), off.cuda())
    assert torch.equal(force, f2) and torch.equal(virial, v2)
    # the source-side partial (multi-GPU form) takes the same two paths
    order, soff = K.group_by_source(src.cuda(), n)
    part = _C().force_assembly_src_partial(grad.cuda(), vec.cuda(), soff, order)
    src_only = truth.force_assembly(grad.numpy(), vec.numpy(), src.numpy(), dst.numpy(), n)
    dst_side = np.zeros((n, 3))
    np.add.at(dst_side, dst.numpy(), grad.numpy().astype(np.float64))
    np.testing.assert_allclose(part[:, :3].cpu().numpy(), src_only[0] - dst_side,
                               rtol=2.0 ** -22, atol=1e-7)
    np.testing.assert_allclose(part[:, 3:].cpu().numpy(), src_only[1], rtol=2.0 ** -22,
                               atol=1e-7)


@pytest.mark.parametrize("parts", [2, 3])
def test_force_dst_range_partition_matches_single_device(cuda, parts):
    # ranks emulated on one GPU: the reduce-scatter becomes a plain sum of the padded partials
    from bysj_b200 import sharding as S

    g = W.c1_box(device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(9)
    grad = torch.randn(g.n_edges, 3, device="cuda", generator=gen)
    off = K.segment_offsets(g.dst, g.n_atoms)
    force, virial = K.force_assembly(grad, g.edge_vec, g.src, g.dst, off)
    plan = [S.make_partition(off, g.src, r, parts) for r in range(parts)]
    partials = [_C().force_assembly_src_partial(p.edges(grad), p.edges(g.edge_vec),
                                                p.src_offsets, p.src_order) for p in plan]
    total = torch.stack(partials).sum(0)
    got_f, got_v = [], []
    for p in plan:
        f, v = S.force_assembly_partitioned(
            p.edges(grad), p.edges(g.edge_vec), p,
            combine=lambda _, q: total[q.rank * q.chunk:(q.rank + 1) * q.chunk])
        got_f.append(f)
        got_v.append(v)
    # fp64 partials: the partitioned sums round to fp32 once, as on one device
    torch.testing.assert_close(torch.cat(got_f), force, rtol=2.0 ** -22, atol=1e-7)
    torch.testing.assert_close(torch.cat(got_v), virial, rtol=2.0 ** -22, atol=1e-7)


def _C():
    from bysj_b200 import _C as ext

    return ext
