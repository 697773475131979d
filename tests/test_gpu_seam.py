"""The DeepMD seam with the real B200 operator bundle on CUDA tensors.

``deepmd_patch`` is installed with its default operators (``bysj_b200.kernels``)
over DeepMD stand-ins -- a softmax namespace, an SO(2) block and a
post-processing namespace whose stock paths are plain torch -- and each
patched call is compared with the stock call on the same CUDA inputs, as the
reference's host stand-in (``tests/python/test_fused_deepmd.py:102-123``)
does on CPU.  Counters must show hits and no fallbacks; the CSR view must be
built on the device (no ``order`` for a destination-sorted edge list).
"""
from __future__ import annotations

import types

import pytest
import torch

from reference import segment_softmax_reference

pytestmark = pytest.mark.gpu

from bysj_b200 import workloads as W  # noqa: E402
from bysj_b200.model import fused_deepmd  # noqa: E402
from test_fused_deepmd import FakeBlock, FakeModel, fake_transform_output  # noqa: E402


def softmax_namespace():
    module = types.ModuleType("fake.sezm_nn.attention")

    def stock(logits, edge_env, dst, n_nodes, z_bias_raw, eps, src_weight=None):
        e, f, h = logits.shape
        d = dst.cpu()
        order = torch.argsort(d, stable=True)
        off = torch.zeros(n_nodes + 1, dtype=torch.int64)
        off[1:] = torch.cumsum(torch.bincount(d, minlength=n_nodes), 0)
        null = torch.log(torch.nn.functional.softplus(z_bias_raw.reshape(-1).cpu()) + eps)
        lg = logits.reshape(e, f * h).cpu()[order]
        env = edge_env.reshape(e).cpu()[order]
        alpha, _ = segment_softmax_reference(lg, env, d[order], off,
                                             null.reshape(1, -1).expand(n_nodes, f * h))
        out = torch.empty_like(alpha)
        out[order] = alpha
        return out.reshape(e, f, h).to(logits.device)

    module.segment_envelope_gated_softmax = stock
    return module


@pytest.fixture
def graph(cuda):
    g = W.c1_box(device="cuda")
    yield g
    fused_deepmd.uninstall()


@pytest.mark.parametrize("shuffle", [False, True])
def test_softmax_seam_with_the_b200_kernels(graph, shuffle):
    g = graph
    gen = torch.Generator(device="cuda").manual_seed(4)
    dst = g.dst
    if shuffle:
        dst = dst[torch.randperm(dst.numel(), device="cuda", generator=gen)].contiguous()
    e = dst.numel()
    logits = torch.randn(e, 2, 4, device="cuda", generator=gen)
    env = torch.rand(e, 1, device="cuda", generator=gen) + 0.05
    bias = torch.randn(2, 4, device="cuda", generator=gen)
    ns = softmax_namespace()
    stats = fused_deepmd.deepmd_patch(FakeModel([]), namespaces=[ns], envelope=False,
                                      verbose=False)
    assert stats.bound_softmax
    got = ns.segment_envelope_gated_softmax(logits, env, dst, g.n_atoms, bias, 1e-6)
    assert got.is_cuda and stats.softmax_hits == 1 and stats.softmax_fallbacks == 0
    offsets, order = fused_deepmd._SESSION.csr.get(dst, g.n_atoms)
    assert offsets.is_cuda and (order is None) == (not shuffle)
    fused_deepmd.uninstall()
    want = ns.segment_envelope_gated_softmax(logits, env, dst, g.n_atoms, bias, 1e-6)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)


def test_envelope_seam_with_the_b200_kernels(graph):
    g = graph
    gen = torch.Generator(device="cuda").manual_seed(5)
    e, n = g.n_edges, g.n_atoms
    cache = types.SimpleNamespace(
        dst=g.dst, edge_env=torch.rand(e, 1, device="cuda", generator=gen) + 0.1,
        inv_sqrt_deg=torch.rand(n, 1, 1, device="cuda", generator=gen) + 0.5,
        edge_src_gate=torch.rand(e, 1, device="cuda", generator=gen))
    message = torch.randn(e, 16, 8, device="cuda", generator=gen)
    x = torch.zeros(n, 16, 8, device="cuda")
    block = FakeBlock(message)
    stats = fused_deepmd.deepmd_patch(FakeModel([block]), softmax=False, verbose=False)
    assert stats.bound_envelope
    got = block.forward_envelope(x, cache, None)
    assert stats.envelope_hits == 1 and stats.envelope_fallbacks == 0
    fused_deepmd.uninstall()
    want = block.forward_envelope(x, cache, None)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("shuffle", [False, True])
def test_force_seam_with_the_b200_kernels(graph, shuffle):
    g = graph
    gen = torch.Generator(device="cuda").manual_seed(6)
    src, dst, vec = g.src, g.dst, g.edge_vec
    if shuffle:
        perm = torch.randperm(g.n_edges, device="cuda", generator=gen)
        src, dst, vec = src[perm].contiguous(), dst[perm].contiguous(), vec[perm].contiguous()
    grad = torch.randn(g.n_edges, 3, device="cuda", generator=gen) * 0.1
    ns = fake_transform_output()
    stats = fused_deepmd.deepmd_patch(FakeModel([]), softmax=False, envelope=False, force=True,
                                      force_namespaces=[ns], verbose=False)
    assert stats.bound_force
    force, virial = ns.edge_force_virial(grad, vec, src, dst, g.n_atoms)
    again = ns.edge_force_virial(grad, vec, src, dst, g.n_atoms)
    assert stats.force_hits == 2 and stats.force_fallbacks == 0
    assert torch.equal(force, again[0]) and torch.equal(virial, again[1])
    fused_deepmd.uninstall()
    # The stock path in float64: its fp32 form sums with atomics in arrival
    # order (a virial element can cancel to ~1e-2 and land 1e-6 off), while
    # the fused kernel sums in fp64 and rounds once.
    stock_force, stock_virial = ns.edge_force_virial(grad.double(), vec.double(), src, dst,
                                                     g.n_atoms)
    torch.testing.assert_close(force.double(), stock_force, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(virial.double(), stock_virial, rtol=1e-5, atol=1e-6)
