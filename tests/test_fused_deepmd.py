"""Host tests of the DeepMD seam with stand-ins (no GPU, no DeepMD).

Modelled on the reference's ``tests/python/test_fused_deepmd.py``: the two
seams run against fake DeepMD modules and an operator bundle that computes
with the CPU oracle, so the patched path can be compared numerically with the
stock one; the counters, restore-on-uninstall, idempotent install, arity
tolerance, wrapper resolution and the module dump are checked.  The fake
bundle also supplies ``segment_offsets`` (the seam builds its CSR view with
the bundle's own builder).
"""
from __future__ import annotations

import contextlib
import io
import types
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import truth
from reference import segment_softmax_reference, segment_sum_reference

from bysj_b200.model import fused_deepmd
from bysj_b200.model.dpa4 import _normalize_fused


def grouped(counts):
    dst = torch.repeat_interleave(torch.arange(len(counts)), torch.tensor(counts))
    off = torch.zeros(len(counts) + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(torch.tensor(counts), 0)
    return dst, off


def dst_from_csr(offsets, order):
    counts = (offsets[1:] - offsets[:-1]).tolist()
    grouped_ids = torch.repeat_interleave(torch.arange(offsets.numel() - 1), torch.tensor(counts))
    if order is None:
        return grouped_ids
    dst = torch.empty_like(grouped_ids)
    dst[order] = grouped_ids
    return dst


class FakeOps:
    def __init__(self):
        self.calls = []

    def segment_offsets(self, dst, n_nodes):
        return torch.from_numpy(truth.segment_offsets(dst.numpy(), n_nodes))

    def segment_softmax(self, logit, env, offsets, null_logit=None, order=None):
        self.calls.append(("softmax", tuple(logit.shape)))
        alpha, null_alpha = segment_softmax_reference(logit, env, dst_from_csr(offsets, order),
                                                      offsets, null_logit)
        return alpha if null_logit is None else (alpha, null_alpha)

    def segment_sum(self, src, dst, offsets, edge_scale=None, node_scale=None, order=None):
        self.calls.append(("sum", tuple(src.shape)))
        return segment_sum_reference(src, dst_from_csr(offsets, order), offsets, edge_scale,
                                     node_scale)

    def group_by_source(self, src, n_nodes):
        order, offsets = truth.group_by_source(src.numpy(), n_nodes)
        return torch.from_numpy(order), torch.from_numpy(offsets)

    def force_assembly(self, grad_edge, edge_vec, src, dst, dst_offsets, src_offsets=None,
                       src_order=None):
        self.calls.append(("force", tuple(grad_edge.shape)))
        # the device kernel walks destination segments in place: dst must be grouped
        assert torch.equal(dst_from_csr(dst_offsets, None), dst)
        f, w = truth.force_assembly(grad_edge.numpy(), edge_vec.numpy(), src.numpy(),
                                    dst.numpy(), dst_offsets.numel() - 1)
        return torch.from_numpy(f).float(), torch.from_numpy(w).float()


class DeviceCsrOps(FakeOps):
    """A bundle with the device CSR view: ``order`` is None for sorted dst."""

    def destination_csr(self, dst, n_nodes):
        self.calls.append(("csr", int(dst.numel())))
        offsets = self.segment_offsets(dst, n_nodes)
        sorted_ = bool((dst[1:] >= dst[:-1]).all()) if dst.numel() > 1 else True
        return offsets, None if sorted_ else torch.argsort(dst, stable=True)


class FakeEdgeCache:
    def __init__(self, counts):
        self.dst, self.offsets = grouped(counts)
        self.edge_env = torch.rand(self.dst.numel(), 1) + 0.1
        self.inv_sqrt_deg = torch.rand(len(counts), 1, 1) + 0.5
        self.edge_src_gate = None


class FakeBlock:
    def __init__(self, message):
        self.training = False
        self._segment_softmax_fn = None
        self._message = message

    def edge_message(self, x, edge_cache, radial_feat):
        return self._message, None

    def forward_envelope(self, x, edge_cache, radial_feat):
        message, _ = self.edge_message(x, edge_cache, radial_feat)
        weight = edge_cache.edge_env if edge_cache.edge_src_gate is None else (
            edge_cache.edge_env * edge_cache.edge_src_gate)
        out = x.new_zeros(x.shape)
        out.index_add_(0, edge_cache.dst, message * weight.unsqueeze(-1))
        return out.mul_(edge_cache.inv_sqrt_deg)


class FakeModel:
    def __init__(self, blocks):
        self._blocks = blocks

    def modules(self):
        return list(self._blocks)


def fake_namespace(name):
    module = types.ModuleType(name)

    def stock(logits, edge_env, dst, n_nodes, z_bias_raw, eps, src_weight=None):
        e, f, h = logits.shape
        off = torch.from_numpy(truth.segment_offsets(dst.numpy(), n_nodes))
        null = torch.log(torch.nn.functional.softplus(z_bias_raw.reshape(-1)) + eps)
        alpha, _ = segment_softmax_reference(logits.reshape(e, f * h), edge_env.reshape(e), dst,
                                             off, null.reshape(1, -1).expand(n_nodes, f * h))
        return alpha.reshape(e, f, h)

    module.segment_envelope_gated_softmax = stock
    return module


@pytest.fixture(autouse=True)
def cpu_seams():
    fused_deepmd._ACCEPT_ANY_DEVICE = True
    yield
    fused_deepmd.uninstall()
    fused_deepmd._ACCEPT_ANY_DEVICE = False


def test_softmax_seam_matches_stock_path():
    ns = fake_namespace("fake.attention")
    ops = FakeOps()
    stats = fused_deepmd.deepmd_patch(FakeModel([]), ops=ops, namespaces=[ns], envelope=False,
                                      verbose=False)
    assert stats.bound_softmax
    dst, _ = grouped([2, 0, 3])
    logits, env, bias = torch.randn(5, 2, 3), torch.rand(5, 1) + 0.1, torch.randn(2, 3)
    got = ns.segment_envelope_gated_softmax(logits, env, dst, 3, bias, 1e-6)
    fused_deepmd.uninstall()
    want = ns.segment_envelope_gated_softmax(logits, env, dst, 3, bias, 1e-6)
    torch.testing.assert_close(got, want, rtol=2e-5, atol=2e-6)
    assert stats.softmax_hits == 1 and ops.calls[0][0] == "softmax"


def test_source_weighted_softmax_falls_back():
    ns = fake_namespace("fake.attention")
    ops = FakeOps()
    fused_deepmd.deepmd_patch(FakeModel([]), ops=ops, namespaces=[ns], envelope=False,
                              verbose=False)
    dst, _ = grouped([2, 0, 3])
    stats = fused_deepmd._SESSION.stats
    ns.segment_envelope_gated_softmax(torch.randn(5, 2, 3), torch.rand(5, 1) + 0.1, dst, 3,
                                      torch.randn(2, 3), 1e-6, torch.rand(5, 1))
    assert (stats.softmax_fallbacks, stats.softmax_hits, ops.calls) == (1, 0, [])


def test_failing_operator_falls_back_and_warns_once():
    class Broken(FakeOps):
        def segment_softmax(self, *args, **kwargs):
            raise RuntimeError("device exploded")

    ns = fake_namespace("fake.attention")
    fused_deepmd.deepmd_patch(FakeModel([]), ops=Broken(), namespaces=[ns], envelope=False,
                              verbose=False)
    dst, _ = grouped([2, 3])
    args = (torch.randn(5, 2, 3), torch.rand(5, 1) + 0.1, dst, 2, torch.randn(2, 3), 1e-6)
    with pytest.warns(RuntimeWarning, match="fell back"):
        out = ns.segment_envelope_gated_softmax(*args)
    assert out.shape == (5, 2, 3)
    ns.segment_envelope_gated_softmax(*args)
    stats = fused_deepmd._SESSION.stats
    assert stats.softmax_fallbacks == 2 and "device exploded" in stats.last_error


def test_envelope_seam_matches_stock_aggregation():
    cache = FakeEdgeCache([2, 1, 3])
    block = FakeBlock(torch.randn(int(cache.dst.numel()), 2, 4))
    ops = FakeOps()
    stats = fused_deepmd.deepmd_patch(FakeModel([block]), ops=ops, softmax=False, verbose=False)
    assert stats.bound_envelope
    x = torch.randn(3, 2, 4)
    got = block.forward_envelope(x, cache, None)
    fused_deepmd.uninstall()
    want = block.forward_envelope(x, cache, None)
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5 * float(want.abs().max()))
    assert stats.envelope_hits == 1 and ops.calls[0][0] == "sum"


def test_training_block_falls_back():
    cache = FakeEdgeCache([2, 1])
    block = FakeBlock(torch.randn(3, 2, 4))
    block.training = True
    stats = fused_deepmd.deepmd_patch(FakeModel([block]), ops=FakeOps(), softmax=False,
                                      verbose=False)
    block.forward_envelope(torch.randn(2, 2, 4), cache, None)
    assert stats.envelope_fallbacks == 1 and stats.envelope_hits == 0


def test_uninstall_restores_every_name():
    ns = fake_namespace("fake.attention")
    original = ns.segment_envelope_gated_softmax
    cache = FakeEdgeCache([1, 2])
    block = FakeBlock(torch.randn(int(cache.dst.numel()), 2, 4))
    fused_deepmd.deepmd_patch(FakeModel([block]), ops=FakeOps(), namespaces=[ns], verbose=False)
    assert ns.segment_envelope_gated_softmax is not original
    assert "forward_envelope" in block.__dict__
    fused_deepmd.uninstall()
    assert ns.segment_envelope_gated_softmax is original
    assert "forward_envelope" not in block.__dict__
    assert block.forward_envelope.__func__ is FakeBlock.forward_envelope


def test_install_without_extension_is_a_noop():
    model = FakeModel([FakeBlock(torch.zeros(2, 1, 1))])
    stats = fused_deepmd.deepmd_patch(model, ops=None, verbose=False)
    assert not (stats.bound_softmax or stats.bound_envelope)
    assert fused_deepmd.status(stats)["blocks"] == 1


def test_installing_twice_keeps_one_patch():
    ns = fake_namespace("fake.attention")
    original = ns.segment_envelope_gated_softmax
    for _ in range(2):
        stats = fused_deepmd.deepmd_patch(FakeModel([]), ops=FakeOps(), namespaces=[ns],
                                          envelope=False, verbose=False)
        assert stats.softmax_hits == 0
    keys = [k for k in fused_deepmd._SAVED if k.endswith(".segment_envelope_gated_softmax")]
    assert len(keys) == 1
    fused_deepmd.uninstall()
    assert ns.segment_envelope_gated_softmax is original
    assert fused_deepmd.status(None) == {}


def test_plain_tensor_return_is_accepted():
    class TensorOps(FakeOps):
        def segment_softmax(self, logit, env, offsets, null_logit=None, order=None):
            return FakeOps.segment_softmax(self, logit, env, offsets, null_logit, order)[0]

    ns = fake_namespace("fake.attention")
    fused_deepmd.deepmd_patch(FakeModel([]), ops=TensorOps(), namespaces=[ns], envelope=False,
                              verbose=False)
    dst, _ = grouped([2, 0, 3])
    alpha = ns.segment_envelope_gated_softmax(torch.randn(5, 2, 3), torch.rand(5, 1) + 0.1, dst, 3,
                                              torch.randn(2, 3), 1e-6)
    assert tuple(alpha.shape) == (5, 2, 3)


def test_csr_view_is_cached_by_dst_storage():
    ops = FakeOps()
    view = fused_deepmd._CsrView(ops.segment_offsets, capacity=2)
    dst, off = grouped([3, 0, 2])
    first = view.get(dst, 3)
    assert view.get(dst, 3) is first
    np.testing.assert_array_equal(first[0].numpy(), off.numpy())
    for k in range(3):  # evict
        view.get(grouped([k + 1, 1])[0], 2)
    assert view.get(dst, 3) is not first


def test_wrapper_resolution():
    root = FakeModel([FakeBlock(torch.zeros(2, 1, 1))])
    assert fused_deepmd._module_root(SimpleNamespace(deep_eval=SimpleNamespace(dp=root))) == (
        root, "deep_eval.dp")
    assert fused_deepmd._module_root(SimpleNamespace(deep_eval=SimpleNamespace(_dpmodel=root))) == (
        root, "deep_eval._dpmodel")
    assert fused_deepmd._module_root(SimpleNamespace(deep_eval=SimpleNamespace())) == (None, "")
    lines = fused_deepmd.describe_module(SimpleNamespace(deep_eval=SimpleNamespace()))
    assert "no nn.Module tree" in "\n".join(lines)
    cache = FakeEdgeCache([2, 1, 3])
    block = FakeBlock(torch.randn(int(cache.dst.numel()), 2, 4))
    wrapper = SimpleNamespace(deep_eval=SimpleNamespace(dp=FakeModel([block])))
    stats = fused_deepmd.deepmd_patch(wrapper, ops=FakeOps(), softmax=False, verbose=False)
    assert stats.bound_envelope and stats.blocks == 1


def test_module_dump_and_verbose_install():
    cache = FakeEdgeCache([2, 1])
    block = FakeBlock(torch.randn(int(cache.dst.numel()), 2, 4))
    text = "\n".join(fused_deepmd.describe_module(FakeModel([block])))
    assert "module: FakeModel" in text
    assert "patch targets: 1 SO(2) block(s)" in text
    assert "forward_envelope -> segment_sum" in text
    buffer = io.StringIO()
    with contextlib.redirect_stdout(buffer):
        fused_deepmd.deepmd_patch(FakeModel([]), ops=FakeOps(),
                                  namespaces=[fake_namespace("fake.attention")], envelope=False)
    out = buffer.getvalue()
    assert "[deepmd_patch] module:" in out and "segment_envelope_gated_softmax" in out


def test_fused_switch_parsing():
    assert _normalize_fused(True) == {"softmax": True, "envelope": True}
    assert _normalize_fused("force") == {"force": True}
    assert _normalize_fused({"force": True}) == {"softmax": False, "envelope": False,
                                                 "force": True}
    assert _normalize_fused("softmax") == {"softmax": True}
    assert _normalize_fused(("envelope",)) == {"envelope": True}
    assert _normalize_fused({"softmax": True, "envelope": False}) == {"softmax": True,
                                                                      "envelope": False}
    for bad in ("flash", {"flash": True}):
        with pytest.raises(ValueError):
            _normalize_fused(bad)
    with pytest.raises(TypeError):
        _normalize_fused(3)
    assert _normalize_fused(False) is None and _normalize_fused(None) is None
    assert _normalize_fused(()) is None


# ---- force seam --------------------------------------------------------------------------

def fake_transform_output(name="fake.transform_output"):
    """Stand-in for DeepMD's post-processing namespace: ``edge_force_virial``
    as four ``index_add_`` scatters in fp32, the stock path the seam replaces."""
    module = types.ModuleType(name)

    def edge_force_virial(g, edge_vec, src, dst, n_ext):
        force = g.new_zeros(n_ext, 3)
        force.index_add_(0, dst, g)
        force.index_add_(0, src, -g)
        virial = g.new_zeros(n_ext, 9)
        virial.index_add_(0, src, -(g[:, :, None] * edge_vec[:, None, :]).reshape(-1, 9))
        return force, virial

    module.edge_force_virial = edge_force_virial
    return module


def toy_system(n=12, seed=0, shuffle=False):
    """Random positions, all directed pairs within 2.5, and a pair energy
    E = sum_e exp(-|v_e|^2) with v_e = r_src - r_dst."""
    gen = torch.Generator().manual_seed(seed)
    pos = (torch.rand(n, 3, generator=gen, dtype=torch.float64) * 4.0).requires_grad_(True)
    d = (pos[None, :, :] - pos[:, None, :]).detach()
    close = (d.norm(dim=-1) < 2.5) & ~torch.eye(n, dtype=torch.bool)
    dst, src = close.nonzero(as_tuple=True)
    if shuffle:
        perm = torch.randperm(dst.numel(), generator=gen)
        dst, src = dst[perm], src[perm]
    vec = pos[src] - pos[dst]
    energy = torch.exp(-(vec * vec).sum(-1)).sum()
    g, = torch.autograd.grad(energy, vec, retain_graph=True)
    forces, = torch.autograd.grad(energy, pos)
    return (g.float().contiguous(), vec.detach().float().contiguous(), src.contiguous(),
            dst.contiguous(), n, -forces)


@pytest.mark.parametrize("shuffle", [False, True])
def test_force_seam_matches_stock_and_minus_the_energy_gradient(shuffle):
    ns = fake_transform_output()
    ops = DeviceCsrOps()
    stats = fused_deepmd.deepmd_patch(FakeModel([]), ops=ops, softmax=False, envelope=False,
                                      force=True, force_namespaces=[ns], verbose=False)
    assert stats.bound_force
    g, vec, src, dst, n, want_force = toy_system(shuffle=shuffle)
    force, virial = ns.edge_force_virial(g, vec, src, dst, n)
    assert stats.force_hits == 1 and ("force", tuple(g.shape)) in ops.calls
    # sign: the assembled forces are minus the gradient of the energy
    torch.testing.assert_close(force.double(), want_force, rtol=1e-5, atol=1e-6)
    # momentum is conserved and the atom virials sum to -sum_e g (x) v
    torch.testing.assert_close(force.double().sum(0), torch.zeros(3, dtype=torch.float64),
                               rtol=0, atol=1e-5)
    total = -(g.double()[:, :, None] * vec.double()[:, None, :]).reshape(-1, 9).sum(0)
    torch.testing.assert_close(virial.double().sum(0), total, rtol=1e-5, atol=1e-6)
    # same as the stock scatters and as the loop oracle
    fused_deepmd.uninstall()
    stock_force, stock_virial = ns.edge_force_virial(g, vec, src, dst, n)
    torch.testing.assert_close(force, stock_force, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(virial, stock_virial, rtol=1e-5, atol=1e-6)
    from oracle import loops

    lf, lw = loops.force_assembly(g.tolist(), vec.tolist(), src.tolist(), dst.tolist(), n)
    np.testing.assert_allclose(force.numpy(), np.asarray(lf), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(virial.numpy(), np.asarray(lw), rtol=1e-5, atol=1e-6)


def test_force_seam_falls_back_and_restores():
    ns = fake_transform_output()
    stock = ns.edge_force_virial
    stats = fused_deepmd.deepmd_patch(FakeModel([]), ops=DeviceCsrOps(), softmax=False,
                                      envelope=False, force=True, force_namespaces=[ns],
                                      verbose=False)
    g, vec, src, dst, n, _ = toy_system(seed=3)
    ns.edge_force_virial(g.double(), vec, src, dst, n)          # not fp32
    ns.edge_force_virial(g.requires_grad_(True), vec, src, dst, n)  # in the autograd graph
    assert stats.force_fallbacks == 2 and stats.force_hits == 0
    fused_deepmd.uninstall()
    assert ns.edge_force_virial is stock
    # a namespace without the name binds nothing
    stats = fused_deepmd.deepmd_patch(FakeModel([]), ops=DeviceCsrOps(), softmax=False,
                                      envelope=False, force=True,
                                      force_namespaces=[types.ModuleType("fake.empty")],
                                      verbose=False)
    assert not stats.bound_force


def test_device_csr_view_keeps_sorted_edges_in_place():
    ns = fake_namespace("fake.attention")
    ops = DeviceCsrOps()
    stats = fused_deepmd.deepmd_patch(FakeModel([]), ops=ops, namespaces=[ns], envelope=False,
                                      verbose=False)
    dst, _ = grouped([2, 0, 3])
    logits, env, bias = torch.randn(5, 2, 3), torch.rand(5, 1) + 0.1, torch.randn(2, 3)
    ns.segment_envelope_gated_softmax(logits, env, dst, 3, bias, 1e-6)
    assert ("csr", 5) in ops.calls and stats.softmax_hits == 1
    view = fused_deepmd._CsrView(csr=ops.destination_csr)
    assert view.get(dst, 3)[1] is None
    shuffled = dst[torch.tensor([4, 0, 3, 1, 2])]
    offsets, order = view.get(shuffled, 3)
    assert torch.equal(shuffled[order], dst)
    # an in-place change of dst is not served the cached view
    before = view.get(shuffled, 3)
    shuffled[0] = 2
    assert view.get(shuffled, 3) is not before
