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
