"""Host-side contracts of the operator wrappers (no GPU).

Ported from the reference's host suite (``tests/python/test_segment_validation.py``,
``test_rmsnorm.py``, ``test_gie.py``, ``test_native_package.py``): validators
accept optional arguments, reject bad inputs with the documented exception
types before any device work, the public entry points stop at the device guard
on CPU tensors, and the autograd wiring dispatches to the extension entry
points (checked with a fake extension that computes with the oracle).

Deliberate difference: the device guard's message names the B200 / CUDA
requirement instead of "DCU".
"""
from __future__ import annotations

import importlib
import math
from types import SimpleNamespace
from unittest.mock import patch

import pytest
import torch

from reference import rmsnorm as reference_rmsnorm
from reference import segment_softmax_reference, segment_sum_reference, zonal_scatter_reference

import bysj_b200.kernels as kernels
from bysj_b200.kernels.segment import (
    _validate_force_assembly,
    _validate_order,
    _validate_segment_softmax,
    _validate_segment_sum,
    force_assembly,
    group_by_source,
    segment_offsets,
    segment_softmax,
    segment_sum,
)

seg_mod = importlib.import_module("bysj_b200.kernels.segment")
norm_mod = importlib.import_module("bysj_b200.kernels.rmsnorm")
gie_mod = importlib.import_module("bysj_b200.kernels.gie")
attn_mod = importlib.import_module("bysj_b200.kernels.attention")
native = importlib.import_module("bysj_b200.kernels.native")

NO_GPU = pytest.mark.skipif(torch.cuda.is_available(), reason="guard behaviour on a CPU host")


def _graph():
    return torch.tensor([0, 0, 1, 2, 2]), torch.tensor([0, 2, 3, 5])


# ---- package surface ---------------------------------------------------------------

def test_package_exports_reference_names_plus_fused_attention():
    reference_names = [
        "force_assembly", "gie_available", "gie_zonal_scatter", "group_by_source", "rmsnorm",
        "rmsnorm_available", "segment_available", "segment_offsets", "segment_softmax",
        "segment_sum", "zonal_scatter",
    ]
    additive = {"segment_attention", "rotate_back_aggregate", "edge_chain"}
    assert sorted(set(kernels.__all__) - additive) == reference_names
    assert kernels.__all__ == sorted(kernels.__all__)
    for name in kernels.__all__:
        assert callable(getattr(kernels, name))


# ---- validators ------------------------------------------------------------------------

def test_segment_sum_validator_optionals():
    dst, offsets = _graph()
    src = torch.randn(5, 4)
    assert _validate_segment_sum(src, dst, offsets, None, None, None) == 3
    assert _validate_segment_sum(src, dst, offsets, torch.rand(5), torch.rand(3),
                                 torch.arange(5)) == 3
    assert _validate_segment_sum(src.bfloat16(), dst, offsets, None, None, None) == 3
    with pytest.raises(ValueError):
        _validate_segment_sum(torch.randn(4, 4), dst, offsets, None, None, None)
    with pytest.raises(TypeError):
        _validate_segment_sum(src.double(), dst, offsets, None, None, None)
    with pytest.raises(ValueError):
        _validate_segment_sum(src, dst, offsets, None, torch.rand(2), None)
    with pytest.raises(ValueError):
        _validate_segment_sum(torch.randn(4, 5).t(), torch.tensor([0, 0, 1, 2, 2]), offsets,
                              None, None, None)


def test_segment_softmax_validator():
    _, offsets = _graph()
    assert _validate_segment_softmax(torch.randn(5, 6), torch.rand(5), offsets, None, None) == (3, 6)
    assert _validate_segment_softmax(torch.randn(5, 6), torch.rand(5), offsets, torch.randn(3, 6),
                                     torch.arange(5)) == (3, 6)
    with pytest.raises(ValueError):
        _validate_segment_softmax(torch.randn(5, 6), torch.rand(5), offsets, torch.randn(2, 6), None)
    with pytest.raises(TypeError):
        _validate_segment_softmax(torch.randn(5, 6).double(), torch.rand(5), offsets, None, None)


def test_order_validator():
    with pytest.raises(TypeError):
        _validate_order(torch.arange(5, dtype=torch.float32), 5, "probe")
    with pytest.raises(ValueError):
        _validate_order(torch.arange(4), 5, "probe")
    assert _validate_order(None, 5, "probe") is None


def test_force_assembly_validator():
    _, off = _graph()
    order = torch.tensor([1, 4, 3, 0, 2])
    assert _validate_force_assembly(torch.randn(5, 3), torch.randn(5, 3), off, off, order) == 3
    with pytest.raises(ValueError):
        _validate_force_assembly(torch.randn(5, 2), torch.randn(5, 2), off, off, order)
    with pytest.raises(ValueError):
        _validate_force_assembly(torch.randn(5, 3), torch.randn(5, 3), off, torch.tensor([0, 5]),
                                 order)


def test_offsets_argument_checks_precede_the_guard():
    with pytest.raises(TypeError):
        segment_offsets([0, 1], 2)
    with pytest.raises(TypeError):
        segment_offsets(torch.tensor([0, 1], dtype=torch.int32), 2)
    with pytest.raises(ValueError):
        segment_offsets(torch.tensor([0, 1]), 0)
    with pytest.raises(TypeError):
        group_by_source(torch.tensor([0.0]), 2)


# ---- device guard ------------------------------------------------------------------------

@NO_GPU
def test_public_entry_points_stop_at_the_device_guard():
    dst, offsets = _graph()
    with pytest.raises(RuntimeError, match="B200|CUDA"):
        segment_sum(torch.randn(5, 4), dst, offsets)
    with pytest.raises(RuntimeError, match="B200|CUDA"):
        segment_softmax(torch.randn(5, 6), torch.rand(5), offsets)
    with pytest.raises(RuntimeError, match="B200|CUDA"):
        force_assembly(torch.randn(5, 3), torch.randn(5, 3), torch.tensor([2, 0, 2, 1, 0]), dst,
                       offsets, offsets, torch.tensor([1, 4, 3, 0, 2]))
    with pytest.raises(RuntimeError, match="B200|CUDA"):
        segment_offsets(dst, 3)
    with pytest.raises(RuntimeError, match="B200|CUDA"):
        kernels.segment_attention(torch.randn(5, 2), torch.randn(5, 1, 4), offsets)
    with pytest.raises(RuntimeError, match="B200|CUDA"):
        kernels.rmsnorm(torch.ones(2, 4))
    assert not kernels.segment_available()
    assert not kernels.rmsnorm_available()
    assert not kernels.gie_available()


def test_guard_rejects_other_architectures_and_cpu_tensors():
    with patch.object(native, "_require_cuda_runtime"), \
            patch.object(native.torch.cuda, "current_device", return_value=0), \
            patch.object(native.torch.cuda, "get_device_capability", return_value=(9, 0)):
        with pytest.raises(RuntimeError, match="sm_90"):
            native.require_dcu()
    with patch.object(native, "_require_cuda_runtime"):
        with pytest.raises(RuntimeError, match="CUDA device"):
            native.require_dcu(torch.ones(1))
    with patch.object(native, "_require_cuda_runtime"), \
            patch.object(native.torch.cuda, "get_device_capability", return_value=(10, 0)), \
            patch.object(native.torch.cuda, "current_device", return_value=0):
        assert native.require_dcu() == torch.device("cuda", 0)


def test_loader_requires_the_named_entry_point():
    ext = SimpleNamespace(rmsnorm_forward=object(), rmsnorm_backward=object())
    with patch.object(native, "_require_cuda_runtime"), \
            patch.object(native.importlib, "import_module", return_value=ext):
        assert native._extension("rmsnorm_forward") is ext
    with patch.object(native, "_require_cuda_runtime"), \
            patch.object(native.importlib, "import_module", return_value=SimpleNamespace()):
        with pytest.raises(RuntimeError, match="no 'rmsnorm_forward' entry point"):
            native._extension("rmsnorm_forward")
    with patch.object(native, "_require_cuda_runtime"), \
            patch.object(native.importlib, "import_module", side_effect=ImportError("x")):
        with pytest.raises(RuntimeError, match="build the B200 extension"):
            native._extension("segment_sum_forward")


# ---- fake-extension dispatch (autograd wiring) --------------------------------------------

class FakeSegmentExtension:
    """Computes with the oracle; checks the wrappers call the right entries."""

    def __init__(self, dst):
        self.dst = dst
        self.calls = []

    def segment_sum_forward(self, src, offsets, edge_scale=None, node_scale=None, order=None):
        self.calls.append("sum_fwd")
        return segment_sum_reference(src, self.dst, offsets, edge_scale, node_scale)

    def segment_sum_backward(self, grad_out, src, dst, offsets, edge_scale=None,
                             node_scale=None, want=False, order=None):
        self.calls.append("sum_bwd")
        with torch.enable_grad():
            s = src.detach().requires_grad_(True)
            n = node_scale.detach().requires_grad_(True) if node_scale is not None else None
            out = segment_sum_reference(s, dst, offsets, edge_scale, n)
            wrt = (s, n) if want else (s,)
            grads = torch.autograd.grad(out, wrt, grad_out)
        return grads[0], (grads[1] if want else None)

    def segment_softmax_forward(self, logit, env, offsets, null_logit=None, order=None):
        self.calls.append("smx_fwd")
        return segment_softmax_reference(logit, env, self.dst, offsets, null_logit)

    def segment_softmax_backward(self, alpha, grad_alpha, env, offsets, null_alpha=None,
                                 grad_null_alpha=None, order=None):
        self.calls.append("smx_bwd")
        s = torch.zeros(offsets.numel() - 1, alpha.shape[1]).index_add_(0, self.dst,
                                                                         alpha * grad_alpha)
        if null_alpha is not None:
            s = s + null_alpha * grad_null_alpha
        gl = alpha * (grad_alpha - s[self.dst])
        gn = null_alpha * (grad_null_alpha - s) if null_alpha is not None else None
        genv = torch.where(env > 0, gl.sum(1) * 2 / env.clamp_min(1e-30), torch.zeros_like(env))
        return gl, gn, genv


def test_segment_sum_dispatch_and_gradients():
    dst, offsets = torch.tensor([0, 0, 1, 2, 2, 2]), torch.tensor([0, 2, 3, 6])
    ext = FakeSegmentExtension(dst)
    src = torch.randn(6, 4, requires_grad=True)
    ns = (torch.rand(3) + 0.5).requires_grad_(True)
    ws = torch.rand(6) + 0.5
    up = torch.randn(3, 4)
    with patch.object(seg_mod, "require_dcu"), patch.object(seg_mod, "_extension",
                                                            return_value=ext):
        out = segment_sum(src, dst, offsets, ws, ns)
        got = torch.autograd.grad(out, (src, ns), up)
    ref_src, ref_ns = src.detach().clone().requires_grad_(True), ns.detach().clone().requires_grad_(True)
    want = torch.autograd.grad(segment_sum_reference(ref_src, dst, offsets, ws, ref_ns),
                               (ref_src, ref_ns), up)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b)
    assert ext.calls == ["sum_fwd", "sum_bwd"]


def test_segment_softmax_dispatch_with_and_without_null():
    dst, offsets = torch.tensor([0, 0, 1, 2, 2, 2]), torch.tensor([0, 2, 3, 6])
    ext = FakeSegmentExtension(dst)
    logit = torch.randn(6, 3, requires_grad=True)
    env = (torch.rand(6) + 0.1).requires_grad_(True)
    null = torch.randn(3, 3, requires_grad=True)
    with patch.object(seg_mod, "require_dcu"), patch.object(seg_mod, "_extension",
                                                            return_value=ext):
        a, n0 = segment_softmax(logit, env, offsets, null)
        got = torch.autograd.grad((a, n0), (logit, env, null), (torch.ones_like(a),
                                                                torch.ones_like(n0)))
        plain = segment_softmax(logit, env, offsets)
        assert isinstance(plain, torch.Tensor)
    rl, re_, rn = (x.detach().clone().requires_grad_(True) for x in (logit, env, null))
    ra, rnull = segment_softmax_reference(rl, re_, dst, offsets, rn)
    want = torch.autograd.grad((ra, rnull), (rl, re_, rn), (torch.ones_like(ra),
                                                           torch.ones_like(rnull)))
    for x, y in zip(got, want):
        torch.testing.assert_close(x, y, rtol=1e-4, atol=1e-6)


def test_rmsnorm_validation_and_dispatch():
    with pytest.raises(TypeError, match="input must be a tensor"):
        kernels.rmsnorm(None)
    with pytest.raises(ValueError, match="contiguous"):
        kernels.rmsnorm(torch.ones(3, 5).t())
    with pytest.raises(ValueError, match="scale must have shape"):
        kernels.rmsnorm(torch.ones(2, 4), torch.ones(3))
    for eps in (0, -1, math.inf, math.nan):
        with pytest.raises(ValueError, match="eps"):
            kernels.rmsnorm(torch.ones(2, 4), eps=eps)
    # per-degree weight table is accepted only with a matching irreps axis
    with pytest.raises(ValueError, match="scale must have shape"):
        kernels.rmsnorm(torch.ones(2, 5, 4), torch.ones(2, 4))

    class Fake:
        @staticmethod
        def rmsnorm_forward(x, scale, eps):
            weight = scale if scale.numel() else None
            return reference_rmsnorm(x, weight, eps), torch.rsqrt(
                x.square().mean(dim=-1) + eps).reshape(-1)

        @staticmethod
        def rmsnorm_backward(g, x, scale, inv, need):
            with torch.enable_grad():
                xx = x.detach().requires_grad_(True)
                ss = scale.detach().requires_grad_(True) if scale.numel() else None
                y = reference_rmsnorm(xx, ss)
                grads = torch.autograd.grad(y, (xx, ss) if need else (xx,), g)
            return grads[0], grads[1] if need else x.new_empty(0)

    x = torch.randn(2, 3, 11, requires_grad=True)
    s = torch.randn(11, requires_grad=True)
    with patch.object(norm_mod, "require_dcu"), patch.object(norm_mod, "_extension",
                                                             return_value=Fake()):
        y = kernels.rmsnorm(x, s)
        got = torch.autograd.grad(y, (x, s), torch.ones_like(y))
    want = torch.autograd.grad(reference_rmsnorm(x, s), (x, s), torch.ones_like(y))
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b)


def _gie_inputs():
    zonal = torch.tensor([[0.2, -0.1, 0.3], [0.4, 0.5, -0.2], [-0.3, 0.6, 0.1], [0.7, -0.2, 0.4]])
    radial = torch.arange(24, dtype=torch.float32).reshape(4, 2, 3) / 10
    return zonal, radial, torch.tensor([1, 0, 1, 1]), torch.tensor([0, 0, 1]), \
        torch.tensor([0.7, 0.5])


def test_gie_validation_and_dispatch():
    valid = _gie_inputs()
    with pytest.raises(TypeError, match="zonal must be a tensor"):
        kernels.zonal_scatter(None, *valid[1:])
    with pytest.raises(ValueError, match="radial must have shape"):
        kernels.zonal_scatter(valid[0], torch.ones(4, 2), *valid[2:])
    with pytest.raises(TypeError, match="dst and radial_slot must be int64"):
        kernels.zonal_scatter(valid[0], valid[1], valid[2].int(), valid[3], valid[4])
    with pytest.raises(TypeError, match="dst_offsets must be a tensor"):
        kernels.zonal_scatter(*valid, dst_offsets=[0, 1, 4])
    with pytest.raises(TypeError, match="dst_offsets must be int64"):
        kernels.zonal_scatter(*valid, dst_offsets=torch.tensor([0, 1, 4], dtype=torch.int32))
    with pytest.raises(ValueError, match=r"dst_offsets must have shape \(n_nodes \+ 1,\)"):
        kernels.zonal_scatter(*valid, dst_offsets=torch.tensor([0, 4]))
    with pytest.raises(ValueError, match="must be contiguous"):
        kernels.zonal_scatter(*valid, dst_offsets=torch.tensor([0, 9, 1, 9, 4, 9])[::2])

    class Fake:
        @staticmethod
        def gie_zonal_scatter_forward(*args):
            assert args[5] is None
            return zonal_scatter_reference(*args[:5])

        @staticmethod
        def gie_zonal_scatter_backward(g, zonal, radial, dst, slot, inv, dst_offsets):
            with torch.enable_grad():
                z, r, i = (t.detach().requires_grad_(True) for t in (zonal, radial, inv))
                return torch.autograd.grad(zonal_scatter_reference(z, r, dst, slot, i), (z, r, i), g)

    z, r = valid[0].clone().requires_grad_(True), valid[1].clone().requires_grad_(True)
    inv = valid[4].clone().requires_grad_(True)
    up = torch.randn(2, 4, 3)
    with patch.object(gie_mod, "require_dcu"), patch.object(gie_mod, "_extension",
                                                            return_value=Fake()):
        out = kernels.gie_zonal_scatter(z, r, valid[2], valid[3], inv)
        got = torch.autograd.grad(out, (z, r, inv), up)
    rz, rr, ri = (t.detach().clone().requires_grad_(True) for t in (z, r, inv))
    want = torch.autograd.grad(zonal_scatter_reference(rz, rr, valid[2], valid[3], ri),
                               (rz, rr, ri), up)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b)


def test_attention_validation():
    _, offsets = _graph()
    with pytest.raises(ValueError, match="heads"):
        kernels.segment_attention(torch.randn(5, 3), torch.randn(5, 2, 4), offsets)
    with pytest.raises(TypeError):
        kernels.segment_attention(torch.randn(5, 2), torch.randn(5, 2, 4).double(), offsets)
    with pytest.raises(ValueError, match="null_logit"):
        kernels.segment_attention(torch.randn(5, 2), torch.randn(5, 2, 4), offsets,
                                  null_logit=torch.randn(2, 2))
    calls = []
    with patch.object(attn_mod, "require_dcu"), patch.object(
            attn_mod, "_extension",
            return_value=SimpleNamespace(segment_attention_forward=lambda *a: calls.append(a) or 7)):
        assert kernels.segment_attention(torch.randn(5, 2), torch.randn(5, 2, 4), offsets) == 7
    assert len(calls) == 1


def test_gie_given_csr_reaches_both_directions():
    # dst_offsets is handed to the forward and, saved with the inputs, to the
    # backward entry point; the gradients keep the reference's contract.
    zonal, radial, _, slot, inv = _gie_inputs()
    dst = torch.tensor([0, 1, 1, 1])
    off = torch.tensor([0, 1, 4])
    seen = []

    class Fake:
        @staticmethod
        def gie_zonal_scatter_forward(zonal, radial, dst, slot, inv, dst_offsets):
            seen.append(("fwd", dst_offsets))
            return zonal_scatter_reference(zonal, radial, dst, slot, inv)

        @staticmethod
        def gie_zonal_scatter_backward(g, zonal, radial, dst, slot, inv, dst_offsets):
            seen.append(("bwd", dst_offsets))
            with torch.enable_grad():
                z, r, i = (t.detach().requires_grad_(True) for t in (zonal, radial, inv))
                return torch.autograd.grad(zonal_scatter_reference(z, r, dst, slot, i), (z, r, i), g)

    z, r, i = (t.clone().requires_grad_(True) for t in (zonal, radial, inv))
    up = torch.randn(2, 4, 3)
    with patch.object(gie_mod, "require_dcu"), patch.object(gie_mod, "_extension",
                                                            return_value=Fake()):
        out = kernels.zonal_scatter(z, r, dst, slot, i, dst_offsets=off)
        got = torch.autograd.grad(out, (z, r, i), up)
    assert [kind for kind, _ in seen] == ["fwd", "bwd"]
    assert all(t is not None and torch.equal(t, off) for _, t in seen)
    rz, rr, ri = (t.detach().clone().requires_grad_(True) for t in (zonal, radial, inv))
    want = torch.autograd.grad(zonal_scatter_reference(rz, rr, dst, slot, ri), (rz, rr, ri), up)
    for a, b in zip(got, want):
        torch.testing.assert_close(a, b)
