"""CUDA-graph capture of the device-side path (B200).

A step built from the operators that do not read anything back to the host
(``segment_offsets_device``, ``segment_attention``, ``segment_softmax``,
``force_assembly`` with a prebuilt source CSR, ``rmsnorm``) can be captured
once and replayed: launches, workspace allocations (from the graph's pool)
and memsets are all stream-ordered.  Replays must reproduce the eager
results bit for bit, also after the inputs change in place.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

from bysj_b200 import _C  # noqa: E402
from bysj_b200 import kernels as K  # noqa: E402
from bysj_b200 import workloads as W  # noqa: E402


def _step(g, flags, logit, value, env, grad, soff, order, x, w):
    offsets = _C.segment_offsets_device(g.dst, g.n_atoms, flags)
    out = _C.segment_attention_forward(logit, value, offsets)
    alpha, _ = _C.segment_softmax_forward(logit, env, offsets)
    force, virial = _C.force_assembly(grad, g.unit, offsets, soff, order)
    y, inv = _C.rmsnorm_forward(x, w, 1e-6)
    return out, alpha, force, virial, y, inv


def test_captured_step_replays_bit_identically(cuda):
    g = W.c1_box(device="cuda")
    e, n = g.n_edges, g.n_atoms
    gen = torch.Generator(device="cuda").manual_seed(21)
    logit = torch.randn(e, 8, device="cuda", generator=gen)
    value = torch.randn(e, 16, 64, device="cuda", generator=gen)
    env = torch.rand(e, device="cuda", generator=gen) + 0.05
    grad = torch.randn(e, 3, device="cuda", generator=gen) * 0.1
    x = torch.randn(n, 16, 128, device="cuda", generator=gen)
    w = torch.rand(4, 128, device="cuda", generator=gen) + 0.5
    order, soff = K.group_by_source(g.src, n)  # built once, outside the graph
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    args = (g, flags, logit, value, env, grad, soff, order, x, w)

    eager = _step(*args)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):  # warm-up on a side stream, as capture requires
        _step(*args)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = _step(*args)
    graph.replay()
    torch.cuda.synchronize()
    assert int(flags.item()) == 0
    for a, b in zip(eager, captured):
        assert torch.equal(a, b)
    # new inputs written in place: the replay recomputes them
    logit.mul_(0.5)
    value.add_(1.0)
    grad.neg_()
    x.mul_(2.0)
    graph.replay()
    fresh = _step(*args)
    torch.cuda.synchronize()
    for a, b in zip(fresh, captured):
        assert torch.equal(a, b)
    del graph
