"""GPU parity of the one-pass edge-stream elementwise chain (B200).

``kernels.edge_chain`` against the float64 ``oracle.truth.edge_chain`` and
the eager fp32 composition (one torch pass per term, as DeepMD runs it): the
three forms the reference's plan names (accumulate, gate, gate + residual),
per-edge and per-channel broadcasts, both activations, a non-contiguous
factor, channel counts that take the 4-wide and the scalar path, an
unaligned factor, bit-identical repeats, the validation errors, and a
[E, 9, 64] chain on the 2.2 M-edge C3 geometry.  Tolerance: rtol 1e-5 /
atol 1e-6 plus 16 units of roundoff of sum|terms| (the terms are summed in
fp32 with fused multiply-adds, the eager form rounds each product).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import truth

pytestmark = pytest.mark.gpu

from bysj_b200 import kernels as K  # noqa: E402


def check(got, terms, shape, activation=None):
    np_terms = [tuple([t[0]] + [f.double().cpu().numpy() for f in t[1:]]) for t in terms]
    want = truth.edge_chain(np_terms, shape, activation)
    mag = truth.edge_chain([tuple([abs(t[0])] + [np.abs(f) for f in t[1:]]) for t in np_terms],
                           shape)
    bound = 1e-6 + 1e-5 * np.abs(want) + 16 * 2.0 ** -24 * mag
    diff = np.abs(got.double().cpu().numpy() - want)
    assert (diff <= bound).all(), float((diff / bound).max())


def eager(terms, shape, activation=None):
    out = torch.zeros(shape, device="cuda")
    for t in terms:
        v = t[0] * t[1]
        if len(t) == 3:
            v = v * t[2]
        out = out + v
    if activation == "silu":
        out = torch.nn.functional.silu(out)
    elif activation == "sigmoid":
        out = torch.sigmoid(out)
    return out


@pytest.mark.parametrize("channels", [64, 6])
@pytest.mark.parametrize("activation", [None, "silu", "sigmoid"])
def test_chain_forms(cuda, channels, activation):
    gen = torch.Generator(device="cuda").manual_seed(channels)
    e, s, c = 1000, 9, channels
    r = lambda *sh: torch.randn(*sh, device="cuda", generator=gen)  # noqa: E731
    x, y, res = r(e, s, c), r(e, s, c), r(e, s, c)
    gate, per_edge, per_channel = r(e, 1, c), r(e, 1, 1), r(c)
    forms = {
        "accumulate": [(1.0, x), (0.5, y), (-2.0, res)],
        "gate": [(1.0, x, gate)],
        "gate+residual": [(1.0, res), (1.0, y, gate)],
        "broadcasts": [(1.0, x, per_edge), (3.0, per_channel), (1.0, y, per_channel)],
    }
    for name, terms in forms.items():
        got = K.edge_chain(terms, (e, s, c), activation)
        assert got.shape == (e, s, c) and got.is_contiguous(), name
        check(got, terms, (e, s, c), activation)
        torch.testing.assert_close(got, eager(terms, (e, s, c), activation), rtol=1e-5,
                                   atol=1e-5)
        assert torch.equal(got, K.edge_chain(terms, (e, s, c), activation))


def test_chain_strided_and_unaligned_factors(cuda):
    gen = torch.Generator(device="cuda").manual_seed(3)
    e, s, c = 513, 10, 64
    base = torch.randn(e, c, s, device="cuda", generator=gen)
    strided = base.transpose(1, 2)                        # [E, S, C], column stride S
    flat = torch.randn(e * s * c + 1, device="cuda", generator=gen)
    unaligned = flat[1:].view(e, s, c)                    # 4-byte offset: scalar path
    terms = [(1.0, strided), (2.0, unaligned), (1.0, strided, unaligned)]
    got = K.edge_chain(terms, (e, s, c))
    check(got, terms, (e, s, c))


def test_chain_validation(cuda):
    x = torch.randn(4, 2, 8, device="cuda")
    with pytest.raises(ValueError):
        K.edge_chain([(1.0, x)] * 9, (4, 2, 8))
    with pytest.raises(ValueError):
        K.edge_chain([(1.0, torch.randn(3, 2, 8, device="cuda"))], (4, 2, 8))
    with pytest.raises(TypeError):
        K.edge_chain([(1.0, x.double())], (4, 2, 8))
    with pytest.raises(ValueError):
        K.edge_chain([(1.0, x)], (4, 2, 8), "relu")
    with pytest.raises(RuntimeError):
        K.edge_chain([(1.0, x.requires_grad_(True))], (4, 2, 8))


def test_chain_c3_stream(cuda):
    # x + y * gate + residual over [E, 9, 64] on the C3 edge count
    e = 2_224_038
    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(e, 9, 64, device="cuda", generator=gen)
    y = torch.randn(e, 9, 64, device="cuda", generator=gen)
    res = torch.randn(e, 9, 64, device="cuda", generator=gen)
    gate = torch.randn(e, 1, 64, device="cuda", generator=gen)
    terms = [(1.0, x), (1.0, y, gate), (1.0, res)]
    got = K.edge_chain(terms, (e, 9, 64))
    for a in range(0, e, 1 << 18):
        b = min(e, a + (1 << 18))
        want = x[a:b].double() + y[a:b].double() * gate[a:b].double() + res[a:b].double()
        mag = x[a:b].double().abs() + (y[a:b].double() * gate[a:b].double()).abs() + \
            res[a:b].double().abs()
        bound = 1e-6 + 1e-5 * want.abs() + 16 * 2.0 ** -24 * mag
        assert bool(((got[a:b].double() - want).abs() <= bound).all())
