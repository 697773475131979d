"""GPU parity through the C ABI alone (ctypes on libbysj_b200.so, no torch shim).

This is how a host that binds only the shared library (a C/C++ plugin, or
the ctypes stub shown in the integration notes) drives the operators: device
pointers, sizes, a caller-owned workspace and the current CUDA stream.
torch only provides device memory here.  Results are checked against the
float64 oracle; status codes and ``bysj_last_error`` against bad calls.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import truth

pytestmark = pytest.mark.gpu

from bysj_b200 import workloads as W  # noqa: E402

LIBRARY = Path(__file__).resolve().parents[1] / "bysj_b200" / "libbysj_b200.so"
P, I64, INT, SZ, F32 = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t,
                        ctypes.c_float)
OK, INVALID, WORKSPACE = 0, 1, 2


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(str(LIBRARY))
    sig = {
        "bysj_segment_offsets_sorted": (INT, [P, I64, I64, P, P, P]),
        "bysj_group_by_key_workspace_size": (SZ, [I64, I64]),
        "bysj_group_by_key": (INT, [P, I64, I64, P, P, P, P, SZ, P]),
        "bysj_segment_sum_workspace_size": (SZ, [I64, I64, I64, INT]),
        "bysj_segment_sum_forward": (INT, [P, INT, I64, I64, P, I64, P, P, P, P, P, SZ, P]),
        "bysj_segment_softmax_workspace_size": (SZ, [I64, I64, I64]),
        "bysj_segment_softmax_forward": (INT, [P, P, P, I64, I64, I64, P, P, P, P, P, SZ, P]),
        "bysj_segment_attention_workspace_size": (SZ, [I64, I64, I64, I64, I64, INT]),
        "bysj_segment_attention_forward": (INT, [P, P, INT, P, P, P, P, I64, I64, I64, I64,
                                                 I64, P, P, SZ, P]),
        "bysj_force_assembly": (INT, [P, P, P, P, P, I64, I64, P, P, P]),
        "bysj_rmsnorm_forward": (INT, [P, INT, I64, I64, P, I64, F32, P, P, P]),
        "bysj_gie_zonal_scatter_workspace_size": (SZ, [I64, I64, I64, I64]),
        "bysj_gie_zonal_scatter_forward": (INT, [P, P, P, P, P, P, I64, I64, I64, I64, I64, P,
                                                 P, SZ, P]),
        "bysj_last_error": (ctypes.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    return lib


def ptr(t):
    return None if t is None else t.data_ptr()


def stream():
    return torch.cuda.current_stream().cuda_stream


def workspace(nbytes):
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device="cuda")


def call(lib, name, *args):
    status = getattr(lib, name)(*args)
    assert status == OK, (name, status, lib.bysj_last_error())
    torch.cuda.synchronize()


@pytest.fixture
def box(cuda):
    g = W.c1_box(device="cuda")
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    offsets = torch.empty(g.n_atoms + 1, dtype=torch.int64, device="cuda")
    return g, flags, offsets


def test_offsets_and_grouping_through_the_abi(lib, box):
    g, flags, offsets = box
    flags.zero_()
    call(lib, "bysj_segment_offsets_sorted", ptr(g.dst), g.n_edges, g.n_atoms, ptr(offsets),
         ptr(flags), stream())
    assert int(flags.item()) == 0
    np.testing.assert_array_equal(offsets.cpu().numpy(),
                                  truth.segment_offsets(g.dst.cpu().numpy(), g.n_atoms))
    order = torch.empty(g.n_edges, dtype=torch.int64, device="cuda")
    soff = torch.empty_like(offsets)
    ws = workspace(lib.bysj_group_by_key_workspace_size(g.n_edges, g.n_atoms))
    flags.zero_()
    call(lib, "bysj_group_by_key", ptr(g.src), g.n_edges, g.n_atoms, ptr(order), ptr(soff),
         ptr(flags), ptr(ws), ws.numel(), stream())
    want_order, want_off = truth.group_by_source(g.src.cpu().numpy(), g.n_atoms)
    np.testing.assert_array_equal(order.cpu().numpy(), want_order)
    np.testing.assert_array_equal(soff.cpu().numpy(), want_off)


def test_segment_sum_softmax_attention_through_the_abi(lib, box):
    g, flags, offsets = box
    flags.zero_()
    call(lib, "bysj_segment_offsets_sorted", ptr(g.dst), g.n_edges, g.n_atoms, ptr(offsets),
         ptr(flags), stream())
    e, n = g.n_edges, g.n_atoms
    gen = torch.Generator(device="cuda").manual_seed(5)
    value = torch.randn(e, 16, 64, device="cuda", generator=gen)
    logit = torch.randn(e, 8, device="cuda", generator=gen) * 2 ** 0.5
    env = torch.rand(e, device="cuda", generator=gen) * 0.9 + 0.1
    dst = g.dst.cpu().numpy()

    out = torch.empty(n, 1024, device="cuda")
    ws = workspace(lib.bysj_segment_sum_workspace_size(e, n, 1024, 0))
    call(lib, "bysj_segment_sum_forward", ptr(value), 0, e, 1024, ptr(offsets), n, None, None,
         None, ptr(out), ptr(ws), ws.numel(), stream())
    want = truth.segment_sum(value.reshape(e, -1).cpu().numpy(), dst, n)
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5,
                               atol=1e-5 * float(np.abs(want).max()))

    alpha = torch.empty_like(logit)
    ws = workspace(lib.bysj_segment_softmax_workspace_size(e, n, 8))
    call(lib, "bysj_segment_softmax_forward", ptr(logit), ptr(env), ptr(offsets), e, n, 8, None,
         None, ptr(alpha), None, ptr(ws), ws.numel(), stream())
    want_alpha = truth.segment_softmax(logit.cpu().numpy(), env.cpu().numpy(), dst, n)
    want_alpha = want_alpha[0] if isinstance(want_alpha, tuple) else want_alpha
    np.testing.assert_allclose(alpha.cpu().numpy(), want_alpha, rtol=1e-5, atol=1e-6)

    att = torch.empty(n, 8, 16, 8, device="cuda")
    ws = workspace(lib.bysj_segment_attention_workspace_size(e, n, 8, 16, 64, 0))
    call(lib, "bysj_segment_attention_forward", ptr(logit), ptr(value), 0, None, None,
         ptr(offsets), None, e, n, 8, 16, 64, ptr(att), ptr(ws), ws.numel(), stream())
    want_att = truth.segment_attention(logit.cpu().numpy(), value.cpu().numpy(), dst, n)
    np.testing.assert_allclose(att.cpu().numpy(), want_att, rtol=1e-5,
                               atol=1e-5 * float(np.abs(want_att).max()))


def test_force_rmsnorm_gie_through_the_abi(lib, box):
    g, flags, offsets = box
    flags.zero_()
    call(lib, "bysj_segment_offsets_sorted", ptr(g.dst), g.n_edges, g.n_atoms, ptr(offsets),
         ptr(flags), stream())
    e, n = g.n_edges, g.n_atoms
    gen = torch.Generator(device="cuda").manual_seed(6)
    grad = torch.randn(e, 3, device="cuda", generator=gen) * 0.1
    order = torch.empty(e, dtype=torch.int64, device="cuda")
    soff = torch.empty_like(offsets)
    ws = workspace(lib.bysj_group_by_key_workspace_size(e, n))
    call(lib, "bysj_group_by_key", ptr(g.src), e, n, ptr(order), ptr(soff), ptr(flags), ptr(ws),
         ws.numel(), stream())
    force = torch.empty(n, 3, device="cuda")
    virial = torch.empty(n, 9, device="cuda")
    call(lib, "bysj_force_assembly", ptr(grad), ptr(g.unit), ptr(offsets), ptr(soff), ptr(order),
         e, n, ptr(force), ptr(virial), stream())
    tf, tv = truth.force_assembly(grad.cpu().numpy(), g.unit.cpu().numpy(), g.src.cpu().numpy(),
                                  g.dst.cpu().numpy(), n)
    np.testing.assert_allclose(force.cpu().numpy(), tf, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(virial.cpu().numpy(), tv, rtol=1e-6, atol=1e-6)

    x = torch.randn(n * 16, 128, device="cuda", generator=gen)
    w = torch.rand(4, 128, device="cuda", generator=gen) + 0.5
    y = torch.empty_like(x)
    inv = torch.empty(n * 16, device="cuda")
    call(lib, "bysj_rmsnorm_forward", ptr(x), 0, n * 16, 128, ptr(w), 4, 1e-6, ptr(y), ptr(inv),
         stream())
    want_y, want_inv = truth.rmsnorm(x.reshape(n, 16, 128).cpu().numpy(), w.cpu().numpy(),
                                     per_degree=True)
    np.testing.assert_allclose(y.reshape(n, 16, 128).cpu().numpy(), want_y, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(inv.cpu().numpy(), want_inv, rtol=1e-5)

    zonal = W.real_sph_zonal(g.unit)
    radial = torch.randn(e, 4, 64, device="cuda", generator=gen)
    slot = W.degree_slots().cuda()
    inv_deg = torch.rsqrt(torch.bincount(g.dst, minlength=n).float() + 1.0)
    out = torch.empty(n, 16, 64, device="cuda")
    ws = workspace(lib.bysj_gie_zonal_scatter_workspace_size(e, n, 15, 64))
    call(lib, "bysj_gie_zonal_scatter_forward", ptr(zonal), ptr(radial), ptr(offsets), None,
         ptr(slot), ptr(inv_deg), e, n, 15, 4, 64, ptr(out), ptr(ws), ws.numel(), stream())
    want = truth.zonal_scatter(zonal.cpu().numpy(), radial.cpu().numpy(), g.dst.cpu().numpy(),
                               slot.cpu().numpy(), inv_deg.cpu().numpy())
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5,
                               atol=1e-5 * float(np.abs(want).max()))


def test_abi_reports_bad_calls(lib, box):
    g, flags, offsets = box
    e, n = g.n_edges, g.n_atoms
    src = torch.randn(e, 8, device="cuda")
    out = torch.empty(n, 8, device="cuda")
    assert lib.bysj_segment_sum_workspace_size(e, n, 8, 0) > 0
    small = workspace(1)
    status = lib.bysj_segment_sum_forward(ptr(src), 0, e, 8, ptr(offsets), n, None, None, None,
                                          ptr(out), ptr(small), 0, stream())
    assert status == WORKSPACE and b"workspace" in lib.bysj_last_error()
    status = lib.bysj_force_assembly(None, None, ptr(offsets), ptr(offsets), None, e, n, None,
                                     None, stream())
    assert status == INVALID and b"NULL" in lib.bysj_last_error()
    status = lib.bysj_segment_softmax_forward(ptr(src), None, ptr(offsets), -1, n, 8, None, None,
                                              ptr(out), None, ptr(small), 1, stream())
    assert status == INVALID
