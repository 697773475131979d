"""The later C-ABI entry points through ctypes alone (no torch shim).

A host that binds only ``libbysj_b200.so`` -- a C/C++ plugin, or the ctypes
stub of the integration notes -- calls the index guard, the edge-stream
chain and the rotate-back aggregation with device pointers, sizes, a
caller-owned workspace and the current CUDA stream.  torch only provides
device memory.  Results are checked against the float64 truth
(``oracle.truth``); the guard's error word against planted bad indices.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import truth

pytestmark = pytest.mark.gpu

LIBRARY = Path(__file__).resolve().parents[1] / "bysj_b200" / "libbysj_b200.so"
P, I64, INT, SZ, F32 = (ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t,
                        ctypes.c_float)
INDEX_OFFSETS, INDEX_ORDER, INDEX_VALUES = 1, 2, 4
ACT_NONE, ACT_SILU = 0, 1


class ChainOperand(ctypes.Structure):
    _fields_ = [("data", P), ("stride", I64 * 3)]


class ChainTerm(ctypes.Structure):
    _fields_ = [("coef", F32), ("a", ChainOperand), ("b", ChainOperand)]


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(str(LIBRARY))
    sig = {
        "bysj_check_indices_workspace_size": (SZ, [I64]),
        "bysj_check_indices": (INT, [P, I64, I64, P, P, I64, I64, P, P, SZ, P]),
        "bysj_edge_chain": (INT, [ctypes.POINTER(ChainTerm), INT, I64, I64, I64, INT, P, P]),
        "bysj_rotate_back_aggregate_workspace_size": (SZ, [I64, I64, I64, I64, I64]),
        "bysj_rotate_back_aggregate": (INT, [P, P, P, P, P, P, I64, I64, I64, I64, I64, P, P,
                                             SZ, P]),
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


def csr(sizes):
    sizes = torch.as_tensor(sizes, dtype=torch.int64)
    dst = torch.repeat_interleave(torch.arange(sizes.numel()), sizes)
    off = torch.zeros(sizes.numel() + 1, dtype=torch.int64)
    off[1:] = torch.cumsum(sizes, 0)
    return dst, off


def guard(lib, offsets, n_edges, order=None, values=None, limit=0):
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws_bytes = lib.bysj_check_indices_workspace_size(n_edges if order is not None else 0)
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device="cuda")
    n_nodes = 0 if offsets is None else offsets.numel() - 1
    status = lib.bysj_check_indices(ptr(offsets), n_nodes, n_edges, ptr(order), ptr(values),
                                    0 if values is None else values.numel(), limit, ptr(error),
                                    ptr(ws), ws.numel(), stream())
    assert status == 0, lib.bysj_last_error()
    return int(error.item())


def test_index_guard_through_the_abi(cuda, lib):
    _, off = csr([3, 0, 4, 2])
    off = off.cuda()
    order = torch.randperm(9, generator=torch.Generator().manual_seed(2)).cuda()
    slots = torch.tensor([0, 1, 3, 3], device="cuda")
    assert guard(lib, off, 9, order, slots, 4) == 0
    bad_off = off.clone()
    bad_off[2] = 8                      # decreasing
    bad_order = order.clone()
    bad_order[0] = bad_order[5]         # a repeat
    bad_slots = torch.tensor([0, 4], device="cuda")
    assert guard(lib, bad_off, 9) == INDEX_OFFSETS
    assert guard(lib, None, 9, bad_order) == INDEX_ORDER
    assert guard(lib, None, 0, None, bad_slots, 4) == INDEX_VALUES
    assert guard(lib, bad_off, 9, bad_order, bad_slots, 4) == (INDEX_OFFSETS | INDEX_ORDER |
                                                               INDEX_VALUES)


def operand(t, shape):
    """Element strides of `t` broadcast to `shape` (0 along broadcast axes)."""
    view = t.expand(shape)
    return ChainOperand(t.data_ptr(), (I64 * 3)(*view.stride()))


def test_edge_chain_through_the_abi(cuda, lib):
    gen = torch.Generator(device="cuda").manual_seed(4)
    e, s, c = 3000, 9, 64
    x = torch.randn(e, s, c, device="cuda", generator=gen)
    y = torch.randn(e, s, c, device="cuda", generator=gen)
    gate = torch.rand(e, 1, c, device="cuda", generator=gen)
    w = torch.randn(c, device="cuda", generator=gen)
    scale = torch.rand(e, 1, 1, device="cuda", generator=gen)
    shape = (e, s, c)
    none = ChainOperand(None, (I64 * 3)(0, 0, 0))
    terms = (ChainTerm * 3)(ChainTerm(1.0, operand(x, shape), none),
                            ChainTerm(0.5, operand(y, shape), operand(gate, shape)),
                            ChainTerm(-2.0, operand(w, shape), operand(scale, shape)))
    out = torch.empty(shape, device="cuda")
    for act, name in ((ACT_NONE, None), (ACT_SILU, "silu")):
        status = lib.bysj_edge_chain(terms, 3, e, s, c, act, ptr(out), stream())
        assert status == 0, lib.bysj_last_error()
        torch.cuda.synchronize()
        want = truth.edge_chain([(1.0, x.cpu().numpy()),
                                 (0.5, y.cpu().numpy(), gate.cpu().numpy()),
                                 (-2.0, w.cpu().numpy(), scale.cpu().numpy())], shape, name)
        np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
    assert lib.bysj_edge_chain(terms, 0, e, s, c, ACT_NONE, ptr(out), stream()) != 0


def test_rotate_back_aggregate_through_the_abi(cuda, lib):
    gen = torch.Generator().manual_seed(6)
    lmax, heads, channels = 3, 4, 16
    comps, width = (lmax + 1) ** 2, sum((2 * l + 1) ** 2 for l in range(lmax + 1))
    dst, off = csr([5, 0, 130, 7, 1])
    e, n = dst.numel(), off.numel() - 1
    x = torch.randn(e, comps, channels, generator=gen)
    rot = torch.randn(e, width, generator=gen)
    scale = torch.rand(e, generator=gen) + 0.5
    alpha = torch.rand(e, heads, generator=gen)
    dev = [t.cuda() for t in (x, rot, scale, alpha, off)]
    out = torch.empty(n, comps, channels, device="cuda")
    ws_bytes = lib.bysj_rotate_back_aggregate_workspace_size(e, n, lmax, heads, channels)
    ws = torch.empty(max(int(ws_bytes), 1), dtype=torch.uint8, device="cuda")
    want = truth.rotate_back_aggregate(x.numpy(), rot.numpy(), scale.numpy(), alpha.numpy(),
                                       dst.numpy(), n, lmax, heads)
    for _ in range(2):  # two calls on the same workspace
        status = lib.bysj_rotate_back_aggregate(*(ptr(t) for t in dev[:4]), ptr(dev[4]), None, e,
                                                n, lmax, heads, channels, ptr(out), ptr(ws),
                                                ws.numel(), stream())
        assert status == 0, lib.bysj_last_error()
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), want, rtol=1e-5, atol=1e-5)
