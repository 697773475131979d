"""The allocation-free fused-attention entry point, called through the C ABI.

``bysj_segment_attention_forward_noalloc`` exists for callers that cannot
allocate device memory or pass a workspace (a plugin hook that only receives
its tensors and a stream, a serving runtime with a frozen memory footprint,
a hot path where cudaMalloc would synchronise the device).  Its scratch is a
fixed 16 MiB device array inside the library.  This test compares it with the
workspace entry point ``bysj_segment_attention_forward`` on two calls in a
row (the second call sees the first call's leftovers in the shared array),
using the same tolerance as the other fp32 parity tests, and checks that a
row too wide for the fixed array is refused.  It is collected last and also
passes on its own in a fresh process.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "bysj_b200" / "libbysj_b200.so"
P, I64, I32, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_size_t


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    handle = ctypes.CDLL(str(LIB))
    handle.bysj_segment_attention_forward_noalloc.argtypes = [
        P, P, I32, P, P, P, P, I64, I64, I64, I64, I64, P, P]
    handle.bysj_segment_attention_forward_noalloc.restype = I32
    handle.bysj_segment_attention_forward.argtypes = [
        P, P, I32, P, P, P, P, I64, I64, I64, I64, I64, P, P, SZ, P]
    handle.bysj_segment_attention_forward.restype = I32
    handle.bysj_segment_attention_workspace_size.argtypes = [I64, I64, I64, I64, I64, I32]
    handle.bysj_segment_attention_workspace_size.restype = SZ
    handle.bysj_last_error.restype = ctypes.c_char_p
    return handle


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def make_case(seed, value_dtype, skewed, comps=16, channels=64, sizes=None):
    gen = torch.Generator().manual_seed(seed)
    if sizes is None and skewed:
        sizes = torch.randint(0, 12, (400,), generator=gen)
        sizes[100], sizes[-1] = 6000, 2500
    elif sizes is None:
        sizes = torch.randint(60, 120, (192,), generator=gen)
    offsets = torch.zeros(sizes.numel() + 1, dtype=torch.int64)
    offsets[1:] = torch.cumsum(sizes, 0)
    e, n = int(offsets[-1]), sizes.numel()
    logit = torch.randn(e, 8, generator=gen) * 2
    value = torch.randn(e, comps, channels, generator=gen).to(value_dtype)
    env = torch.rand(e, generator=gen) + 0.05
    null = torch.randn(n, 8, generator=gen)
    return [t.cuda() for t in (logit, value, env, null, offsets)]


def dtype_code(t):
    return 1 if t.dtype == torch.bfloat16 else 0


def workspace_bytes(lib, logit, value, offsets):
    e, h = logit.shape
    _, comps, channels = value.shape
    return lib.bysj_segment_attention_workspace_size(e, offsets.numel() - 1, h, comps, channels,
                                                     dtype_code(value))


def with_workspace(lib, logit, value, env, null, offsets):
    e, h = logit.shape
    _, comps, channels = value.shape
    n = offsets.numel() - 1
    out = torch.empty(n, h, comps, channels // h, device="cuda")
    size = workspace_bytes(lib, logit, value, offsets)
    ws = torch.empty(max(size, 1), dtype=torch.uint8, device="cuda")
    status = lib.bysj_segment_attention_forward(
        ptr(logit), ptr(value), dtype_code(value), ptr(env), ptr(null), ptr(offsets), None,
        e, n, h, comps, channels, ptr(out), ptr(ws), size, stream())
    assert status == 0, lib.bysj_last_error()
    return out


def without_workspace(lib, logit, value, env, null, offsets):
    e, h = logit.shape
    _, comps, channels = value.shape
    n = offsets.numel() - 1
    out = torch.empty(n, h, comps, channels // h, device="cuda")
    status = lib.bysj_segment_attention_forward_noalloc(
        ptr(logit), ptr(value), dtype_code(value), ptr(env), ptr(null), ptr(offsets), None,
        e, n, h, comps, channels, ptr(out), stream())
    assert status == 0, lib.bysj_last_error()
    return out


def test_noalloc_matches_the_workspace_entry_point_on_two_calls_in_a_row(lib):
    first = make_case(1, torch.float32, skewed=True)
    second = make_case(2, torch.bfloat16, skewed=False)
    out1 = without_workspace(lib, *first)
    out2 = without_workspace(lib, *second)
    torch.cuda.synchronize()
    torch.testing.assert_close(out1, with_workspace(lib, *first), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(out2, with_workspace(lib, *second), rtol=1e-5, atol=1e-6)
    # Leftovers of the previous call in the shared scratch do not leak into results.
    assert torch.equal(without_workspace(lib, *first), out1)


def test_noalloc_capped_plan_matches_the_workspace_entry_point(lib):
    # Cases whose workspace plan (one partition per resident warp) needs more
    # than the fixed 16 MiB, so the entry point runs the capped plan: fewer,
    # longer partitions and segments split over several of them.
    cap = 16 * 1024 * 1024
    gen = torch.Generator().manual_seed(7)
    # about 54k edges with the headline's [16, 64] rows
    frame = make_case(3, torch.float32, False,
                      sizes=torch.randint(60, 120, (600,), generator=gen))
    # 16 x 1024 rows (cap of ~127 partitions) with one 3000-edge hub segment
    sizes = torch.randint(0, 12, (300,), generator=gen)
    sizes[150] = 3000
    wide = make_case(4, torch.float32, False, comps=16, channels=1024, sizes=sizes)
    for case in (frame, wide):
        logit, value, _, _, offsets = case
        assert workspace_bytes(lib, logit, value, offsets) > cap
        first = without_workspace(lib, *case)
        second = without_workspace(lib, *case)
        torch.cuda.synchronize()
        torch.testing.assert_close(first, with_workspace(lib, *case), rtol=1e-5, atol=1e-6)
        assert torch.equal(first, second)


def test_noalloc_refuses_rows_too_wide_for_the_fixed_scratch(lib):
    # 2^22-element rows cannot fit one partition's slots in 16 MiB; with zero
    # nodes and edges nothing could be launched even if the check were absent.
    dummy = torch.zeros(16, device="cuda")
    status = lib.bysj_segment_attention_forward_noalloc(
        ptr(dummy), ptr(dummy), 0, None, None, ptr(dummy), None, 0, 0, 1, 1 << 20, 4,
        ptr(dummy), stream())
    assert status == 6  # BYSJ_ERR_TOO_LARGE
    assert b"scratch" in lib.bysj_last_error()
