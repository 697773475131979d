"""The C-ABI library loads without a GPU and exports what its header declares.

No compute call is made here (that needs a GPU): only the library load, the
symbol table, and the pure host helpers (version, status strings).
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "bysj_b200.h"
LIBRARY = ROOT / "bysj_b200" / "libbysj_b200.so"


def declared_symbols() -> list[str]:
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^BYSJ_API\s+[\w\s\*]+?\b(bysj_\w+)\s*\(", text, re.M)))


@pytest.fixture(scope="module")
def lib():
    if not LIBRARY.exists():
        pytest.skip("libbysj_b200.so not built (python -m bysj_b200._build)")
    return ctypes.CDLL(str(LIBRARY))


def test_header_declares_the_reference_replacements():
    names = declared_symbols()
    for required in (
        "bysj_segment_offsets_sorted", "bysj_segment_offsets_histogram",
        "bysj_segment_sum_forward", "bysj_segment_sum_backward",
        "bysj_segment_softmax_forward", "bysj_segment_softmax_backward",
        "bysj_segment_attention_forward", "bysj_force_assembly",
        "bysj_rmsnorm_forward", "bysj_rmsnorm_backward",
        "bysj_gie_zonal_scatter_forward", "bysj_gie_zonal_scatter_backward",
    ):
        assert required in names
    assert len(names) >= 26


def test_library_exports_every_declared_symbol(lib):
    missing = [name for name in declared_symbols() if not hasattr(lib, name)]
    assert missing == []


def test_host_helpers_answer_without_a_gpu(lib):
    lib.bysj_version.restype = ctypes.c_int
    assert lib.bysj_version() >= 10000
    lib.bysj_status_string.restype = ctypes.c_char_p
    assert lib.bysj_status_string(0) == b"ok"
    assert b"workspace" in lib.bysj_status_string(2)
    lib.bysj_last_error.restype = ctypes.c_char_p
    assert isinstance(lib.bysj_last_error(), bytes)


def test_only_sm100a_code_is_embedded():
    # the build passes exactly one -gencode (compute_100a -> sm_100a)
    from bysj_b200 import _build

    assert _build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert "-lineinfo" in _build.NVCC_FLAGS
    assert "--use_fast_math" not in _build.NVCC_FLAGS
    sources = {p.name for p in (ROOT / "bysj_b200" / "csrc").glob("*.cu")}
    assert sources == set(_build.CU_SOURCES)
