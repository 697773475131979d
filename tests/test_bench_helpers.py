"""Host-side pieces of bench.py that fix what its JSON lines report (no GPU).

The per-frame algorithmic bytes of the chain mode are the sum of each
operator's input read once and output written once; the chain's frames are
dealt out round-robin over the ranks, as in the frame-sharded default mode.
"""
from __future__ import annotations

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402
from bysj_b200 import sharding as S  # noqa: E402


def test_chain_bytes_is_the_sum_of_the_operators():
    e, n, c = 2_224_038, 24_576, 32
    offsets = 8 * e + 8 * (n + 1)
    rmsnorm = 2 * n * 16 * c * 4 + 4 * n * 16 + 4 * 4 * c
    attention = e * (32 + 16 * c * 4) + n * 16 * c * 4 + 8 * (n + 1)
    zonal = e * (60 + 8 + 3 * c * 4) + n * (16 * c * 4 + 4)
    group = 16 * e + 8 * (n + 1)
    force = 32 * e + 64 * n
    assert bench.chain_bytes(e, n, c) == offsets + rmsnorm + attention + zonal + group + force
    assert 5.9e9 < bench.chain_bytes(e, n) < 6.0e9  # the C3 geometry at C = 32


def test_attention_bytes_matches_the_c3_roofline_figure():
    # 32 B of logits and 4 KB of fp32 values per edge, 4 KB of output per node
    assert abs(bench.attention_bytes(2_224_038, 24_576, 4) - 9.2817e9) < 1e6


def test_chain_frames_cover_the_job_once_at_every_world_size():
    for world in (1, 2, 4, 8):
        dealt = sorted(f for r in range(world) for f in S.frame_share(64, r, world))
        assert dealt == list(range(64))
        assert {len(S.frame_share(64, r, world)) for r in range(world)} == {64 // world}
