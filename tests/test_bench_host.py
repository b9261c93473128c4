"""Host-side logic of bench.py (no GPU): the DRAM-traffic figures it reports
are derived from the committed ncu captures, either whole-launch or scaled
per unit of work (slices of the bf16 attention shape, elements of the
streaming pair)."""
from __future__ import annotations

import json
import os

import bench

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _table():
    return json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))


def test_traffic_table_matches_committed_captures():
    t = bench.traffic_table()
    assert t == _table()
    for key in ("gemm_f16_4096", "fa_causal", "fa_bf16_per_slice", "stream_fused_per_elem",
                "gemm_f32_4096"):
        assert key in t and t[key] > 0


def test_flash_traffic_whole_launch_or_per_slice():
    t = _table()
    # a whole-launch capture is reported as captured, whatever the slice count
    assert bench.flash_traffic("fa_causal", 128) == t["fa_causal"]
    # per-slice figures scale with the slices a launch (or a rank) processes
    assert bench.flash_traffic("fa_bf16", 1024) == int(t["fa_bf16_per_slice"] * 1024)
    assert bench.flash_traffic("fa_bf16", 128) == int(t["fa_bf16_per_slice"] * 128)
    # no capture: no figure
    assert bench.flash_traffic("fa_f32", 1) is None


def test_stream_traffic_per_element_near_algorithmic():
    t = _table()
    n = 1 << 30
    assert bench.stream_traffic(n) == int(t["stream_fused_per_elem"] * n)
    # the fused vadd + sum moves 12 bytes per element; the capture agrees
    assert 11.5 <= t["stream_fused_per_elem"] <= 12.5


def test_shard_covers_range_once():
    for total in (0, 1, 7, 1024, (1 << 30) + 3):
        for world in (1, 2, 3, 8):
            spans = [bench.shard(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0 and a0 <= a1
