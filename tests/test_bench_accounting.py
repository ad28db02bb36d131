"""The benchmark's byte accounting (no GPU): the algorithmic bytes of a selected
page are its K and V codes plus the scales the format needs, and the L2
statement of a bench line matches the size of its inputs."""

import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import bench  # noqa: E402

PS, D = 16, 128


def test_page_bytes_per_format():
    # codes: F16 2 B, FP8 / INT8 1 B, INT4 0.5 B, INT4_RESIDUAL 2 x 0.5 B per element; K and V planes
    codes = {1: 2 * D, 2: D, 3: D, 4: D // 2, 5: D}
    scales = {1: 0, 2: 1, 3: 1, 4: 1, 5: 2}           # scale rows per plane (residual: two)
    for ns in (1, D // 32, D):
        for f in codes:
            assert bench.page_bytes(f, PS, D, ns) == 2 * (codes[f] * PS + scales[f] * ns * 4)


def test_step_bytes_is_the_sum_over_units():
    w = dict(PS=PS, D=D, B=3, Hkv=2, scale_mode="group32")
    fmt = np.array([1, 2, 3, 4, 5, 2], np.int32)
    per_unit = sum(bench.page_bytes(int(f), PS, D, D // 32) for f in fmt)
    assert bench.step_bytes(w, fmt) == per_unit * 3 * 2


def test_c2_selected_bytes_match_the_published_figure():
    """C2's 1024 selected pages per (sequence, kv head) at 30 / 40 / 30 % F16 / FP8 / INT8 with page
    scales: 5,457,512 B per unit, 1,397,123,072 B per step of 32 sequences x 8 kv heads."""
    n = 1024
    fmt = np.array([1] * round(0.3 * n) + [2] * round(0.4 * n) + [3] * (n - round(0.3 * n) - round(0.4 * n)))
    w = dict(PS=PS, D=D, B=1, Hkv=1, scale_mode="page")
    assert bench.step_bytes(w, fmt) == 5_457_512
    assert bench.step_bytes(dict(w, B=32, Hkv=8), fmt) == 1_397_123_072


def test_l2_statement_follows_the_input_size():
    assert bench.l2_note(2 * bench.L2_BYTES, "selected KV").startswith("inputs larger than L2")
    small = bench.l2_note(1_820_992, "selected KV")
    assert small.startswith("inputs smaller than L2") and "not flushed" in small


def test_ncu_traffic_scales_with_the_batch():
    t, note = bench.ncu_traffic("c2", 32, 1_397_123_072)
    assert t == 356_055_552 * 4 and "1.019x the algorithmic bytes" in note
    t, note = bench.ncu_traffic("c3", 64, 1_082_769_408)
    assert t == 142_390_528 * 8 and "1.052x" in note
    t, note = bench.ncu_traffic("c4", 64, 438_860_288)
    assert t == 58_652_672 * 8 and "1.069x" in note
    t, note = bench.ncu_traffic("prefill", 2, None)
    assert t == 140_648_704 and "algorithmic" not in note
    # a sequence-sharded launch reads its share of the pages
    t, note = bench.ncu_traffic("c5", 8, 2_043_910_656 // 8, shards=8)
    assert t == 261_946_112 and "1.025x" in note
    assert bench.ncu_traffic("route", 32, 1) == (None, "null (no ncu capture of this workload)")
