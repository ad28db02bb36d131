"""The prefill oracle vs outputs of the reference itself (CPU, no GPU)."""

import numpy as np
import pytest

import inputs as gi
from oracle import prefill as op

CASES = [("e2e_causal", gi.E2E_LAYOUT, (1, 2, 448, 64), 448, True),
         ("e2e_chunk", gi.E2E_LAYOUT, (2, 2, 16, 64), 448, False),
         ("partial_causal", gi.PREFILL_PARTIAL_LAYOUT, (2, 3, 100, 32), 100, True),
         ("gap_causal", gi.PREFILL_GAP_LAYOUT, (1, 2, 96, 32), 96, True),
         ("partial_causal_d128", gi.PREFILL_PARTIAL_LAYOUT, (1, 2, 100, 128), 100, True)]


def _inputs(i, qshape, T_kv):
    B, H, M, D = qshape
    return (gi.normal(600 + 3 * i, qshape), gi.normal(601 + 3 * i, (B, H, T_kv, D)),
            gi.normal(602 + 3 * i, (B, H, T_kv, D)))


@pytest.mark.parametrize("i", range(len(CASES)))
def test_semantic_block_attention_matches_reference(golden, i):
    name, spec, qshape, T_kv, causal = CASES[i]
    q, k, v = _inputs(i, qshape, T_kv)
    ref = golden("prefill_golden.npz")[name]
    got = op.semantic_block_attention(q, k, v, spec, causal)
    assert np.array_equal(np.isnan(got), np.isnan(ref))
    ok = ~np.isnan(ref)
    np.testing.assert_allclose(got[ok], ref[ok], atol=2e-5, rtol=1e-4)


@pytest.mark.parametrize("PS", [8, 16, 32])
@pytest.mark.parametrize("i", range(len(CASES)))
def test_paged_prefill_with_row_masks_equals_exact_token_attention(golden, i, PS):
    """Pages + per-page row masks + original positions reproduce the exact-token
    reference (rows the reference leaves NaN are 0 here)."""
    name, spec, qshape, T_kv, causal = CASES[i]
    q, k, v = _inputs(i, qshape, T_kv)
    B, H, M, D = qshape
    pages, masks = op.layout_pages(spec, PS)
    n_log = (T_kv + PS - 1) // PS
    # one unit per (b, h): physical page = (b*H + h) * n_log + logical; float32
    # pools stand in for F16 so the comparison is exact
    kp = np.zeros((B * H * n_log, PS, D), np.float32)
    vp = np.zeros_like(kp)
    pad = n_log * PS - T_kv
    for b in range(B):
        for h in range(H):
            u = b * H + h
            kp[u * n_log:(u + 1) * n_log] = np.pad(k[b, h], ((0, pad), (0, 0))).reshape(n_log, PS, D)
            vp[u * n_log:(u + 1) * n_log] = np.pad(v[b, h], ((0, pad), (0, 0))).reshape(n_log, PS, D)
    bases = (np.arange(B * H) * n_log).astype(np.int64)
    table = (bases.reshape(B, H, 1) + pages.reshape(1, 1, -1)).astype(np.int32)
    row_masks = np.tile(masks, (B, 1))
    tags = np.ones(B * H * n_log, np.uint8)
    got = op.paged_prefill(q, table, None, tags, {1: "F16"}, {"k_f16": kp, "v_f16": vp}, bases=bases,
                           row_masks=row_masks, causal=causal)
    ref = golden("prefill_golden.npz")[name]
    np.testing.assert_allclose(got, np.nan_to_num(ref, nan=0.0), atol=2e-5, rtol=1e-4)


def test_layout_pages_threshold_selection():
    spec = [("a", 0, 10, "ALWAYS", None), ("b", 10, 20, "ATTEND", 0.4), ("c", 20, 30, "ATTEND", 0.6),
            ("d", 30, 35, "SKIP", None)]
    pages, masks = op.layout_pages(spec, 8)
    assert pages.tolist() == [0, 1, 2, 3] and int(masks[3]) == 0b111111
    pages, masks = op.layout_pages(spec, 8, threshold=0.5)
    # ATTEND 0.4 dropped: page 1 keeps rows 0-1 (tokens 8, 9), page 2 rows 4-7
    assert pages.tolist() == [0, 1, 2, 3]
    assert int(masks[1]) == 0b11 and int(masks[2]) == 0b11110000 and int(masks[3]) == 0b111111
