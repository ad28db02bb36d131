"""GPU parity of the multi-query (prefill) attention over selected pages:
the tcgen05 kernel and the CUDA-core kernel vs the numpy oracle (pinned to the
reference's semantic_block_attention), and through the drop-in entry point
vs the reference's own outputs.

Tolerance (north star): atol 2e-3 / rtol 1e-2.
"""

import numpy as np
import pytest
import torch

import inputs as gi
from gpu_cases import ORACLE_FMT, NAME_OF, oracle_pools, tag_map_for
from oracle import prefill as op

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
ALL = ("F16", "FP8", "INT8", "INT4", "INT4R")


def _case(seed, B=2, Ht=2, G=2, M=70, D=128, PS=16, n_log=10, formats=ALL, scale_mode="page", causal=True,
          masks=True, q_dtype=torch.bfloat16, counts=True, pad=True, q_offset=0):
    """Units own n_log logical pages each (physical = unit * n_log + logical);
    the table lists a random subset of them in random order."""
    from intent_attention import PagePool
    g = np.random.default_rng(seed)
    units = B * Ht
    NP = units * n_log
    k = g.standard_normal((NP, PS, D)).astype(np.float32)
    v = g.standard_normal((NP, PS, D)).astype(np.float32)
    fm = g.choice([NAME_OF[f] for f in formats], size=NP).astype(np.uint8)
    fm = np.where(g.random(NP) < 0.05, 0, fm).astype(np.uint8)          # a few SKIP-tagged pages
    pool = PagePool.allocate(NP, PS, D, formats, scale_mode, "cuda", zero=True)
    pool.quantize_(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), torch.from_numpy(fm).cuda())
    W = n_log
    bases = (np.arange(units) * n_log).reshape(B, Ht).astype(np.int32)
    table = np.stack([np.stack([bases[b, h] + g.permutation(n_log) for h in range(Ht)]) for b in range(B)])
    table = table.astype(np.int32)
    if pad:
        table = np.where(g.random(table.shape) < 0.1, -1, table).astype(np.int32)
    cnt = g.integers(W // 2, W + 1, size=(B, Ht)).astype(np.int32) if counts else None
    rm = None
    if masks:
        full = (1 << PS) - 1 if PS < 64 else (1 << 64) - 1
        rm = np.where(g.random((B, W)) < 0.5, full, g.integers(0, 1 << min(PS, 62), size=(B, W))).astype(np.uint64)
    q = g.standard_normal((B, Ht * G, M, D)).astype(np.float32)
    qt = torch.from_numpy(q).to("cuda", q_dtype)
    qpos = (q_offset + np.arange(M))[None].repeat(B, 0).astype(np.int32)
    return dict(pool=pool, table=table, counts=cnt, bases=bases, masks=rm, tags=fm, q=qt, np_q=qt.float().cpu().numpy(),
                qpos=qpos, causal=causal, scale_mode=scale_mode, formats=formats)


def _run(c, kernel, out_dtype=torch.float32):
    from intent_attention.paged import paged_prefill
    rm = None if c["masks"] is None else torch.from_numpy(c["masks"].view(np.int64)).cuda()
    return paged_prefill(c["q"], c["pool"], torch.from_numpy(c["table"]).cuda(),
                         None if c["counts"] is None else torch.from_numpy(c["counts"]).cuda(),
                         torch.from_numpy(c["tags"]).cuda(), tag_map_for(c["formats"]),
                         q_positions=torch.from_numpy(c["qpos"]).cuda(), causal=c["causal"],
                         bases=torch.from_numpy(c["bases"]).cuda(), row_masks=rm, out_dtype=out_dtype, kernel=kernel)


def _oracle(c):
    pools, sc = oracle_pools(c["pool"])
    return op.paged_prefill(c["np_q"], c["table"], c["counts"], c["tags"], ORACLE_FMT, pools, sc, c["scale_mode"],
                            bases=c["bases"], row_masks=c["masks"], q_positions=c["qpos"], causal=c["causal"])


def _close(got, ref):
    np.testing.assert_allclose(got.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("kernel", ["tensor", "generic"])
@pytest.mark.parametrize("PS", [8, 16, 32, 64])
def test_page_sizes(kernel, PS):
    c = _case(PS, PS=PS, n_log=max(4, 160 // PS), M=150, q_offset=20)
    _close(_run(c, kernel), _oracle(c))


@pytest.mark.parametrize("kernel", ["tensor", "generic"])
@pytest.mark.parametrize("mode", ["page", "group32", "channel"])
def test_scale_modes_all_formats(kernel, mode):
    c = _case(11 + len(mode), scale_mode=mode)
    _close(_run(c, kernel), _oracle(c))


@pytest.mark.parametrize("kernel", ["tensor", "generic"])
@pytest.mark.parametrize("G,M", [(1, 200), (4, 33), (8, 40), (16, 9)])
def test_gqa_groups_and_ragged_tiles(kernel, G, M):
    c = _case(20 + G, G=G, M=M, Ht=2, q_offset=100)
    _close(_run(c, kernel), _oracle(c))


@pytest.mark.parametrize("kernel", ["tensor", "generic"])
def test_non_causal_chunk(kernel):
    c = _case(31, causal=False, M=16)
    _close(_run(c, kernel), _oracle(c))


@pytest.mark.parametrize("kernel", ["tensor", "generic"])
@pytest.mark.parametrize("q_dtype", [torch.float16, torch.float32])
def test_query_dtypes_and_output_dtypes(kernel, q_dtype):
    c = _case(41, q_dtype=q_dtype, masks=False, counts=False)
    ref = _oracle(c)
    _close(_run(c, kernel), ref)
    np.testing.assert_allclose(_run(c, kernel, out_dtype=torch.bfloat16).float().cpu().numpy(), ref, atol=2e-2,
                               rtol=2e-2)


@pytest.mark.parametrize("kernel", ["tensor", "generic"])
def test_rows_without_visible_keys_are_zero(kernel):
    """Causal queries before every selected key (and empty units) give 0."""
    c = _case(51, q_offset=-60, M=90)            # the first queries precede every page
    c["counts"][1, 1] = 0                         # an empty unit
    got = _run(c, kernel).float().cpu().numpy()
    ref = _oracle(c)
    np.testing.assert_allclose(got, ref, atol=ATOL, rtol=RTOL)
    assert (got[1, 2:4] == 0).all() and np.isfinite(got).all()
    assert (got[:, :, 0] == 0).all()


def test_tensor_and_generic_agree_on_a_long_table():
    c = _case(61, B=1, Ht=2, G=4, M=256, PS=16, n_log=200, q_offset=3000)
    a = _run(c, "tensor").float().cpu().numpy()
    b = _run(c, "generic").float().cpu().numpy()
    np.testing.assert_allclose(a, b, atol=ATOL, rtol=RTOL)
    _close(torch.from_numpy(a), _oracle(c))


@pytest.mark.parametrize("i", range(5))
def test_reference_golden_through_pages(golden, i):
    """The reference's own semantic_block_attention outputs (exact tokens,
    original positions) through F16 pages, layout row masks and the tensor
    kernel; rows the reference leaves NaN are 0 here."""
    from intent_attention import PagePool
    from intent_attention.paged import paged_prefill, make_tag_map
    cases = [("e2e_causal", gi.E2E_LAYOUT, (1, 2, 448, 64), 448, True),
             ("e2e_chunk", gi.E2E_LAYOUT, (2, 2, 16, 64), 448, False),
             ("partial_causal", gi.PREFILL_PARTIAL_LAYOUT, (2, 3, 100, 32), 100, True),
             ("gap_causal", gi.PREFILL_GAP_LAYOUT, (1, 2, 96, 32), 96, True),
             ("partial_causal_d128", gi.PREFILL_PARTIAL_LAYOUT, (1, 2, 100, 128), 100, True)]
    name, spec, qshape, T_kv, causal = cases[i]
    B, H, M, D = qshape
    q = gi.normal(600 + 3 * i, qshape)
    k = gi.normal(601 + 3 * i, (B, H, T_kv, D))
    v = gi.normal(602 + 3 * i, (B, H, T_kv, D))
    PS = 16
    pages, masks = op.layout_pages(spec, PS)
    n_log = (T_kv + PS - 1) // PS
    pad = n_log * PS - T_kv
    kp = np.pad(k, ((0, 0), (0, 0), (0, pad), (0, 0))).reshape(B * H * n_log, PS, D)
    vp = np.pad(v, ((0, 0), (0, 0), (0, pad), (0, 0))).reshape(B * H * n_log, PS, D)
    pool = PagePool.allocate(B * H * n_log, PS, D, ["F16"], "page", "cuda")
    pool.quantize_(torch.from_numpy(kp).cuda(), torch.from_numpy(vp).cuda(), ["F16"] * (B * H * n_log))
    bases = (np.arange(B * H) * n_log).reshape(B, H).astype(np.int32)
    table = (bases[:, :, None] + pages[None, None, :]).astype(np.int32)
    rm = np.tile(masks, (B, 1)).view(np.int64)
    tags = torch.ones(B * H * n_log, dtype=torch.uint8, device="cuda")
    got = paged_prefill(torch.from_numpy(q).cuda(), pool, torch.from_numpy(table).cuda(), None, tags,
                        make_tag_map({1: "F16"}), causal=causal, bases=torch.from_numpy(bases).cuda(),
                        row_masks=torch.from_numpy(rm).cuda(), kernel="generic" if D != 128 else "auto")
    ref = np.nan_to_num(golden("prefill_golden.npz")[name], nan=0.0)
    # K / V pass through f16 pages: 2e-3 covers the rounding
    np.testing.assert_allclose(got.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


def test_non_positive_scale_runs_on_the_cuda_core_kernel():
    """The tensor-core softmax takes each slot's max score times a positive scale:
    kernel="tensor" refuses another scale, "auto" runs the CUDA-core kernel."""
    from intent_attention.paged import paged_prefill
    c = _case(71, M=40)
    rm = torch.from_numpy(c["masks"].view(np.int64)).cuda()
    args = (c["q"], c["pool"], torch.from_numpy(c["table"]).cuda(), torch.from_numpy(c["counts"]).cuda(),
            torch.from_numpy(c["tags"]).cuda(), tag_map_for(c["formats"]))
    kw = dict(q_positions=torch.from_numpy(c["qpos"]).cuda(), causal=True, bases=torch.from_numpy(c["bases"]).cuda(),
              row_masks=rm, sm_scale=-0.05)
    with pytest.raises(Exception):
        paged_prefill(*args, kernel="tensor", **kw)
    got = paged_prefill(*args, kernel="auto", **kw)
    pools, sc = oracle_pools(c["pool"])
    ref = op.paged_prefill(c["np_q"], c["table"], c["counts"], c["tags"], ORACLE_FMT, pools, sc, c["scale_mode"],
                           bases=c["bases"], row_masks=c["masks"], q_positions=c["qpos"], causal=True, sm_scale=-0.05)
    _close(got, ref)
