"""GPU parity at the shapes of the five BASELINE configurations.

Each case builds its workload exactly as ``bench.py`` does (the router's page
lists, format mix, scale mode, GQA group, head counts, context length and
synthetic value distribution of the configuration; only the batch is cut to
one or two sequences) and compares the decode that ``bench.py`` times (the
tensor-core path, through the C ABI) with the numpy oracle on the very pages
the GPU quantiser wrote.

Oracle semantics: ``intent_quant_attention.py:20-119``
(``intent_quant_attention_reference``: dequantise the selected blocks, then
dense attention over them), with the page quantisation rules of
``intent_quant.py:258-307`` (INT8 / INT4 / INT4_RESIDUAL) and, for C4, the
absorbed latent decode of ``mla.py:61-92``.

Tolerance: atol 2e-3 / rtol 1e-2 on fp32-accumulated
outputs.  The stress cases at the end push the kernel's own numeric choices
(the two-term int8 query of the integer MMA path, the V scale folded into fp16
probabilities, the fp16 query fragments of the FP16 / FP8 path) with inputs
the random N(0, 1) cases never produce.
"""

import json
import os

import numpy as np
import pytest
import torch

import bench
from gpu_cases import compact_oracle_view, make_case, run_gpu, run_oracle
from intent_attention import paged_decode
from intent_attention.paged import make_tag_map
from intent_attention.split_kv import block_floats, decode_partial_block, merge_partial_blocks, shard_page_lists
from oracle import decode as odec

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
ORACLE_FMT = {1: "F16", 2: "FP8", 3: "INT8", 4: "INT4", 5: "INT4R"}
_BUILT = {}
# worst errors per configuration; written as JSON to $IAK_PARITY_REPORT (when set) after the module
_REPORT = {}


def _close(got, ref, atol=ATOL, rtol=RTOL, key=None):
    got = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else got
    if key is not None:
        err = np.abs(got.astype(np.float64) - ref)
        _REPORT[key] = {"max_abs": float(err.max()), "max_abs_over_max_ref": float(err.max() / np.abs(ref).max()),
                        "max_rel_where_ref_above_atol": float(np.max((err / np.abs(ref))[np.abs(ref) > atol], initial=0.0)),
                        "elements": int(ref.size), "atol": atol, "rtol": rtol}
    np.testing.assert_allclose(got, ref, atol=atol, rtol=rtol)


def teardown_module(module):
    path = os.environ.get("IAK_PARITY_REPORT")
    if path and _REPORT:
        with open(path, "w") as f:
            json.dump(_REPORT, f, indent=1)


def _config(name, batch):
    """(workload, pool, table, counts, tags, q, tag_map, oracle output) of a config at `batch`, built once."""
    key = (name, batch)
    if key not in _BUILT:
        _BUILT.clear()                      # one configuration's pools on the device at a time
        torch.cuda.empty_cache()
        w = bench.workload(name)
        w["B"] = batch
        ids, fmt = bench.select_pages(w)
        dev = torch.device("cuda", 0)
        pool, table, counts, tags, q = bench.build_gpu_workload(w, ids, fmt, dev, 0)
        tag_map = make_tag_map({c: (f if f in w["mix"] else "SKIP") for f, c in bench.FMT_CODE.items()})
        np_table, np_counts, np_tags, pools, scales = compact_oracle_view(pool, table, counts, tags)
        ref = odec.paged_decode(q.float().cpu().numpy(), np_table, np_counts, np_tags, ORACLE_FMT, pools, scales,
                                w["scale_mode"], default_fmt="SKIP")
        _BUILT[key] = (w, ids, fmt, pool, table, counts, tags, q, tag_map, ref)
    return _BUILT[key]


def _decode(cfg, **kw):
    w, ids, fmt, pool, table, counts, tags, q, tag_map, _ = cfg
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    return paged_decode(q, pool, table, counts, tags, tag_map, 0, out=out, kernel="tensor", **kw)


# ------------------------------------------------------------------ C1-C5 at their shapes
def test_c1_config_shape():
    """C1: MHA, head_dim 64, 1440 tokens, 74 of 90 pages: FP16 system / recent pages,
    INT8 retrieved pages (per-page, per-head absmax), the tool-output pages skipped."""
    cfg = _config("c1", 1)
    w, ids, fmt = cfg[:3]
    assert ids.size == 74 and set(np.unique(fmt)) == {1, 3}
    assert (fmt[(ids >= 8) & (ids < 64)] == 3).all() and (fmt[(ids < 8) | (ids >= 80)] == 1).all()
    _close(_decode(cfg), cfg[-1], key="C1")


@pytest.mark.parametrize("batch", [1, 2])
def test_c2_config_shape(batch):
    """C2: Llama-3-8B GQA (32 / 8 heads), 1024 of 2048 pages per (sequence, kv head),
    30 / 40 / 30 % FP16 / FP8 / INT8 with per-page scales, 1 % x8 outliers, bf16 q."""
    cfg = _config("c2", batch)
    w, ids, fmt = cfg[:3]
    assert ids.size == 1024 and w["Hq"] == 32 and w["Hkv"] == 8 and cfg[7].dtype == torch.bfloat16
    assert np.bincount(fmt, minlength=6)[[1, 2, 3]].tolist() == [307, 410, 307]
    _close(_decode(cfg), cfg[-1], key=f"C2 batch {batch}")


def test_c3_config_shape():
    """C3: Llama-3-70B low-bit (64 / 8 heads, G = 8), all 512 pages, group-32 scales,
    20 / 40 / 40 % FP16 / INT4 / INT4_RESIDUAL, q ~ N(0, 0.5)."""
    cfg = _config("c3", 1)
    w, ids, fmt = cfg[:3]
    assert ids.size == 512 and w["Hq"] // w["Hkv"] == 8 and w["scale_mode"] == "group32"
    assert np.bincount(fmt, minlength=6)[[1, 4, 5]].tolist() == [102, 205, 205]
    _close(_decode(cfg), cfg[-1], key="C3")


def test_c5_config_shape():
    """C5: 524288-token context, 8192 selected pages per (sequence, kv head),
    10 / 30 / 30 / 30 % FP16 / FP8 / INT8 / INT4 with per-page scales."""
    cfg = _config("c5", 1)
    w, ids, fmt = cfg[:3]
    assert ids.size == 8192 and w["T"] == 524288
    _close(_decode(cfg), cfg[-1], key="C5")


def test_c5_config_shape_eight_shards_merged():
    """C5 cut as on 8 GPUs: every page list in 8 contiguous ranges, each decoded
    into a partial block, the blocks LSE-merged with iak_merge_partial_blocks."""
    cfg = _config("c5", 1)
    w, ids, fmt, pool, table, counts, tags, q, tag_map, ref = cfg
    B, Hq, D = q.shape
    rows, world = B * Hq, 8
    blocks = torch.empty(world * block_floats(rows, D), dtype=torch.float32, device=q.device)
    for r in range(world):
        t_r, c_r = shard_page_lists(table, counts, r, world)
        decode_partial_block(q, pool, t_r, c_r, tags, tag_map, block=blocks.view(world, -1)[r], kernel="tensor")
    out = merge_partial_blocks(blocks, rows, D).view(B, Hq, D)
    _close(out, ref, key="C5 as 8 sequence shards")


@pytest.mark.parametrize("splits", [1, 5])
def test_c2_config_shape_fixed_splits(splits):
    """The same C2 batch with the split count forced (one item per unit, and a ragged split)."""
    cfg = _config("c2", 1)
    _close(_decode(cfg, num_splits=splits), cfg[-1])


def test_c4_config_shape():
    """C4: DeepSeek-V2 absorbed MLA, 128 heads, d_qk 576 / d_v 512, 64-token pages,
    154 selected pages per sequence: the last 32 BF16, 122 FP8 with per-page scales."""
    from intent_attention.triton_mla_decode import make_mla_tag_map, mla_paged_decode
    from oracle import mla as omla
    _BUILT.clear()
    torch.cuda.empty_cache()
    w = dict(bench.C4)
    w["B"] = 2
    ids, tags_sel = bench.select_mla_pages(w)
    assert ids.size == 154 and int((tags_sel == 0).sum()) == 32
    dev = torch.device("cuda", 0)
    dense, fp8, scale, tags, table, q = bench.build_mla_workload(w, ids, tags_sel, dev, 0)
    tmap = make_mla_tag_map({0: "DENSE", 1: "FP8", 2: "SKIP"})
    sm = 1.0 / np.sqrt(w["Dqk"])
    out = mla_paged_decode(q, table, None, dense_pages=dense, fp8_pages=fp8, fp8_scale=scale, page_tags=tags,
                           tag_map=tmap, d_v=w["Dv"], sm_scale=sm, out_dtype=torch.float32, kernel="tensor")
    # compact oracle view of the selected latent pages
    uniq = torch.unique(table.long())
    ct = torch.searchsorted(uniq, table.long()).cpu().numpy()
    pools = {"bf16": dense.index_select(0, uniq).float().cpu().numpy(),
             "fp8": fp8.index_select(0, uniq).cpu().numpy()}
    ref = omla.mla_paged_decode(q.float().cpu().numpy(), ct, None, tags.long().index_select(0, uniq).cpu().numpy(),
                                pools, scale.index_select(0, uniq).cpu().numpy(), w["Dv"], sm)
    _close(out, ref, key="C4")


# ------------------------------------------------------------------ stress cases
def _requantised(case, k, v):
    """Rewrite the case's pools from new dense K / V pages (same formats and tags)."""
    case["pool"].quantize_(torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), case["tags"])
    return case


@pytest.mark.parametrize("fmts", [("INT8",), ("INT4", "INT4R"), ("F16", "FP8", "INT8", "INT4", "INT4R")])
@pytest.mark.parametrize("mode", ["page", "group32"])
def test_stress_query_outlier_channels(fmts, mode):
    """A few query channels x50: the integer-MMA path represents q as s1*i1 + s2*i2
    (two int8 terms per head), whose error grows with the head's absmax."""
    case = make_case(501, B=2, Hq=16, Ht=2, D=128, W=200, NP=600, formats=fmts, scale_mode=mode,
                     counts="full", pad_frac=0.0, skip_frac=0.0)
    g = np.random.default_rng(502)
    q = case["np_q"].copy()
    for b in range(q.shape[0]):
        for h in range(q.shape[1]):
            q[b, h, g.choice(128, 3, replace=False)] *= 50.0
    case["q"] = torch.from_numpy(q).to("cuda", torch.bfloat16)
    case["np_q"] = case["q"].float().cpu().numpy()
    _close(run_gpu(case), run_oracle(case))


@pytest.mark.parametrize("mode", ["page", "group32"])
def test_stress_value_scales_span_seven_decades(mode):
    """V pages whose absmax spans 1e-4 .. 1e3: the V scale is folded into the
    fp16 probabilities (page scales) or applied to the accumulators (group scales)."""
    case = make_case(511, B=2, Hq=8, Ht=2, D=128, W=160, NP=400, scale_mode=mode, counts="full",
                     pad_frac=0.0, skip_frac=0.0)
    g = np.random.default_rng(512)
    mag = 10.0 ** g.uniform(-4.0, 3.0, size=case["dense_v"].shape[0])
    v = (case["dense_v"] / np.abs(case["dense_v"]).reshape(len(mag), -1).max(1)[:, None, None]
         * mag[:, None, None]).astype(np.float32)
    _requantised(case, case["dense_k"], v)
    _close(run_gpu(case), run_oracle(case))


@pytest.mark.parametrize("fmts", [("F16",), ("FP8",), ("F16", "FP8", "INT8", "INT4", "INT4R")])
def test_stress_bf16_queries_outside_fp16_range(fmts):
    """bf16 queries beyond fp16's largest finite value (65504) and inside its
    subnormal range: the fp16 query fragments of the FP16 / FP8 path must neither
    overflow nor lose the small heads' precision."""
    case = make_case(521, B=2, Hq=8, Ht=2, D=128, W=120, NP=300, formats=fmts, counts="full",
                     pad_frac=0.0, skip_frac=0.0, q_dtype=torch.bfloat16)
    q = case["np_q"].copy()
    q[0, 0] *= 3.0e5                       # |q| up to ~1e6
    q[0, 1] *= 1.0e-6                      # fp16 subnormal range
    q[1, 2] *= 7.0e4
    case["q"] = torch.from_numpy(q).to("cuda", torch.bfloat16)
    case["np_q"] = case["q"].float().cpu().numpy()
    assert case["q"].float().abs().max() > 65504
    _close(run_gpu(case), run_oracle(case))
