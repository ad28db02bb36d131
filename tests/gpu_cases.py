"""Seeded GPU test cases: dense pages -> GPU quantiser -> pools, plus the
numpy-oracle view of the very same pools (test infrastructure)."""

from __future__ import annotations

import numpy as np
import torch

from intent_attention import PagePool, paged_decode
from intent_attention.paged import make_tag_map
from oracle import decode as odec

# tag = IAK format code in these cases
TAG_MAP = {0: "SKIP", 1: "F16", 2: "FP8", 3: "INT8", 4: "INT4", 5: "INT4R"}
NAME_OF = {"SKIP": 0, "F16": 1, "FP8": 2, "INT8": 3, "INT4": 4, "INT4R": 5}
ORACLE_FMT = {0: "SKIP", 1: "F16", 2: "FP8", 3: "INT8", 4: "INT4", 5: "INT4R"}


def make_case(seed, B=2, Hq=8, Ht=2, D=128, PS=16, W=40, NP=200, formats=("F16", "FP8", "INT8", "INT4", "INT4R"),
              probs=None, scale_mode="page", q_dtype=torch.bfloat16, counts="ragged", pad_frac=0.1,
              skip_frac=0.05, device="cuda", outliers=0.01):
    g = np.random.default_rng(seed)
    k = g.standard_normal((NP, PS, D)).astype(np.float32)
    v = g.standard_normal((NP, PS, D)).astype(np.float32)
    if outliers:
        k = np.where(g.random(k.shape) < outliers, k * 8, k).astype(np.float32)
        v = np.where(g.random(v.shape) < outliers, v * 8, v).astype(np.float32)
    fm = g.choice([NAME_OF[f] for f in formats], size=NP, p=probs).astype(np.uint8)
    fm = np.where(g.random(NP) < skip_frac, 0, fm).astype(np.uint8)
    pool = PagePool.allocate(NP, PS, D, formats, scale_mode, device, zero=True)
    pool.quantize_(torch.from_numpy(k).to(device), torch.from_numpy(v).to(device), torch.from_numpy(fm).to(device))
    table = np.stack([np.stack([g.permutation(NP)[:W] for _ in range(Ht)]) for _ in range(B)]).astype(np.int32)
    table = np.where(g.random(table.shape) < pad_frac, -1, table).astype(np.int32)
    if counts == "ragged":
        cnt = g.integers(0, W + 1, size=(B, Ht)).astype(np.int32)
        cnt[0, 0] = W
    elif counts == "full":
        cnt = np.full((B, Ht), W, np.int32)
    else:
        cnt = None
    q = g.standard_normal((B, Hq, D)).astype(np.float32)
    qt = torch.from_numpy(q).to(device=device, dtype=q_dtype)
    return {"pool": pool, "table": torch.from_numpy(table).to(device),
            "counts": None if cnt is None else torch.from_numpy(cnt).to(device),
            "tags": torch.from_numpy(fm).to(device), "q": qt, "np_table": table, "np_counts": cnt,
            "np_tags": fm, "np_q": qt.float().cpu().numpy(), "scale_mode": scale_mode, "dense_k": k, "dense_v": v,
            "formats": tuple(formats)}


def oracle_pools(pool: PagePool):
    names = ("k_f16", "v_f16", "k_fp8", "v_fp8", "k_i8", "v_i8", "k_i4", "v_i4", "k_i4r", "v_i4r")
    pools = {n: getattr(pool, n).cpu().numpy() for n in names if getattr(pool, n) is not None}
    sc = {}
    for n in ("k_scale", "v_scale", "k_res_scale", "v_res_scale"):
        t = getattr(pool, n)
        if t is not None:
            sc[n] = t.cpu().numpy()
    return pools, sc


def tag_map_for(formats):
    """Tags of formats without a pool in this case map to SKIP (no page carries them)."""
    return make_tag_map({t: (f if f in formats else "SKIP") for t, f in TAG_MAP.items()})


def run_gpu(case, out_dtype=torch.float32, num_splits=0, sm_scale=None, kernel="auto"):
    return paged_decode(case["q"], case["pool"], case["table"], case["counts"], case["tags"],
                        tag_map_for(case["formats"]), 0, sm_scale=sm_scale, out_dtype=out_dtype,
                        num_splits=num_splits, kernel=kernel)


def run_oracle(case, sm_scale=None):
    pools, sc = oracle_pools(case["pool"])
    return odec.paged_decode(case["np_q"], case["np_table"], case["np_counts"], case["np_tags"], ORACLE_FMT, pools,
                             sc, case["scale_mode"], sm_scale=sm_scale, default_fmt="SKIP")


POOL_PLANES = ("k_f16", "v_f16", "k_fp8", "v_fp8", "k_i8", "v_i8", "k_i4", "v_i4", "k_i4r", "v_i4r")
SCALE_PLANES = ("k_scale", "v_scale", "k_res_scale", "v_res_scale")


def compact_oracle_view(pool: PagePool, table: torch.Tensor, counts, tags: torch.Tensor):
    """The oracle's view of only the pages a decode can reach.

    Gathers, on the device, every pool plane and scale row of the distinct valid
    page ids of ``table`` (slots below ``counts``), copies them to the host and
    renumbers the table to the compact ids, so that configurations whose pools
    span millions of pages stay cheap to check.  Returns (np_table, np_counts,
    np_tags, pools, scales) for ``oracle.decode.paged_decode``.
    """
    t = table.long()
    W = t.shape[-1]
    if counts is not None:
        live = torch.arange(W, device=t.device)[None, None, :] < counts.long()[:, :, None]
        t = torch.where(live, t, torch.full_like(t, -1))
    t = torch.where((t >= 0) & (t < pool.num_pages), t, torch.full_like(t, -1))
    uniq = torch.unique(t[t >= 0])
    compact = torch.searchsorted(uniq, t.clamp(min=0))
    compact = torch.where(t >= 0, compact, torch.full_like(compact, -1))
    pools = {n: getattr(pool, n).index_select(0, uniq).cpu().numpy() for n in POOL_PLANES
             if getattr(pool, n) is not None}
    scales = {n: getattr(pool, n).index_select(0, uniq).cpu().numpy() for n in SCALE_PLANES
              if getattr(pool, n) is not None}
    np_tags = tags.long().index_select(0, uniq).cpu().numpy()
    return compact.int().cpu().numpy(), None, np_tags, pools, scales
