"""Oracle paged decode (numpy).  TEST INFRASTRUCTURE ONLY.

Restates the single-query paged decode of the reference:

* ``fused_selected_quant_decode.py:267-336`` (``fused_selected_quant_decode_reference``):
  for each (b, h), walk ``page_table[b, h, :page_counts[b, h]]``, look up the
  page's precision tag, skip SKIP pages, dequantise INT8 pages as
  ``code * scale[page]``, score ``q . k / sqrt(D)``, online softmax, output
  ``acc / max(l, 1e-8)`` (zeros when nothing was attended).
* ``triton_intent_quant_attention.py:272-332``: the same walk with -1 padded
  page ids, six tags, and FP8/INT4/INT4_RESIDUAL read through the INT8 buffers.
* ``triton_adaptive_format_attention.py:153-222``: all table slots, -1 = unused,
  SPARSE contributes nothing (the reference kernel masks it to -inf).
* the (m, l, acc) algebra of the online softmax (``fused_selected_quant_decode.py:323-332``)
  gives the split-KV LSE merge (``lse_merge``).

One generalised routine, ``paged_decode``, covers all of them: a page table
per (batch, page-table head) unit, G = Hq / Hpt query heads per unit (GQA; the
reference is the G = 1 case), a tag -> format map chosen per entry point, and
this project's page formats (FP16, FP8-e4m3, INT8, packed INT4, INT4_RESIDUAL)
with per-page / per-32-group / per-channel scales.  Attention is evaluated in
float64 on float32 dequantised values; softmax is permutation invariant, so
evaluating all of a unit's tokens at once equals the reference's page-by-page
online recurrence up to rounding.
"""

from __future__ import annotations

from typing import Dict, Mapping, Optional, Tuple

import numpy as np

from .quant import F32, e4m3_to_f32, expand_scales, unpack_int4

FORMATS = ("SKIP", "F16", "FP8", "INT8", "INT4", "INT4R", "SPARSE")


def _dequant_page_set(fmt: str, pids: np.ndarray, plane: str, pools: Mapping, scales: Mapping,
                      scale_mode: str, head_dim: int) -> np.ndarray:
    """Dequantise pages ``pids`` of one format and one plane ('k' or 'v') -> [n, PS, D]."""
    if fmt == "F16":
        return np.asarray(pools[f"{plane}_f16"])[pids].astype(F32)
    if fmt == "SPARSE":
        # reference kernel: SPARSE pages are masked out; callers drop them
        raise ValueError("SPARSE pages contribute nothing and are filtered earlier")
    s = np.asarray(scales[f"{plane}_scale"])[pids]
    se = expand_scales(s, scale_mode, head_dim)
    if fmt == "FP8":
        return (e4m3_to_f32(np.asarray(pools[f"{plane}_fp8"])[pids]) * se).astype(F32)
    if fmt == "INT8":
        return (np.asarray(pools[f"{plane}_i8"])[pids].astype(F32) * se).astype(F32)
    if fmt == "INT4":
        codes = unpack_int4(np.asarray(pools[f"{plane}_i4"])[pids])
        return (codes.astype(F32) * se).astype(F32)
    if fmt == "INT4R":
        base = unpack_int4(np.asarray(pools[f"{plane}_i4"])[pids]).astype(F32) * se
        rs = np.asarray(scales[f"{plane}_res_scale"])[pids]
        rse = expand_scales(rs, scale_mode, head_dim)
        res = unpack_int4(np.asarray(pools[f"{plane}_i4r"])[pids]).astype(F32) * rse
        return (base.astype(F32) + res.astype(F32)).astype(F32)
    raise ValueError(f"unknown format {fmt}")


def unit_pages(page_table: np.ndarray, counts: Optional[np.ndarray], b: int, hk: int,
               num_pages: int) -> np.ndarray:
    """Valid page ids of one unit, in table order (slots < count, id in [0, NP))."""
    row = np.asarray(page_table[b, hk]).astype(np.int64)
    n = row.shape[0] if counts is None else int(min(max(int(counts[b, hk]), 0), row.shape[0]))
    row = row[:n]
    return row[(row >= 0) & (row < num_pages)]


def unit_partial(q: np.ndarray, pids: np.ndarray, tags: np.ndarray, tag_map: Mapping[int, str],
                 default_fmt: str, pools: Mapping, scales: Mapping, scale_mode: str,
                 sm_scale: float) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(m, l, acc) of G queries ``q`` [G, D] over pages ``pids`` (natural-log domain).

    Empty -> m = -inf, l = 0, acc = 0.
    """
    G, D = q.shape
    fmts = np.array([tag_map.get(int(tags[p]), default_fmt) for p in pids], dtype=object)
    keep = (fmts != "SKIP") & (fmts != "SPARSE")
    pids, fmts = pids[keep], fmts[keep]
    if pids.size == 0:
        return (np.full(G, -np.inf), np.zeros(G), np.zeros((G, D)))
    ks, vs = [], []
    for fmt in FORMATS:
        sel = pids[fmts == fmt]
        if sel.size == 0:
            continue
        ks.append(_dequant_page_set(fmt, sel, "k", pools, scales, scale_mode, D))
        vs.append(_dequant_page_set(fmt, sel, "v", pools, scales, scale_mode, D))
    K = np.concatenate(ks, axis=0).reshape(-1, D).astype(np.float64)
    V = np.concatenate(vs, axis=0).reshape(-1, D).astype(np.float64)
    s = (q.astype(np.float64) @ K.T) * sm_scale          # [G, T]
    m = s.max(axis=1)
    p = np.exp(s - m[:, None])
    return m, p.sum(axis=1), p @ V


def paged_decode(q: np.ndarray, page_table: np.ndarray, counts: Optional[np.ndarray],
                 tags: np.ndarray, tag_map: Mapping[int, str], pools: Mapping,
                 scales: Optional[Mapping] = None, scale_mode: str = "page",
                 sm_scale: Optional[float] = None, default_fmt: str = "SKIP",
                 return_partials: bool = False):
    """Generalised paged decode.

    q [B, Hq, D] float; page_table [B, Hpt, W] int (Hq % Hpt == 0, G = Hq/Hpt);
    counts [B, Hpt] or None (all slots, -1 = unused); tags [NP] per physical page;
    ``tag_map`` maps a tag to one of ``FORMATS``; unknown tags -> ``default_fmt``.
    Returns out [B, Hq, D] float64 (and (m, l, acc) when ``return_partials``).
    """
    q = np.asarray(q, dtype=np.float64)
    B, Hq, D = q.shape
    Hpt = page_table.shape[1]
    G = Hq // Hpt
    scales = scales or {}
    if sm_scale is None:
        sm_scale = 1.0 / np.sqrt(D)
    tags = np.asarray(tags).astype(np.int64)
    NP = tags.shape[0]
    out = np.zeros((B, Hq, D))
    ms = np.zeros((B, Hq)); ls = np.zeros((B, Hq)); accs = np.zeros((B, Hq, D))
    for b in range(B):
        for hk in range(Hpt):
            pids = unit_pages(page_table, counts, b, hk, NP)
            m, l, acc = unit_partial(q[b, hk * G:(hk + 1) * G], pids, tags, tag_map, default_fmt,
                                     pools, scales, scale_mode, sm_scale)
            sl = slice(hk * G, (hk + 1) * G)
            ms[b, sl], ls[b, sl], accs[b, sl] = m, l, acc
            out[b, sl] = np.where(l[:, None] > 0, acc / np.maximum(l, 1e-300)[:, None], 0.0)
    if return_partials:
        return out, (ms, ls, accs)
    return out


def lse_merge(m: np.ndarray, l: np.ndarray, acc: np.ndarray) -> np.ndarray:
    """Merge split partials along axis -1 of ``m``/``l`` (axis -2 of ``acc``).

    m_* = max_i m_i; l_* = sum_i l_i e^(m_i - m_*); o = sum_i acc_i e^(m_i - m_*) / l_*.
    Splits with l_i = 0 (m_i = -inf) contribute nothing; all-empty -> 0.
    """
    m = np.asarray(m, dtype=np.float64)
    l = np.asarray(l, dtype=np.float64)
    acc = np.asarray(acc, dtype=np.float64)
    mstar = m.max(axis=-1, keepdims=True)
    safe = np.where(np.isfinite(mstar), mstar, 0.0)
    w = np.where(l > 0, np.exp(np.where(np.isfinite(m), m, safe) - safe), 0.0)
    lstar = (l * w).sum(axis=-1)
    o = (acc * w[..., None]).sum(axis=-2)
    return np.where(lstar[..., None] > 0, o / np.where(lstar > 0, lstar, 1.0)[..., None], 0.0)


# --------------------------------------------------------------------------- #
#  Reference entry-point semantics
# --------------------------------------------------------------------------- #

FUSED_TAG_MAP = {0: "F16", 1: "INT8", 2: "SKIP"}           # FusedKVPrecision
TRITON6_TAG_MAP = {0: "F16", 1: "INT8", 2: "INT8", 3: "INT8", 4: "INT8", 5: "SKIP"}
ADAPTIVE_TAG_MAP = {0: "F16", 1: "INT8", 2: "SPARSE", 3: "SKIP"}


def fused_selected_quant_decode_ref(query, k_fp16, v_fp16, k_i8, v_i8, k_scales, v_scales,
                                    page_table, page_precision, page_counts) -> np.ndarray:
    """``fused_selected_quant_decode.py:267-336`` restated; returns float64 [B, H, 1, D].

    (The reference then casts to float16.)  Scales are used as stored (the
    reference upcasts them with ``.float()``), so fp16 scales stay fp16-rounded.
    """
    q = np.asarray(query, dtype=np.float32)[:, :, 0, :]
    pools = {"k_f16": k_fp16, "v_f16": v_fp16, "k_i8": k_i8, "v_i8": v_i8}
    sc = {"k_scale": np.asarray(k_scales, dtype=F32).reshape(-1, 1),
          "v_scale": np.asarray(v_scales, dtype=F32).reshape(-1, 1)}
    out = paged_decode(q, np.asarray(page_table), np.asarray(page_counts), np.asarray(page_precision),
                       FUSED_TAG_MAP, pools, sc, "page", default_fmt="SKIP")
    return out[:, :, None, :]


def intent_quant_decode_triton_ref(q, k_fp16, v_fp16, k_i8, v_i8, k_scales, v_scales,
                                   page_ids, page_count, page_precision) -> np.ndarray:
    """``triton_intent_quant_attention.py:255-335`` semantics -> float64 [B, H, D]."""
    pools = {"k_f16": k_fp16, "v_f16": v_fp16, "k_i8": k_i8, "v_i8": v_i8}
    sc = {"k_scale": np.asarray(k_scales, dtype=F32).reshape(-1, 1),
          "v_scale": np.asarray(v_scales, dtype=F32).reshape(-1, 1)}
    return paged_decode(np.asarray(q, dtype=np.float32), np.asarray(page_ids), np.asarray(page_count),
                        np.asarray(page_precision), TRITON6_TAG_MAP, pools, sc, "page",
                        default_fmt="INT8")


def adaptive_decode_triton_ref(q, page_ids, page_formats, k_fp16, v_fp16, k_i8=None, v_i8=None,
                               k_scales=None, v_scales=None) -> np.ndarray:
    """``triton_adaptive_format_attention.py:137-225`` semantics -> float64 [B, H, D]."""
    NP = np.asarray(page_formats).shape[0]
    shape = np.asarray(k_fp16).shape
    pools = {"k_f16": k_fp16, "v_f16": v_fp16,
             "k_i8": np.zeros(shape, np.int8) if k_i8 is None else k_i8,
             "v_i8": np.zeros(shape, np.int8) if v_i8 is None else v_i8}
    ones = np.ones((NP, 1), F32)
    sc = {"k_scale": ones if k_scales is None else np.asarray(k_scales, dtype=F32).reshape(-1, 1),
          "v_scale": ones if v_scales is None else np.asarray(v_scales, dtype=F32).reshape(-1, 1)}
    return paged_decode(np.asarray(q, dtype=np.float32), np.asarray(page_ids), None,
                        np.asarray(page_formats), ADAPTIVE_TAG_MAP, pools, sc, "page",
                        default_fmt="SKIP")
