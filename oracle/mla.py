"""Oracle MLA (absorbed latent) decode (numpy).  TEST INFRASTRUCTURE ONLY.

* ``mla_decode_cpu`` restates ``triton_mla_decode.py:155-186`` (``_mla_decode_cpu``):
  per (batch, query row) an online softmax over the pages listed in a shared
  page table, latent page ``C[pid*ps:(pid+1)*ps]`` used as both key and value,
  scale ``1/sqrt(d_c)``, then ``context @ W_VO``; no pages -> zeros.
* ``mla_sparse_decode_reference`` (``mla.py:61-92``) is the same computation
  after ``q_absorb = q_flat @ W_QK`` with heads collapsed into one query row.
* ``mla_paged_decode`` is the per-head restatement used for the DeepSeek-V2
  shape: query rows are heads, the key is the full latent+rope vector
  (``d_qk`` channels), the value is its first ``d_v`` channels, pages are BF16
  or FP8-e4m3 with one scale per page.
"""

from __future__ import annotations

from typing import Mapping, Optional

import numpy as np

from .attention import softmax_lastdim
from .quant import F32, e4m3_to_f32


def mla_decode_cpu(q_absorb: np.ndarray, C: np.ndarray, W_VO: np.ndarray,
                   page_table: np.ndarray, page_size: int = 64) -> np.ndarray:
    """``triton_mla_decode.py:155-186`` -> [batch, q_len, d_out] float64."""
    q = np.asarray(q_absorb, dtype=np.float64)
    C = np.asarray(C, dtype=np.float64)
    W = np.asarray(W_VO, dtype=np.float64)
    batch, q_len, d_c = q.shape
    rows = [C[int(p) * page_size:(int(p) + 1) * page_size] for p in np.asarray(page_table).reshape(-1)]
    if not rows:
        return np.zeros((batch, q_len, W.shape[1]))
    Ct = np.concatenate(rows, axis=0)
    if Ct.shape[0] == 0:
        return np.zeros((batch, q_len, W.shape[1]))
    s = (q @ Ct.T) / np.sqrt(d_c)
    ctx = softmax_lastdim(s) @ Ct
    return ctx @ W


def mla_paged_decode(q: np.ndarray, page_table: np.ndarray, counts: Optional[np.ndarray],
                     tags: np.ndarray, pools: Mapping, scales: Optional[np.ndarray],
                     d_v: int, sm_scale: float) -> np.ndarray:
    """Per-head absorbed MLA decode over paged latents.

    q [B, H, Dqk]; page_table [B, W]; counts [B] or None; tags [NP] with
    0 = BF16 (``pools['bf16']`` float32 values already bf16-rounded),
    1 = FP8 (``pools['fp8']`` e4m3 codes, ``scales`` [NP] per page), 2 = SKIP.
    Returns context [B, H, d_v] float64 (zeros when no page is attended).
    """
    q = np.asarray(q, dtype=np.float64)
    B, H, Dqk = q.shape
    NP = np.asarray(tags).shape[0]
    out = np.zeros((B, H, d_v))
    for b in range(B):
        row = np.asarray(page_table[b]).astype(np.int64)
        n = row.shape[0] if counts is None else min(int(counts[b]), row.shape[0])
        row = row[:n]
        row = row[(row >= 0) & (row < NP)]
        lat = []
        for p in row:
            t = int(tags[p])
            if t == 0:
                lat.append(np.asarray(pools["bf16"][p], dtype=F32))
            elif t == 1:
                lat.append(e4m3_to_f32(pools["fp8"][p]) * F32(scales[p]))
        if not lat:
            continue
        Cb = np.concatenate(lat, axis=0).astype(np.float64)
        s = (q[b] @ Cb.T) * sm_scale
        out[b] = softmax_lastdim(s) @ Cb[:, :d_v]
    return out
