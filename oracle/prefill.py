"""Oracle multi-query (prefill) attention over selected pages (numpy).
TEST INFRASTRUCTURE ONLY.

* ``semantic_block_attention`` restates ``reference.py:82-130``
  (``semantic_block_attention``, the exact-token CPU path): the selected
  tokens are every token of the blocks whose policy is ALWAYS / ATTEND /
  RECENT / GLOBAL (``block_metadata.py:72-79``), in layout order; attention is
  ``reference.py:16-45`` ``dense_attention`` with, when causal, query i at
  position i and key j visible iff ``i >= original position of j``.  A query
  that sees no key gets NaN there (softmax over an all -inf row); the product
  writes 0 for such rows instead.
* ``paged_prefill`` is the same attention over page pools: for every
  (sequence, page-table head) the keys are the rows of the listed pages that
  the slot's row mask selects, at token position ``(page - base) * PS + row``;
  G = Hq / Ht query heads share a unit (the reference is G = 1); formats and
  scales as ``oracle.decode``.  Queries that see no key give 0.

Evaluated in float64 on float32 dequantised values.
"""

from __future__ import annotations

from typing import Mapping, Optional, Sequence, Tuple

import numpy as np

from .decode import _dequant_page_set

SELECTED_POLICIES = ("ALWAYS", "ATTEND", "RECENT", "GLOBAL")


def selected_token_indices(spec: Sequence[Tuple]) -> np.ndarray:
    """block_metadata.py:75-79: tokens of the selected-policy blocks, in layout order."""
    idx = []
    for _name, start, end, policy, _score in spec:
        if policy in SELECTED_POLICIES:
            idx.extend(range(start, end))
    return np.asarray(idx, dtype=np.int64)


def semantic_block_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, spec: Sequence[Tuple],
                             causal: bool) -> np.ndarray:
    """q [B, H, M, D], k / v [B, H, T, D] -> [B, H, M, D] (float64, NaN rows as the reference)."""
    q = np.asarray(q, np.float64)
    idx = selected_token_indices(spec)
    if idx.size == 0:
        return np.zeros(q.shape)
    ks = np.asarray(k, np.float64)[..., idx, :]
    vs = np.asarray(v, np.float64)[..., idx, :]
    s = np.matmul(q, np.swapaxes(ks, -1, -2)) / np.sqrt(q.shape[-1])
    if causal:
        qpos = np.arange(q.shape[-2])
        s = np.where(qpos[:, None] < idx[None, :], -np.inf, s)
    with np.errstate(invalid="ignore"):
        m = s.max(axis=-1, keepdims=True)
        e = np.exp(s - m)
        return np.matmul(e / e.sum(axis=-1, keepdims=True), vs)


def unit_tokens(page_table, counts, bases, row_masks, tags, tag_map, default_fmt, pools, scales, scale_mode,
                b: int, h: int, page_size: int, head_dim: int, page_positions=None):
    """Selected keys / values / positions of one (sequence, table head) unit."""
    Ht = page_table.shape[1]
    row = np.asarray(page_table[b, h]).astype(np.int64)
    n = row.shape[0] if counts is None else int(min(max(int(counts[b, h]), 0), row.shape[0]))
    NP = np.asarray(tags).shape[0]
    base = 0 if bases is None else int(np.asarray(bases).reshape(-1)[b * Ht + h])
    ks, vs, pos = [], [], []
    for o in range(n):
        pid = int(row[o])
        if pid < 0 or pid >= NP:
            continue
        fmt = tag_map.get(int(tags[pid]), default_fmt)
        if fmt in ("SKIP", "SPARSE"):
            continue
        mask = ~np.uint64(0) if row_masks is None else np.uint64(row_masks[b, o])
        rows = [r for r in range(page_size) if (int(mask) >> r) & 1]
        if not rows:
            continue
        kp = _dequant_page_set(fmt, np.array([pid]), "k", pools, scales, scale_mode, head_dim)[0]
        vp = _dequant_page_set(fmt, np.array([pid]), "v", pools, scales, scale_mode, head_dim)[0]
        ks.append(kp[rows])
        vs.append(vp[rows])
        pos0 = (pid - base) * page_size if page_positions is None else int(page_positions[b, h, o])
        pos.extend(pos0 + r for r in rows)
    if not ks:
        return np.zeros((0, head_dim)), np.zeros((0, head_dim)), np.zeros(0, np.int64)
    return (np.concatenate(ks).astype(np.float64), np.concatenate(vs).astype(np.float64),
            np.asarray(pos, np.int64))


def paged_prefill(q: np.ndarray, page_table: np.ndarray, counts: Optional[np.ndarray], tags: np.ndarray,
                  tag_map: Mapping[int, str], pools: Mapping, scales: Optional[Mapping] = None,
                  scale_mode: str = "page", bases: Optional[np.ndarray] = None,
                  row_masks: Optional[np.ndarray] = None, q_positions: Optional[np.ndarray] = None,
                  causal: bool = True, sm_scale: Optional[float] = None, default_fmt: str = "SKIP",
                  page_positions: Optional[np.ndarray] = None) -> np.ndarray:
    """q [B, Hq, M, D]; page_table [B, Ht, W]; row_masks [B, W] uint64 (bit r = row r) or None;
    q_positions [B, M] or None (= m); page_positions [B, Ht, W] (position of row 0 of each
    slot) or None.  Returns [B, Hq, M, D] float64; rows that see no key are 0."""
    q = np.asarray(q, np.float64)
    B, Hq, M, D = q.shape
    Ht = page_table.shape[1]
    G = Hq // Ht
    page_size = next(np.asarray(pools[k]).shape[1] for k in pools if np.asarray(pools[k]).ndim == 3)
    scale = 1.0 / np.sqrt(D) if sm_scale is None else sm_scale
    out = np.zeros((B, Hq, M, D))
    for b in range(B):
        qpos = np.arange(M) if q_positions is None else np.asarray(q_positions[b], np.int64)
        for h in range(Ht):
            K, V, pos = unit_tokens(page_table, counts, bases, row_masks, tags, tag_map, default_fmt, pools,
                                    scales or {}, scale_mode, b, h, page_size, D, page_positions)
            if pos.size == 0:
                continue
            for g in range(G):
                s = (q[b, h * G + g] @ K.T) * scale                     # [M, T]
                vis = (pos[None, :] <= qpos[:, None]) if causal else np.ones(s.shape, bool)
                s = np.where(vis, s, -np.inf)
                has = vis.any(axis=1)
                m = np.where(has, s.max(axis=1), 0.0)
                e = np.where(vis, np.exp(s - m[:, None]), 0.0)
                l = e.sum(axis=1)
                o = (e @ V) / np.where(has, l, 1.0)[:, None]
                out[b, h * G + g] = np.where(has[:, None], o, 0.0)
    return out


def layout_pages(spec: Sequence[Tuple], page_size: int, threshold: Optional[float] = None):
    """Logical pages and row masks of a layout's selected tokens, pages in
    first-occurrence order of the selected blocks (layout order).

    ``threshold`` None: the exact-token CPU path's selection (every
    ALWAYS / ATTEND / RECENT / GLOBAL block).  A number: the GPU path's
    selection (``triton_kernel.py:437-445``: SKIP dropped, ATTEND kept only
    with a score >= threshold)."""
    pages, masks = [], {}
    for _name, start, end, policy, score in spec:
        if policy == "SKIP":
            continue
        if threshold is not None and policy == "ATTEND" and (score is None or score < threshold):
            continue
        if threshold is None and policy not in SELECTED_POLICIES:
            continue
        for t in range(start, end):
            pg = t // page_size
            if pg not in masks:
                masks[pg] = 0
                pages.append(pg)
            masks[pg] |= 1 << (t - pg * page_size)
    return np.asarray(pages, np.int64), np.asarray([masks[p] for p in pages], np.uint64)


def semantic_paged_attention(query: np.ndarray, key_cache: np.ndarray, value_cache: np.ndarray,
                             block_table: np.ndarray, spec: Sequence[Tuple], block_size: int,
                             causal: bool) -> np.ndarray:
    """Per-head attention of query [T, H, D] over the selected cache blocks
    ([NB, H, D, BS] caches) with the block selection of ``vllm_bridge.py:37-58``
    and the compacted-index causal mask of ``dense_attention(causal=True)``
    (``reference.py:27-40``): query i sees the first i + 1 concatenated keys.
    The reference itself contracts over the head axis (a defect); this is the
    per-head attention its docstring describes."""
    num_logical = len(block_table)
    phys = {}
    for _name, start, end, policy, score in spec:
        if policy == "SKIP" or (policy == "ATTEND" and score is not None and score < 0.5):
            continue
        for logical in range(start // block_size, min((end + block_size - 1) // block_size, num_logical)):
            phys.setdefault(int(block_table[logical]), None)
    T, H, D = query.shape
    if not phys:
        return np.zeros((T, H, D))
    ids = list(phys)
    K = np.concatenate([np.asarray(key_cache[p], np.float64).transpose(2, 0, 1) for p in ids])    # [N, H, D]
    V = np.concatenate([np.asarray(value_cache[p], np.float64).transpose(2, 0, 1) for p in ids])
    out = np.zeros((T, H, D))
    for h in range(H):
        s = np.asarray(query[:, h], np.float64) @ K[:, h].T / np.sqrt(D)        # [T, N]
        if causal:
            s = np.where(np.arange(K.shape[0])[None, :] > np.arange(T)[:, None], -np.inf, s)
        m = s.max(axis=1, keepdims=True)
        e = np.exp(s - m)
        out[:, h] = (e / e.sum(axis=1, keepdims=True)) @ V[:, h]
    return out
