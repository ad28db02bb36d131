"""Drop-in for the reference's ``triton_kernel.py``: multi-query selected-block
attention over dense K / V (``semantic_block_attention_triton``).

The reference (``triton_kernel.py:427-498`` ``_triton_impl``, ``:564-641``
``_triton_impl_quant``, ``:668-760``) selects the non-SKIP blocks whose ATTEND
score is >= ``threshold``, lists the 128-token pages they touch and runs a
Triton flash kernel over whole pages.  Here the selected tokens are exact:
each page slot carries a row mask of the tokens its selected blocks cover, and
causal masks compare ORIGINAL token positions (the semantics of the
reference's exact-token path, ``reference.py:82-130``).  The reference's GPU
path instead attends to every token of a touched page (its README notes the
missing partial-page bounds) and leaves rows that see nothing NaN; those rows
are 0 here.

K / V are quantised on write into page pools of this build (``use_quant``:
INT8 with one scale per page and channel, the reference's
``_quant_kernel`` granularity, ``triton_kernel.py:186-279``; otherwise F16)
and the attention runs in ``iak_prefill`` (tcgen05 kernel for head_dim 128).
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Sequence, Tuple, Union

import torch

from . import _native as N
from .block_metadata import BlockLayout, BlockPolicy, SemanticBlock
from .paged import PagePool, make_tag_map, paged_prefill

# page size of the pools built here: the largest the row masks and the tensor-core kernel take
_PAGE_SIZE = 64


def is_triton_available() -> bool:
    """True when the compiled kernels can run (the reference's name for its GPU-path probe)."""
    return N.available() and torch.cuda.is_available()


def is_cuda_available() -> bool:
    return torch.cuda.is_available()


def _unique_preserve_order(pages: torch.Tensor) -> torch.Tensor:
    seen: Dict[int, None] = {}
    for p in pages.tolist():
        seen.setdefault(int(p), None)
    return torch.tensor(list(seen), dtype=pages.dtype, device=pages.device)


def _threshold_blocks(layout: BlockLayout, threshold: float) -> List[SemanticBlock]:
    """triton_kernel.py:437-445: SKIP dropped, ATTEND kept only with a score >= threshold."""
    out = []
    for blk in layout.blocks:
        if blk.policy == BlockPolicy.SKIP:
            continue
        if blk.policy == BlockPolicy.ATTEND and (blk.score is None or blk.score < threshold):
            continue
        out.append(blk)
    return out


def _compute_selected_page_ids(layout: BlockLayout, kv_len: int, threshold: float = 0.5,
                               page_size: int = 128) -> torch.Tensor:
    """triton_kernel.py:644-665: pages touched by the selected blocks, first occurrence first."""
    pages: Dict[int, None] = {}
    for blk in _threshold_blocks(layout, threshold):
        for pid in range(blk.start // page_size, (blk.end + page_size - 1) // page_size):
            pages.setdefault(pid, None)
    return torch.tensor(list(pages), dtype=torch.int32)


def block_pages_and_masks(blocks: Sequence[SemanticBlock], page_size: int) -> Tuple[List[int], List[int]]:
    """Logical pages of the blocks' tokens (first occurrence first) and, per
    page, the bit mask of the rows the blocks cover."""
    masks: Dict[int, int] = {}
    for blk in blocks:
        t = blk.start
        while t < blk.end:
            pg = t // page_size
            hi = min(blk.end, (pg + 1) * page_size)
            lo_r, hi_r = t - pg * page_size, hi - pg * page_size
            masks[pg] = masks.get(pg, 0) | (((1 << (hi_r - lo_r)) - 1) << lo_r)
            t = hi
    pages = list(masks)
    return pages, [masks[p] for p in pages]


def _to_signed64(mask: int) -> int:
    return mask - (1 << 64) if mask >= (1 << 63) else mask


def blocks_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, blocks: Sequence[SemanticBlock],
                     causal: bool, use_quant: bool = False, kernel: str = "auto") -> torch.Tensor:
    """Attention of q [B, Hq, M, D] over exactly the tokens of ``blocks`` of
    k / v [B, Hk, T, D] (Hq a multiple of Hk), causal on original positions
    (query m at position m)."""
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("this build runs only on CUDA tensors (no CPU fallback)")
    B, Hq, M, D = q.shape
    Hk, T = k.shape[1], k.shape[2]
    if not blocks:
        return torch.zeros_like(q)
    PS = _PAGE_SIZE
    n_log = (T + PS - 1) // PS
    units = B * Hk
    pages, masks = block_pages_and_masks(blocks, PS)
    n = len(pages)
    idx = torch.tensor(pages, dtype=torch.int64, device=q.device)
    # only the touched pages are quantised; each slot carries its page's token position
    pad = n_log * PS - T
    kp = torch.nn.functional.pad(k, (0, 0, 0, pad)).reshape(units, n_log, PS, D)[:, idx].reshape(units * n, PS, D)
    vp = torch.nn.functional.pad(v, (0, 0, 0, pad)).reshape(units, n_log, PS, D)[:, idx].reshape(units * n, PS, D)
    fmt = "INT8" if use_quant else "F16"
    pool = PagePool.allocate(units * n, PS, D, [fmt], "channel" if use_quant else "page", q.device)
    pool.quantize_(kp.contiguous(), vp.contiguous(), [fmt] * (units * n))
    table = torch.arange(units * n, dtype=torch.int32, device=q.device).view(B, Hk, n)
    positions = (idx.to(torch.int32) * PS)[None, None, :].expand(B, Hk, n).contiguous()
    row_masks = torch.tensor([_to_signed64(m) for m in masks], dtype=torch.int64, device=q.device)
    row_masks = row_masks[None, :].expand(B, -1).contiguous()
    tags = torch.ones(units * n, dtype=torch.uint8, device=q.device)
    return paged_prefill(q, pool, table, None, tags, make_tag_map({1: fmt}), causal=causal, row_masks=row_masks,
                         page_positions=positions, out_dtype=q.dtype, kernel=kernel)


def semantic_block_attention_triton(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layout: BlockLayout,
                                    causal: bool = False, threshold: float = 0.5, return_debug: bool = False,
                                    use_quant: bool = False, prefetch: bool = False
                                    ) -> Union[torch.Tensor, Tuple[torch.Tensor, Dict[str, Any]]]:
    """Same signature and debug keys as the reference (``triton_kernel.py:668-760``);
    ``prefetch`` predicts nothing here (``prefetched_page_ids`` is empty)."""
    kv_tokens = k.size(-2)
    layout.validate(kv_tokens)
    blocks = _threshold_blocks(layout, threshold)
    out = blocks_attention(q, k, v, blocks, causal, use_quant)
    if return_debug:
        count = sum(b.end - b.start for b in blocks)
        return out, {"selected_token_count": count, "selected_block_names": [b.name for b in blocks],
                     "total_kv_tokens": kv_tokens, "selected_kv_tokens": count, "prefetched_page_ids": []}
    return out
