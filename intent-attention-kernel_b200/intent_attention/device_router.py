"""Device router: ``BlockRouter`` page selection for a batch of sequences on the GPU.

One launch of ``iak_route_pages`` does, for every sequence of a batch, what
the reference does on the host per request before each decode step:

* ``block_router.py:101-266`` ``BlockRouter.route_layout`` (with
  ``intent_quant.py:77-131`` ``IntentQuantizer.assign_block_precision`` as the
  precision policy),
* ``block_router.py:283-296`` ``selected_page_ids`` and the page precision map
  of ``block_router.py:383-421`` ``routing_to_kernel_metadata``,
* the page-table packing that ``iak_pack_metadata`` does for a host list,

so the decode kernel's page table, counts and per-page format tags are built
without a host round trip.  The layout checks of ``BlockLayout.validate``
(``block_metadata.py:41-70``) run on the device too; a sequence that fails them
gets ``num_selected == -1`` and an empty row, where the reference raises
``ValueError`` (``route_layouts`` raises it on the host before the launch).

Scores travel as float64 so that the threshold tests compare exactly as the
reference's Python floats do; NaN stands for ``None``.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Mapping, Optional, Sequence

import torch

from . import _native as N
from .block_metadata import BlockLayout, BlockPolicy
from .block_router import RouterConfig
from .intent_quant import IntentQuantizer, KVPrecision
from .paged import _require_cuda, _stream

POLICY_CODES = {BlockPolicy.ALWAYS: N.POLICY_ALWAYS, BlockPolicy.ATTEND: N.POLICY_ATTEND,
                BlockPolicy.SKIP: N.POLICY_SKIP, BlockPolicy.RECENT: N.POLICY_RECENT,
                BlockPolicy.GLOBAL: N.POLICY_GLOBAL}
PRECISION_CODES = {KVPrecision.FP16: N.PREC_FP16, KVPrecision.FP8: N.PREC_FP8, KVPrecision.INT8: N.PREC_INT8,
                   KVPrecision.INT4: N.PREC_INT4, KVPrecision.INT4_RESIDUAL: N.PREC_INT4_RESIDUAL,
                   KVPrecision.SKIP: N.PREC_SKIP}
PRECISIONS = {v: k for k, v in PRECISION_CODES.items()}


@dataclass
class LayoutBatch:
    """Block layouts of a batch on the device.

    ``start``/``end`` int32, ``policy`` uint8 and ``scores`` float64 are
    ``[batch, num_blocks]`` (row b holds sequence b's blocks in layout order;
    rows shorter than ``num_blocks`` are padded and ``counts`` gives their
    length).  A batch that shares one layout may pass 1-row ``start``/``end``/
    ``policy`` with per-sequence ``scores``.
    """

    start: torch.Tensor
    end: torch.Tensor
    policy: torch.Tensor
    scores: torch.Tensor
    counts: Optional[torch.Tensor] = None

    @property
    def batch(self) -> int:
        return self.scores.shape[0]

    @property
    def num_blocks(self) -> int:
        return self.start.shape[-1]


@dataclass
class RoutedPages:
    """Device outputs of one routing launch."""

    page_table: torch.Tensor     # [B, Ht, W] int32, pad_value padded
    page_counts: torch.Tensor    # [B, Ht] int32, min(n, W)
    num_selected: torch.Tensor   # [B] int32, n before truncation, -1 for an invalid layout
    page_prec: torch.Tensor      # [B, W] uint8 precision code per listed page (PREC_SKIP padding)
    row_masks: Optional[torch.Tensor] = None   # [B, W] int64 bit masks of the selected rows (0 padding)


def encode_layouts(layouts: Sequence[BlockLayout], device, scores: Optional[Sequence[Sequence[float]]] = None,
                   num_blocks: Optional[int] = None) -> LayoutBatch:
    """Pack host ``BlockLayout`` objects into a ``LayoutBatch`` on ``device``.

    ``scores`` (per layout, per block) overrides the blocks' own ``score``
    fields; ``None`` entries become NaN.
    """
    B = len(layouts)
    nb = max([len(l.blocks) for l in layouts] + [0]) if num_blocks is None else num_blocks
    start = torch.zeros((B, max(nb, 1)), dtype=torch.int32)
    end = torch.ones((B, max(nb, 1)), dtype=torch.int32)
    policy = torch.zeros((B, max(nb, 1)), dtype=torch.uint8)
    sc = torch.full((B, max(nb, 1)), math.nan, dtype=torch.float64)
    counts = torch.zeros(B, dtype=torch.int32)
    for b, layout in enumerate(layouts):
        n = len(layout.blocks)
        if n > nb:
            raise ValueError(f"layout {b} has {n} blocks > num_blocks={nb}")
        counts[b] = n
        for i, blk in enumerate(layout.blocks):
            start[b, i], end[b, i], policy[b, i] = blk.start, blk.end, POLICY_CODES[blk.policy]
            s = scores[b][i] if scores is not None else blk.score
            sc[b, i] = math.nan if s is None else float(s)
    to = lambda t: t[:, :nb].contiguous().to(device) if nb else t[:, :1].contiguous().to(device)  # noqa: E731
    return LayoutBatch(to(start), to(end), to(policy), to(sc), counts.to(device))


def route_pages(layouts: LayoutBatch, config: RouterConfig, page_size: int, table_width: int,
                table_heads: int = 1, quantizer: Optional[IntentQuantizer] = None,
                bases: Optional[torch.Tensor] = None, seq_lens: Optional[torch.Tensor] = None,
                page_tags: Optional[torch.Tensor] = None,
                prec_to_tag: Optional[Mapping[KVPrecision, int]] = None, pad_value: int = -1,
                out: Optional[RoutedPages] = None, row_masks: bool = False) -> RoutedPages:
    """Route every sequence of ``layouts`` and write its page-table rows on the device.

    ``config`` and ``quantizer`` mean what they mean for ``BlockRouter``
    (``quantizer=None`` builds the router's default from ``config``).
    Physical page id = ``bases[b, h]`` + logical page id.  With ``page_tags``
    (uint8, one per physical page) and ``prec_to_tag`` (precision -> decode
    tag), every listed page's tag is written too.  ``row_masks`` also returns,
    per listed page, the bit mask of its rows inside selected blocks (the
    exact-token bounds ``paged_prefill`` takes; page_size <= 64).  Never
    synchronises.
    """
    dev = layouts.scores.device
    _require_cuda(layouts.scores, "layouts.scores")
    q = quantizer or IntentQuantizer(memory_pressure=config.memory_pressure, preserve_recent=config.preserve_recent,
                                     preserve_global=config.preserve_system_prompt)
    B, nb = layouts.batch, layouts.num_blocks
    if nb > N.ROUTE_MAX_BLOCKS:
        raise ValueError(f"{nb} blocks exceed the device router's limit of {N.ROUTE_MAX_BLOCKS}")
    for name in ("start", "end", "policy", "scores"):
        t = getattr(layouts, name)
        if t.device != dev or not t.is_contiguous() or t.dim() != 2:
            raise ValueError(f"layouts.{name} must be a contiguous 2-D tensor on {dev}")
    if layouts.scores.dtype != torch.float64:
        raise ValueError("layouts.scores must be float64")
    shared = layouts.start.shape[0] == 1 and B != 1
    if not shared and layouts.start.shape[0] != B:
        raise ValueError("layout rows must be 1 (shared) or batch")
    if out is None:
        out = RoutedPages(torch.empty((B, table_heads, table_width), dtype=torch.int32, device=dev),
                          torch.empty((B, table_heads), dtype=torch.int32, device=dev),
                          torch.empty(B, dtype=torch.int32, device=dev),
                          torch.empty((B, table_width), dtype=torch.uint8, device=dev))
    if row_masks and out.row_masks is None:
        out.row_masks = torch.empty((B, table_width), dtype=torch.int64, device=dev)
    a = N.RouteArgs()
    a.num_blocks = nb
    keep = []   # temporaries must outlive the launch's argument capture
    if layouts.counts is not None:
        counts = layouts.counts.to(device=dev, dtype=torch.int32).contiguous()
        if counts.numel() != B:
            raise ValueError("layouts.counts must have one entry per sequence")
        keep.append(counts)
        a.block_counts = counts.data_ptr()
    a.block_start, a.block_end = layouts.start.data_ptr(), layouts.end.data_ptr()
    a.block_policy = layouts.policy.data_ptr()
    a.layout_stride = 0 if shared else layouts.start.stride(0)
    a.scores, a.score_stride = layouts.scores.data_ptr(), layouts.scores.stride(0)
    if seq_lens is not None:
        seq_lens = seq_lens.to(device=dev, dtype=torch.int32).contiguous()
        keep.append(seq_lens)
        a.seq_lens = seq_lens.data_ptr()
    a.batch, a.num_table_heads, a.page_size = B, table_heads, page_size
    a.top_k_blocks = config.top_k_blocks
    a.preserve_recent, a.preserve_global = int(bool(q.preserve_recent)), int(bool(q.preserve_global))
    a.score_threshold, a.memory_pressure = float(config.score_threshold), float(q.memory_pressure)
    a.high_score_threshold, a.medium_score_threshold = float(q.high_score_threshold), float(q.medium_score_threshold)
    if bases is not None:
        bases = bases.to(device=dev, dtype=torch.int32).contiguous()
        keep.append(bases)
        a.bases = bases.data_ptr()
    a.table_width, a.pad_value = table_width, pad_value
    a.page_table, a.page_counts = out.page_table.data_ptr(), out.page_counts.data_ptr()
    a.num_selected = out.num_selected.data_ptr()
    a.page_prec = out.page_prec.data_ptr()
    if page_tags is not None:
        if page_tags.dtype != torch.uint8 or page_tags.device != dev:
            raise ValueError("page_tags must be a uint8 tensor on the layouts' device")
        if prec_to_tag is None:
            raise ValueError("page_tags needs prec_to_tag")
        a.page_tags, a.num_tag_pages = page_tags.data_ptr(), page_tags.numel()
        for prec, code in PRECISION_CODES.items():
            a.prec_to_tag[code] = int(prec_to_tag.get(prec, 0))
    if out.row_masks is not None:
        if out.row_masks.dtype != torch.int64 or tuple(out.row_masks.shape) != (B, table_width):
            raise ValueError("row_masks must be int64 [B, table_width]")
        a.row_masks = out.row_masks.data_ptr()
    N.check(N.lib().iak_route_pages(ctypes.byref(a), _stream(dev)), "iak_route_pages")
    return out


def route_layouts(router, layouts: Sequence[BlockLayout], total_tokens: Sequence[int], page_size: int,
                  table_width: int, device, **kwargs) -> RoutedPages:
    """``BlockRouter``-facing form: validate on the host (raising ``ValueError``
    as ``route_layout`` does), encode, and route on ``device``."""
    for layout, n in zip(layouts, total_tokens):
        layout.validate(n)
    batch = encode_layouts(layouts, device)
    seq_lens = torch.tensor(list(total_tokens), dtype=torch.int32).to(device)
    return route_pages(batch, router.config, page_size, table_width, quantizer=router.quantizer,
                       seq_lens=seq_lens, **kwargs)
