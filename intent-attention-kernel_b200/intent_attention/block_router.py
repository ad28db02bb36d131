"""Block router (drop-in for the reference's ``block_router.py:18-421``).

Routing decisions, precisions, reasons and the kernel metadata dict are the
same as the reference's (pinned by ``tests/test_router_golden.py`` against the
reference's own outputs).  What changes is cost: the reference builds page
lists with a Python loop over every selected TOKEN (``block_router.py:283-296,
405-410``); here each block contributes its page RANGE, so
``selected_page_ids`` / ``routing_to_kernel_metadata`` are O(blocks + pages).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import torch

from .block_metadata import BlockLayout, BlockPolicy, SemanticBlock, _NamedEnum
from .intent_quant import _BYTES_PER_VALUE, IntentQuantizer, KVPrecision


class BlockDecision(_NamedEnum):
    SELECT = "SELECT"
    SKIP = "SKIP"
    PREFETCH = "PREFETCH"
    QUANTIZE = "QUANTIZE"
    PIN_HIGH_PRECISION = "PIN_HIGH_PRECISION"


_SELECTED = (BlockDecision.SELECT, BlockDecision.PIN_HIGH_PRECISION, BlockDecision.QUANTIZE)


@dataclass
class RoutedBlock:
    name: str
    start: int
    end: int
    policy: BlockPolicy
    score: Optional[float]
    decision: BlockDecision
    precision: KVPrecision
    reason: str


@dataclass
class RouterConfig:
    top_k_blocks: int = 8
    score_threshold: float = 0.35
    recent_window_tokens: int = 2048
    memory_pressure: float = 0.5
    prefetch_top_k: int = 4
    preserve_system_prompt: bool = True
    preserve_recent: bool = True


def compute_block_scores(query_vector: torch.Tensor, block_representations: Dict[str, torch.Tensor]) -> Dict[str, float]:
    """Cosine similarity of the query with each block representation, clamped to [0, 1]."""
    q = query_vector.flatten().float()
    qn = q / (q.norm(p=2) + 1e-10)
    out: Dict[str, float] = {}
    for name, rep in block_representations.items():
        r = rep.flatten().float()
        sim = float(torch.dot(qn, r / (r.norm(p=2) + 1e-10)).item())
        out[name] = min(1.0, max(0.0, sim))
    return out


def _pages_of(start: int, end: int, page_size: int) -> range:
    """Pages touched by tokens [start, end)."""
    return range(start // page_size, (end - 1) // page_size + 1)


class BlockRouter:
    """Converts semantic blocks into selected pages, precisions, prefetch hints and reasons."""

    def __init__(self, config: RouterConfig, quantizer: Optional[IntentQuantizer] = None) -> None:
        self.config = config
        self.quantizer = quantizer or IntentQuantizer(memory_pressure=config.memory_pressure,
                                                      preserve_recent=config.preserve_recent,
                                                      preserve_global=config.preserve_system_prompt)

    def _routed(self, b: SemanticBlock, decision: BlockDecision, precision: KVPrecision, reason: str) -> RoutedBlock:
        return RoutedBlock(b.name, b.start, b.end, b.policy, b.score, decision, precision, reason)

    def route_layout(self, layout: BlockLayout, total_tokens: int, query_vector: Optional[torch.Tensor] = None,
                     block_representations: Optional[Dict[str, torch.Tensor]] = None) -> List[RoutedBlock]:
        layout.validate(total_tokens)
        cfg = self.config
        qs = compute_block_scores(query_vector, block_representations) \
            if query_vector is not None and block_representations is not None else {}
        pinned = (BlockPolicy.ALWAYS, BlockPolicy.GLOBAL, BlockPolicy.RECENT)
        high = [b for b in layout.blocks if b.policy in pinned]
        attend = []
        for b in layout.blocks:
            if b.policy == BlockPolicy.ATTEND:
                if b.score is None and b.name in qs:
                    b = SemanticBlock(b.name, b.start, b.end, b.policy, qs[b.name])
                attend.append(b)
        others = [b for b in layout.blocks if b.policy not in pinned and b.policy != BlockPolicy.ATTEND]
        # stable descending sort by score; ATTEND blocks without a score are dropped
        ranked = sorted((b for b in attend if b.score is not None), key=lambda b: b.score or 0.0, reverse=True)
        top, rest = ranked[:cfg.top_k_blocks], ranked[cfg.top_k_blocks:]

        routed: List[RoutedBlock] = []
        assign = lambda b: self.quantizer.assign_block_precision(b).precision  # noqa: E731
        for b in high:
            if b.policy in (BlockPolicy.ALWAYS, BlockPolicy.GLOBAL):
                routed.append(self._routed(b, BlockDecision.PIN_HIGH_PRECISION, assign(b),
                                           f"{b.policy.value} block, always selected"))
            else:
                routed.append(self._routed(b, BlockDecision.SELECT, assign(b), "recent context, always selected"))
        for b in top:
            prec = assign(b)
            if prec == KVPrecision.SKIP:
                routed.append(self._routed(b, BlockDecision.SKIP, prec, "low-score attend, skipped under memory pressure"))
            else:
                decision = BlockDecision.SELECT if prec == KVPrecision.FP16 else BlockDecision.QUANTIZE
                routed.append(self._routed(b, decision, prec,
                                           f"attend score={b.score:.3f} >= threshold={cfg.score_threshold}"))
        for b in rest:
            why = "below top-k"
            if cfg.memory_pressure > 0.5 and b.score is not None and b.score < cfg.score_threshold:
                why += ", low score with pressure"
            routed.append(self._routed(b, BlockDecision.SKIP, assign(b), why))
        for b in others:
            prec = assign(b)
            if b.score is not None and b.score >= cfg.score_threshold:
                routed.append(self._routed(b, BlockDecision.SELECT, prec,
                                           "SKIP block with unexpectedly high score, selected"))
            else:
                routed.append(self._routed(b, BlockDecision.SKIP, KVPrecision.SKIP, "SKIP block, not selected"))
        return routed

    def selected_blocks(self, routed_blocks: List[RoutedBlock]) -> List[RoutedBlock]:
        return [b for b in routed_blocks if b.decision in _SELECTED]

    def skipped_blocks(self, routed_blocks: List[RoutedBlock]) -> List[RoutedBlock]:
        return [b for b in routed_blocks if b.decision == BlockDecision.SKIP]

    def selected_token_indices(self, routed_blocks: List[RoutedBlock]) -> List[int]:
        out: List[int] = []
        for b in self.selected_blocks(routed_blocks):
            out.extend(range(b.start, b.end))
        return out

    def selected_page_ids(self, routed_blocks: List[RoutedBlock], page_size: int) -> List[int]:
        """Order-preserving, de-duplicated pages of the selected blocks."""
        seen = set()
        ids: List[int] = []
        for b in self.selected_blocks(routed_blocks):
            if b.end <= b.start:
                continue
            for pid in _pages_of(b.start, b.end, page_size):
                if pid not in seen:
                    seen.add(pid)
                    ids.append(pid)
        return ids

    def prefetch_page_ids(self, routed_blocks: List[RoutedBlock], page_size: int) -> List[int]:
        cfg = self.config
        best: Dict[int, float] = {}

        def offer(pid: int, score: float) -> None:
            if pid not in best or score > best[pid]:
                best[pid] = score

        for b in routed_blocks:
            if b.decision == BlockDecision.SKIP and b.score is not None and b.score >= cfg.score_threshold \
                    and b.end > b.start:
                for pid in _pages_of(b.start, b.end, page_size):
                    offer(pid, b.score)
        for b in self.selected_blocks(routed_blocks):
            left = max(0, b.start // page_size - 1)
            right = (b.end + page_size - 1) // page_size
            for pid in range(left, right + 1):
                offer(pid, 1.0)
        ranked = sorted(best.items(), key=lambda kv: (-kv[1], kv[0]))
        return [pid for pid, _ in ranked][:cfg.prefetch_top_k]

    def routing_summary(self, routed_blocks: List[RoutedBlock]) -> Dict:
        """Decision summary; byte estimates assume head_dim 64, K+V, fp16 baseline."""
        sel = self.selected_blocks(routed_blocks)
        total = sum(b.end - b.start for b in routed_blocks)
        sel_tok = sum(b.end - b.start for b in sel)
        dist: Dict[str, int] = {}
        fp16 = 0
        quant = 0.0
        for b in sel:
            n = b.end - b.start
            fp16 += 2 * n * 64 * 2
            quant += 2 * n * 64 * _BYTES_PER_VALUE.get(b.precision, 2.0)
            dist[b.precision.value] = dist.get(b.precision.value, 0) + n
        saved = (1.0 - quant / max(fp16, 1)) * 100.0 if fp16 > 0 else 0.0
        return {"total_blocks": len(routed_blocks), "selected_blocks": len(sel),
                "skipped_blocks": len(self.skipped_blocks(routed_blocks)), "total_tokens": total,
                "selected_tokens": sel_tok, "skipped_tokens": total - sel_tok,
                "estimated_fp16_mb": round(fp16 / (1024 * 1024), 3),
                "estimated_quant_mb": round(quant / (1024 * 1024), 3),
                "bytes_saved_pct": round(saved, 2), "precision_distribution": dist}


def routing_to_kernel_metadata(routed_blocks: List[RoutedBlock], page_size: int) -> Dict:
    """Flat metadata for the decode kernels (same keys and values as the reference).

    As in the reference, prefetch ids use a default ``RouterConfig`` (not the
    caller's), and a page shared by two selected blocks takes the precision of
    the first block that touches it.
    """
    router = BlockRouter(RouterConfig())
    sel = router.selected_blocks(routed_blocks)
    prec_by_page: Dict[int, KVPrecision] = {}
    for b in sel:
        if b.end <= b.start:
            continue
        for pid in _pages_of(b.start, b.end, page_size):
            prec_by_page.setdefault(pid, b.precision)
    return {
        "selected_page_ids": router.selected_page_ids(routed_blocks, page_size),
        "prefetch_page_ids": router.prefetch_page_ids(routed_blocks, page_size),
        "block_precision_by_page": {str(k): v.value for k, v in sorted(prec_by_page.items())},
        "selected_block_names": [b.name for b in sel],
        "skipped_block_names": [b.name for b in router.skipped_blocks(routed_blocks)],
        "reasons_by_block": {b.name: b.reason for b in routed_blocks},
    }
