"""Precision policy (drop-in for the reference's ``intent_quant.py:14-213``).

``IntentQuantizer.assign_block_precision`` maps a block's policy, score and
the memory pressure to a ``KVPrecision`` exactly as the reference's decision
table (``intent_quant.py:77-131``).  The reference's CPU fake quantisation
(``fake_quantize_tensor``) is not part of this package: real page formats are
produced on the GPU by ``PagePool.quantize_`` (``iak_quantize_pages``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Dict, List

from .block_metadata import BlockLayout, BlockPolicy, SemanticBlock, _NamedEnum


class KVPrecision(_NamedEnum):
    FP16 = "FP16"
    FP8 = "FP8"
    INT8 = "INT8"
    INT4 = "INT4"
    INT4_RESIDUAL = "INT4_RESIDUAL"
    SKIP = "SKIP"


_BYTES_PER_VALUE: Dict[KVPrecision, float] = {
    KVPrecision.FP16: 2.0, KVPrecision.FP8: 1.0, KVPrecision.INT8: 1.0,
    KVPrecision.INT4: 0.5, KVPrecision.INT4_RESIDUAL: 1.0, KVPrecision.SKIP: 0.0,
}


@dataclass
class QuantPolicy:
    precision: KVPrecision
    reason: str = ""
    estimated_bytes_per_value: float = field(init=False)
    requires_scale: bool = field(init=False)
    uses_residual: bool = field(init=False)

    def __post_init__(self) -> None:
        self.estimated_bytes_per_value = _BYTES_PER_VALUE[self.precision]
        self.requires_scale = self.precision in (KVPrecision.INT8, KVPrecision.INT4, KVPrecision.INT4_RESIDUAL)
        self.uses_residual = self.precision == KVPrecision.INT4_RESIDUAL


class IntentQuantizer:
    """Per-block precision from policy, score, recency and memory pressure."""

    def __init__(self, memory_pressure: float = 0.0, preserve_recent: bool = True, preserve_global: bool = True,
                 high_score_threshold: float = 0.75, medium_score_threshold: float = 0.40) -> None:
        if not 0.0 <= memory_pressure <= 1.0:
            raise ValueError(f"memory_pressure must be in [0, 1], got {memory_pressure}")
        self.memory_pressure = memory_pressure
        self.preserve_recent = preserve_recent
        self.preserve_global = preserve_global
        self.high_score_threshold = high_score_threshold
        self.medium_score_threshold = medium_score_threshold

    # decision tables, evaluated top to bottom: (predicate on pressure, precision, reason)
    def _pinned(self, policy: BlockPolicy, mp: float) -> QuantPolicy:
        if policy == BlockPolicy.GLOBAL and self.preserve_global:
            if mp > 0.8:
                return QuantPolicy(KVPrecision.INT8, "global, extreme pressure")
            return QuantPolicy(KVPrecision.FP16, "global, preserved")
        for limit, prec, why in ((0.9, KVPrecision.INT8, "always, extreme pressure"),
                                 (0.7, KVPrecision.FP8, "always, high pressure")):
            if mp > limit:
                return QuantPolicy(prec, why)
        return QuantPolicy(KVPrecision.FP16, "always, full precision")

    def _recent(self, mp: float) -> QuantPolicy:
        if self.preserve_recent:
            if mp > 0.8:
                return QuantPolicy(KVPrecision.INT8, "recent, extreme pressure")
            return QuantPolicy(KVPrecision.FP8, "recent, moderate pressure" if mp > 0.5 else "recent, preserved")
        if mp > 0.6:
            return QuantPolicy(KVPrecision.INT4_RESIDUAL, "recent, high pressure, not preserved")
        return QuantPolicy(KVPrecision.INT8, "recent, not preserved")

    def _attend(self, score, mp: float) -> QuantPolicy:
        if score is None:
            return QuantPolicy(KVPrecision.INT8 if mp > 0.5 else KVPrecision.FP16, "attend, no score")
        if score >= self.high_score_threshold:
            if mp > 0.8:
                return QuantPolicy(KVPrecision.INT8, "high-score, extreme pressure")
            if mp > 0.5:
                return QuantPolicy(KVPrecision.FP8, "high-score, moderate pressure")
            return QuantPolicy(KVPrecision.INT8, "high-score attend")
        if score >= self.medium_score_threshold:
            if mp > 0.6:
                return QuantPolicy(KVPrecision.INT4, "medium-score, high pressure")
            return QuantPolicy(KVPrecision.INT4_RESIDUAL, "medium-score attend")
        if mp > 0.3:
            return QuantPolicy(KVPrecision.SKIP, "low-score, pressure")
        return QuantPolicy(KVPrecision.INT4, "low-score attend")

    def assign_block_precision(self, block: SemanticBlock) -> QuantPolicy:
        mp = self.memory_pressure
        pol = block.policy
        if pol in (BlockPolicy.ALWAYS, BlockPolicy.GLOBAL):
            return self._pinned(pol, mp)
        if pol == BlockPolicy.RECENT:
            return self._recent(mp)
        if pol == BlockPolicy.ATTEND:
            return self._attend(block.score, mp)
        if pol == BlockPolicy.SKIP:
            return QuantPolicy(KVPrecision.SKIP, "skipped block")
        return QuantPolicy(KVPrecision.FP16, "default")

    def assign_layout_precision(self, layout: BlockLayout) -> Dict[str, QuantPolicy]:
        return {b.name: self.assign_block_precision(b) for b in layout.blocks}

    def estimate_layout_bytes(self, layout: BlockLayout, heads: int, head_dim: int, kv_tensors: int = 2) -> Dict[str, Any]:
        pol = self.assign_layout_precision(layout)
        dense = 0
        quant = 0.0
        dist: Dict[str, int] = {}
        fp16_tokens = 0
        for b in layout.blocks:
            p = pol[b.name]
            n = b.end - b.start
            dense += kv_tensors * n * head_dim * 2
            quant += kv_tensors * n * head_dim * p.estimated_bytes_per_value
            dist[p.precision.value] = dist.get(p.precision.value, 0) + n
            if p.precision == KVPrecision.FP16:
                fp16_tokens += n
        saved_pct = (1.0 - quant / dense) * 100.0 if dense > 0 else 0.0
        return {"total_tokens": layout.total_token_count(), "dense_fp16_bytes": dense,
                "intent_quant_bytes": int(round(quant)), "bytes_saved": int(round(dense - quant)),
                "bytes_saved_pct": round(saved_pct, 2), "precision_distribution": dist,
                "critical_full_precision_tokens": fp16_tokens}

    def summary_table(self, layout: BlockLayout, heads: int, head_dim: int) -> List[Dict[str, Any]]:
        pol = self.assign_layout_precision(layout)
        rows = []
        for b in layout.blocks:
            p = pol[b.name]
            n = b.end - b.start
            rows.append({"block": b.name, "policy": b.policy.value, "score": b.score, "tokens": n,
                         "precision": p.precision.value, "reason": p.reason, "dense_fp16_bytes": 2 * n * head_dim * 2,
                         "quant_bytes": int(round(2 * n * head_dim * p.estimated_bytes_per_value))})
        return rows
