"""Semantic layout types (drop-in for the reference's ``block_metadata.py:10-93``).

``BlockPolicy`` values are the member names, ``SemanticBlock`` is a plain
record, and ``BlockLayout.validate`` raises ``ValueError`` on the same
conditions as the reference (empty name, negative start, empty or
out-of-range span, ATTEND without a score, unsorted or overlapping blocks).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from enum import Enum
from typing import Dict, List, Optional


class _NamedEnum(Enum):
    """Enum whose auto values are the member names; str() gives the value."""

    @staticmethod
    def _generate_next_value_(name, start, count, last_values):
        return name

    def __str__(self) -> str:
        return self.value

    def __repr__(self) -> str:
        return f"{type(self).__name__}.{self.value}"


class BlockPolicy(_NamedEnum):
    ALWAYS = "ALWAYS"
    ATTEND = "ATTEND"
    SKIP = "SKIP"
    RECENT = "RECENT"
    GLOBAL = "GLOBAL"


SELECTED_POLICIES = frozenset({BlockPolicy.ALWAYS, BlockPolicy.ATTEND, BlockPolicy.RECENT, BlockPolicy.GLOBAL})


@dataclass
class SemanticBlock:
    name: str
    start: int
    end: int
    policy: BlockPolicy
    score: Optional[float] = None


@dataclass
class BlockLayout:
    blocks: List[SemanticBlock] = field(default_factory=list)

    def validate(self, total_tokens: int) -> None:
        prev: Optional[SemanticBlock] = None
        for i, blk in enumerate(self.blocks):
            if not blk.name:
                raise ValueError(f"Block at index {i} has empty name")
            if blk.start < 0:
                raise ValueError(f"Block '{blk.name}' has start={blk.start} < 0")
            if blk.end <= blk.start:
                raise ValueError(f"Block '{blk.name}' has end={blk.end} <= start={blk.start}")
            if blk.end > total_tokens:
                raise ValueError(f"Block '{blk.name}' has end={blk.end} > total_tokens={total_tokens}")
            if blk.policy == BlockPolicy.ATTEND and blk.score is None:
                raise ValueError(f"Block '{blk.name}' has policy ATTEND but score is None")
            if prev is not None:
                if blk.start < prev.start:
                    raise ValueError(f"Blocks not sorted: '{blk.name}' start={blk.start} "
                                     f"< '{prev.name}' start={prev.start}")
                if blk.start < prev.end:
                    raise ValueError(f"Blocks overlap: '{prev.name}' end={prev.end} "
                                     f"> '{blk.name}' start={blk.start}")
            prev = blk

    def selected_blocks(self) -> List[SemanticBlock]:
        return [b for b in self.blocks if b.policy in SELECTED_POLICIES]

    def selected_token_indices(self) -> List[int]:
        out: List[int] = []
        for b in self.selected_blocks():
            out.extend(range(b.start, b.end))
        return out

    def selected_token_count(self) -> int:
        return sum(b.end - b.start for b in self.selected_blocks())

    def total_token_count(self) -> int:
        return sum(b.end - b.start for b in self.blocks)

    def summary(self) -> Dict[str, int]:
        return {"total_blocks": len(self.blocks), "selected_blocks": len(self.selected_blocks()),
                "total_token_count": self.total_token_count(),
                "selected_token_count": self.selected_token_count()}
