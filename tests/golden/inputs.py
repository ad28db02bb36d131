"""Seeded numpy input generators shared by the golden-vector script and the tests.

Inputs are regenerated from seeds instead of being stored, so the committed
fixtures hold only the reference's outputs.  numpy's PCG64 stream is stable
across platforms and numpy versions for ``standard_normal`` / ``integers``.
"""

from __future__ import annotations

import numpy as np


def rng(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def normal(seed: int, shape, outlier_frac: float = 0.0, outlier_mult: float = 8.0,
           std: float = 1.0) -> np.ndarray:
    """float32 N(0, std^2) with an optional Bernoulli(outlier_frac) x outlier_mult."""
    g = rng(seed)
    x = g.standard_normal(shape).astype(np.float32) * np.float32(std)
    if outlier_frac > 0:
        mask = g.random(shape) < outlier_frac
        x = np.where(mask, x * np.float32(outlier_mult), x).astype(np.float32)
    return x


# Layout used by the reference's own end-to-end router test (448 tokens).
E2E_LAYOUT = [
    ("system", 0, 64, "ALWAYS", None),
    ("doc_high", 64, 192, "ATTEND", 0.85),
    ("doc_low", 192, 320, "ATTEND", 0.15),
    ("recent", 320, 384, "RECENT", None),
    ("unused", 384, 448, "SKIP", None),
]

# Layout used by the reference's oracle tests (64 tokens).
BASIC_LAYOUT = [
    ("always", 0, 16, "ALWAYS", None),
    ("attend_high", 16, 32, "ATTEND", 0.9),
    ("attend_low", 32, 48, "ATTEND", 0.3),
    ("skip", 48, 64, "SKIP", None),
]

# BASELINE config 1 (CPU-runnable): 1440 tokens, page 16.
C1_LAYOUT = [
    ("system", 0, 128, "ALWAYS", None),
    ("retrieved", 128, 1024, "ATTEND", 0.9),
    ("tool_output", 1024, 1280, "SKIP", None),
    ("recent", 1280, 1440, "RECENT", None),
]


def many_attend_layout(seed: int, n_blocks: int = 24, block_tokens: int = 64,
                       head: int = 128, tail: int = 128):
    """ALWAYS head, n ATTEND blocks with seeded scores, a SKIP block, RECENT tail."""
    g = rng(seed)
    blocks = [("sys", 0, head, "ALWAYS", None)]
    cur = head
    for i in range(n_blocks):
        blocks.append((f"doc{i}", cur, cur + block_tokens, "ATTEND", float(np.round(g.random(), 4))))
        cur += block_tokens
    blocks.append(("tool", cur, cur + 96, "SKIP", float(np.round(g.random(), 4))))
    cur += 96
    blocks.append(("recent", cur, cur + tail, "RECENT", None))
    return blocks


# Layouts with block boundaries inside pages (prefill parity cases).
PREFILL_PARTIAL_LAYOUT = [
    ("sys", 0, 13, "ALWAYS", None),
    ("tool", 13, 50, "SKIP", None),
    ("doc", 50, 77, "ATTEND", 0.9),
    ("doc_low", 77, 85, "ATTEND", 0.2),
    ("recent", 85, 100, "RECENT", None),
]
# The first 32 tokens are skipped: causal queries 0..31 see no key.
PREFILL_GAP_LAYOUT = [
    ("skipped", 0, 32, "SKIP", None),
    ("doc", 32, 80, "ATTEND", 0.7),
    ("recent", 80, 96, "RECENT", None),
]
