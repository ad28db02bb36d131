"""Oracle attention over selected blocks (numpy).  TEST INFRASTRUCTURE ONLY.

* ``dense_attention`` restates ``reference.py:16-45`` (non-causal):
  ``softmax(q k^T / sqrt(D)) v``.
* ``intent_quant_attention`` restates ``intent_quant_attention.py:20-86``:
  per selected block, fake-quantise the K and V slices with the block's
  precision (``intent_quant.py:229-312``), concatenate the reconstructions in
  block order, then run dense attention.  Zero selected blocks -> zeros
  (``intent_quant_attention.py:41-45``).

Attention is evaluated in float64 on the float32 reconstructions; the
reference's float32 evaluation agrees to ~1e-6 (pinned by the golden tests).
"""

from __future__ import annotations

from typing import Iterable, Optional, Sequence, Tuple

import numpy as np

from .quant import fake_quantize


def softmax_lastdim(s: np.ndarray) -> np.ndarray:
    m = s.max(axis=-1, keepdims=True)
    e = np.exp(s - m)
    return e / e.sum(axis=-1, keepdims=True)


def dense_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                    sm_scale: Optional[float] = None) -> np.ndarray:
    """[..., Lq, D] x [..., Lk, D] x [..., Lk, Dv] -> [..., Lq, Dv] (float64)."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    scale = 1.0 / np.sqrt(q.shape[-1]) if sm_scale is None else float(sm_scale)
    s = np.matmul(q, np.swapaxes(k, -1, -2)) * scale
    return np.matmul(softmax_lastdim(s), v)


def intent_quant_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                           blocks: Iterable[Tuple[int, int, str]]) -> np.ndarray:
    """Selected-block fake-quant attention.

    ``blocks``: (start, end, precision) for each SELECTED block, in layout
    order.  q [B, H, Lq, D], k/v [B, H, T, D] (float32).  GQA callers pass
    q viewed as [B, Hkv, G*Lq, D].
    """
    k_parts, v_parts = [], []
    for start, end, prec in blocks:
        k_parts.append(fake_quantize(np.ascontiguousarray(k[..., start:end, :]), prec)["recon"])
        v_parts.append(fake_quantize(np.ascontiguousarray(v[..., start:end, :]), prec)["recon"])
    if not k_parts:
        return np.zeros(q.shape, dtype=np.float64)
    kk = np.concatenate(k_parts, axis=-2)
    vv = np.concatenate(v_parts, axis=-2)
    return dense_attention(q, kk, vv)
