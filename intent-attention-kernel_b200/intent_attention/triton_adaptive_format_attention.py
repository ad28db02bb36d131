"""Adaptive-format decode (drop-in for ``triton_adaptive_format_attention.py``).

``AdaptivePageFormat`` (``:33-38``), ``AdaptiveFormatKernelConfig``
(``:42-50``), ``adaptive_format_decode_attention_triton`` (``:237-329``) and
``make_adaptive_page_tables`` (``:420-468``) keep the reference's contract:
every table slot is visited, ``-1`` marks an unused slot, FP16 pages are
read directly, INT8 pages as ``code * scale[page]``, SKIP pages are skipped and
SPARSE pages contribute nothing, which is what the reference kernel computes
for them (it masks SPARSE tokens to -inf, ``:204-211``).  The sparse buffers
are accepted for signature compatibility.  The decode runs the sm_100a kernel
of libiak_b200.so; CPU tensors raise.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum
from typing import Optional, Tuple

import torch

from . import _native as N
from .paged import PagePool, make_tag_map, paged_decode
from .triton_intent_quant_attention import make_page_tables_from_selected_pages


class AdaptivePageFormat(IntEnum):
    """Storage format tag for one physical KV page."""

    FP16 = 0
    INT8 = 1
    SPARSE = 2
    SKIP = 3


@dataclass(frozen=True)
class AdaptiveFormatKernelConfig:
    page_size: int = 16
    head_dim: int = 64
    max_selected_pages: int = 64
    block_d: int = 64
    sparse_max_nnz: int = 256


_TAG_MAP = make_tag_map({0: "F16", 1: "INT8", 2: "SPARSE", 3: "SKIP"})


def is_triton_available() -> bool:
    """True when the GPU kernel backend (libiak_b200.so) is loadable."""
    return N.available()


def is_cuda_available() -> bool:
    return torch.cuda.is_available()


def _require_triton_cuda() -> None:
    if not is_triton_available():
        raise RuntimeError("Triton is not installed: the adaptive-format GPU kernel library (libiak_b200.so) "
                           "is not built.")
    if not is_cuda_available():
        raise RuntimeError("CUDA is not available.  This build has no CPU path for the decode kernels.")


def adaptive_format_decode_attention_triton(
    q: torch.Tensor, page_ids: torch.Tensor, page_formats: torch.Tensor, fp16_k_pages: torch.Tensor,
    fp16_v_pages: torch.Tensor, int8_k_pages: Optional[torch.Tensor] = None, int8_v_pages: Optional[torch.Tensor] = None,
    int8_k_scales: Optional[torch.Tensor] = None, int8_v_scales: Optional[torch.Tensor] = None,
    sparse_k_indices: Optional[torch.Tensor] = None, sparse_k_values: Optional[torch.Tensor] = None,
    sparse_v_indices: Optional[torch.Tensor] = None, sparse_v_values: Optional[torch.Tensor] = None,
    sparse_nnz: Optional[torch.Tensor] = None, *, config: Optional[AdaptiveFormatKernelConfig] = None,
    out: Optional[torch.Tensor] = None, num_splits: int = 0,
) -> torch.Tensor:
    """Adaptive-format decode over -1 padded page_ids [B, H, W] -> [B, H, D] in q's dtype."""
    _require_triton_cuda()
    cfg = config or AdaptiveFormatKernelConfig()
    if not q.is_cuda:
        raise ValueError("q must be a CUDA tensor")
    B, H, D = q.shape
    if cfg.block_d < D:
        raise ValueError("block_d must be >= D")
    if page_ids.ndim != 3 or page_ids.shape[0] != B or H % page_ids.shape[1]:
        raise ValueError(f"page_ids must be [B, H, W] matching q, got {tuple(page_ids.shape)}")
    NP, PS = fp16_k_pages.shape[0], fp16_k_pages.shape[1]
    pool = PagePool(NP, PS, D, "page")
    pool.k_f16, pool.v_f16 = fp16_k_pages.to(torch.float16).contiguous(), fp16_v_pages.to(torch.float16).contiguous()
    if int8_k_pages is None or int8_v_pages is None:
        pool.k_i8 = torch.zeros((NP, PS, D), dtype=torch.int8, device=q.device)
        pool.v_i8 = pool.k_i8
    else:
        pool.k_i8, pool.v_i8 = int8_k_pages.to(torch.int8).contiguous(), int8_v_pages.to(torch.int8).contiguous()
    ones = torch.ones((NP, 1), dtype=torch.float32, device=q.device)
    pool.k_scale = ones if int8_k_scales is None else int8_k_scales.to(torch.float32).reshape(NP, 1).contiguous()
    pool.v_scale = ones if int8_v_scales is None else int8_v_scales.to(torch.float32).reshape(NP, 1).contiguous()
    tags = page_formats if page_formats.dtype in (torch.uint8, torch.int32) else page_formats.to(torch.int32)
    return paged_decode(q, pool, page_ids, None, tags.contiguous(), _TAG_MAP, N.FMT_SKIP, out=out,
                        out_dtype=q.dtype, num_splits=num_splits)


def make_adaptive_page_tables(selected_pages: torch.Tensor, batch: int, heads: int,
                              max_selected_pages: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Same contract as the reference helper (-1 padded page_ids, counts)."""
    if selected_pages.ndim not in (1, 3):
        raise ValueError("selected_pages must have shape [N] or [B, H, N]")
    try:
        return make_page_tables_from_selected_pages(selected_pages, batch, heads, max_selected_pages)
    except ValueError as e:
        if "length exceeds" in str(e):
            raise ValueError("selected_pages exceeds max_selected_pages") from None
        raise
