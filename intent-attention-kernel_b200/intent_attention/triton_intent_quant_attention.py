"""Six-tag IntentQuant decode (drop-in for ``triton_intent_quant_attention.py``).

The module keeps the reference's names and contracts (``TritonKVPrecision``
``:40-48``, ``IntentQuantKernelConfig`` ``:51-58``, the validation errors of
``:93-123`` and ``:396-430``, the page-table helpers ``:126-203`` /
``:499-536``, ``fake_int8_pages_from_fp16`` ``:460-496``) while the decode
itself is the sm_100a kernel of libiak_b200.so.

Tag semantics.  Called exactly like the reference, FP8 / INT4 /
INT4_RESIDUAL tags are read through the INT8 buffers as ``code * scale``,
which is what the reference kernel does (``:250-253, :302-318``).  When the
real page pools are passed as keyword arguments (``k_pages_fp8``,
``k_pages_int4``, ``k_pages_int4r`` ... ), those tags read the real FP8-e4m3 /
packed INT4 / INT4+residual formats instead.  SKIP pages and -1 slots
contribute nothing; unlike the reference kernel, an invalid FIRST slot does
not zero the head (the reference evaluates exp(-inf - -inf) there).
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum
from typing import Optional, Tuple

import torch

from . import _native as N
from .paged import PagePool, make_tag_map, pack_metadata, paged_decode


class TritonKVPrecision(IntEnum):
    """Integer precision tags passed to the decode kernel."""

    FP16 = 0
    FP8 = 1
    INT8 = 2
    INT4 = 3
    INT4_RESIDUAL = 4
    SKIP = 5


@dataclass(frozen=True)
class IntentQuantKernelConfig:
    page_size: int = 16
    head_dim: int = 64
    max_selected_pages: int = 64
    block_d: int = 64


def is_triton_available() -> bool:
    """True when the GPU kernel backend (libiak_b200.so) is loadable."""
    return N.available()


def is_cuda_available() -> bool:
    return torch.cuda.is_available()


def _require_triton_cuda() -> None:
    if not is_triton_available():
        raise RuntimeError("Triton is not installed: the IntentQuant GPU kernel library (libiak_b200.so) "
                           "is not built; run intent-attention-kernel_b200/build.py.")
    if not is_cuda_available():
        raise RuntimeError("CUDA is not available. The IntentQuant decode kernel requires an NVIDIA GPU.")


def _validate_decode_inputs(q, page_ids, page_count, page_precision, out) -> None:
    if q.ndim != 3:
        raise ValueError(f"q must have shape [B, H, D], got {tuple(q.shape)}")
    if page_ids.ndim != 3:
        raise ValueError(f"page_ids must have shape [B, H, max_selected_pages], got {tuple(page_ids.shape)}")
    if page_count.ndim != 2:
        raise ValueError(f"page_count must have shape [B, H], got {tuple(page_count.shape)}")
    if page_precision.ndim != 1:
        raise ValueError(f"page_precision must have shape [num_pages], got {tuple(page_precision.shape)}")
    if page_ids.shape[0] != q.shape[0] or q.shape[1] % page_ids.shape[1]:
        raise ValueError("page_ids batch/head dimensions must match q")
    if page_count.shape[0] != page_ids.shape[0] or page_count.shape[1] != page_ids.shape[1]:
        raise ValueError("page_count batch/head dimensions must match q")
    if out is not None and out.shape != q.shape:
        raise ValueError(f"out must have shape {tuple(q.shape)}, got {tuple(out.shape)}")


def make_page_tables_from_selected_pages(selected_pages: torch.Tensor, batch: int, heads: int,
                                         max_selected_pages: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """[N] (shared) or [B, H, N] selected pages -> (-1 padded page_ids [B, H, W], page_count [B, H])."""
    dev = selected_pages.device
    if selected_pages.ndim == 1:
        n = selected_pages.numel()
        width = max_selected_pages or n
        if n > width:
            raise ValueError("selected_pages length exceeds max_selected_pages")
        if dev.type == "cuda" and n > 0:
            return pack_metadata(selected_pages, batch, heads, width, pad_value=-1)
        ids = torch.full((batch, heads, width), -1, dtype=torch.int32, device=dev)
        ids[:, :, :n] = selected_pages.to(torch.int32).view(1, 1, n)
        return ids, torch.full((batch, heads), n, dtype=torch.int32, device=dev)
    if selected_pages.ndim == 3:
        if selected_pages.shape[0] != batch or selected_pages.shape[1] != heads:
            raise ValueError("selected_pages [B, H, N] must match batch and heads")
        n = selected_pages.shape[2]
        width = max_selected_pages or n
        if n > width:
            raise ValueError("selected_pages width exceeds max_selected_pages")
        ids = torch.full((batch, heads, width), -1, dtype=torch.int32, device=dev)
        ids[:, :, :n] = selected_pages.to(torch.int32)
        return ids, torch.full((batch, heads), n, dtype=torch.int32, device=dev)
    raise ValueError("selected_pages must have shape [N] or [B, H, N]")


def intent_quant_decode_attention_triton(
    q: torch.Tensor, k_pages_fp16: torch.Tensor, v_pages_fp16: torch.Tensor, k_pages_i8: torch.Tensor,
    v_pages_i8: torch.Tensor, k_i8_scales: torch.Tensor, v_i8_scales: torch.Tensor, page_ids: torch.Tensor,
    page_count: torch.Tensor, page_precision: torch.Tensor, *, config: Optional[IntentQuantKernelConfig] = None,
    out: Optional[torch.Tensor] = None,
    k_pages_fp8: Optional[torch.Tensor] = None, v_pages_fp8: Optional[torch.Tensor] = None,
    k_pages_int4: Optional[torch.Tensor] = None, v_pages_int4: Optional[torch.Tensor] = None,
    k_pages_int4r: Optional[torch.Tensor] = None, v_pages_int4r: Optional[torch.Tensor] = None,
    k_res_scales: Optional[torch.Tensor] = None, v_res_scales: Optional[torch.Tensor] = None,
    scale_mode: str = "page", sm_scale: Optional[float] = None, num_splits: int = 0,
) -> torch.Tensor:
    """Single-token decode over selected pages -> [B, H, D] in q's dtype.

    ``page_ids`` may also be [B, Hkv, W] with H a multiple of Hkv (grouped-query
    attention: H/Hkv query heads share one page list).  Keyword-only
    extensions: real FP8 / INT4 / INT4_RESIDUAL pools (with
    ``k/v_res_scales`` for the residual), ``scale_mode`` ("page", "group32",
    "channel"; scales then are [NP, n_scales]), ``sm_scale``, ``num_splits``.
    """
    _require_triton_cuda()
    cfg = config or IntentQuantKernelConfig()
    _validate_decode_inputs(q, page_ids, page_count, page_precision, out)
    if not q.is_cuda:
        raise ValueError("q must be a CUDA tensor")
    bsz, heads, dim = q.shape
    if dim != cfg.head_dim:
        raise ValueError(f"q head_dim={dim} does not match config.head_dim={cfg.head_dim}")
    if cfg.block_d < dim:
        raise ValueError("This prototype expects block_d >= head_dim so one program handles the full head.")
    if k_pages_fp16.shape != v_pages_fp16.shape:
        raise ValueError("k_pages_fp16 and v_pages_fp16 must have the same shape")
    if k_pages_i8.shape != v_pages_i8.shape:
        raise ValueError("k_pages_i8 and v_pages_i8 must have the same shape")
    if k_pages_fp16.ndim != 3:
        raise ValueError("page tensors must have shape [num_pages, page_size, D]")
    if k_pages_fp16.shape[1] != cfg.page_size:
        raise ValueError("page_size mismatch")
    if k_pages_fp16.shape[2] != dim:
        raise ValueError("page head_dim mismatch")
    if page_ids.shape[2] != cfg.max_selected_pages:
        raise ValueError("page_ids width must match config.max_selected_pages")
    dev = q.device
    NP = k_pages_fp16.shape[0]
    pool = PagePool(NP, cfg.page_size, dim, scale_mode)
    pool.k_f16, pool.v_f16 = k_pages_fp16.to(torch.float16).contiguous(), v_pages_fp16.to(torch.float16).contiguous()
    pool.k_i8, pool.v_i8 = k_pages_i8.contiguous(), v_pages_i8.contiguous()
    ns = {"page": 1, "group32": dim // 32, "channel": dim}[scale_mode]
    pool.k_scale = k_i8_scales.to(torch.float32).reshape(NP, ns).contiguous()
    pool.v_scale = v_i8_scales.to(torch.float32).reshape(NP, ns).contiguous()
    mapping = {0: "F16", 1: "INT8", 2: "INT8", 3: "INT8", 4: "INT8", 5: "SKIP"}
    default = N.FMT_INT8
    if k_pages_fp8 is not None:
        pool.k_fp8, pool.v_fp8 = k_pages_fp8.view(torch.uint8).contiguous(), v_pages_fp8.view(torch.uint8).contiguous()
        mapping[1] = "FP8"
    if k_pages_int4 is not None:
        pool.k_i4, pool.v_i4 = k_pages_int4.contiguous(), v_pages_int4.contiguous()
        mapping[3] = "INT4"
    if k_pages_int4r is not None:
        if k_pages_int4 is None or k_res_scales is None or v_res_scales is None:
            raise ValueError("INT4_RESIDUAL pages need k/v_pages_int4 (base), k/v_pages_int4r and k/v_res_scales")
        pool.k_i4r, pool.v_i4r = k_pages_int4r.contiguous(), v_pages_int4r.contiguous()
        pool.k_res_scale = k_res_scales.to(torch.float32).reshape(NP, ns).contiguous()
        pool.v_res_scale = v_res_scales.to(torch.float32).reshape(NP, ns).contiguous()
        mapping[4] = "INT4R"
    tags = page_precision if page_precision.dtype in (torch.uint8, torch.int32) else page_precision.to(torch.int32)
    res = paged_decode(q, pool, page_ids, page_count, tags.contiguous(), make_tag_map(mapping), default,
                       sm_scale=sm_scale, out=out, out_dtype=q.dtype, num_splits=num_splits)
    return res


def fake_int8_pages_from_fp16(pages: torch.Tensor, *, eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-page symmetric INT8 (``:460-496``): fp32 scale = max(absmax, eps)/127, codes clamp(round(x/s), +-127)."""
    if pages.ndim != 3:
        raise ValueError("pages must have shape [num_pages, page_size, D]")
    P = pages.shape[0]
    flat = pages.float().reshape(P, -1)
    scales = flat.abs().amax(dim=1).clamp_min(eps) / 127.0
    codes = torch.round(flat / scales[:, None]).clamp(-127, 127).to(torch.int8).reshape_as(pages)
    return codes, scales.to(torch.float32)


def make_precision_tensor(num_pages: int, fp16_pages: Optional[torch.Tensor] = None,
                          int8_pages: Optional[torch.Tensor] = None, *, device=None) -> torch.Tensor:
    """[num_pages] int32 tags, INT8 by default, FP16 / INT8 at the given pages."""
    prec = torch.full((num_pages,), int(TritonKVPrecision.INT8), dtype=torch.int32, device=device)
    if fp16_pages is not None:
        prec[fp16_pages.to(device=device, dtype=torch.long)] = int(TritonKVPrecision.FP16)
    if int8_pages is not None:
        prec[int8_pages.to(device=device, dtype=torch.long)] = int(TritonKVPrecision.INT8)
    return prec
