"""Fused selected-quant decode (drop-in for ``fused_selected_quant_decode.py``).

Same names, arguments, shapes and errors as the reference module
(``FusedKVPrecision`` / ``FusedDecodeConfig`` ``:29-49``,
``metadata_to_kernel_tensors`` ``:344-400``, ``fused_selected_quant_decode``
``:408-464``, ``fake_int8_pages_from_fp16`` ``:521-542``).  The decode runs
the sm_100a kernels of libiak_b200.so; unlike the reference there is no CPU
fallback: CPU tensors raise ``RuntimeError``.

Semantics kept from the reference CPU path (``:290-334``): FP16 pages are read
directly, INT8 pages as ``code * scale[page]``, SKIP pages contribute nothing,
``page_counts`` bounds each (b, h) (clamped to the table width, as the
reference kernel does), the output is ``acc / l`` (0 when nothing is
attended) cast to float16 ``[B, H, 1, D]``.  Negative page ids are unused
slots.
"""

from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum
from typing import Dict, Optional, Tuple

import torch

from . import _native as N
from .paged import PagePool, make_tag_map, pack_metadata, paged_decode


class FusedKVPrecision(IntEnum):
    """Precision tags for per-page load decisions inside the kernel."""

    FP16 = 0
    INT8 = 1
    SKIP = 2


@dataclass(frozen=True)
class FusedDecodeConfig:
    page_size: int = 16
    head_dim: int = 64
    max_selected_pages: int = 64
    block_d: int = 64


_TAG_MAP = make_tag_map({0: "F16", 1: "INT8", 2: "SKIP"})


def is_triton_available() -> bool:
    """True when the GPU kernel backend (libiak_b200.so) is loadable."""
    return N.available()


def is_cuda_available() -> bool:
    return torch.cuda.is_available()


def _precision_code(prec: str) -> int:
    # the reference's lossy mapping (:384-389): FP8 -> FP16, INT4* -> INT8
    if prec == "SKIP":
        return int(FusedKVPrecision.SKIP)
    if prec in ("INT8", "INT4", "INT4_RESIDUAL"):
        return int(FusedKVPrecision.INT8)
    return int(FusedKVPrecision.FP16)


def metadata_to_kernel_tensors(meta: Dict, num_pages: int, B: int = 1, H: int = 1,
                               config: Optional[FusedDecodeConfig] = None,
                               device: Optional[torch.device] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Router metadata -> (page_table [B, H, W] int32 zero-padded,
    page_precision [num_pages] int32 (default FP16), page_counts [B, H] int32).

    On a CUDA ``device`` the table and counts are packed by one device
    launch (``iak_pack_metadata``) instead of a Python loop per element.
    """
    cfg = config or FusedDecodeConfig()
    dev = torch.device("cpu") if device is None else torch.device(device)
    W = cfg.max_selected_pages
    prec = torch.full((num_pages,), int(FusedKVPrecision.FP16), dtype=torch.int32)
    for pid_s, p in meta.get("block_precision_by_page", {}).items():
        try:
            pid = int(pid_s)
        except ValueError:
            continue
        prec[pid] = _precision_code(p)
    ids = list(meta.get("selected_page_ids", []))
    n = min(len(ids), W)
    if dev.type == "cuda":
        ids_t = torch.tensor(ids[:n] if n else [0], dtype=torch.int32).to(dev, non_blocking=True)
        if n == 0:
            ids_t = ids_t[:0]
        table, counts = pack_metadata(ids_t, B, H, W, pad_value=0)
        return table, prec.to(dev), counts
    table = torch.zeros(B, H, W, dtype=torch.int32)
    if n:
        table[:, :, :n] = torch.tensor(ids[:n], dtype=torch.int32)
    counts = torch.full((B, H), n, dtype=torch.int32)
    return table, prec, counts


def fused_selected_quant_decode(query: torch.Tensor, k_pages_fp16: torch.Tensor, v_pages_fp16: torch.Tensor,
                                k_pages_int8: torch.Tensor, v_pages_int8: torch.Tensor, k_scales: torch.Tensor,
                                v_scales: torch.Tensor, page_table: torch.Tensor, page_precision: torch.Tensor,
                                page_counts: torch.Tensor, config: FusedDecodeConfig = FusedDecodeConfig(),
                                *, num_splits: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Fused selected-quant decode attention -> [B, H, 1, D] float16.

    query [B, H, 1, D]; k/v_pages_fp16 [NP, page_size, D] float16;
    k/v_pages_int8 [NP, page_size, D] int8; k/v_scales [NP] per-page scales;
    page_table [B, H, W] int32; page_precision [NP] FusedKVPrecision tags;
    page_counts [B, H] int32.
    """
    B, H, _, D = query.shape
    if D != config.head_dim:
        raise ValueError(f"head_dim {D} != config.head_dim {config.head_dim}")
    if query.device.type != "cuda":
        raise RuntimeError("fused_selected_quant_decode runs only on CUDA tensors (this build has no CPU fallback)")
    NP, PS = k_pages_fp16.shape[0], k_pages_fp16.shape[1]
    dev = query.device
    pool = PagePool(NP, PS, D, "page")
    pool.k_f16, pool.v_f16 = k_pages_fp16.to(dev, torch.float16).contiguous(), v_pages_fp16.to(dev, torch.float16).contiguous()
    pool.k_i8, pool.v_i8 = k_pages_int8.to(dev, torch.int8).contiguous(), v_pages_int8.to(dev, torch.int8).contiguous()
    pool.k_scale = k_scales.to(dev, torch.float32).reshape(NP, 1).contiguous()
    pool.v_scale = v_scales.to(dev, torch.float32).reshape(NP, 1).contiguous()
    q = query[:, :, 0, :]
    res = paged_decode(q, pool, page_table.to(dev), page_counts.to(dev), page_precision.to(dev).contiguous(),
                       _TAG_MAP, N.FMT_SKIP, out_dtype=torch.float16, num_splits=num_splits,
                       out=None if out is None else out[:, :, 0, :])
    return res.unsqueeze(2) if out is None else out


def fake_int8_pages_from_fp16(pages: torch.Tensor, eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-page symmetric INT8 (``:521-542``): scale = max(absmax, eps)/127 in the
    input dtype, codes = clamp(round(x / scale), -128, 127)."""
    P = pages.shape[0]
    flat = pages.view(P, -1)
    scales = flat.abs().max(dim=1, keepdim=True).values.clamp(min=eps) / 127.0
    codes = (flat / scales).round().clamp(-128, 127).to(torch.int8).view(pages.shape)
    return codes, scales.squeeze(-1)
