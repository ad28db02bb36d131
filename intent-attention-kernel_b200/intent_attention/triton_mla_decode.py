"""MLA (absorbed latent attention) decode over selected latent pages.

Drop-in for the reference module ``intent_attention/triton_mla_decode.py``:

* ``mla_decode_triton(q_absorb, C, W_VO_fused, page_table, page_size=64)``
  keeps the reference's signature and result (``triton_mla_decode.py:110-152``):
  every (batch, position) row attends over the listed latent pages of ``C``
  (key = value = the latent row, scale 1/sqrt(d_c)), the context is
  projected by ``W_VO_fused`` and returned in ``q_absorb``'s dtype; an empty
  page table gives zeros.  It runs in libiak_b200.so (``iak_mla_decode``);
  there is no Triton and no CPU fallback: CPU tensors raise RuntimeError.
* ``mla_paged_decode`` is the per-head paged form used for the
  DeepSeek-V2 shape: q ``[B, H, d_qk]``, one page list per sequence, dense
  (BF16 / F16 / F32) and FP8-e4m3 (per-page scale) latent pools picked by a
  per-page tag, value = the first ``d_v`` latent channels.  At d_qk = 576,
  d_v = 512, H <= 128 it runs on the tcgen05 / TMEM kernel.

The W_VO projection after the attention is a plain GEMM and stays a torch
matmul (cuBLAS); everything before it runs in the library's kernels.
"""

from __future__ import annotations

import ctypes
import math
from typing import Mapping, Optional, Tuple

import torch

from . import _native as N
from .paged import _DT, _require_cuda, _stream, _workspace

MLA_FORMATS = {"SKIP": N.MLA_SKIP, "DENSE": N.MLA_DENSE, "BF16": N.MLA_DENSE, "F16": N.MLA_DENSE,
               "FP16": N.MLA_DENSE, "F32": N.MLA_DENSE, "FP8": N.MLA_FP8}


def is_triton_available() -> bool:
    """The reference's probe; this build has no Triton path (always False)."""
    return False


def is_cuda_available() -> bool:
    return torch.cuda.is_available()


def is_native_available() -> bool:
    """True when libiak_b200.so is built and loadable."""
    return N.available()


def _can_run_gpu_kernel() -> bool:
    return is_cuda_available() and is_native_available()


def make_mla_tag_map(mapping: Mapping[int, str]) -> Tuple[int, ...]:
    tm = [N.MLA_SKIP] * 16
    for tag, fmt in mapping.items():
        tm[int(tag)] = MLA_FORMATS[fmt.upper()] if isinstance(fmt, str) else int(fmt)
    return tuple(tm)


def mla_paged_decode(q: torch.Tensor, page_table: torch.Tensor, page_counts: Optional[torch.Tensor] = None,
                     dense_pages: Optional[torch.Tensor] = None, fp8_pages: Optional[torch.Tensor] = None,
                     fp8_scale: Optional[torch.Tensor] = None, page_tags: Optional[torch.Tensor] = None,
                     tag_map: Optional[Tuple[int, ...]] = None, tag_default: int = N.MLA_SKIP,
                     d_v: Optional[int] = None, sm_scale: Optional[float] = None,
                     out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                     num_splits: int = 0, kernel: str = "auto",
                     partial: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None) -> torch.Tensor:
    """Per-head MLA decode -> context ``[B, H, d_v]``.

    ``page_table`` is ``[B, W]`` (or ``[W]``, shared by every sequence), ids
    < 0 unused; ``page_counts`` ``[B]`` limits each row.  ``dense_pages`` /
    ``fp8_pages`` are ``[num_pages, page_size, d_qk]`` pools (``fp8_pages``
    uint8 e4m3 codes with ``fp8_scale`` ``[num_pages]``); ``page_tags`` +
    ``tag_map`` (see ``make_mla_tag_map``) choose a page's pool; without tags
    every page is dense.  ``sm_scale`` defaults to 1/sqrt(d_qk).  With
    ``partial=(m, l, acc)`` ([B*H], [B*H], [B*H, d_v] fp32) the unnormalised
    partials are written instead of ``out`` (merge with
    ``split_kv.merge_partial_blocks``)."""
    _require_cuda(q, "q")
    if q.dim() != 3:
        raise ValueError(f"q must be [B, H, d_qk], got {tuple(q.shape)}")
    if q.dtype not in _DT:
        raise ValueError(f"q dtype {q.dtype} unsupported")
    if q.stride(-1) != 1:
        q = q.contiguous()
    B, H, Dqk = q.shape
    Dv = Dqk if d_v is None else int(d_v)
    dev = q.device
    pools = [t for t in (dense_pages, fp8_pages) if t is not None]
    if not pools:
        raise ValueError("need dense_pages and/or fp8_pages")
    NP, PS = pools[0].shape[0], pools[0].shape[1]
    for t, name in ((dense_pages, "dense_pages"), (fp8_pages, "fp8_pages")):
        if t is None:
            continue
        _require_cuda(t, name)
        if t.dim() != 3 or tuple(t.shape) != (NP, PS, Dqk) or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous [{NP}, {PS}, {Dqk}] tensor, got {tuple(t.shape)}")
    if dense_pages is not None and dense_pages.dtype not in _DT:
        raise ValueError(f"dense_pages dtype {dense_pages.dtype} unsupported")
    if fp8_pages is not None:
        if fp8_pages.dtype not in (torch.uint8, torch.float8_e4m3fn):
            raise ValueError("fp8_pages must hold e4m3 codes (uint8 or float8_e4m3fn)")
        if fp8_scale is None or fp8_scale.numel() < NP:
            raise ValueError("fp8_pages need fp8_scale [num_pages]")
        _require_cuda(fp8_scale, "fp8_scale")
        fp8_scale = fp8_scale.to(torch.float32).contiguous()
    _require_cuda(page_table, "page_table")
    pt = page_table.to(torch.int32)
    if pt.dim() == 1:
        pt = pt.contiguous()
        pt_sb = 0
    elif pt.dim() == 2 and pt.shape[0] == B:
        pt = pt.contiguous()
        pt_sb = pt.stride(0)
    else:
        raise ValueError(f"page_table must be [W] or [B={B}, W], got {tuple(page_table.shape)}")
    W = pt.shape[-1]
    if page_counts is not None:
        _require_cuda(page_counts, "page_counts")
        page_counts = page_counts.to(torch.int32).contiguous()
        if page_counts.numel() != B:
            raise ValueError(f"page_counts must have {B} entries")
    if page_tags is not None:
        _require_cuda(page_tags, "page_tags")
        if page_tags.dtype not in (torch.uint8, torch.int32):
            page_tags = page_tags.to(torch.int32)
        page_tags = page_tags.contiguous()
        if page_tags.numel() < NP:
            raise ValueError(f"page_tags must have num_pages={NP} entries")
        if tag_map is None:
            raise ValueError("page_tags need a tag_map")
    if out is None and partial is None:
        out = torch.empty((B, H, Dv), dtype=out_dtype or q.dtype, device=dev)
    if out is not None:
        _require_cuda(out, "out")
        if tuple(out.shape) != (B, H, Dv) or out.stride(-1) != 1 or out.dtype not in _DT:
            raise ValueError(f"out must be a [{B}, {H}, {Dv}] float tensor with a contiguous last dim")

    a = N.MlaArgs()
    a.q, a.q_dtype, a.q_stride_b, a.q_stride_h = q.data_ptr(), _DT[q.dtype], q.stride(0), q.stride(1)
    if out is not None:
        a.out, a.out_dtype, a.out_stride_b, a.out_stride_h = out.data_ptr(), _DT[out.dtype], out.stride(0), out.stride(1)
    a.batch, a.num_heads, a.d_qk, a.d_v = B, H, Dqk, Dv
    if dense_pages is not None:
        a.dense_pages, a.dense_dtype = dense_pages.data_ptr(), _DT[dense_pages.dtype]
    if fp8_pages is not None:
        a.fp8_pages, a.fp8_scale = fp8_pages.data_ptr(), fp8_scale.data_ptr()
    a.num_pages, a.page_size = NP, PS
    a.page_table, a.pt_stride_b, a.table_width = pt.data_ptr(), pt_sb, W
    if page_counts is not None:
        a.page_counts = page_counts.data_ptr()
    if page_tags is not None:
        a.page_tags, a.tag_bytes = page_tags.data_ptr(), page_tags.element_size()
        for i, f in enumerate(tag_map):
            a.tag_map[i] = f
        a.tag_default = tag_default
    a.sm_scale = float(1.0 / math.sqrt(Dqk) if sm_scale is None else sm_scale)
    if partial is not None:
        m, l, acc = partial
        for t, n in ((m, B * H), (l, B * H), (acc, B * H * Dv)):
            _require_cuda(t, "partial")
            if t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != n:
                raise ValueError("partial must be contiguous fp32 (m [B*H], l [B*H], acc [B*H, d_v])")
        a.partial_m, a.partial_l, a.partial_acc = m.data_ptr(), l.data_ptr(), acc.data_ptr()
    a.num_splits = int(num_splits)
    a.kernel = N.KERNELS[kernel]
    L = N.lib()
    nbytes = ctypes.c_size_t(0)
    N.check(L.iak_mla_workspace_size(ctypes.byref(a), ctypes.byref(nbytes)), "iak_mla_workspace_size")
    ws = _workspace(dev, nbytes.value)
    N.check(L.iak_mla_decode(ctypes.byref(a), None if ws is None else ws.data_ptr(),
                             0 if ws is None else ws.numel(), _stream(dev)), "iak_mla_decode")
    return out


def mla_decode_triton(q_absorb: torch.Tensor, C: torch.Tensor, W_VO_fused: torch.Tensor,
                      page_table: torch.Tensor, page_size: int = 64) -> torch.Tensor:
    """MLA decode over page-table selected latent pages (reference signature).

    q_absorb [batch, q_len, d_c]; C [total_tokens, d_c] (page p = rows
    p*page_size .. (p+1)*page_size); W_VO_fused [d_c, d_out]; page_table
    [n_selected] int.  Returns [batch, q_len, d_out] in q_absorb's dtype on
    q_absorb's device; zeros when no page is selected."""
    for t, n in ((q_absorb, "q_absorb"), (C, "C"), (W_VO_fused, "W_VO_fused"), (page_table, "page_table")):
        _require_cuda(t, n)
    if q_absorb.dim() != 3 or C.dim() != 2 or W_VO_fused.dim() != 2:
        raise ValueError("expected q_absorb [batch, q_len, d_c], C [tokens, d_c], W_VO_fused [d_c, d_out]")
    batch, q_len, d_c = q_absorb.shape
    if C.shape[1] != d_c or W_VO_fused.shape[0] != d_c:
        raise ValueError(f"d_c mismatch: q_absorb {d_c}, C {C.shape[1]}, W_VO_fused {W_VO_fused.shape[0]}")
    if page_size <= 0:
        raise ValueError("page_size must be positive")
    d_out = W_VO_fused.shape[1]
    Cc = C if C.dtype in _DT else C.float()
    Cc = Cc.contiguous()
    tokens = Cc.shape[0]
    if page_table.numel() == 0 or tokens == 0:
        return torch.zeros((batch, q_len, d_out), dtype=q_absorb.dtype, device=q_absorb.device)
    if tokens % page_size:
        raise ValueError(f"C has {tokens} rows, not a multiple of page_size={page_size} (pages must be whole)")
    pages = Cc.view(tokens // page_size, page_size, d_c)
    q = q_absorb if q_absorb.dtype in _DT else q_absorb.float()
    ctx = mla_paged_decode(q, page_table.reshape(-1), None, dense_pages=pages, sm_scale=1.0 / math.sqrt(d_c),
                           out_dtype=torch.float32)
    return torch.matmul(ctx, W_VO_fused.to(torch.float32)).to(q_absorb.dtype)
