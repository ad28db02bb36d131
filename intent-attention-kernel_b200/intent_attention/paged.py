"""Device page pools, quantise-on-write, metadata packing and the decode call.

This is the thin host layer over the C ABI that every reference-compatible
entry point (``fused_selected_quant_decode``, ``intent_quant_decode_attention_triton``,
``adaptive_format_decode_attention_triton``) funnels into.  PyTorch is used
only for device memory and the current stream; all arithmetic runs in the
sm_100a kernels of libiak_b200.so.

Page model (as in the reference, ``fused_selected_quant_decode.py:428-431``):
pages are single-head, ``[num_pages, page_size, head_dim]`` per pool, and a
page table row lists the physical pages one (batch, table-head) attends to.
G = Hq / Ht query heads share a row (grouped-query attention; G = 1 is the
reference's layout).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass, field
from typing import Dict, Mapping, Optional, Sequence, Tuple

import torch

from . import _native as N

FORMAT_CODES = {"SKIP": N.FMT_SKIP, "F16": N.FMT_F16, "FP16": N.FMT_F16, "FP8": N.FMT_FP8, "INT8": N.FMT_INT8,
                "INT4": N.FMT_INT4, "INT4R": N.FMT_INT4R, "INT4_RESIDUAL": N.FMT_INT4R, "SPARSE": N.FMT_SPARSE}
_DT = {torch.float32: N.DT_F32, torch.float16: N.DT_F16, torch.bfloat16: N.DT_BF16}


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or t.device.type != "cuda":
        raise RuntimeError(f"{name} must be a CUDA tensor: this build runs only on the GPU (no CPU fallback)")


def n_scales(scale_mode: str, head_dim: int) -> int:
    return {"page": 1, "group32": head_dim // 32, "channel": head_dim}[scale_mode]


@dataclass
class PagePool:
    """K/V page pools of one layer on one device.

    Each format keeps its own ``[num_pages, page_size, row]`` pool (``row`` =
    head_dim bytes for 8-bit formats, head_dim/2 for packed INT4); a page's tag
    selects which pool holds it.  Scales are ``[num_pages, n_scales]`` fp32.
    """

    num_pages: int
    page_size: int
    head_dim: int
    scale_mode: str = "page"
    k_f16: Optional[torch.Tensor] = None
    v_f16: Optional[torch.Tensor] = None
    k_fp8: Optional[torch.Tensor] = None
    v_fp8: Optional[torch.Tensor] = None
    k_i8: Optional[torch.Tensor] = None
    v_i8: Optional[torch.Tensor] = None
    k_i4: Optional[torch.Tensor] = None
    v_i4: Optional[torch.Tensor] = None
    k_i4r: Optional[torch.Tensor] = None
    v_i4r: Optional[torch.Tensor] = None
    k_scale: Optional[torch.Tensor] = None
    v_scale: Optional[torch.Tensor] = None
    k_res_scale: Optional[torch.Tensor] = None
    v_res_scale: Optional[torch.Tensor] = None

    @classmethod
    def allocate(cls, num_pages: int, page_size: int, head_dim: int,
                 formats: Sequence[str] = ("F16", "FP8", "INT8", "INT4", "INT4R"),
                 scale_mode: str = "page", device="cuda", zero: bool = False) -> "PagePool":
        dev = torch.device(device)
        mk = torch.zeros if zero else torch.empty
        shape = (num_pages, page_size, head_dim)
        p = cls(num_pages, page_size, head_dim, scale_mode)
        fm = {f.upper() for f in formats}
        if fm & {"F16", "FP16"}:
            p.k_f16, p.v_f16 = mk(shape, dtype=torch.float16, device=dev), mk(shape, dtype=torch.float16, device=dev)
        if "FP8" in fm:
            p.k_fp8, p.v_fp8 = mk(shape, dtype=torch.uint8, device=dev), mk(shape, dtype=torch.uint8, device=dev)
        if "INT8" in fm:
            p.k_i8, p.v_i8 = mk(shape, dtype=torch.int8, device=dev), mk(shape, dtype=torch.int8, device=dev)
        half = (num_pages, page_size, head_dim // 2)
        if fm & {"INT4", "INT4R", "INT4_RESIDUAL"}:
            p.k_i4, p.v_i4 = mk(half, dtype=torch.uint8, device=dev), mk(half, dtype=torch.uint8, device=dev)
        if fm & {"INT4R", "INT4_RESIDUAL"}:
            p.k_i4r, p.v_i4r = mk(half, dtype=torch.uint8, device=dev), mk(half, dtype=torch.uint8, device=dev)
        if fm - {"F16", "FP16"}:
            ns = n_scales(scale_mode, head_dim)
            p.k_scale = torch.ones((num_pages, ns), dtype=torch.float32, device=dev)
            p.v_scale = torch.ones((num_pages, ns), dtype=torch.float32, device=dev)
            if fm & {"INT4R", "INT4_RESIDUAL"}:
                p.k_res_scale = torch.ones((num_pages, ns), dtype=torch.float32, device=dev)
                p.v_res_scale = torch.ones((num_pages, ns), dtype=torch.float32, device=dev)
        return p

    def tensors(self):
        return [t for t in (self.k_f16, self.v_f16, self.k_fp8, self.v_fp8, self.k_i8, self.v_i8, self.k_i4,
                            self.v_i4, self.k_i4r, self.v_i4r, self.k_scale, self.v_scale, self.k_res_scale,
                            self.v_res_scale) if t is not None]

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.tensors())

    def struct(self) -> N.PagePools:
        for t in self.tensors():
            _require_cuda(t, "page pool")
            if not t.is_contiguous():
                raise ValueError("page pools must be contiguous")
            if t.data_ptr() % 16:
                raise ValueError("page pools must be 16-byte aligned")
        s = N.PagePools()
        for name in ("k_f16", "v_f16", "k_fp8", "v_fp8", "k_i8", "v_i8", "k_i4", "v_i4", "k_i4r", "v_i4r",
                     "k_scale", "v_scale", "k_res_scale", "v_res_scale"):
            setattr(s, name, _ptr(getattr(self, name)))
        s.num_pages, s.page_size, s.head_dim = self.num_pages, self.page_size, self.head_dim
        s.scale_mode = N.SCALE_MODES[self.scale_mode]
        return s

    # ------------------------------------------------------------------ #
    def quantize_(self, k: torch.Tensor, v: torch.Tensor, formats, dst_ids: Optional[torch.Tensor] = None,
                  k_scales=None, v_scales=None, k_res_scales=None, v_res_scales=None) -> "PagePool":
        """Quantise dense pages k/v [P, page_size, head_dim] into the pools.

        ``formats`` is a [P] tensor / sequence of format names or IAK_FMT codes;
        page i is written to pool page ``dst_ids[i]`` (default i).  Optional
        ``*_scales`` ([P, n_scales]) replace the per-page absmax scales.
        """
        fm = _format_tensor(formats, k.shape[0], k.device)
        for plane, x, sc, rs in (("k", k, k_scales, k_res_scales), ("v", v, v_scales, v_res_scales)):
            quantize_plane(self, plane, x, fm, dst_ids, sc, rs)
        return self


def _format_tensor(formats, P: int, device) -> torch.Tensor:
    if isinstance(formats, torch.Tensor):
        fm = formats.to(device=device, dtype=torch.uint8)
    else:
        codes = [FORMAT_CODES[f.upper()] if isinstance(f, str) else int(f) for f in formats]
        fm = torch.tensor(codes, dtype=torch.uint8, device=device)
    if fm.numel() != P:
        raise ValueError(f"formats has {fm.numel()} entries for {P} pages")
    return fm.contiguous()


def quantize_plane(pool: PagePool, plane: str, x: torch.Tensor, formats: torch.Tensor,
                   dst_ids: Optional[torch.Tensor] = None, given_scale: Optional[torch.Tensor] = None,
                   given_res_scale: Optional[torch.Tensor] = None) -> None:
    """One plane (``'k'`` or ``'v'``) of ``PagePool.quantize_``."""
    _require_cuda(x, "x")
    if x.dim() != 3 or x.shape[1] != pool.page_size or x.shape[2] != pool.head_dim:
        raise ValueError(f"x must be [P, {pool.page_size}, {pool.head_dim}], got {tuple(x.shape)}")
    if x.dtype not in _DT:
        raise ValueError(f"x dtype {x.dtype} unsupported")
    x = x.contiguous()
    P = x.shape[0]
    if dst_ids is not None:
        dst_ids = dst_ids.to(device=x.device, dtype=torch.int32).contiguous()
        if dst_ids.numel() != P:
            raise ValueError("dst_ids must have one entry per source page")
    ns = n_scales(pool.scale_mode, pool.head_dim)
    for name, g in (("given_scale", given_scale), ("given_res_scale", given_res_scale)):
        if g is not None and tuple(g.shape) != (P, ns):
            raise ValueError(f"{name} must be [{P}, {ns}]")
    given_scale = None if given_scale is None else given_scale.to(x.device, torch.float32).contiguous()
    given_res_scale = None if given_res_scale is None else given_res_scale.to(x.device, torch.float32).contiguous()
    a = N.QuantArgs()
    a.x, a.x_dtype, a.num_src_pages = x.data_ptr(), _DT[x.dtype], P
    a.dst_ids, a.formats = _ptr(dst_ids), formats.data_ptr()
    a.given_scale, a.given_res_scale = _ptr(given_scale), _ptr(given_res_scale)
    a.f16, a.fp8, a.i8 = _ptr(getattr(pool, f"{plane}_f16")), _ptr(getattr(pool, f"{plane}_fp8")), _ptr(getattr(pool, f"{plane}_i8"))
    a.i4, a.i4r = _ptr(getattr(pool, f"{plane}_i4")), _ptr(getattr(pool, f"{plane}_i4r"))
    a.scale, a.res_scale = _ptr(getattr(pool, f"{plane}_scale")), _ptr(getattr(pool, f"{plane}_res_scale"))
    a.num_pages, a.page_size, a.head_dim = pool.num_pages, pool.page_size, pool.head_dim
    a.scale_mode = N.SCALE_MODES[pool.scale_mode]
    N.check(N.lib().iak_quantize_pages(ctypes.byref(a), _stream(x.device)), "iak_quantize_pages")


# ---------------------------------------------------------------------- #
#  Decode
# ---------------------------------------------------------------------- #

_workspaces: Dict[int, torch.Tensor] = {}


def _workspace(device: torch.device, nbytes: int) -> Optional[torch.Tensor]:
    if nbytes == 0:
        return None
    idx = device.index if device.index is not None else torch.cuda.current_device()
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[idx] = ws
    return ws


def reserve_workspace(device, nbytes: int) -> None:
    """Pre-size the per-device workspace (e.g. before CUDA-graph capture)."""
    _workspace(torch.device(device), nbytes)


def make_tag_map(mapping: Mapping[int, str]) -> Tuple[int, ...]:
    tm = [N.FMT_SKIP] * 16
    for tag, fmt in mapping.items():
        tm[int(tag)] = FORMAT_CODES[fmt] if isinstance(fmt, str) else int(fmt)
    return tuple(tm)


def _decode_structs(q, pool, page_table, page_counts, page_tags, tag_map, tag_default, sm_scale, out,
                    partial, num_splits, kernel="auto", status=None, wait_budget_ns=0):
    B, Hq, D = q.shape
    if page_table.dim() != 3 or page_table.shape[0] != B:
        raise ValueError(f"page_table must be [B, Ht, W] with B={B}, got {tuple(page_table.shape)}")
    Ht, W = page_table.shape[1], page_table.shape[2]
    if Ht == 0 or Hq % Ht:
        raise ValueError(f"query heads ({Hq}) must be a multiple of page-table heads ({Ht})")
    if D != pool.head_dim:
        raise ValueError(f"q head_dim {D} does not match the pool head_dim {pool.head_dim}")
    args = N.DecodeArgs()
    args.q, args.q_dtype, args.q_stride_b, args.q_stride_h = q.data_ptr(), _DT[q.dtype], q.stride(0), q.stride(1)
    if out is not None:
        args.out, args.out_dtype = out.data_ptr(), _DT[out.dtype]
        args.out_stride_b, args.out_stride_h = out.stride(0), out.stride(1)
    args.batch, args.num_q_heads, args.num_table_heads = B, Hq, Ht
    args.page_table, args.pt_stride_b, args.pt_stride_h = page_table.data_ptr(), page_table.stride(0), page_table.stride(1)
    args.table_width = W
    if page_counts is not None:
        args.page_counts, args.pc_stride_b = page_counts.data_ptr(), page_counts.stride(0)
    args.page_tags, args.tag_bytes = page_tags.data_ptr(), page_tags.element_size()
    for i, f in enumerate(tag_map):
        args.tag_map[i] = f
    args.tag_default = tag_default
    args.sm_scale = float(1.0 / math.sqrt(D) if sm_scale is None else sm_scale)
    if partial is not None:
        m, l, acc = partial
        args.partial_m, args.partial_l, args.partial_acc = m.data_ptr(), l.data_ptr(), acc.data_ptr()
    args.num_splits = int(num_splits)
    args.kernel = N.KERNELS[kernel]
    if status is not None:
        _require_cuda(status, "status")
        if status.dtype not in (torch.int32, torch.uint32) or status.numel() < 1:
            raise ValueError("status must be a 32-bit integer CUDA tensor")
        args.status = status.data_ptr()
    args.wait_budget_ns = int(wait_budget_ns)
    return pool.struct(), args


def paged_decode(q: torch.Tensor, pool: PagePool, page_table: torch.Tensor, page_counts: Optional[torch.Tensor],
                 page_tags: torch.Tensor, tag_map: Sequence[int], tag_default: int = N.FMT_SKIP,
                 sm_scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                 out_dtype: Optional[torch.dtype] = None, num_splits: int = 0,
                 partial: Optional[Tuple[torch.Tensor, torch.Tensor, torch.Tensor]] = None,
                 kernel: str = "auto", status: Optional[torch.Tensor] = None,
                 wait_budget_ns: int = 0) -> torch.Tensor:
    """Single-query paged decode over selected pages -> out [B, Hq, D].

    ``status`` (a 32-bit CUDA tensor, optional) collects ``IAK_STATUS_*`` bits:
    bit 0 is set when a bounded device-side wait of the tensor-core decode gave
    up (each wait's budget is ``wait_budget_ns`` nanoseconds, 0 = about 2 s); it is never
    cleared here, and reading it does not stall the launch.  The output of a
    call that timed out is undefined.

    ``tag_map`` (16 IAK_FMT codes, see ``make_tag_map``) translates the
    caller's precision enum; tags outside 0..15 use ``tag_default``.  With
    ``partial=(m, l, acc)`` ([B*Hq], [B*Hq], [B*Hq, D] fp32) the unnormalised
    split-KV partials are written instead of ``out``.  ``kernel`` selects
    "auto" (tensor-core path when the shape allows it), "generic" or "tensor".
    """
    _require_cuda(q, "q")
    if q.dim() != 3:
        raise ValueError(f"q must be [B, H, D], got {tuple(q.shape)}")
    if q.dtype not in _DT:
        raise ValueError(f"q dtype {q.dtype} unsupported")
    if q.stride(-1) != 1:
        q = q.contiguous()
    dev = q.device
    for name, t in (("page_table", page_table), ("page_tags", page_tags)):
        _require_cuda(t, name)
        if t.device != dev:
            raise ValueError(f"{name} is on {t.device}, q on {dev}")
    if page_table.dtype != torch.int32:
        page_table = page_table.to(torch.int32)
    if page_table.stride(-1) != 1:
        page_table = page_table.contiguous()
    if page_counts is not None:
        _require_cuda(page_counts, "page_counts")
        if page_counts.dtype != torch.int32 or page_counts.dim() != 2 or page_counts.stride(1) != 1:
            page_counts = page_counts.to(torch.int32).contiguous()
    if page_tags.dtype not in (torch.uint8, torch.int32):
        page_tags = page_tags.to(torch.int32)
    if page_tags.dim() != 1 or page_tags.numel() < pool.num_pages or not page_tags.is_contiguous():
        raise ValueError(f"page_tags must be a contiguous [num_pages={pool.num_pages}] tensor")
    if out is None and partial is None:
        out = torch.empty(q.shape, dtype=out_dtype or q.dtype, device=dev)
    if out is not None:
        _require_cuda(out, "out")
        if out.shape != q.shape or out.stride(-1) != 1 or out.dtype not in _DT:
            raise ValueError(f"out must be a {tuple(q.shape)} float tensor with a contiguous last dim")
    pools, args = _decode_structs(q, pool, page_table, page_counts, page_tags, tag_map, tag_default, sm_scale,
                                  out, partial, num_splits, kernel, status, wait_budget_ns)
    L = N.lib()
    nbytes = ctypes.c_size_t(0)
    N.check(L.iak_decode_workspace_size(ctypes.byref(pools), ctypes.byref(args), ctypes.byref(nbytes)),
            "iak_decode_workspace_size")
    ws = _workspace(dev, nbytes.value)
    N.check(L.iak_decode(ctypes.byref(pools), ctypes.byref(args), _ptr(ws), 0 if ws is None else ws.numel(),
                         _stream(dev)), "iak_decode")
    return out


def merge_partials(m: torch.Tensor, l: torch.Tensor, acc: torch.Tensor,
                   out: Optional[torch.Tensor] = None, out_dtype=torch.float32) -> torch.Tensor:
    """LSE-merge split partials: m/l [rows, S], acc [rows, S, D] -> [rows, D]."""
    _require_cuda(acc, "acc")
    rows, S, D = acc.shape
    m, l, acc = (t.to(torch.float32).contiguous() for t in (m, l, acc))
    if tuple(m.shape) != (rows, S) or tuple(l.shape) != (rows, S):
        raise ValueError("m and l must be [rows, splits]")
    if out is None:
        out = torch.empty((rows, D), dtype=out_dtype, device=acc.device)
    N.check(N.lib().iak_merge_partials(m.data_ptr(), l.data_ptr(), acc.data_ptr(), rows, S, D, out.data_ptr(),
                                       _DT[out.dtype], out.stride(0), _stream(acc.device)), "iak_merge_partials")
    return out


def pack_metadata(logical_ids: torch.Tensor, batch: int, table_heads: int, width: int,
                  bases: Optional[torch.Tensor] = None, logical_tags: Optional[torch.Tensor] = None,
                  page_tags: Optional[torch.Tensor] = None, pad_value: int = -1,
                  page_table: Optional[torch.Tensor] = None, page_counts: Optional[torch.Tensor] = None):
    """Device packing of one shared page list into [B, Ht, W] tables.

    physical id = bases[b, h] + logical id; slots >= min(n, W) get ``pad_value``;
    ``logical_tags`` (per logical page) are scattered into ``page_tags``.
    Returns (page_table, page_counts).
    """
    dev = logical_ids.device
    _require_cuda(logical_ids, "logical_ids")
    ids = logical_ids.to(torch.int32).contiguous()
    if page_table is None:
        page_table = torch.empty((batch, table_heads, width), dtype=torch.int32, device=dev)
    if page_counts is None:
        page_counts = torch.empty((batch, table_heads), dtype=torch.int32, device=dev)
    a = N.PackArgs()
    a.logical_ids, a.num_ids = ids.data_ptr(), ids.numel()
    if logical_tags is not None:
        logical_tags = logical_tags.to(device=dev, dtype=torch.uint8).contiguous()
        if page_tags is None or page_tags.dtype != torch.uint8:
            raise ValueError("logical_tags needs a uint8 page_tags output")
        a.logical_tags, a.num_logical_pages, a.page_tags = logical_tags.data_ptr(), logical_tags.numel(), page_tags.data_ptr()
        a.num_tag_pages = page_tags.numel()
    if bases is not None:
        bases = bases.to(device=dev, dtype=torch.int32).contiguous()
        a.bases = bases.data_ptr()
    a.batch, a.num_table_heads, a.table_width = batch, table_heads, width
    a.page_table, a.page_counts, a.pad_value = page_table.data_ptr(), page_counts.data_ptr(), pad_value
    N.check(N.lib().iak_pack_metadata(ctypes.byref(a), _stream(dev)), "iak_pack_metadata")
    return page_table, page_counts


# --------------------------------------------------------------------------- #
#  KV append (quantise-on-write) and page format transitions
# --------------------------------------------------------------------------- #

@dataclass
class KVStage:
    """fp32 rows of every (sequence, table head)'s open page, [units, PS, D]
    per plane, kept between ``append_tokens`` calls."""

    k: torch.Tensor
    v: torch.Tensor

    @classmethod
    def allocate(cls, units: int, pool: PagePool, device=None) -> "KVStage":
        dev = torch.device(device) if device is not None else pool.tensors()[0].device
        shape = (units, pool.page_size, pool.head_dim)
        return cls(torch.zeros(shape, dtype=torch.float32, device=dev),
                   torch.zeros(shape, dtype=torch.float32, device=dev))


def _tags_args(page_tags: torch.Tensor):
    _require_cuda(page_tags, "page_tags")
    if page_tags.dtype not in (torch.uint8, torch.int32) or not page_tags.is_contiguous():
        raise ValueError("page_tags must be a contiguous uint8 or int32 tensor")
    return page_tags.data_ptr(), page_tags.element_size()


def append_tokens(pool: PagePool, k_new: torch.Tensor, v_new: torch.Tensor, positions: torch.Tensor,
                  page_tags: torch.Tensor, tag_map: Sequence[int], stage: KVStage,
                  bases: Optional[torch.Tensor] = None, new_lengths: Optional[torch.Tensor] = None,
                  dropped: Optional[torch.Tensor] = None, tag_default: int = N.FMT_SKIP) -> None:
    """Append ``k_new``/``v_new`` [B, Ht, n, D] at token ``positions[b]`` of
    every (b, h) and re-quantise each touched page in the format its tag names.

    Physical page of token t = ``bases[b, h]`` + t // page_size.  A page
    always ends up holding what ``PagePool.quantize_`` gives for its dense
    rows (zeros past the last appended row).  Never synchronises.
    """
    _require_cuda(k_new, "k_new")
    if k_new.shape != v_new.shape or k_new.dim() != 4 or k_new.shape[-1] != pool.head_dim:
        raise ValueError(f"k_new / v_new must both be [B, Ht, n, {pool.head_dim}]")
    if k_new.dtype != v_new.dtype or k_new.dtype not in _DT:
        raise ValueError("k_new / v_new must share a float32 / float16 / bfloat16 dtype")
    B, Ht, n, _ = k_new.shape
    dev = k_new.device
    k_new, v_new = k_new.contiguous(), v_new.contiguous()
    positions = positions.to(device=dev, dtype=torch.int32).contiguous()
    if positions.numel() != B:
        raise ValueError("positions must hold one entry per sequence")
    for t in (stage.k, stage.v):
        if t.dtype != torch.float32 or tuple(t.shape) != (B * Ht, pool.page_size, pool.head_dim) \
                or not t.is_contiguous():
            raise ValueError(f"stage planes must be contiguous float32 [{B * Ht}, {pool.page_size}, {pool.head_dim}]")
    keep = [k_new, v_new, positions]
    a = N.AppendArgs()
    a.k_new, a.v_new, a.new_dtype = k_new.data_ptr(), v_new.data_ptr(), _DT[k_new.dtype]
    a.batch, a.num_table_heads, a.num_new = B, Ht, n
    a.positions = positions.data_ptr()
    if new_lengths is not None:
        if new_lengths.dtype != torch.int32 or new_lengths.numel() != B or new_lengths.data_ptr() == positions.data_ptr():
            raise ValueError("new_lengths must be a separate int32 tensor of B entries")
        a.new_lengths = new_lengths.data_ptr()
    if bases is not None:
        bases = bases.to(device=dev, dtype=torch.int32).contiguous()
        keep.append(bases)
        a.bases = bases.data_ptr()
    a.page_tags, a.tag_bytes = _tags_args(page_tags)
    for i, f in enumerate(tag_map):
        a.tag_map[i] = f
    a.tag_default = tag_default
    a.k_stage, a.v_stage = stage.k.data_ptr(), stage.v.data_ptr()
    if dropped is not None:
        a.dropped = dropped.data_ptr()
    s = pool.struct()
    N.check(N.lib().iak_append_tokens(ctypes.byref(s), ctypes.byref(a), _stream(dev)), "iak_append_tokens")


def convert_pages(pool: PagePool, page_ids: torch.Tensor, new_formats, page_tags: torch.Tensor,
                  tag_map: Sequence[int], fmt_to_tag: Mapping[str, int], tag_default: int = N.FMT_SKIP,
                  rejected: Optional[torch.Tensor] = None) -> None:
    """Demote / promote pool pages: read each page in its current format,
    re-quantise it into ``new_formats`` (names or IAK_FMT codes) and store
    ``fmt_to_tag[format name]`` as its tag.  Never synchronises."""
    dev = page_ids.device
    _require_cuda(page_ids, "page_ids")
    ids = page_ids.to(torch.int32).contiguous()
    fm = _format_tensor(new_formats, ids.numel(), dev)
    a = N.ConvertArgs()
    a.page_ids, a.num_ids, a.new_formats = ids.data_ptr(), ids.numel(), fm.data_ptr()
    a.page_tags, a.tag_bytes = _tags_args(page_tags)
    for i, f in enumerate(tag_map):
        a.tag_map[i] = f
    a.tag_default = tag_default
    for name, tag in fmt_to_tag.items():
        a.fmt_to_tag[FORMAT_CODES[name.upper()]] = int(tag)
    if rejected is not None:
        a.rejected = rejected.data_ptr()
    s = pool.struct()
    N.check(N.lib().iak_convert_pages(ctypes.byref(s), ctypes.byref(a), _stream(dev)), "iak_convert_pages")


# --------------------------------------------------------------------------- #
#  Multi-query (prefill) attention over selected pages
# --------------------------------------------------------------------------- #

def paged_prefill(q: torch.Tensor, pool: PagePool, page_table: torch.Tensor, page_counts: Optional[torch.Tensor],
                  page_tags: torch.Tensor, tag_map: Sequence[int], q_positions: Optional[torch.Tensor] = None,
                  causal: bool = True, bases: Optional[torch.Tensor] = None,
                  row_masks: Optional[torch.Tensor] = None, sm_scale: Optional[float] = None,
                  out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                  tag_default: int = N.FMT_SKIP, kernel: str = "auto",
                  page_positions: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention of ``q`` [B, Hq, M, D] over the selected pages -> [B, Hq, M, D].

    Unit (b, h) attends to the rows of ``page_table[b, h, :page_counts[b, h]]``
    that ``row_masks[b, slot]`` (uint64 bit masks, None = every row) selects;
    a row of page ``pid`` sits at token position ``(pid - bases[b, h]) *
    page_size + row``.  With ``causal`` a key is visible to query m iff its
    position <= ``q_positions[b, m]`` (default m).  ``page_positions`` [B, Ht, W]
    (int32) gives the position of row 0 of each slot's page directly instead.
    Rows that see no key are 0.

    ``kernel``: "auto" runs the tcgen05 kernel when it applies (head_dim 128,
    page_size 8..64, at most 1024 table slots, 16-byte aligned pools, a
    positive ``sm_scale``) and the CUDA-core kernel otherwise; "tensor" raises
    on calls outside those bounds; "generic" always runs the CUDA-core kernel.
    """
    _require_cuda(q, "q")
    if q.dim() != 4:
        raise ValueError("q must be [B, Hq, M, D]")
    B, Hq, M, D = q.shape
    if D != pool.head_dim:
        raise ValueError(f"q head_dim {D} does not match the pool head_dim {pool.head_dim}")
    if q.dtype not in _DT:
        raise ValueError("q must be float32 / float16 / bfloat16")
    if page_table.dim() != 3 or page_table.shape[0] != B or page_table.dtype != torch.int32:
        raise ValueError(f"page_table must be int32 [B, Ht, W] with B={B}")
    Ht, W = page_table.shape[1], page_table.shape[2]
    dev = q.device
    keep = []
    if out is None:
        out = torch.empty((B, Hq, M, D), dtype=out_dtype or q.dtype, device=dev)
    a = N.PrefillArgs()
    a.q, a.q_dtype = q.data_ptr(), _DT[q.dtype]
    a.q_stride_b, a.q_stride_h, a.q_stride_m = q.stride(0), q.stride(1), q.stride(2)
    if q.stride(3) != 1 or out.stride(3) != 1:
        raise ValueError("q and out need a unit stride along head_dim")
    a.out, a.out_dtype = out.data_ptr(), _DT[out.dtype]
    a.out_stride_b, a.out_stride_h, a.out_stride_m = out.stride(0), out.stride(1), out.stride(2)
    a.batch, a.num_q_heads, a.num_table_heads, a.num_queries = B, Hq, Ht, M
    if q_positions is not None:
        q_positions = q_positions.to(device=dev, dtype=torch.int32).contiguous()
        if tuple(q_positions.shape) != (B, M):
            raise ValueError("q_positions must be [B, M]")
        keep.append(q_positions)
        a.q_positions, a.qp_stride_b = q_positions.data_ptr(), M
    a.causal = 1 if causal else 0
    a.page_table, a.pt_stride_b, a.pt_stride_h = page_table.data_ptr(), page_table.stride(0), page_table.stride(1)
    if page_table.stride(2) != 1:
        raise ValueError("page_table rows must be contiguous")
    a.table_width = W
    if page_counts is not None:
        if page_counts.dtype != torch.int32 or page_counts.dim() != 2 or page_counts.stride(1) != 1:
            raise ValueError("page_counts must be int32 [B, Ht] with contiguous rows")
        a.page_counts, a.pc_stride_b = page_counts.data_ptr(), page_counts.stride(0)
    if bases is not None:
        bases = bases.to(device=dev, dtype=torch.int32).contiguous()
        keep.append(bases)
        a.bases = bases.data_ptr()
    if page_positions is not None:
        page_positions = page_positions.to(device=dev, dtype=torch.int32).contiguous()
        if tuple(page_positions.shape) != (B, Ht, W):
            raise ValueError("page_positions must be [B, Ht, W]")
        keep.append(page_positions)
        a.page_positions, a.pp_stride_b, a.pp_stride_h = page_positions.data_ptr(), Ht * W, W
    if row_masks is not None:
        if row_masks.dtype not in (torch.int64, torch.uint64) or tuple(row_masks.shape) != (B, W) \
                or row_masks.stride(1) != 1:
            raise ValueError("row_masks must be 64-bit [B, W] with contiguous rows")
        a.row_masks, a.rm_stride_b = row_masks.data_ptr(), row_masks.stride(0)
    a.page_tags, a.tag_bytes = _tags_args(page_tags)
    for i, f in enumerate(tag_map):
        a.tag_map[i] = f
    a.tag_default = tag_default
    a.sm_scale = float(1.0 / math.sqrt(D) if sm_scale is None else sm_scale)
    a.kernel = N.KERNELS[kernel]
    s = pool.struct()
    N.check(N.lib().iak_prefill(ctypes.byref(s), ctypes.byref(a), _stream(dev)), "iak_prefill")
    return out
