"""Sequence-sharded split-KV decode across GPUs (one process per GPU).

No counterpart in the reference, which decodes on one device.  For very long
contexts every (sequence, kv head)'s selected page list is cut into ``world``
contiguous ranges, one per rank.  Each rank decodes its range into a *partial
block* (m, l, acc per query row), one NCCL all-gather exchanges the blocks
(rows * (D + 2) fp32 per rank), and every rank merges them with the
online-softmax recurrence of the reference's decode loop
(``fused_selected_quant_decode.py:323-334``), applied across ranks:

    m = max_i m_i,  l = sum_i l_i e^(m_i - m),  o = sum_i acc_i e^(m_i - m) / l

Block layout (``IAK_PARTIAL_BLOCK_FLOATS`` in the C header):
``[m: rows][l: rows][acc: rows x D]`` with rows = B * Hq, row = b * Hq + h.

The decode and merge run in libiak_b200.so; this module only cuts page
lists, allocates blocks and drives the exchange: either one NCCL all-gather
(``transport="nccl"``) or stores straight into the peers' exchange areas over
NVLink with epoch flags and a bounded wait (``transport="p2p"``, CUDA IPC,
``PeerExchange``).  ``shard_bounds``,
``block_views`` and ``shard_page_lists`` are plain index helpers that also
run on CPU tensors.
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from . import _native as N
from .paged import PagePool, _DT, _decode_structs, _require_cuda, _stream, _workspace, paged_decode


def shard_bounds(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous range [start, stop) of ``n`` ordered items owned by ``rank``
    (sizes differ by at most one; earlier ranks get the larger shares)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    if n < 0:
        raise ValueError("n must be >= 0")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_page_lists(page_table: torch.Tensor, page_counts: Optional[torch.Tensor], rank: int,
                     world: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Cut each row of a [B, Ht, W] page table into ``world`` contiguous
    ranges of its first ``count`` slots and return rank's range as a
    -1-padded [B, Ht, W_r] table (W_r = ceil(W / world)) with its counts."""
    if page_table.dim() != 3:
        raise ValueError(f"page_table must be [B, Ht, W], got {tuple(page_table.shape)}")
    B, Ht, W = page_table.shape
    dev = page_table.device
    if page_counts is None:
        counts = torch.full((B, Ht), W, dtype=torch.int64, device=dev)
    else:
        if tuple(page_counts.shape) != (B, Ht):
            raise ValueError(f"page_counts must be [{B}, {Ht}], got {tuple(page_counts.shape)}")
        counts = page_counts.to(torch.int64).clamp(0, W)
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    base, extra = counts // world, counts % world
    start = rank * base + torch.clamp(extra, max=rank)
    size = base + (extra > rank).to(torch.int64)
    width = (W + world - 1) // world
    idx = start[..., None] + torch.arange(width, device=dev)
    valid = torch.arange(width, device=dev) < size[..., None]
    local = torch.gather(page_table.to(torch.int32), 2, torch.where(valid, idx, 0).clamp(max=max(W - 1, 0)))
    local = torch.where(valid, local, torch.full_like(local, -1))
    return local.contiguous(), size.to(torch.int32).contiguous()


def block_floats(rows: int, head_dim: int) -> int:
    return rows * (head_dim + 2)


def block_views(block: torch.Tensor, rows: int, head_dim: int):
    """(m [rows], l [rows], acc [rows, D]) views of a flat partial block."""
    if block.numel() != block_floats(rows, head_dim):
        raise ValueError(f"block must hold rows*(D+2) = {block_floats(rows, head_dim)} floats")
    return block[:rows], block[rows:2 * rows], block[2 * rows:].view(rows, head_dim)


def decode_partial_block(q: torch.Tensor, pool: PagePool, page_table: torch.Tensor,
                         page_counts: Optional[torch.Tensor], page_tags: torch.Tensor, tag_map: Sequence[int],
                         tag_default: int = N.FMT_SKIP, sm_scale: Optional[float] = None,
                         block: Optional[torch.Tensor] = None, num_splits: int = 0,
                         kernel: str = "auto") -> torch.Tensor:
    """Decode this rank's pages into a partial block (see the module doc)."""
    _require_cuda(q, "q")
    B, Hq, D = q.shape
    rows = B * Hq
    if block is None:
        block = torch.empty(block_floats(rows, D), dtype=torch.float32, device=q.device)
    elif block.dtype != torch.float32 or not block.is_contiguous() or block.numel() != block_floats(rows, D):
        raise ValueError("block must be a contiguous fp32 tensor of rows*(D+2) floats")
    paged_decode(q, pool, page_table, page_counts, page_tags, tag_map, tag_default, sm_scale,
                 partial=block_views(block, rows, D), num_splits=num_splits, kernel=kernel)
    return block


def decode_exchange(q: torch.Tensor, pool: PagePool, page_table: torch.Tensor, page_counts: Optional[torch.Tensor],
                    page_tags: torch.Tensor, tag_map: Sequence[int], x: "PeerExchange",
                    tag_default: int = N.FMT_SKIP, sm_scale: Optional[float] = None, num_splits: int = 0) -> None:
    """Decode this rank's pages with the push fused in (``iak_decode_exchange``): the
    decode kernel stores every query row's partial into slot ``x.rank`` of every
    rank's receive array and raises this rank's flags; ``x.merge(out)`` follows."""
    import ctypes
    _require_cuda(q, "q")
    if q.dim() != 3 or q.stride(-1) != 1:
        raise ValueError("q must be a [B, Hq, D] tensor with a contiguous last dim")
    if page_table.dtype != torch.int32 or page_table.stride(-1) != 1:
        page_table = page_table.to(torch.int32).contiguous()
    if page_counts is not None and (page_counts.dtype != torch.int32 or page_counts.stride(-1) != 1):
        page_counts = page_counts.to(torch.int32).contiguous()
    pools, args = _decode_structs(q, pool, page_table, page_counts, page_tags, tag_map, tag_default, sm_scale,
                                  None, None, num_splits, "tensor")
    L = N.lib()
    nbytes = ctypes.c_size_t(0)
    N.check(L.iak_decode_workspace_size(ctypes.byref(pools), ctypes.byref(args), ctypes.byref(nbytes)),
            "iak_decode_workspace_size")
    ws = _workspace(q.device, nbytes.value)
    N.check(L.iak_decode_exchange(ctypes.byref(pools), ctypes.byref(args), ctypes.byref(x.x),
                                  None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(),
                                  _stream(q.device)), "iak_decode_exchange")


def merge_partial_blocks(blocks: torch.Tensor, rows: int, head_dim: int,
                         out: Optional[torch.Tensor] = None, out_dtype=torch.float32) -> torch.Tensor:
    """LSE-merge ``S`` partial blocks ([S, rows*(D+2)] or flat) -> [rows, D]."""
    _require_cuda(blocks, "blocks")
    blk = block_floats(rows, head_dim)
    if blocks.dtype != torch.float32 or not blocks.is_contiguous() or blocks.numel() % blk or blocks.numel() == 0:
        raise ValueError("blocks must be a contiguous fp32 tensor of S * rows*(D+2) floats")
    parts = blocks.numel() // blk
    if out is None:
        out = torch.empty((rows, head_dim), dtype=out_dtype, device=blocks.device)
    if out.dim() < 2 or out.stride(-1) != 1 or out.numel() != rows * head_dim or out.dtype not in _DT:
        raise ValueError("out must hold rows x head_dim floats with a contiguous last dim")
    o2 = out.view(rows, head_dim)
    N.check(N.lib().iak_merge_partial_blocks(blocks.data_ptr(), parts, rows, head_dim, o2.data_ptr(),
                                             _DT[out.dtype], o2.stride(0), _stream(blocks.device)),
            "iak_merge_partial_blocks")
    return out


class _DeviceArray:
    """Minimal __cuda_array_interface__ wrapper to view raw device memory as a tensor."""

    def __init__(self, ptr: int, n: int, device: torch.device):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}
        self.device = device


class PeerExchange:
    """Exchange areas of all ranks mapped into this process over CUDA IPC, for
    the NVLink peer-store exchange of partial blocks (``iak_exchange_*``).

    Collective to construct (every rank of ``group``); afterwards a step is
    decode into ``staging`` (this rank's partial block), ``push()`` (stores it
    into every rank's area over NVLink and raises this rank's flags) and
    ``merge(out)`` (bounded wait for every rank, then the LSE merge).  The
    epoch counter lives in device memory, so a step can be captured in a CUDA
    graph and replayed.  ``check()`` raises if any wait ran out."""

    def __init__(self, rows: int, head_dim: int, device: torch.device, group=None, timeout_us: int = 2_000_000):
        import ctypes
        import torch.distributed as dist
        self.dist, self.group = dist, group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        if self.world > N.MAX_PEERS:
            raise ValueError(f"peer exchange supports at most {N.MAX_PEERS} ranks")
        self.rows, self.head_dim, self.device, self.timeout_us = rows, head_dim, device, timeout_us
        L = N.lib()
        nbytes = ctypes.c_size_t(0)
        N.check(L.iak_exchange_area_bytes(self.world, rows, head_dim, ctypes.byref(nbytes)), "iak_exchange_area_bytes")
        handle = (ctypes.c_uint8 * 64)()
        own = ctypes.c_void_p(0)
        with torch.cuda.device(device):
            N.check(L.iak_ipc_alloc(nbytes.value, ctypes.byref(own), handle), "iak_ipc_alloc")
        self._own = own.value
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened = []
        x = N.PeerExchange()
        with torch.cuda.device(device):
            for r in range(self.world):
                if r == self.rank:
                    x.areas[r] = self._own
                    continue
                ptr = ctypes.c_void_p(0)
                buf = (ctypes.c_uint8 * 64).from_buffer_copy(handles[r])
                N.check(L.iak_ipc_open(buf, ctypes.byref(ptr)), "iak_ipc_open")
                x.areas[r] = ptr.value
                self._opened.append(ptr.value)
        x.rank, x.world, x.rows, x.head_dim = self.rank, self.world, rows, head_dim
        self.x = x
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        ptr = L.iak_exchange_staging_ptr(self._own, self.world, rows, head_dim)
        self.staging = torch.as_tensor(_DeviceArray(ptr, block_floats(rows, head_dim), device), device=device)

    def push(self) -> None:
        import ctypes
        N.check(N.lib().iak_exchange_push(ctypes.byref(self.x), _stream(self.device)), "iak_exchange_push")

    def merge(self, out: torch.Tensor) -> torch.Tensor:
        import ctypes
        o2 = out.view(self.rows, self.head_dim)
        N.check(N.lib().iak_exchange_merge(ctypes.byref(self.x), o2.data_ptr(), _DT[out.dtype], o2.stride(0),
                                           self.status.data_ptr(), self.timeout_us, _stream(self.device)),
                "iak_exchange_merge")
        return out

    def check(self) -> None:
        """Raise if a bounded wait for a peer ran out (synchronises the device)."""
        if int(self.status.item()):
            raise RuntimeError("peer exchange: a rank's partial block did not arrive within the timeout")

    def close(self) -> None:
        L = N.lib()
        with torch.cuda.device(self.device):
            torch.cuda.synchronize(self.device)
            for ptr in self._opened:
                L.iak_ipc_close(ptr)
            self._opened = []
            if self._own:
                L.iak_ipc_free(self._own)
                self._own = 0
        self.staging = None


class SequenceShardedDecoder:
    """Per-rank driver of the sharded decode: owns the send / receive blocks
    so that repeated steps allocate nothing.

    ``decode(q, pool, local_table, local_counts, tags, tag_map)`` decodes the
    rank's pages (``local_table`` indexes this rank's ``pool``), all-gathers
    the partial blocks over ``group`` and returns the merged [B, Hq, D]
    output on every rank.  Every rank must call it with the same q shape."""

    def __init__(self, group=None, transport: str = "nccl"):
        import torch.distributed as dist
        if transport not in ("nccl", "p2p"):
            raise ValueError("transport must be 'nccl' or 'p2p'")
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.transport = transport
        self._send = None
        self._recv = None
        self._x = None

    def _buffers(self, rows, D, device):
        n = block_floats(rows, D)
        if self._send is None or self._send.numel() != n or self._send.device != device:
            self._send = torch.empty(n, dtype=torch.float32, device=device)
            self._recv = torch.empty(self.world * n, dtype=torch.float32, device=device)
        return self._send, self._recv

    def exchange(self, send: torch.Tensor, recv: Optional[torch.Tensor] = None) -> torch.Tensor:
        """All-gather this rank's flat partial block -> [world * block] in rank
        order (the block itself when world == 1)."""
        if self.world == 1:
            return send
        if recv is None:
            recv = torch.empty(self.world * send.numel(), dtype=send.dtype, device=send.device)
        self.dist.all_gather_into_tensor(recv, send, group=self.group)
        return recv

    def peer_exchange(self, rows: int, head_dim: int, device) -> PeerExchange:
        if self._x is None or self._x.rows != rows or self._x.head_dim != head_dim:
            if self._x is not None:
                self._x.close()
            self._x = PeerExchange(rows, head_dim, device, self.group)
        return self._x

    def close(self) -> None:
        if self._x is not None:
            self._x.close()
            self._x = None

    def decode(self, q, pool, local_table, local_counts, page_tags, tag_map, tag_default=N.FMT_SKIP,
               sm_scale=None, out=None, num_splits: int = 0, kernel: str = "auto"):
        B, Hq, D = q.shape
        rows = B * Hq
        if out is None:
            out = torch.empty(q.shape, dtype=q.dtype, device=q.device)
        if self.transport == "p2p":
            x = self.peer_exchange(rows, D, q.device)
            if kernel != "generic" and pool.page_size == 16 and D in (64, 128) and q.dtype != torch.float32 \
                    and pool.scale_mode != "channel" and (pool.scale_mode == "page" or D == 128):
                # the decode kernel stores each row's partial into every rank's receive slot over
                # NVLink and raises this rank's flags itself; one bounded-wait + merge launch follows
                decode_exchange(q, pool, local_table, local_counts, page_tags, tag_map, x, tag_default, sm_scale,
                                num_splits)
            else:
                # decode into this rank's staging block, then push it to every rank
                decode_partial_block(q, pool, local_table, local_counts, page_tags, tag_map, tag_default, sm_scale,
                                     block=x.staging, num_splits=num_splits, kernel=kernel)
                x.push()
            return x.merge(out)
        send, recv = self._buffers(rows, D, q.device)
        decode_partial_block(q, pool, local_table, local_counts, page_tags, tag_map, tag_default, sm_scale,
                             block=send, num_splits=num_splits, kernel=kernel)
        blocks = self.exchange(send, recv)
        merge_partial_blocks(blocks, rows, D, out=out)
        return out
