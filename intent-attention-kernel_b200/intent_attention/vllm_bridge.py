"""Drop-in for the reference's vLLM bridge, ``vllm_bridge.py:12-76``
``semantic_paged_attention``: attention of ``query`` [T, H, D] over the
selected blocks of a vLLM-layout paged cache (``key_cache`` / ``value_cache``
[num_blocks, H, head_size, block_size]) on CUDA.

Selection as the reference: non-SKIP blocks, ATTEND blocks with a score < 0.5
dropped (no score keeps them), logical cache blocks ``start // block_size ..
ceil(end / block_size)`` (clipped to the table), mapped through
``block_table`` and de-duplicated in first-occurrence order; whole cache
blocks are attended.  Causal masking follows the reference's
``dense_attention(causal=True)`` over the concatenated keys: query i sees the
first i + 1 of them.

The reference concatenates the blocks as [1, N, H, D] and calls
``dense_attention`` on [1, T, H, D] queries, whose matmul contracts over the
head axis (it attends across heads, and only runs when T == N or T == 1);
here every head attends over the selected tokens, which is what the bridge
describes.  The selected blocks are gathered into this build's page layout
(64-token pages at most, the tensor-core kernel's limit) and attended by
``iak_prefill``.
"""

from __future__ import annotations

from typing import List

import torch

from .block_metadata import BlockLayout, BlockPolicy
from .paged import PagePool, make_tag_map, paged_prefill


def selected_physical_blocks(layout: BlockLayout, block_table: torch.Tensor, block_size: int) -> List[int]:
    """vllm_bridge.py:37-58: physical cache blocks of the selected logical ranges, first occurrence first."""
    num_logical = int(block_table.shape[0])
    table = block_table.tolist()
    out: dict = {}
    for blk in layout.blocks:
        if blk.policy == BlockPolicy.SKIP:
            continue
        if blk.policy == BlockPolicy.ATTEND and blk.score is not None and blk.score < 0.5:
            continue
        for logical in range(blk.start // block_size, min((blk.end + block_size - 1) // block_size, num_logical)):
            out.setdefault(int(table[logical]), None)
    return list(out)


def semantic_paged_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                             block_table: torch.Tensor, layout: BlockLayout, block_size: int = 128,
                             causal: bool = True) -> torch.Tensor:
    if not (query.is_cuda and key_cache.is_cuda and value_cache.is_cuda):
        raise RuntimeError("this build runs only on CUDA tensors (no CPU fallback)")
    T, H, D = query.shape
    if key_cache.dim() != 4 or key_cache.shape[1] != H or key_cache.shape[2] != D or key_cache.shape[3] != block_size:
        raise ValueError("key_cache must be [num_blocks, heads, head_size, block_size]")
    phys = selected_physical_blocks(layout, block_table, block_size)
    if not phys:
        return torch.zeros(T, H, D, device=query.device, dtype=query.dtype)
    # split cache blocks into pages of at most 64 tokens
    PS = block_size
    while PS > 64 and PS % 2 == 0:
        PS //= 2
    per = block_size // PS
    n = len(phys) * per
    idx = torch.tensor(phys, dtype=torch.int64, device=query.device)

    def gather(cache: torch.Tensor) -> torch.Tensor:
        # [n_blk, H, D, BS] -> [H, n_blk, BS, D] -> pages [H * n, PS, D]
        x = cache[idx].permute(1, 0, 3, 2)
        return x.reshape(H, len(phys) * per, PS, D).reshape(H * n, PS, D).contiguous()

    pool = PagePool.allocate(H * n, PS, D, ["F16"], "page", query.device)
    pool.quantize_(gather(key_cache), gather(value_cache), ["F16"] * (H * n))
    table = torch.arange(H * n, dtype=torch.int32, device=query.device).view(1, H, n)
    positions = (torch.arange(n, dtype=torch.int32, device=query.device) * PS)[None, None, :].expand(1, H, n)
    tags = torch.ones(H * n, dtype=torch.uint8, device=query.device)
    q = query.permute(1, 0, 2).unsqueeze(0)                       # [1, H, T, D]
    out = paged_prefill(q, pool, table, None, tags, make_tag_map({1: "F16"}), causal=causal,
                        page_positions=positions.contiguous(), out_dtype=query.dtype)
    return out[0].permute(1, 0, 2).contiguous()
