"""intent_attention -- B200 (sm_100a) drop-in for the fused selected-quant
paged decode path of manishklach/intent-attention-kernel.

Exports the reference's hot-path surface (layout types, precision policy,
router + kernel metadata, the fused / six-tag / adaptive decode entry points
and their helpers) backed by libiak_b200.so, plus the B200 extensions
(``PagePool`` quantise-on-write pools, device metadata packing, split-KV
partial export / merge).  As in the reference package, the name
``fused_selected_quant_decode`` refers to the function (the submodule is
still importable with ``from intent_attention.fused_selected_quant_decode import ...``).
"""

from .block_metadata import BlockLayout, BlockPolicy, SemanticBlock
from .block_router import (
    BlockDecision,
    BlockRouter,
    RoutedBlock,
    RouterConfig,
    compute_block_scores,
    routing_to_kernel_metadata,
)
from .intent_quant import IntentQuantizer, KVPrecision, QuantPolicy
from .fused_selected_quant_decode import (
    FusedDecodeConfig,
    FusedKVPrecision,
    fused_selected_quant_decode,
    metadata_to_kernel_tensors,
)
from .triton_intent_quant_attention import (
    IntentQuantKernelConfig,
    TritonKVPrecision,
    fake_int8_pages_from_fp16,
    intent_quant_decode_attention_triton,
    is_cuda_available,
    is_triton_available,
    make_page_tables_from_selected_pages,
    make_precision_tensor,
)
from .triton_adaptive_format_attention import (
    AdaptiveFormatKernelConfig,
    AdaptivePageFormat,
    adaptive_format_decode_attention_triton,
    make_adaptive_page_tables,
)
from .paged import KVStage, PagePool, append_tokens, convert_pages, merge_partials, pack_metadata, paged_decode
from .device_router import LayoutBatch, RoutedPages, encode_layouts, route_layouts, route_pages
from .split_kv import (
    SequenceShardedDecoder,
    decode_partial_block,
    merge_partial_blocks,
    shard_bounds,
    shard_page_lists,
)

__all__ = [
    "BlockLayout", "BlockPolicy", "SemanticBlock",
    "BlockDecision", "BlockRouter", "RoutedBlock", "RouterConfig", "compute_block_scores",
    "routing_to_kernel_metadata",
    "IntentQuantizer", "KVPrecision", "QuantPolicy",
    "FusedDecodeConfig", "FusedKVPrecision", "fused_selected_quant_decode", "metadata_to_kernel_tensors",
    "IntentQuantKernelConfig", "TritonKVPrecision", "fake_int8_pages_from_fp16",
    "intent_quant_decode_attention_triton", "is_cuda_available", "is_triton_available",
    "make_page_tables_from_selected_pages", "make_precision_tensor",
    "AdaptiveFormatKernelConfig", "AdaptivePageFormat", "adaptive_format_decode_attention_triton",
    "make_adaptive_page_tables",
    "PagePool", "merge_partials", "pack_metadata", "paged_decode", "KVStage", "append_tokens", "convert_pages",
    "LayoutBatch", "RoutedPages", "encode_layouts", "route_layouts", "route_pages",
    "SequenceShardedDecoder", "decode_partial_block", "merge_partial_blocks", "shard_bounds", "shard_page_lists",
]
