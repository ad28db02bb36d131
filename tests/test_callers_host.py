"""Host logic of the prefill callers (no GPU): block selection, page lists
and row masks, the vLLM block mapping, and the HF module detection."""

import torch

from intent_attention import BlockLayout, BlockPolicy, SemanticBlock
from intent_attention.triton_kernel import (_compute_selected_page_ids, _threshold_blocks, block_pages_and_masks)
from intent_attention.vllm_bridge import selected_physical_blocks

import inputs as gi
from oracle import prefill as op


def _layout(spec):
    return BlockLayout([SemanticBlock(n, s, e, BlockPolicy[p], score=sc) for n, s, e, p, sc in spec])


def test_threshold_selection_matches_gpu_path_rule():
    lay = _layout([("a", 0, 10, "ALWAYS", None), ("b", 10, 20, "ATTEND", 0.4), ("c", 20, 30, "ATTEND", 0.6),
                   ("d", 30, 35, "SKIP", None), ("e", 35, 40, "RECENT", None), ("f", 40, 50, "ATTEND", 0.5)])
    assert [b.name for b in _threshold_blocks(lay, 0.5)] == ["a", "c", "e", "f"]
    assert _compute_selected_page_ids(lay, 50, 0.5, 16).tolist() == [0, 1, 2, 3]
    assert _compute_selected_page_ids(lay, 50, 0.7, 16).tolist() == [0, 2]


def test_row_masks_equal_the_oracle_layout_pages():
    for spec in (gi.E2E_LAYOUT, gi.PREFILL_PARTIAL_LAYOUT, gi.PREFILL_GAP_LAYOUT):
        for ps in (8, 16, 64):
            blocks = [b for b in _layout(spec).blocks if b.policy != BlockPolicy.SKIP]
            pages, masks = block_pages_and_masks(blocks, ps)
            ref_pages, ref_masks = op.layout_pages(spec, ps)
            assert pages == ref_pages.tolist()
            assert masks == [int(m) for m in ref_masks]


def test_vllm_block_selection():
    lay = _layout([("a", 0, 100, "ALWAYS", None), ("b", 100, 300, "ATTEND", 0.3), ("c", 300, 400, "ATTEND", None),
                   ("d", 400, 500, "SKIP", None), ("e", 500, 530, "RECENT", None)])
    table = torch.tensor([7, 3, 9, 1, 4], dtype=torch.int32)     # 5 logical blocks of 128
    # a -> logical 0; b dropped (score < 0.5); c (no score) -> logical 2, 3; e -> 3, 4 (4 clipped to the table)
    assert selected_physical_blocks(lay, table, 128) == [7, 9, 1, 4]


def test_hf_attention_module_detection():
    import torch.nn as nn
    from intent_attention.hf_patch import _is_attention_module, _layer_index

    class LlamaAttn(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = self.k_proj = self.v_proj = self.o_proj = nn.Identity()

    class SelfAttention(nn.Module):
        def __init__(self):
            super().__init__()
            self.proj = nn.Identity()

    class Leaf(nn.Module):
        pass

    assert _is_attention_module(LlamaAttn()) and _is_attention_module(SelfAttention())
    assert not _is_attention_module(Leaf()) and not _is_attention_module(nn.Linear(2, 2))
    assert _layer_index("model.layers.12.self_attn") == 12 and _layer_index("attn") == 0
