"""Drop-in for the reference's exact-token selected-block attention,
``reference.py:82-130`` ``semantic_block_attention`` (the function the
reference's HF SDPA hook calls, ``hf_patch.py:61-99``), on CUDA tensors.

Selected tokens: every token of the ALWAYS / ATTEND / RECENT / GLOBAL blocks
(``block_metadata.py:72-79``; scores do not select here), attended with causal
masks on their original positions (``reference.py:16-45``).  Runs in
``iak_prefill``; a query row that sees no key is 0 where the reference gives
NaN.  ATTEND blocks without a score are accepted (the reference scores them
with its BlockScorer before validating; the score does not change which tokens
this path attends to, so no scoring is done).
"""

from __future__ import annotations

from typing import Any, Dict, Tuple, Union

import torch

from .block_metadata import SELECTED_POLICIES, BlockLayout, BlockPolicy, SemanticBlock
from .triton_kernel import blocks_attention


def semantic_block_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layout: BlockLayout,
                             causal: bool = False, return_debug: bool = False, threshold: float = 0.5
                             ) -> Union[torch.Tensor, Tuple[torch.Tensor, Dict[str, Any]]]:
    kv_tokens = k.size(-2)
    # validate as the reference does after resolving missing ATTEND scores
    BlockLayout([SemanticBlock(b.name, b.start, b.end, b.policy,
                               0.0 if (b.policy == BlockPolicy.ATTEND and b.score is None) else b.score)
                 for b in layout.blocks]).validate(kv_tokens)
    blocks = [b for b in layout.blocks if b.policy in SELECTED_POLICIES]
    out = blocks_attention(q, k, v, blocks, causal)
    if return_debug:
        count = sum(b.end - b.start for b in blocks)
        return out, {"selected_token_count": count, "selected_block_names": [b.name for b in blocks],
                     "total_kv_tokens": kv_tokens, "selected_kv_tokens": count}
    return out
