"""Drop-in for the reference's Hugging Face hook, ``hf_patch.py:16-180``:
``patch_model(model, layout_fn)`` routes the attention of every attention
module through ``reference.semantic_block_attention`` (this build's CUDA
selected-block attention) whenever ``layout_fn(layer_idx)`` returns a layout.

As in the reference: a module counts as attention when it has the
q/k/v/o (Llama-style) or c_attn/c_proj (GPT-2-style) projections, or its class
name contains "attention" / "attn" and it has children; the layer index is the
first integer component of its name; inside the patched ``forward``,
``torch.nn.functional.scaled_dot_product_attention`` is replaced by the
selected-block attention (non-causal, the reference's call), and an ``_attn``
method, where present, is replaced the same way.  The reference's per-call
savings print uses its cost model (out of scope here); this hook prints the
selected / total key counts when ``verbose``.
"""

from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .block_metadata import BlockLayout
from .reference import semantic_block_attention

_LLAMA_PROJ = frozenset({"q_proj", "k_proj", "v_proj", "o_proj"})
_GPT2_PROJ = frozenset({"c_attn", "c_proj"})


def _layer_index(name: str) -> int:
    return next((int(part) for part in name.split(".") if part.isdigit()), 0)


def _is_attention_module(module: nn.Module) -> bool:
    children = {n for n, _ in module.named_children()}
    if _LLAMA_PROJ <= children or _GPT2_PROJ <= children:
        return True
    cls = type(module).__name__.lower()
    return ("attention" in cls or "attn" in cls) and bool(children)


def _patch_forward(module: nn.Module, name: str, layer: int, layout_fn, verbose: bool) -> None:
    original = module.forward

    def forward(*args, **kwargs):
        layout = layout_fn(layer)
        if layout is None:
            return original(*args, **kwargs)
        saved = F.scaled_dot_product_attention

        def sdpa(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, **kw):
            if verbose:
                print(f"  [{name}] KV: {key.size(-2)} -> {layout.selected_token_count()} tokens")
            return semantic_block_attention(query, key, value, layout, causal=False)

        F.scaled_dot_product_attention = sdpa
        try:
            return original(*args, **kwargs)
        finally:
            F.scaled_dot_product_attention = saved

    module.forward = forward


def _patch_attn(module: nn.Module, layer: int, layout_fn) -> None:
    if not hasattr(module, "_attn"):
        return
    original = module._attn

    def _attn(query, key, value, attention_mask=None, head_mask=None) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        layout = layout_fn(layer)
        if layout is None:
            return original(query, key, value, attention_mask, head_mask)
        return semantic_block_attention(query, key, value, layout, causal=False), None

    module._attn = _attn


def patch_model(model: nn.Module, layout_fn: Callable[[int], Optional[BlockLayout]], verbose: bool = True) -> nn.Module:
    count = 0
    for name, module in model.named_modules():
        if _is_attention_module(module):
            layer = _layer_index(name)
            _patch_forward(module, name, layer, layout_fn, verbose)
            _patch_attn(module, layer, layout_fn)
            count += 1
            if verbose:
                print(f"  Patched {name} (layer {layer})")
    if verbose:
        print(f"Patched {count} attention modules.")
    return model
