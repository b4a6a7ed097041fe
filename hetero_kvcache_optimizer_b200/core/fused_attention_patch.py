"""GQA-aware fused attention hook for HuggingFace models.

Rebuilds the fused path of ``patch_model_for_fused_attention``
(reference: src/core/fused_attention_patch.py:33-210). The reference swaps
``torch.nn.functional.scaled_dot_product_attention`` for a mixed bf16 / Triton
version fed from ``cache._dram_quant_kv``; it has no GQA, and HF models reach
their attention through transformers' ``ALL_ATTENTION_FUNCTIONS`` rather than
that module attribute.

Here the context manager registers an attention implementation with
transformers' ``AttentionInterface`` and selects it on every config of the model
while the context is open. For a decode step (one query position, inference,
head_dim 128, G = Hq / Hkv <= 8) of a layer that a ``FusedHeteroCache`` holds,
the attention is one launch of the fused INT4 decode kernel over that layer's
[sink ; INT4 body ; tail] (``cache.attend``); the key/value tensors HF passes in
are not read. Every other call (prefill, training, other shapes, layers the
cache does not hold) goes to the implementation the model had before.

The fused path attends to every cached token of every sequence: batches must
hold sequences of equal length (no padding mask), as the cache does.
"""
from __future__ import annotations

import contextlib
from typing import Any, Dict, List

import torch
from transformers import AttentionInterface
from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

FUSED_ATTENTION_NAME = "hetero_kv_fused"


def _all_configs(model: torch.nn.Module) -> List[Any]:
    """Every config object of the model (module configs and their sub-configs), once."""
    found: Dict[int, Any] = {}

    def visit(cfg):
        if cfg is None or id(cfg) in found or not hasattr(cfg, "_attn_implementation_internal"):
            return
        found[id(cfg)] = cfg
        for key in getattr(cfg, "sub_configs", {}) or {}:
            visit(getattr(cfg, key, None))

    visit(getattr(model, "config", None))
    for mod in model.modules():
        visit(getattr(mod, "config", None))
    return list(found.values())


@contextlib.contextmanager
def patch_model_for_fused_attention(model: torch.nn.Module, cache, enable_fused: bool = True):
    """Route the model's decode-step attention through ``cache.attend`` (the fused
    INT4 kernel) while the context is open; see the module docstring.

    Usage (``self_healing=False``: the cache then hands HF only its HBM tokens,
    and no step dequantises the INT4 body for a stock attention)::

        cache = FusedHeteroCache(num_layers=model.config.num_hidden_layers, self_healing=False, ...)
        with patch_model_for_fused_attention(model, cache):
            out = model.generate(input_ids, past_key_values=cache, max_new_tokens=64)
    """
    if not enable_fused:
        yield
        return
    configs = _all_configs(model)
    original = {id(c): c._attn_implementation_internal for c in configs}

    def fallback(module):
        name = original.get(id(getattr(module, "config", None)))
        if name is None or name == FUSED_ATTENTION_NAME:
            name = "sdpa"
        from transformers.models.llama.modeling_llama import eager_attention_forward
        return ALL_ATTENTION_FUNCTIONS.get_interface(name, eager_attention_forward)

    def fused_attention(module, query, key, value, attention_mask, dropout: float = 0.0, scaling=None, **kwargs):
        layer = getattr(module, "layer_idx", None)
        fused = (query.shape[2] == 1 and not module.training and layer is not None
                 and query.shape[-1] == 128 and query.shape[1] % key.shape[1] == 0
                 and query.shape[1] // key.shape[1] <= 8 and cache.holds_layer(layer))
        if not fused:
            return fallback(module)(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                    **kwargs)
        out = cache.attend(query, layer, sm_scale=scaling)  # [B, Hq, 1, 128] in query.dtype
        return out.transpose(1, 2), None                     # [B, 1, Hq, 128], as HF's interfaces

    AttentionInterface.register(FUSED_ATTENTION_NAME, fused_attention)
    for c in configs:
        c._attn_implementation_internal = FUSED_ATTENTION_NAME
    try:
        yield
    finally:
        for c in configs:
            c._attn_implementation_internal = original[id(c)]
