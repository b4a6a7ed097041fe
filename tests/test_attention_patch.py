"""Host logic of the HF attention hook (core/fused_attention_patch.py) on CPU:
a tiny random-init Llama whose decode steps go through ``cache.attend`` inside
the context (here a stand-in cache computing the same attention in torch, so
the logits must match the stock model's), prefill through the original
implementation, and the model's configuration restored afterwards."""
import pytest
import torch
from transformers import LlamaConfig, LlamaForCausalLM
from transformers.cache_utils import DynamicCache

from hetero_kvcache_optimizer_b200.core.fused_attention_patch import (FUSED_ATTENTION_NAME,
                                                                        patch_model_for_fused_attention)


class _TorchAttendCache(DynamicCache):
    """DynamicCache whose ``attend`` is plain fp32 GQA attention over its own K/V."""

    def __init__(self):
        super().__init__()
        self.calls = []

    def holds_layer(self, layer_idx):
        return layer_idx < len(self.layers) and self.layers[layer_idx].is_initialized

    def attend(self, q, layer_idx, sm_scale=None):
        self.calls.append((layer_idx, tuple(q.shape)))
        k, v = self.layers[layer_idx].keys.float(), self.layers[layer_idx].values.float()
        g = q.shape[1] // k.shape[1]
        k, v = k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1)
        s = torch.matmul(q.float(), k.transpose(-1, -2)) * sm_scale
        return torch.matmul(torch.softmax(s, dim=-1), v).to(q.dtype)


def _model():
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=97, hidden_size=512, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=128,
                      max_position_embeddings=256, attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).eval()


def _decode(model, cache, ids, steps):
    logits = []
    with torch.no_grad():
        out = model(input_ids=ids, past_key_values=cache, use_cache=True)
        nxt = out.logits[:, -1:].argmax(-1)
        for _ in range(steps):
            out = model(input_ids=nxt, past_key_values=cache, use_cache=True)
            logits.append(out.logits[:, -1])
            nxt = out.logits[:, -1:].argmax(-1)
    return torch.stack(logits)


def test_decode_steps_route_through_attend():
    model = _model()
    ids = torch.randint(0, 97, (2, 11), generator=torch.Generator().manual_seed(1))
    ref = _decode(model, DynamicCache(), ids, 4)
    cache = _TorchAttendCache()
    with patch_model_for_fused_attention(model, cache):
        assert model.config._attn_implementation == FUSED_ATTENTION_NAME
        got = _decode(model, cache, ids, 4)
    assert model.config._attn_implementation == "sdpa"
    # 2 layers x 4 decode steps, query [B, Hq, 1, 128]; the prefill took the stock path
    assert cache.calls == [(l, (2, 4, 1, 128)) for _ in range(4) for l in range(2)]
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4)


def test_disabled_patch_changes_nothing():
    model = _model()
    cache = _TorchAttendCache()
    with patch_model_for_fused_attention(model, cache, enable_fused=False):
        assert model.config._attn_implementation == "sdpa"
        _decode(model, cache, torch.randint(0, 97, (1, 5)), 2)
    assert cache.calls == []
