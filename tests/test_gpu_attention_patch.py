"""GPU: a tiny random-init HF Llama decoding with FusedHeteroCache through the
attention hook (core/fused_attention_patch.py): every decode step's attention
is one fused INT4 decode launch over [sink ; INT4 body ; tail]. The reference
run uses the same hook and cache type, but its ``attend`` computes fp32 torch
attention over the cache's own contents (INT4 body dequantised, sink and ring
rows as stored); with the same token sequence fed to both (teacher forcing) the
logits must agree to the attention tolerance."""
import pytest
import torch
from transformers import LlamaConfig, LlamaForCausalLM

from hetero_kvcache_optimizer_b200 import kvstore as kv
from hetero_kvcache_optimizer_b200.core.engine_wrapper import FusedHeteroCache
from hetero_kvcache_optimizer_b200.core.fused_attention_patch import patch_model_for_fused_attention

pytestmark = pytest.mark.gpu


class _TorchAttendCache(FusedHeteroCache):
    def attend(self, q, layer_idx, sm_scale=None, out_dtype=None):
        m = self._manager
        nb, nd = m._body_len[layer_idx], m._dense_len[layer_idx]
        d = m._dense[layer_idx]
        k, v = d.k[:, :, :nd].float(), d.v[:, :, :nd].float()
        if nb:
            st = m._body[layer_idx]
            k = torch.cat([kv.dequantize_pack(st, 0, 0, nb, dtype=torch.float32), k], dim=2)
            v = torch.cat([kv.dequantize_pack(st, 1, 0, nb, dtype=torch.float32), v], dim=2)
        g = q.shape[1] // k.shape[1]
        k, v = k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1)
        s = torch.matmul(q.float(), k.transpose(-1, -2)) * sm_scale
        return torch.matmul(torch.softmax(s, dim=-1), v).to(out_dtype or q.dtype)


def _model():
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=97, hidden_size=1024, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                      max_position_embeddings=1024, attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).eval().to("cuda", torch.float16)


def _decode(model, cache, ids, steps):
    """Prefill ids[:, :-steps], then feed ids[:, -steps:] one token at a time."""
    logits = []
    with torch.no_grad():
        with patch_model_for_fused_attention(model, cache):
            model(input_ids=ids[:, :-steps], past_key_values=cache, use_cache=True)
            for i in range(steps):
                t = ids.shape[1] - steps + i
                out = model(input_ids=ids[:, t:t + 1], past_key_values=cache, use_cache=True)
                logits.append(out.logits[:, -1].float())
    return torch.stack(logits)


@pytest.mark.parametrize("group", [32, 128])
def test_fused_hook_matches_torch_attention_over_the_cache(group):
    model = _model()
    ids = torch.randint(0, 97, (2, 304), generator=torch.Generator().manual_seed(3)).cuda()
    kw = dict(num_layers=2, sink_tokens=16, keep_tail=64, device="cuda:0", group_size=group,
              enable_prefetch=False, self_healing=False)
    fused_cache = FusedHeteroCache(**kw)
    fused = _decode(model, fused_cache, ids, 4)
    ref = _decode(model, _TorchAttendCache(**kw), ids, 4)
    m = fused_cache._manager
    assert m._body_len[0] > 0 and m._body_len[1] > 0, "the context must reach the INT4 body"
    assert torch.isfinite(fused).all()
    torch.testing.assert_close(fused, ref, rtol=2e-2, atol=2e-2)
