"""GPU parity of the multi-layer decode engine (decode_engine.TieredKVDecoder):
per layer and step, append (new token -> recent ring, oldest ring row -> INT4
body) then split-KV attention, eagerly and as one captured CUDA graph replayed
every step (the path bench.py times). After each step the output must equal the
oracle attention over what the cache then holds: the sink and ring rows (fp16)
and the INT4 body read back from the pages.

Tolerance (benchmark spec): max |out - ref| <= 2e-3 * ||ref||_2 per (b, head).
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from tests.hkv_testutil import dequant_side, t16

pytestmark = pytest.mark.gpu
TOL = 2e-3
K, V = 0, 1


def _oracle_step(eng, q: torch.Tensor) -> np.ndarray:
    """[L, B, Hq, 128] attention over every layer's current cache contents."""
    outs = []
    for l in range(eng.num_layers):
        st, d = eng.stores[l], eng.dense[l]
        nb = int(st.lengths[0].item())
        nd = int(d.lengths[0].item())
        kd = np.concatenate([dequant_side(st, K, nb), d.k[:, :, :nd].float().cpu().numpy()], axis=2)
        vd = np.concatenate([dequant_side(st, V, nb), d.v[:, :, :nd].float().cpu().numpy()], axis=2)
        outs.append(ko.decode_attention(q[l].float().cpu().numpy(), kd, vd))
    return np.stack(outs)


def _engine(fmt, group, fused=True):
    from hetero_kvcache_optimizer_b200.decode_engine import TieredKVDecoder
    L_, B, Hq, Hkv, S = 2, 2, 8, 2, 300
    eng = TieredKVDecoder(L_, B, Hq, Hkv, sink=16, recent=64, body_capacity=1024, fmt=fmt, group=group,
                          fused_append=fused)
    k, v = ko.make_kv(7, B, Hkv, S)
    for l in range(L_):
        eng.prefill_layer(l, t16(k * (1 + 0.1 * l)), t16(v * (1 - 0.1 * l)))
    return eng


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("fmt,group", [("fp16min", 32), ("ref", 32), ("fp16min", 128)])
def test_engine_steps_eager_and_graph(fmt, group, fused):
    """Eager steps and graph replays; fused: one decode-append launch per layer,
    else append_kv then decode."""
    rng = np.random.default_rng(11)
    eager, graph = _engine(fmt, group, fused), _engine(fmt, group, fused)
    L_, B, Hq, Hkv = eager.num_layers, eager.batch, eager.q_heads, eager.kv_heads
    graph.capture(max_steps=4)
    q_s, kn_s, vn_s, out_s = graph.static_buffers
    for step in range(3):
        q = torch.from_numpy(rng.standard_normal((L_, B, Hq, 128)).astype(np.float32)).cuda().bfloat16()
        kn = torch.from_numpy(rng.standard_normal((L_, B, Hkv, 128)).astype(np.float32)).cuda().half()
        vn = torch.from_numpy(rng.standard_normal((L_, B, Hkv, 128)).astype(np.float32)).cuda().half()
        out_e = eager.step(q, kn, vn).cpu().numpy()
        q_s.copy_(q)
        kn_s.copy_(kn)
        vn_s.copy_(vn)
        graph.replay()
        torch.cuda.synchronize()
        out_g = out_s.cpu().numpy()
        ref = _oracle_step(eager, q)
        assert ko.rel_err(out_e, ref) < TOL, (fmt, group, step, "eager")
        assert ko.rel_err(out_g, ref) < TOL, (fmt, group, step, "graph")
        # both engines hold the same cache after the step (pool bytes past the
        # body length are never written and may differ)
        for l in range(L_):
            assert torch.equal(eager.stores[l].lengths, graph.stores[l].lengths)
            assert torch.equal(eager.dense[l].ring_head, graph.dense[l].ring_head)
            nb = int(eager.stores[l].lengths[0].item())
            for role in (K, V):
                assert np.array_equal(dequant_side(eager.stores[l], role, nb), dequant_side(graph.stores[l], role, nb))
            assert torch.equal(eager.dense[l].k, graph.dense[l].k)
            assert torch.equal(eager.dense[l].v, graph.dense[l].v)


def test_pipelined_host_step_matches_graph():
    """step_host over the engine's own pinned buffers (per-layer copies on side
    streams inside the captured graph) gives exactly the plain graph's outputs."""
    rng = np.random.default_rng(12)
    a, b = _engine("fp16min", 32), _engine("fp16min", 32)
    L_, B, Hq, Hkv = a.num_layers, a.batch, a.q_heads, a.kv_heads
    a.capture(max_steps=4)
    b.capture(max_steps=4)
    b.capture_host()
    hq, hk, hv, ho = b.host_buffers
    q_s, kn_s, vn_s, out_s = a.static_buffers
    for step in range(3):
        q = torch.from_numpy(rng.standard_normal((L_, B, Hq, 128)).astype(np.float32)).bfloat16()
        kn = torch.from_numpy(rng.standard_normal((L_, B, Hkv, 128)).astype(np.float32)).half()
        vn = torch.from_numpy(rng.standard_normal((L_, B, Hkv, 128)).astype(np.float32)).half()
        q_s.copy_(q)
        kn_s.copy_(kn)
        vn_s.copy_(vn)
        a.replay()
        hq.copy_(q)
        hk.copy_(kn)
        hv.copy_(vn)
        b.step_host(hq, hk, hv, ho)
        torch.cuda.synchronize()
        assert torch.equal(out_s.cpu(), ho), step
        assert a.body_len == b.body_len


def test_engine_many_query_heads_per_kv_head():
    """16 query heads per KV head: the engine runs the two launches (append, then
    the attention in groups of 8 heads), eager and replayed, against the oracle."""
    from hetero_kvcache_optimizer_b200.decode_engine import TieredKVDecoder
    L_, B, Hq, Hkv, S = 2, 2, 32, 2, 300
    rng = np.random.default_rng(13)
    engs = []
    for _ in range(2):
        eng = TieredKVDecoder(L_, B, Hq, Hkv, sink=16, recent=64, body_capacity=1024, fmt="fp16min", group=32)
        assert not eng.fused_append
        k, v = ko.make_kv(9, B, Hkv, S)
        for l in range(L_):
            eng.prefill_layer(l, t16(k), t16(v))
        engs.append(eng)
    eager, graph = engs
    graph.capture(max_steps=3)
    q_s, kn_s, vn_s, out_s = graph.static_buffers
    for step in range(2):
        q = torch.from_numpy(rng.standard_normal((L_, B, Hq, 128)).astype(np.float32)).cuda().bfloat16()
        kn = torch.from_numpy(rng.standard_normal((L_, B, Hkv, 128)).astype(np.float32)).cuda().half()
        vn = torch.from_numpy(rng.standard_normal((L_, B, Hkv, 128)).astype(np.float32)).cuda().half()
        out_e = eager.step(q, kn, vn).cpu().numpy()
        q_s.copy_(q)
        kn_s.copy_(kn)
        vn_s.copy_(vn)
        graph.replay()
        torch.cuda.synchronize()
        ref = _oracle_step(eager, q)
        assert ko.rel_err(out_e, ref) < TOL, step
        assert ko.rel_err(out_s.cpu().numpy(), ref) < TOL, step
    with pytest.raises(ValueError):
        TieredKVDecoder(1, B, Hq, Hkv, sink=16, recent=64, body_capacity=1024, fused_append=True)
