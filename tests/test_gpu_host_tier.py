"""The host (DRAM) tier of HeteroKVManager's INT4 body (memory/host_tier.py) and
the reference's adaptive self-healing retrievals (src/memory/manager.py:823-1056):

* with ``hbm_body_pages`` set, most of the body lives in pinned host memory;
  ``attend`` stages a layer's host pages (layer-ahead) and reads them through
  the page table: the output equals, bit for bit, that of a manager holding
  the whole body in HBM, and the oracle within 2e-3 * ||ref|| per row, through
  prefill and through decode steps that move pages to the host;
* ``get_dram_chunks_quantized_adaptive`` / ``decompress_dram_chunks_adaptive``
  return the top-w chunks by attention score, in eviction order, bit-exact with
  the reference quantiser; ``FusedHeteroCache`` serves paths A and B with them.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from tests.test_gpu_manager import GROUP, SINK, TAIL, _oracle_context, _seq

pytestmark = pytest.mark.gpu
TOL = 2e-3


def _pair(layers=2, resident=2, cap=4096):
    from hetero_kvcache_optimizer_b200.memory.manager import HeteroKVManager
    kw = dict(num_layers=layers, sink_tokens=SINK, hbm_budget_tokens=SINK + TAIL, group_size=GROUP,
              body_capacity=cap)
    return HeteroKVManager(**kw, hbm_body_pages=resident), HeteroKVManager(**kw)


def test_host_tier_attention_equals_all_in_hbm():
    B, H, G, S = 2, 4, 4, 64 + 2000 + TAIL
    tiered, plain = _pair()
    seqs = [_seq(10 + l, B, H, S) for l in range(2)]
    for l, (k, v) in enumerate(seqs):
        for m in (tiered, plain):
            m.update(l, k.cuda(), v.cuda(), mode="prefill")
    summ = tiered.memory_summary()["host_tier"]
    # 2000 body tokens = 8 pages per unit; 2 stay in HBM, 6 live on the host
    assert summ["host_pages"] == [6 * B * H] * 2 and summ["device_body_pages"] == [2 * B * H] * 2
    q = torch.randn(B, H * G, 128, generator=torch.Generator().manual_seed(3)).half().cuda()
    k_all = [s[0] for s in seqs]
    v_all = [s[1] for s in seqs]
    for step in range(0, 520):
        if step in (0, 1, 255, 256, 519):
            for l in range(2):
                a = tiered.attend(l, q)
                b = plain.attend(l, q)
                torch.cuda.synchronize()
                assert torch.equal(a, b), (step, l)
                ref_k, ref_v = _oracle_context(k_all[l].float().numpy(), v_all[l].float().numpy(), SINK, TAIL,
                                               GROUP)
                ref = ko.decode_attention(q.float().cpu().numpy(), ref_k, ref_v)
                assert ko.rel_err(a.float().cpu().numpy(), ref) < TOL, (step, l)
        for l in range(2):
            kn, vn = _seq(1000 + step * 2 + l, B, H, 1)
            for m in (tiered, plain):
                m.update(l, kn.cuda(), vn.cuda(), mode="decode", seq_offset=S + step)
            k_all[l] = torch.cat([k_all[l], kn], dim=2)
            v_all[l] = torch.cat([v_all[l], vn], dim=2)
    # 520 decode steps: every step evicts one token, the body grew by 520 tokens
    summ = tiered.memory_summary()["host_tier"]
    assert summ["host_pages"][0] == (tiered.count_dram_tokens(0) // 256 + 1 - 2) * B * H
    assert summ["host_pages"][0] > summ["device_body_pages"][0]
    assert summ["d2h_bytes"] > 0 and summ["h2d_bytes"] > 0
    # the full-retrieval path reads through the tier as well
    kd, vd, n = tiered.decompress_dram_chunks(0)
    kp, vp, n2 = plain.decompress_dram_chunks(0)
    assert n == n2 and torch.equal(kd, kp) and torch.equal(vd, vp)
    from hetero_kvcache_optimizer_b200 import _lib
    assert _lib.device_error() == 0


def test_adaptive_retrieval_top_w_in_eviction_order():
    from hetero_kvcache_optimizer_b200.memory.manager import HeteroKVManager
    B, H = 1, 2
    m = HeteroKVManager(num_layers=1, sink_tokens=SINK, hbm_budget_tokens=SINK + TAIL, group_size=GROUP,
                        body_capacity=4096)
    k, v = _seq(30, B, H, 1400)
    # chunked prefill: every chunk after the first evicts its overflow as one DRAM chunk
    bounds = [0, 500, 700, 950, 1400]
    for a, b in zip(bounds[:-1], bounds[1:]):
        m.update(0, k[:, :, a:b].cuda(), v[:, :, a:b].cuda(), mode="prefill", seq_offset=a)
    keys = [key for key in m._chunk_eviction_order if key.startswith("l0_")]
    assert len(keys) == 4
    # body token ranges of the chunks, in eviction order
    ranges, t = [], SINK
    for key in keys:
        n = m._chunk_tokens[key]
        ranges.append((t, t + n))
        t += n
    # the scores decide the pick; the result keeps eviction order
    scores = {keys[0]: 0.1, keys[1]: 0.9, keys[2]: 0.05, keys[3]: 0.5}
    m._chunk_attention_scores.update(scores)
    q = m.get_dram_chunks_quantized_adaptive(0, window_size=2)
    picked = [1, 3]
    kk = np.concatenate([k[:, :, ranges[i][0]:ranges[i][1]].float().numpy() for i in picked], axis=2)
    vv = np.concatenate([v[:, :, ranges[i][0]:ranges[i][1]].float().numpy() for i in picked], axis=2)
    for name, x in (("k", kk), ("v", vv)):
        c, s, z = ko.quantize_ref(x, GROUP)
        assert np.array_equal(q[name + "_data"].cpu().numpy(), c), name
        assert np.array_equal(q[name + "_scales"].cpu().numpy(), s), name
        assert np.array_equal(q[name + "_zps"].cpu().numpy(), z), name
    dk, dv, n = m.decompress_dram_chunks_adaptive(0, window_size=2)
    assert n == kk.shape[2] and dk.dtype == torch.bfloat16
    ref = ko.dequantize_ref(*ko.quantize_ref(kk, GROUP), GROUP).reshape(kk.shape)
    # the reference decompresses straight to bf16 here (manager.py:893-894)
    assert torch.equal(dk.cpu(), torch.from_numpy(ref).to(torch.bfloat16))
    # no window given: the controller's w (w_min = 2 on a first call) picks the same two
    q2 = m.get_dram_chunks_quantized_adaptive(0)
    assert torch.equal(q2["k_data"], q["k_data"])
    # every chunk: the reference's _get_dram_kv_quantized, in eviction order
    allq = m._get_dram_kv_quantized(0)
    assert allq["k_data"].shape[2] == sum(b - a for a, b in ranges)
    assert m.get_dram_chunks_quantized_adaptive(0, window_size=100)["k_data"].shape[2] == allq["k_data"].shape[2]


def test_fused_cache_adaptive_paths():
    from hetero_kvcache_optimizer_b200.core.engine_wrapper import FusedHeteroCache
    B, H = 1, 2
    k, v = _seq(40, B, H, 900, dtype=torch.bfloat16)
    for triton in (True, False):
        cache = FusedHeteroCache(num_layers=1, sink_tokens=SINK, keep_tail=SINK + TAIL, device="cuda:0",
                                 group_size=GROUP, body_capacity=4096, adaptive_self_healing=True,
                                 enable_triton=triton)
        for a, b in ((0, 400), (400, 900)):
            cache.update(k[:, :, a:b].cuda(), v[:, :, a:b].cuda(), 0)
        kn, vn = _seq(41, B, H, 1, dtype=torch.bfloat16)
        rk, rv = cache.update(kn.cuda(), vn.cuda(), 0)
        m = cache._manager
        chunks = [key for key in m._chunk_eviction_order if key.startswith("l0_")]
        assert len(chunks) == 2
        if triton:  # path A: INT4 chunks on the device, [sink ; tail] returned as is
            assert cache._dram_quant_kv is not None and cache._dram_quant_kv["k_data"].is_cuda
            assert rk.shape[2] == SINK + TAIL
        else:  # path B: the top-w chunks (w = 2: both) dequantised in front
            total = sum(m._chunk_tokens[c] for c in chunks)
            assert rk.shape[2] == total + SINK + TAIL
            assert cache.get_seq_length(0) == SINK + TAIL + total
