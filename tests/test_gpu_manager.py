"""HeteroKVManager / FusedHeteroCache drop-ins (reference src/memory/manager.py,
src/core/engine_wrapper.py): zone bookkeeping, INT4 eviction bit-exact with
KVCompressor, and the fused attention over [sink ; INT4 body ; tail] against
the oracle's dequant-then-softmax on the same logical sequence."""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu

SINK, TAIL, GROUP = 64, 256, 128


def _oracle_context(k_all, v_all, sink, tail, group):
    """The manager's logical context for a sequence of S tokens: sink and the
    last `tail` tokens exact, everything between INT4 (reference format)."""
    S = k_all.shape[2]
    ns = min(S, sink)
    nt = min(S - ns, tail)
    body = slice(ns, S - nt)

    def deq(x):
        if x.shape[2] == 0:
            return x
        c, s, z = ko.quantize_ref(x, group)
        return ko.dequantize_ref(c, s, z, group).reshape(x.shape)

    k = np.concatenate([k_all[:, :, :ns], deq(k_all[:, :, body]), k_all[:, :, S - nt:]], axis=2)
    v = np.concatenate([v_all[:, :, :ns], deq(v_all[:, :, body]), v_all[:, :, S - nt:]], axis=2)
    return k, v


def _check_attend(mgr, layer, q16, k_all, v_all, tol=2e-3):
    ref_k, ref_v = _oracle_context(k_all, v_all, SINK, TAIL, GROUP)
    ref = ko.decode_attention(q16.float().cpu().numpy(), ref_k, ref_v)
    out = mgr.attend(layer, q16).float().cpu().numpy()
    err = np.abs(out - ref).max(axis=-1)
    nrm = np.linalg.norm(ref, axis=-1)
    assert np.all(err <= tol * nrm), float((err / nrm).max())


def _seq(seed, B, H, S, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn(B, H, S, 128, generator=g).to(dtype)
    v = torch.randn(B, H, S, 128, generator=g).to(dtype)
    return k, v


def test_manager_prefill_decode_and_fused_attention():
    from hetero_kvcache_optimizer_b200.memory.manager import HeteroKVManager
    B, H, G, S = 2, 4, 4, 700
    mgr = HeteroKVManager(num_layers=2, sink_tokens=SINK, hbm_budget_tokens=SINK + TAIL, group_size=GROUP,
                          body_capacity=2048)
    k, v = _seq(0, B, H, S)
    kd, vd = k.cuda(), v.cuda()
    ok, ov = mgr.update(0, kd, vd, mode="prefill")
    assert ok.shape[2] == S  # prefill returns the full sequence (as the reference)
    hk, hv = mgr.get_hbm_kv(0)
    assert torch.equal(hk.cpu(), torch.cat([k[:, :, :SINK], k[:, :, S - TAIL:]], dim=2))
    assert mgr.count_dram_tokens(0) == S - SINK - TAIL
    # the legacy DRAM entry is KVCompressor.compress of the evicted body, bit-exact
    e = mgr._dram_table["l0_e0"]
    c, s, z = ko.quantize_ref(k[:, :, SINK:S - TAIL].float().numpy(), GROUP)
    assert np.array_equal(e["k_data"].cpu().numpy(), c.reshape(e["k_data"].shape))
    assert np.array_equal(e["k_scales"].cpu().numpy().reshape(-1), s)
    assert np.array_equal(e["k_zps"].cpu().numpy().reshape(-1), z)
    q = torch.randn(B, H * G, 128, generator=torch.Generator().manual_seed(9)).half().cuda()
    _check_attend(mgr, 0, q, k.float().numpy(), v.float().numpy())
    # decode: 300 new tokens; once the tail is full every step evicts one token to INT4
    k_all, v_all = k, v
    for step in range(300):
        kn, vn = _seq(100 + step, B, H, 1)
        rk, rv = mgr.update(0, kn.cuda(), vn.cuda(), mode="decode", seq_offset=S + step)
        k_all = torch.cat([k_all, kn], dim=2)
        v_all = torch.cat([v_all, vn], dim=2)
        if step in (0, 77, 299):
            T = k_all.shape[2]
            assert torch.equal(rk.cpu(), torch.cat([k_all[:, :, :SINK], k_all[:, :, T - TAIL:]], dim=2))
            _check_attend(mgr, 0, q, k_all.float().numpy(), v_all.float().numpy())
    assert mgr.get_seq_offset(0) == S + 300
    assert mgr.count_dram_tokens(0) == k_all.shape[2] - SINK - TAIL
    summ = mgr.memory_summary()
    assert summ["hbm_tokens"] == SINK + TAIL and summ["int4_tokens"] == k_all.shape[2] - SINK - TAIL
    # compress(): the tail joins the INT4 body
    n = mgr.compress(0)
    assert n == TAIL and mgr.count_dram_tokens(0) == k_all.shape[2] - SINK
    from hetero_kvcache_optimizer_b200 import _lib
    assert _lib.device_error() == 0


def test_manager_chunked_prefill():
    from hetero_kvcache_optimizer_b200.memory.manager import HeteroKVManager
    B, H, G = 1, 8, 4
    mgr = HeteroKVManager(num_layers=1, sink_tokens=SINK, hbm_budget_tokens=SINK + TAIL, group_size=GROUP,
                          body_capacity=4096, kv_format="ref")
    k, v = _seq(3, B, H, 1000, dtype=torch.bfloat16)
    chunks = [(0, 100), (100, 450), (450, 1000)]
    for a, b in chunks:
        rk, _ = mgr.update(0, k[:, :, a:b].cuda(), v[:, :, a:b].cuda(), mode="prefill", seq_offset=a)
    assert mgr.count_dram_tokens(0) == 1000 - SINK - TAIL
    hk, _ = mgr.get_hbm_kv(0)
    assert torch.equal(hk.cpu(), torch.cat([k[:, :, :SINK], k[:, :, 1000 - TAIL:]], dim=2))
    q = torch.randn(B, H * G, 128, generator=torch.Generator().manual_seed(5)).bfloat16().cuda()
    _check_attend(mgr, 0, q, k.float().numpy(), v.float().numpy())


def test_fused_hetero_cache_dropin():
    from hetero_kvcache_optimizer_b200.core.engine_wrapper import FusedHeteroCache
    B, H, G, S = 1, 4, 4, 600
    cache = FusedHeteroCache(num_layers=1, sink_tokens=SINK, keep_tail=SINK + TAIL, device="cuda:0",
                             group_size=GROUP, body_capacity=2048)
    k, v = _seq(7, B, H, S, dtype=torch.bfloat16)
    ok, _ = cache.update(k.cuda(), v.cuda(), 0)
    assert ok.shape[2] == S and cache.seen_tokens == S
    body = S - SINK - TAIL
    kn, vn = _seq(8, B, H, 1, dtype=torch.bfloat16)
    cache.update(kn.cuda(), vn.cuda(), 0)  # first decode step: the swap-in count is refreshed after it
    kn2, vn2 = _seq(9, B, H, 1, dtype=torch.bfloat16)
    rk, rv = cache.update(kn2.cuda(), vn2.cuda(), 0)
    # self-healing full retrieval: [INT4 body dequantised ; sink ; tail]
    nb = cache._manager.count_dram_tokens(0)
    assert rk.shape[2] == nb + SINK + TAIL
    assert cache.get_seq_length(0) == SINK + TAIL + nb
    assert cache.get_mask_sizes(torch.arange(1), 0) == (SINK + TAIL + nb, 0)
    k_all = torch.cat([k, kn, kn2], dim=2)
    v_all = torch.cat([v, vn, vn2], dim=2)
    q = torch.randn(B, H * G, 1, 128, generator=torch.Generator().manual_seed(2)).bfloat16().cuda()
    out = cache.attend(q, 0, out_dtype=torch.float32)
    ref_k, ref_v = _oracle_context(k_all.float().numpy(), v_all.float().numpy(), SINK, TAIL, GROUP)
    ref = ko.decode_attention(q[:, :, 0].float().cpu().numpy(), ref_k, ref_v)
    err = np.abs(out[:, :, 0].cpu().numpy() - ref).max(axis=-1)
    assert np.all(err <= 2e-3 * np.linalg.norm(ref, axis=-1))
    # fused attention on one swapped DRAM chunk (the prefill body, key l0_e0)
    qs = q[:, :H]  # one query head per KV head: the legacy single-query API has no GQA
    o2 = cache.fused_attn_on_swapped(qs, "l0_e0")
    kb, vb = k[:, :, SINK:SINK + body].float().numpy(), v[:, :, SINK:SINK + body].float().numpy()
    dk = ko.dequantize_ref(*ko.quantize_ref(kb, GROUP), GROUP).reshape(kb.shape)
    dv = ko.dequantize_ref(*ko.quantize_ref(vb, GROUP), GROUP).reshape(vb.shape)
    ref2 = ko.decode_attention(qs[:, :, 0].float().cpu().numpy(), dk, dv)
    err2 = np.abs(o2[:, :, 0].float().cpu().numpy() - ref2).max(axis=-1)
    assert np.all(err2 <= 2e-3 * np.linalg.norm(ref2, axis=-1))
