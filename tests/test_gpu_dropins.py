"""The reference-facing drop-ins its callers use, against the oracle and the
reference's golden digests:

* AsyncPrefetcher.submit_prefetch_task / fetch_if_ready / clear / pending_keys
  (reference src/policy/prefetcher.py:47-122): both dict protocols, BF16 (K, V)
  bit-exact with the reference's decompress(...).to(bfloat16) on the same codes;
* HeteroKVManager.schedule_prefetch / swap_in / swap_in_quantized
  (src/memory/manager.py:233-348);
* DRAMStorageManager.store / store_entry / retrieve / remove /
  transfer_to_device and its capacity caps (src/memory/dram_storage.py:57-194);
* the legacy fused_dequant_attn_* signatures: repeated calls with unchanged
  INT4 tensors reuse one packed store, a modified tensor is repacked; the
  score-only fused_dequant_attention.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu

GROUP = 128


def _expected_bf16(codes: np.ndarray, scales: np.ndarray, zps: np.ndarray, group: int) -> torch.Tensor:
    """The reference's decompress(q, s, z) (fp16 target by default,
    kv_compressor.py:100-132) followed by .to(torch.bfloat16), prefetcher.py:82-83."""
    deq = ko.dequantize_ref(codes, scales.reshape(-1), zps.reshape(-1), group).reshape(codes.shape)
    return torch.from_numpy(deq).half().to(torch.bfloat16)


def _entry(seed, B=1, H=4, S=300, group=GROUP, pinned=True):
    k, v = ko.make_kv(seed, B, H, S)
    kq, ks, kz = ko.quantize_ref(k, group)
    vq, vs, vz = ko.quantize_ref(v, group)

    def host(x):
        t = torch.from_numpy(np.ascontiguousarray(x))
        return t.pin_memory() if pinned else t

    e = {"k_data": host(kq.reshape(k.shape)), "k_scales": host(ks), "k_zps": host(kz),
         "v_data": host(vq.reshape(v.shape)), "v_scales": host(vs), "v_zps": host(vz)}
    return e, (kq.reshape(k.shape), ks, kz), (vq.reshape(v.shape), vs, vz)


def test_async_prefetcher_split_protocol_bit_exact():
    from hetero_kvcache_optimizer_b200.policy.prefetcher import AsyncPrefetcher
    from hetero_kvcache_optimizer_b200.quantization.kv_compressor import KVCompressor
    pf = AsyncPrefetcher(torch.device("cuda"))
    comp = KVCompressor(group_size=GROUP)
    entries = {f"l0_e{i}": _entry(40 + i) for i in range(3)}
    for key, (e, _, _) in entries.items():
        pf.submit_prefetch_task(key, e, comp)
    assert sorted(pf.pending_keys) == sorted(entries)
    pf.submit_prefetch_task("l0_e0", entries["l0_e0"][0], comp)  # a second submit is a no-op
    assert len(pf.pending_keys) == 3
    for key, (_, kk, vv) in entries.items():
        got = pf.fetch_if_ready(key)
        assert got is not None
        k, v = got
        assert k.dtype == torch.bfloat16 and k.is_cuda
        assert torch.equal(k.cpu(), _expected_bf16(*kk, GROUP))
        assert torch.equal(v.cpu(), _expected_bf16(*vv, GROUP))
        assert pf.fetch_if_ready(key) is None  # popped
    assert pf.fetch_if_ready("missing") is None
    pf.submit_prefetch_task("x", {"unrelated": 1}, comp)  # neither protocol: ignored
    assert pf.pending_keys == []


def test_async_prefetcher_merged_protocol_and_clear():
    from hetero_kvcache_optimizer_b200.policy.prefetcher import AsyncPrefetcher
    from hetero_kvcache_optimizer_b200.quantization.kv_compressor import KVCompressor
    pf = AsyncPrefetcher(torch.device("cuda"))
    comp = KVCompressor(group_size=32)
    x, _ = ko.make_kv(5, 1, 2, 64)
    c, s, z = ko.quantize_ref(x, 32)
    data = {"q_data": torch.from_numpy(c.reshape(x.shape)).pin_memory(),
            "scales": torch.from_numpy(s).pin_memory(), "zps": torch.from_numpy(z).pin_memory()}
    pf.submit_prefetch_task("m", data, comp)
    k, v = pf.fetch_if_ready("m")
    assert k is v  # the merged protocol restores one tensor for both (prefetcher.py:83-91)
    assert torch.equal(k.cpu(), _expected_bf16(c.reshape(x.shape), s, z, 32))
    pf.submit_prefetch_task("m2", data, comp)
    pf.clear()
    assert pf.pending_keys == [] and pf.fetch_if_ready("m2") is None


def test_manager_swap_in_with_and_without_prefetch():
    """The prefill body is one DRAM entry (l0_e0); swap_in returns it as BF16
    (K, V) and removes it, whether schedule_prefetch ran first or not."""
    from hetero_kvcache_optimizer_b200.memory.manager import HeteroKVManager
    sink, tail, S = 16, 64, 400
    for prefetch in (True, False):
        mgr = HeteroKVManager(num_layers=1, sink_tokens=sink, hbm_budget_tokens=sink + tail, group_size=GROUP,
                              body_capacity=1024)
        k, v = ko.make_kv(61, 1, 4, S)
        mgr.update(0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), mode="prefill")
        key = "l0_e0"
        q = mgr.swap_in_quantized(0, key)
        assert q is not None and q["k_data"].is_cuda
        kb, vb = k[:, :, sink:S - tail], v[:, :, sink:S - tail]
        kc, ks, kz = ko.quantize_ref(kb, GROUP)
        vc, vs, vz = ko.quantize_ref(vb, GROUP)
        assert np.array_equal(q["k_data"].cpu().numpy().reshape(-1), kc.reshape(-1))
        assert np.array_equal(q["v_scales"].cpu().numpy().reshape(-1), vs)
        if prefetch:
            mgr.schedule_prefetch(key)
            assert key in mgr._prefetcher.pending_keys
        out = mgr.swap_in(0, key)
        assert out is not None
        assert torch.equal(out[0].cpu(), _expected_bf16(kc.reshape(kb.shape), ks, kz, GROUP))
        assert torch.equal(out[1].cpu(), _expected_bf16(vc.reshape(vb.shape), vs, vz, GROUP))
        assert mgr.swap_in(0, key) is None  # the entry left DRAM
        assert mgr.swap_in_quantized(0, key) is None
        mgr.schedule_prefetch("missing")  # unknown keys are ignored


def test_dram_storage_crud_and_transfer():
    from hetero_kvcache_optimizer_b200.memory.dram_storage import DRAMStorageManager
    dram = DRAMStorageManager()
    e, _, _ = _entry(70, pinned=False)
    dev = {k: t.cuda() for k, t in e.items()}
    nbytes = sum(t.element_size() * t.nelement() for t in e.values())
    assert dram.store("l0_e0", dev["k_data"], dev["k_scales"], dev["k_zps"],
                      dev["v_data"], dev["v_scales"], dev["v_zps"])
    assert dram.store_entry("l0_e1", e)
    assert dram.total_bytes == 2 * nbytes and dram.num_entries == 2
    assert dram.contains("l0_e0") and "l0_e1" in dram
    r = dram.retrieve("l0_e0")
    for k, t in e.items():
        assert r[k].device.type == "cpu" and r[k].is_pinned()
        assert torch.equal(r[k], t), k
    t = dram.transfer_to_device("l0_e1", torch.device("cuda"))
    torch.cuda.synchronize()
    for k, x in e.items():
        assert t[k].is_cuda and torch.equal(t[k].cpu(), x), k
    assert dram.transfer_to_device("nope", torch.device("cuda")) is None
    assert dram.retrieve("nope") is None and dram.remove("nope") is None
    popped = dram.remove("l0_e0")
    assert popped is not None and torch.equal(popped["k_data"], e["k_data"])
    assert dram.num_entries == 1 and dram.total_bytes == nbytes
    # re-storing a key replaces it without double counting
    assert dram.store_entry("l0_e1", e)
    assert dram.num_entries == 1 and dram.total_bytes == nbytes
    with pytest.raises(ValueError):
        dram.store_entry("bad", {"k_data": e["k_data"]})
    s = dram.memory_summary()
    assert s["num_entries"] == 1 and s["total_bytes"] == nbytes


def test_dram_storage_capacity_caps():
    """The caps refuse with False and leave the table unchanged
    (reference dram_storage.py:76-86 and :123-128)."""
    from hetero_kvcache_optimizer_b200.memory.dram_storage import DRAMStorageManager
    e, _, _ = _entry(71, pinned=False)
    nbytes = sum(t.element_size() * t.nelement() for t in e.values())
    by_count = DRAMStorageManager(max_entries=1)
    assert by_count.store_entry("a", e)
    assert not by_count.store_entry("b", e)
    assert not by_count.store("c", *[e[k] for k in ("k_data", "k_scales", "k_zps", "v_data", "v_scales", "v_zps")])
    assert by_count.keys == ["a"] and by_count.total_bytes == nbytes
    by_bytes = DRAMStorageManager(max_bytes=nbytes + nbytes // 2)
    assert by_bytes.store_entry("a", e)
    assert not by_bytes.store_entry("b", e)
    assert by_bytes.keys == ["a"] and by_bytes.total_bytes == nbytes


def test_dram_storage_pinned_alloc_failure_leaves_table_intact(monkeypatch):
    """An injected page-locked allocation failure (host side: the arena's
    allocator raises) propagates, and neither the entry being replaced nor the
    byte count changes."""
    from hetero_kvcache_optimizer_b200.memory import dram_storage as ds
    dram = ds.DRAMStorageManager()
    e, _, _ = _entry(72, pinned=False)
    nbytes = sum(t.element_size() * t.nelement() for t in e.values())
    assert dram.store_entry("a", e)
    calls = {"n": 0}
    real = ds._PinnedArena.alloc

    def failing(self, n):
        calls["n"] += 1
        if calls["n"] == 3:
            raise RuntimeError("injected: cudaHostAlloc failed")
        return real(self, n)

    monkeypatch.setattr(ds._PinnedArena, "alloc", failing)
    e2, _, _ = _entry(73, pinned=False)
    with pytest.raises(RuntimeError, match="injected"):
        dram.store_entry("a", e2)
    assert dram.keys == ["a"] and dram.total_bytes == nbytes
    assert torch.equal(dram.retrieve("a")["v_data"], e["v_data"])
    monkeypatch.setattr(ds._PinnedArena, "alloc", real)
    assert dram.store_entry("a", e2)
    assert torch.equal(dram.retrieve("a")["v_data"], e2["v_data"])


def test_legacy_decode_reuses_packed_store():
    from hetero_kvcache_optimizer_b200.quantization import _legacy
    from hetero_kvcache_optimizer_b200.quantization.fused_dequant_attn import fused_dequant_attn_decode
    k, v = ko.make_kv(81, 1, 4, 500)
    kq, ks, kz = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in ko.quantize_ref(k, 32))
    vq, vs, vz = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in ko.quantize_ref(v, 32))
    kq, vq = kq.reshape(k.shape), vq.reshape(v.shape)
    q = torch.from_numpy(ko.make_q(81, 1, 4).astype(np.float16)).cuda()[:, :, None, :]
    _legacy._STORE_CACHE.clear()
    a = fused_dequant_attn_decode(q, kq, ks, kz, vq, vs, vz)
    store = _legacy.build_store(kq, ks, kz, vq, vs, vz)
    assert len(_legacy._STORE_CACHE) == 1
    b = fused_dequant_attn_decode(q, kq, ks, kz, vq, vs, vz)
    assert torch.equal(a, b) and _legacy.build_store(kq, ks, kz, vq, vs, vz) is store
    kd = ko.dequantize_ref(*ko.quantize_ref(k, 32), 32).reshape(k.shape)
    vd = ko.dequantize_ref(*ko.quantize_ref(v, 32), 32).reshape(v.shape)
    ref = ko.decode_attention(q[:, :, 0].float().cpu().numpy(), kd, vd)
    assert ko.rel_err(a[:, :, 0].cpu().numpy(), ref) < 2e-3
    # an in-place change of the codes bumps the tensor's version: repacked
    vq.zero_()
    c = fused_dequant_attn_decode(q, kq, ks, kz, vq, vs, vz)
    assert _legacy.build_store(kq, ks, kz, vq, vs, vz) is not store
    vd0 = ko.dequantize_ref(np.zeros_like(vq.cpu().numpy()), vs.cpu().numpy(), vz.cpu().numpy(), 32)
    ref0 = ko.decode_attention(q[:, :, 0].float().cpu().numpy(), kd, vd0.reshape(v.shape))
    assert ko.rel_err(c[:, :, 0].cpu().numpy(), ref0) < 2e-3


@pytest.mark.parametrize("qdtype", [torch.float16, torch.bfloat16, torch.float32])
def test_legacy_score_function_vs_oracle(qdtype):
    """fused_dequant_attention: per-key scale/zero-point (the reference reshapes
    them to [seq_k], fused_dequant_attn.py:354-355), fp32 scores q . dequant(K)."""
    from hetero_kvcache_optimizer_b200.quantization.fused_dequant_attn import fused_dequant_attention
    from hetero_kvcache_optimizer_b200.quantization.kernels.fused_dequant_attn import (
        fused_dequant_attention as twin)
    S, D = 777, 128
    k, _ = ko.make_kv(91, 1, 1, S)
    c, s, z = ko.quantize_ref(k[0, 0], D)
    q = torch.from_numpy(ko.make_q(91, 1, 1)[0, 0]).to(qdtype)
    kd = ko.dequantize_ref(c, s, z, D).reshape(S, D)
    ref = kd.astype(np.float64) @ q.float().numpy().astype(np.float64)
    out = fused_dequant_attention(q.cuda(), torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda(),
                                  torch.from_numpy(z).cuda())
    assert out.dtype == torch.float32 and out.shape == (S,)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
    o2 = twin(q.cuda(), torch.from_numpy(c).cuda(), torch.from_numpy(s).cuda(), torch.from_numpy(z).cuda())
    assert o2.dtype == qdtype
    np.testing.assert_allclose(o2.float().cpu().numpy(), ref, rtol=1e-2, atol=1e-2 * np.abs(ref).max())
