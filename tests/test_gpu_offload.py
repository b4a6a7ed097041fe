"""Tiered offload (config 3): pages prefetched layer-ahead from pinned host
memory give exactly the attention of the same pages held resident in HBM."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("window", [None, 2])
def test_prefetched_pages_match_resident(window):
    from hetero_kvcache_optimizer_b200 import _lib, kvstore as kv
    from hetero_kvcache_optimizer_b200.offload import TieredOffloadDecoder
    dev = torch.device("cuda", 0)
    Lyr, B, Hq, Hkv, R, C = 3, 2, 8, 2, 2, 5
    dec = TieredOffloadDecoder(Lyr, B, Hq, Hkv, resident_pages=R, cold_pages=C, window_pages=window,
                               sink=16, recent=48, device=dev)
    gen = torch.Generator(device=dev).manual_seed(11)
    dec.fill(gen)
    q = torch.randn(Lyr, B, Hq, 128, device=dev, generator=gen).bfloat16()
    out = torch.empty(Lyr, B, Hq, 128, device=dev)
    for _ in range(2):  # two steps: the second one reuses both staging areas
        out.fill_(float("nan"))
        dec.step(q, out, transfer=True)
        torch.cuda.synchronize()
        W, U = dec.window, dec.units
        host = dec.host.to(dev).view(U, C, dec.page_bytes)
        for l in range(Lyr):
            ref_store = kv.Int4KVStore(B, Hkv, (R + W) * 256, fmt=dec.fmt, group=dec.group, device=dev)
            pages = ref_store.pool.view(U, ref_store.max_pages, dec.page_bytes)
            res = dec.pool[l * U * R:(l + 1) * U * R].view(U, R, dec.page_bytes)
            pages[:, :R] = res
            pages[:, R:R + W] = host[:, C - W:]
            ref_store.set_lengths((R + W) * 256)
            d = dec.dense[l]
            ref = kv.decode(q[l], ref_store, d, dense_len=d.len_hint)
            assert torch.equal(out[l], ref), l
    assert _lib.device_error() == 0
    assert dec.prefetcher.bytes_submitted >= 2 * Lyr * dec.stage_pages * dec.page_bytes
