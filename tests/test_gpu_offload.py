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


@pytest.mark.parametrize("window,delta", [(4, 1), (4, 2), (3, 0), (4, 4)])
@pytest.mark.parametrize("mode", ["eager", "graph-copy", "graph-gather"])
def test_sliding_window_cache_matches_resident(window, delta, mode):
    """Residency-aware window: the pages cached in HBM across steps plus the
    ``delta`` new ones copied each step give exactly the attention of the same
    pages (resident pages, then the window's pages in window order) held in a
    plain store; the copies per step are the delta only. ``graph-*``: the steps
    replay CUDA graphs (two eager steps first, so the step starts > 0) whose page
    moves are copy nodes retargeted to each step's host rows (``copy``) or
    zero-copy gather kernels driven by the device step counter (``gather``)."""
    from hetero_kvcache_optimizer_b200 import _lib, kvstore as kv
    from hetero_kvcache_optimizer_b200.offload import SlidingWindowOffload
    dev = torch.device("cuda", 0)
    Lyr, B, Hq, Hkv, R, C = 3, 2, 8, 2, 2, 9
    dec = SlidingWindowOffload(Lyr, B, Hq, Hkv, resident_pages=R, cold_pages=C, window_pages=window,
                               delta=delta, sink=16, recent=48, device=dev)
    gen = torch.Generator(device=dev).manual_seed(12)
    dec.fill(gen)
    q = torch.randn(Lyr, B, Hq, 128, device=dev, generator=gen).bfloat16()
    out = torch.empty(Lyr, B, Hq, 128, device=dev)
    U, W = dec.units, dec.window
    host = dec.host.to(dev).view(C, U, dec.page_bytes).transpose(0, 1)  # page-major arena
    fetched0 = dec.fetched_pages
    graph = mode.startswith("graph")
    for s in range(12 if graph else 7):  # past the ring's period and around the cold set
        if graph and s == 2:
            dec.capture(q, out, transport=mode.split("-")[1])
        out.fill_(float("nan"))
        if graph and s >= 2:
            dec.replay(transfer=True)
        else:
            dec.step(q, out, transfer=True)
        torch.cuda.synchronize()
        win = [(s * delta + i) % C for i in range(W)]
        for l in range(Lyr):
            ref_store = kv.Int4KVStore(B, Hkv, (R + W) * 256, fmt=dec.fmt, group=dec.group, device=dev)
            pages = ref_store.pool.view(U, ref_store.max_pages, dec.page_bytes)
            pages[:, :R] = dec.pool[l * U * R:(l + 1) * U * R].view(U, R, dec.page_bytes)
            pages[:, R:R + W] = host[:, win]
            ref_store.set_lengths((R + W) * 256)
            d = dec.dense[l]
            ref = kv.decode(q[l], ref_store, d, dense_len=d.len_hint)
            assert torch.equal(out[l], ref), (s, l)
    assert _lib.device_error() == 0
    # after step 0, each step copies only the pages entering the window
    steps_after_first = 11 if graph else 6
    per_step = Lyr * U * delta
    assert dec.fetched_pages - fetched0 <= (steps_after_first + 2) * per_step + Lyr * U * delta
    assert dec.h2d_bytes_per_step() == per_step * dec.page_bytes
    # a layer's fetch is one run of pages (two where the ring or the cold set wraps)
    before = dec.prefetcher.bytes_submitted
    dec.prefetch(0, dec.step_idx)
    torch.cuda.synchronize()
    assert dec.prefetcher.bytes_submitted - before == U * delta * dec.page_bytes


def test_page_gather_kernel():
    """hkv_prefetch_gather: device id arrays, scattered pages, the step-counter
    shift with wrap-around, and ids outside the pools skipped with
    HKV_DEVERR_BAD_PAGE (checked in the kernel, nothing dereferenced)."""
    from hetero_kvcache_optimizer_b200 import _lib
    from hetero_kvcache_optimizer_b200.policy.prefetcher import PagePrefetcher
    dev = torch.device("cuda", 0)
    pb, nh, nd = 20480, 13, 11
    host = torch.randint(0, 256, (nh, pb), dtype=torch.uint8).pin_memory()
    pool = torch.zeros(nd, pb, dtype=torch.uint8, device=dev)
    pf = PagePrefetcher(host, pool)
    src = torch.tensor([12, 0, 5, 5, 7], dtype=torch.int32, device=dev)
    dst = torch.tensor([0, 3, 10, 4, 6], dtype=torch.int32, device=dev)
    pf.gather(src, dst)
    torch.cuda.synchronize()
    hd = host.to(dev)
    for s_, d_ in zip(src.tolist(), dst.tolist()):
        assert torch.equal(pool[d_], hd[s_])
    assert not pool[[1, 2, 5, 7, 8, 9]].any()
    # the step counter shifts the host pages: (src + (step + add) * mul) mod nh
    step = torch.tensor([4], dtype=torch.int64, device=dev)
    pool.zero_()
    pf.gather(src, dst, step=step, step_mul=3, step_add=1)
    torch.cuda.synchronize()
    for s_, d_ in zip(src.tolist(), dst.tolist()):
        assert torch.equal(pool[d_], hd[(s_ + 5 * 3) % nh])
    assert _lib.device_error() == 0
    # out-of-range ids: skipped and flagged, the valid entry still lands
    pool.zero_()
    bad_src = torch.tensor([nh, 2, -1], dtype=torch.int32, device=dev)
    bad_dst = torch.tensor([1, 2, 3], dtype=torch.int32, device=dev)
    pf.gather(bad_src, bad_dst)
    pf.gather(torch.tensor([1], dtype=torch.int32, device=dev), torch.tensor([nd], dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert torch.equal(pool[2], hd[2]) and not pool[1].any() and not pool[3].any()
    assert _lib.device_error(clear=True) & _lib.DEVERR_BAD_PAGE
    assert pf.bytes_submitted == (5 + 5 + 3 + 1) * pb
