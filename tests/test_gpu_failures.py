"""Failure detection, made to happen without a GPU fault or hang:

* the host-side bounded event wait (hkv_event_wait) gives up with
  HKV_ERR_TIMEOUT while the stream is busy with a bounded spin kernel, then
  succeeds once it has finished;
* the device-side bounded wait every kernel uses (mbarrier phase with a time
  limit) runs out when nothing arrives: the self-test kernel returns, the
  device error word reports HKV_DEVERR_TIMEOUT, the call returns
  HKV_ERR_DEVICE and the context stays usable (a decode afterwards is right);
* a missing page (page table entry -1) and a page id past the pool are
  skipped and reported as HKV_DEVERR_BAD_PAGE by the decode kernel and the
  quantiser; a write past the body's capacity is refused on the host
  (HKV_ERR_CAPACITY) or reported as HKV_DEVERR_CAPACITY by the append kernel.
Injected host-side failures of the DRAM tier live in test_gpu_dropins.py.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from tests.hkv_testutil import dequant_side, t16

pytestmark = pytest.mark.gpu
K, V = 0, 1


@pytest.fixture(scope="module")
def hkv():
    from hetero_kvcache_optimizer_b200 import kvstore
    return kvstore


@pytest.fixture(scope="module")
def L():
    from hetero_kvcache_optimizer_b200 import _lib
    _lib.device_error(clear=True)
    return _lib


def test_event_wait_times_out_then_completes(L):
    from hetero_kvcache_optimizer_b200.policy.prefetcher import PagePrefetcher
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        torch.cuda._sleep(int(4e8))  # a bounded spin of ~0.2 s on the device
        ev = torch.cuda.Event()
        ev.record(s)
    with pytest.raises(L.HkvError) as info:
        PagePrefetcher.host_wait(ev, timeout_us=2000)
    assert info.value.status == L.HKV_ERR_TIMEOUT
    PagePrefetcher.host_wait(ev, timeout_us=10_000_000)
    assert ev.query()


def test_device_bounded_wait_runs_out_and_context_survives(hkv, L):
    assert hkv.selftest_bounded_wait(20_000_000, arrive=True) == L.HKV_OK
    assert L.device_error() == 0
    assert hkv.selftest_bounded_wait(20_000_000, arrive=False) == L.HKV_ERR_DEVICE
    assert L.device_error() & L.DEVERR_TIMEOUT
    assert L.device_error() == 0  # cleared by the read above
    assert L.load().hkv_selftest_bounded_wait(0, 0, None) == L.HKV_ERR_ARG
    assert L.load().hkv_selftest_bounded_wait(2_000_000_000, 0, None) == L.HKV_ERR_ARG
    # the context is usable: a decode afterwards matches the oracle
    k, v = ko.make_kv(3, 1, 2, 300)
    store = hkv.Int4KVStore(1, 2, 300)
    hkv.prefill(store, t16(k), t16(v))
    q = ko.make_q(3, 1, 8).astype(np.float16).astype(np.float32)
    out = hkv.decode(t16(q), store, None).cpu().numpy()
    ref = ko.decode_attention(q, dequant_side(store, K, 300), dequant_side(store, V, 300))
    assert ko.rel_err(out, ref) < 2e-3
    assert L.device_error() == 0


def test_missing_and_out_of_pool_pages_are_reported(hkv, L):
    B, Hkv, S = 1, 2, 600
    k, v = ko.make_kv(4, B, Hkv, S)
    store = hkv.Int4KVStore(B, Hkv, 768, fmt="ref", num_pages=8)
    store.page_table.copy_(torch.arange(6, dtype=torch.int32).reshape(2, 3).cuda())
    hkv.prefill(store, t16(k), t16(v))
    assert L.device_error() == 0
    q = t16(ko.make_q(4, B, Hkv * 4))
    hkv.decode(q, store, None)
    assert L.device_error() == 0
    for bad in (-1, 8, 1 << 30):
        store.page_table[1, 2] = bad
        hkv.decode(q, store, None)
        assert L.device_error() & L.DEVERR_BAD_PAGE, bad
        hkv.quantize_pack(t16(k[:, :, :10]), store, K, 520)  # lands in the bad page
        assert L.device_error() & L.DEVERR_BAD_PAGE, bad
    store.page_table[1, 2] = 5
    out = hkv.decode(q, store, None)
    assert L.device_error() == 0 and torch.isfinite(out).all()


def test_capacity_refused_or_reported(hkv, L):
    B, Hkv = 1, 2
    store = hkv.Int4KVStore(B, Hkv, 256)
    x = t16(ko.make_kv(5, B, Hkv, 64)[0])
    with pytest.raises(L.HkvError) as info:
        hkv.quantize_pack(x, store, K, 256 - 10)  # host-side start: refused before launch
    assert info.value.status == L.HKV_ERR_CAPACITY
    # a full body: the append kernel has nowhere to put the evicted row
    dense = hkv.DenseKV(B, Hkv, 8)
    dense.set_lengths(8)
    store.set_lengths(256)
    kn = t16(ko.make_kv(6, B, Hkv, 1)[0][:, :, 0])
    hkv.append_kv(kn, kn, dense, 4, store)
    assert L.device_error() & L.DEVERR_CAPACITY
    assert int(store.lengths[0]) == 257 or int(store.lengths[0]) == 256
