"""hkv_decode_append: the decode step's append and the attention over the
updated cache in ONE launch, against the two-launch path it replaces
(hkv_append_kv then hkv_decode_attn) and the CPU oracle:

* the cache afterwards is identical byte for byte: packed INT4 pages (the
  evicted row quantised by the same code), the dense sink/ring rows, and the
  state arrays (dense length, ring head, body length);
* the output is within the north-star tolerance, max |out - ref| <= 2e-3 *
  ||ref||_2 per (b, head), of the oracle's dequant-then-softmax over the cache
  after the append;
over the ring-filling, ring-evicting and no-ring regimes, ragged per-sequence
states, both formats, f16/bf16 caches, GQA 4/7/8 and grids from 1 CTA (one CTA
appends every unit) to one per SM.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from tests.hkv_testutil import dequant_side, t16

pytestmark = pytest.mark.gpu
TOL = 2e-3
K, V = 0, 1


@pytest.fixture(scope="module")
def hkv():
    from hetero_kvcache_optimizer_b200 import kvstore
    return kvstore


def _cache(hkv, seed, B, Hkv, body, sink, ring, dense_lens, fmt, group, dtype):
    """A store with `body` INT4 tokens and a dense segment of sink + ring rows,
    sequence b holding dense_lens[b] of them (ring head 0)."""
    k, v = ko.make_kv(seed, B, Hkv, body + sink + ring)
    store = hkv.Int4KVStore(B, Hkv, body + 1024, fmt=fmt, group=group, page_tokens=256)
    if body:
        hkv.prefill(store, t16(k[:, :, :body], dtype=dtype), t16(v[:, :, :body], dtype=dtype))
    store.set_lengths(body)
    dense = hkv.DenseKV(B, Hkv, sink + ring, dtype=dtype)
    dense.k.copy_(t16(k[:, :, body:], dtype=dtype))
    dense.v.copy_(t16(v[:, :, body:], dtype=dtype))
    dense.lengths.copy_(torch.tensor(dense_lens, dtype=torch.int32))
    dense.len_hint = sink + ring
    dense.ring_head.zero_()
    return store, dense


def _clone(hkv, store, dense):
    s2 = hkv.Int4KVStore(store.batch, store.kv_heads, store.capacity, fmt=store.fmt, group=store.group,
                         page_tokens=store.page_tokens)
    s2.pool.copy_(store.pool)
    s2.lengths.copy_(store.lengths)
    s2.len_hint = store.len_hint
    d2 = hkv.DenseKV(dense.batch, dense.kv_heads, dense.capacity, dtype=dense.dtype)
    d2.k.copy_(dense.k)
    d2.v.copy_(dense.v)
    d2.lengths.copy_(dense.lengths)
    d2.ring_head.copy_(dense.ring_head)
    d2.len_hint = dense.len_hint
    return s2, d2


def _oracle_out(q, store, dense):
    """Oracle attention over the cache as it stands: INT4 body tokens
    [0, body_len[b]) dequantised, dense rows [0, dense_len[b])."""
    bl = store.lengths.cpu().numpy()
    dl = dense.lengths.cpu().numpy()
    nb = int(bl.max())
    kd, vd = dequant_side(store, K, max(nb, 1)), dequant_side(store, V, max(nb, 1))
    dk, dv = dense.k.float().cpu().numpy(), dense.v.float().cpu().numpy()
    outs = []
    for b in range(q.shape[0]):
        kk = np.concatenate([kd[b:b + 1, :, :bl[b]], dk[b:b + 1, :, :dl[b]]], axis=2)
        vv = np.concatenate([vd[b:b + 1, :, :bl[b]], dv[b:b + 1, :, :dl[b]]], axis=2)
        outs.append(ko.decode_attention(q[b:b + 1], kk, vv))
    return np.concatenate(outs)


def _assert_same_cache(a_store, a_dense, b_store, b_dense):
    torch.cuda.synchronize()
    assert torch.equal(a_store.lengths, b_store.lengths)
    assert torch.equal(a_dense.lengths, b_dense.lengths)
    assert torch.equal(a_dense.ring_head, b_dense.ring_head)
    assert torch.equal(a_dense.k, b_dense.k) and torch.equal(a_dense.v, b_dense.v)
    # the INT4 pool, raw bytes of every page (both started from the same pool)
    assert torch.equal(a_store.pool, b_store.pool)


@pytest.mark.parametrize("fmt,group", [("fp16min", 32), ("ref", 32), ("fp16min", 128), ("ref", 64)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_fused_step_equals_two_launches(hkv, fmt, group, dtype):
    """Ragged states in one batch: sequence 0's ring is full (evicts), 1 fills
    its last free row, 2 fills a middle row, 3 evicts with an empty body."""
    B, Hkv, G, sink, ring = 4, 2, 4, 8, 40
    dense_lens = [sink + ring, sink + ring - 1, sink + 5, sink + ring]
    store, dense = _cache(hkv, 3, B, Hkv, 600, sink, ring, dense_lens, fmt, group, dtype)
    store.lengths[3] = 0  # sequence 3: nothing evicted yet
    s2, d2 = _clone(hkv, store, dense)
    rng = ko.rng_for(9)
    for step in range(3):
        # queries in the cache's dtype, as a model computes them (a bf16 model's
        # q is bf16: the dense tiles multiply q and P in the cache's dtype)
        qt = t16(rng.standard_normal((B, Hkv * G, 128), dtype=np.float32), dtype=dtype)
        q = qt.float().cpu().numpy()
        kn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
        vn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
        for ctas in ((0,) if step else (0, 1, 3)):
            if ctas != 0:  # replay the same step from the same state with another grid
                s3, d3 = _clone(hkv, store, dense)
                o3 = hkv.decode_append(qt, t16(kn, dtype=dtype), t16(vn, dtype=dtype), d3, sink, s3,
                                       ctas=ctas, body_len=601, dense_len=sink + ring)
                _assert_same_cache(s3, d3, *_clone_after(hkv, store, dense, kn, vn, sink, dtype))
                assert ko.rel_err(o3.cpu().numpy(), _oracle_out(q, s3, d3)) < TOL
                continue
            out = hkv.decode_append(qt, t16(kn, dtype=dtype), t16(vn, dtype=dtype), dense, sink, store,
                                    body_len=600 + step + 1, dense_len=sink + ring)
            hkv.append_kv(t16(kn, dtype=dtype), t16(vn, dtype=dtype), d2, sink, s2)
            ref2 = hkv.decode(qt, s2, d2, body_len=600 + step + 1, dense_len=sink + ring)
            _assert_same_cache(store, dense, s2, d2)
            oracle = _oracle_out(q, store, dense)
            assert ko.rel_err(ref2.cpu().numpy(), oracle) < TOL, ("two launches", fmt, group, step)
            assert ko.rel_err(out.cpu().numpy(), oracle) < TOL, ("fused", fmt, group, step)
    from hetero_kvcache_optimizer_b200 import _lib
    assert _lib.device_error() == 0


def _clone_after(hkv, store, dense, kn, vn, sink, dtype):
    """A clone of the cache advanced by the two-launch append."""
    s, d = _clone(hkv, store, dense)
    hkv.append_kv(t16(kn, dtype=dtype), t16(vn, dtype=dtype), d, sink, s)
    return s, d


@pytest.mark.parametrize("G", [1, 7, 8])
def test_fused_no_ring_and_gqa(hkv, G):
    """capacity == sink: every new token goes straight to the INT4 body."""
    B, Hkv, sink = 2, 3, 16
    store, dense = _cache(hkv, 4, B, Hkv, 300, sink, 0, [sink, sink], "ref", 32, torch.float16)
    s2, d2 = _clone(hkv, store, dense)
    rng = ko.rng_for(G)
    for step in range(4):
        q = rng.standard_normal((B, Hkv * G, 128), dtype=np.float32).astype(np.float16).astype(np.float32)
        kn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
        vn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
        out = hkv.decode_append(t16(q), t16(kn), t16(vn), dense, sink, store, body_len=300 + step + 1,
                                dense_len=sink, ctas=2)
        hkv.append_kv(t16(kn), t16(vn), d2, sink, s2)
        _assert_same_cache(store, dense, s2, d2)
        assert ko.rel_err(out.cpu().numpy(), _oracle_out(q, store, dense)) < TOL


def test_fused_many_steps_through_eviction(hkv):
    """200 fused steps from an empty ring: the ring fills, then every step
    evicts; the cache tracks the two-launch path exactly all the way."""
    B, Hkv, G, sink, ring = 2, 4, 4, 16, 48
    store, dense = _cache(hkv, 5, B, Hkv, 256, sink, ring, [sink, sink + 10], "fp16min", 32, torch.float16)
    s2, d2 = _clone(hkv, store, dense)
    rng = ko.rng_for(11)
    for step in range(200):
        q = rng.standard_normal((B, Hkv * G, 128), dtype=np.float32).astype(np.float16).astype(np.float32)
        kn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
        vn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
        out = hkv.decode_append(t16(q), t16(kn), t16(vn), dense, sink, store, body_len=256 + step + 1,
                                dense_len=sink + ring)
        hkv.append_kv(t16(kn), t16(vn), d2, sink, s2)
        if step % 50 == 49 or step in (0, 37, 38, 39):
            _assert_same_cache(store, dense, s2, d2)
            assert ko.rel_err(out.cpu().numpy(), _oracle_out(q, store, dense)) < TOL, step
    _assert_same_cache(store, dense, s2, d2)
    from hetero_kvcache_optimizer_b200 import _lib
    assert _lib.device_error() == 0


@pytest.mark.parametrize("fmt", ["fp16min", "ref"])
def test_fused_early_mode_layers_interleaved(hkv, fmt):
    """Early mode as a multi-layer step uses it: two layers' caches alternate on
    the stream, so the launch before each fused launch never writes its cache;
    the caches track the two-launch path exactly over 60 steps (the rings fill,
    then evict) and the outputs stay within tolerance of the oracle."""
    B, Hkv, G, sink, ring = 2, 4, 4, 16, 48
    caches = [_cache(hkv, 20 + l, B, Hkv, 500, sink, ring, [sink + ring - 3, sink + ring - 40], fmt, 32,
                     torch.float16) for l in range(2)]
    twins = [_clone(hkv, *c) for c in caches]
    rng = ko.rng_for(21)
    for step in range(60):
        for l in range(2):
            store, dense = caches[l]
            q = rng.standard_normal((B, Hkv * G, 128), dtype=np.float32).astype(np.float16).astype(np.float32)
            kn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
            vn = rng.standard_normal((B, Hkv, 128), dtype=np.float32)
            out = hkv.decode_append(t16(q), t16(kn), t16(vn), dense, sink, store, body_len=500 + step + 1,
                                    dense_len=sink + ring, early=True)
            hkv.append_kv(t16(kn), t16(vn), twins[l][1], sink, twins[l][0])
            if step in (0, 3, 45, 59):
                _assert_same_cache(store, dense, *twins[l])
                assert ko.rel_err(out.cpu().numpy(), _oracle_out(q, store, dense)) < TOL, (fmt, step, l)
    from hetero_kvcache_optimizer_b200 import _lib
    assert _lib.device_error() == 0


def test_fused_rejects_mismatched_state_arrays(hkv):
    from hetero_kvcache_optimizer_b200 import _lib as L
    store, dense = _cache(hkv, 6, 1, 2, 128, 8, 8, [16], "ref", 32, torch.float16)
    q = torch.zeros(1, 8, 128, dtype=torch.float16, device="cuda")
    kn = torch.zeros(1, 2, 128, dtype=torch.float16, device="cuda")
    other = torch.zeros(1, dtype=torch.int32, device="cuda")
    store.lengths, saved = other, store.lengths  # the attention would read other lengths than the append
    st = store.struct()
    store.lengths = saved
    import ctypes
    ds = dense.struct()
    ws = hkv.workspace(1 << 22, q.device)
    out = torch.empty(1, 8, 128, device="cuda")
    rc = L.load().hkv_decode_append(q.data_ptr(), L.DT_F16, q.stride(0), q.stride(1), kn.data_ptr(), kn.data_ptr(),
                                    kn.stride(0), kn.stride(1), ctypes.byref(st), ctypes.byref(ds), 8,
                                    dense.lengths.data_ptr(), dense.ring_head.data_ptr(), saved.data_ptr(), 1, 8, 2,
                                    128, 0.088, 0, ws.data_ptr(), ws.numel(), out.data_ptr(), L.DT_F32,
                                    out.stride(0), out.stride(1), 0, None)
    assert rc == L.HKV_ERR_ARG


def test_fused_refuses_more_ctas_than_sms(hkv):
    """A unit's last pipeline piece waits for the append job of another CTA, so
    every CTA must be resident at once: a grid larger than the SM count is
    refused before anything is launched, and the cache is left untouched."""
    store, dense = _cache(hkv, 7, 1, 2, 128, 8, 8, [16], "fp16min", 32, torch.float16)
    before = (store.pool.clone(), dense.k.clone(), store.lengths.clone(), dense.lengths.clone())
    q = torch.zeros(1, 8, 128, dtype=torch.float16, device="cuda")
    kn = torch.zeros(1, 2, 128, dtype=torch.float16, device="cuda")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    with pytest.raises(RuntimeError, match="ARG"):
        hkv.decode_append(q, kn, kn, dense, 8, store, ctas=sms + 1)
    torch.cuda.synchronize()
    after = (store.pool, dense.k, store.lengths, dense.lengths)
    assert all(torch.equal(a, b) for a, b in zip(before, after))
