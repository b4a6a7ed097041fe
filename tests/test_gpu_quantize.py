"""GPU parity of the INT4 quantiser, packer, append step and dequantisers
against the CPU oracle and the reference's golden digests (bit-exact)."""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from tests.hkv_testutil import dequant_side, read_side, t16

pytestmark = pytest.mark.gpu

K, V = 0, 1


@pytest.fixture(scope="module")
def hkv():
    from hetero_kvcache_optimizer_b200 import kvstore
    return kvstore


def _torch_input(x: np.ndarray, dt: str) -> torch.Tensor:
    if dt == "fp16":
        return torch.from_numpy(x.astype(np.float16)).cuda()
    return torch.from_numpy(x.astype(np.float32)).cuda().to(torch.bfloat16)


def test_quantize_flat_matches_reference_sweep(hkv, golden):
    """KVCompressor.compress contract on the reference's own regression shapes."""
    digests, _ = golden
    names = sorted(k for k in digests if k.startswith("compress_"))
    assert names
    for name in names:
        d = digests[name]
        x = ko.make_input(d["seed"], tuple(d["shape"]), d["dtype"])
        q, s, z = hkv.quantize_flat(_torch_input(x, d["dtype"]), d["group"])
        torch.cuda.synchronize()
        assert ko.sha256(q.cpu().numpy()) == d["codes"], name
        assert ko.sha256(s.cpu().numpy()) == d["scales"], name
        assert ko.sha256(z.cpu().numpy()) == d["zps"], name
        deq = hkv.dequantize_flat(q, s, z, d["group"], dtype=torch.float32)
        assert ko.sha256(deq.cpu().numpy()) == d["decompress_f32"], name


def test_quantize_rounding_boundaries(hkv):
    """Values whose quotient x/scale + zp sits on, or one or two ulps either side
    of, a .5 rounding boundary, over scales from 1e-6 to 1e3 (fp32 input): codes
    must equal the IEEE-division oracle's exactly."""
    rng = np.random.default_rng(123)
    G, ngroups = 32, 4096
    x = np.zeros((ngroups, G), np.float32)
    for g in range(ngroups):
        mag = np.float32(10.0 ** rng.uniform(-5, 4))
        mn, mx = np.float32(-rng.uniform(0.05, 1.0) * mag), np.float32(rng.uniform(0.05, 1.0) * mag)
        scale = np.maximum(np.float32((mx - mn) / np.float32(15.0)), np.float32(1e-8))
        zp = np.clip(np.rint(np.float32(-mn / scale)), 0, 15).astype(np.float32)
        vals = [mn, mx]
        while len(vals) < G:
            k = rng.integers(0, 16)
            b = np.float32((np.float32(k) + np.float32(0.5) - zp) * scale)
            for _ in range(int(rng.integers(-2, 3))):
                b = np.nextafter(b, np.float32(np.inf), dtype=np.float32)
            vals.append(np.float32(np.clip(b, mn, mx)))
        x[g] = np.array(vals, np.float32)
    q, s_, z = hkv.quantize_flat(torch.from_numpy(x).cuda(), G)
    qc, qs, qz = ko.quantize_ref(x, G)
    assert np.array_equal(s_.cpu().numpy().reshape(-1), qs)
    assert np.array_equal(z.cpu().numpy().reshape(-1), qz)
    assert np.array_equal(q.cpu().numpy().reshape(qc.shape), qc)


@pytest.mark.parametrize("page_tokens", [256, 4096])
def test_quantize_pack_cfg0_bit_exact(hkv, golden, page_tokens):
    """Config 0 K/V packed into pages, unpacked by the oracle: codes, scales and
    zero-points equal the reference's KVCompressor(group_size=32) output."""
    digests, _ = golden
    d = digests["cfg0"]
    k, v = ko.make_kv(d["seed"], d["B"], d["Hkv"], d["S"])
    store = hkv.Int4KVStore(1, 8, 4096, fmt="ref", group=32, page_tokens=page_tokens)
    hkv.prefill(store, t16(k), t16(v))
    for role, name in ((K, "k"), (V, "v")):
        codes, sc, zp = read_side(store, role)
        assert ko.sha256(codes[:, :, :4096]) == d[name + "_codes"]
        assert ko.sha256(sc[:, :, :4096].reshape(-1)) == d[name + "_scales"]
        assert ko.sha256(zp[:, :, :4096].reshape(-1)) == d[name + "_zps"]
    assert int(store.lengths[0]) == 4096


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_quantize_pack_formats_vs_oracle(hkv, group, dtype):
    B, H, T = 2, 3, 300
    x = ko.make_input(77 + group, (B, H, T, 128), dtype)
    for fmt in ("ref", "fp16min"):
        store = hkv.Int4KVStore(B, H, 512, fmt=fmt, group=group, page_tokens=256)
        hkv.quantize_pack(_torch_input(x, dtype), store, K, 0)
        hkv.quantize_pack(_torch_input(x, dtype), store, V, 0)
        for role in (K, V):
            codes, a, z = read_side(store, role)
            if fmt == "ref":
                qc, qs, qz = ko.quantize_ref(x, group)
                assert np.array_equal(codes[:, :, :T], qc)
                assert np.array_equal(a[:, :, :T].reshape(-1), qs)
                assert np.array_equal(z[:, :, :T].reshape(-1), qz)
            else:
                qc, qs, qm = ko.quantize_fp16min(x, group)
                assert np.array_equal(codes[:, :, :T], qc)
                assert np.array_equal(a[:, :, :T].view(np.uint16), qs.view(np.uint16))
                assert np.array_equal(z[:, :, :T].view(np.uint16), qm.view(np.uint16))


def test_quantize_pack_odd_offsets_and_paged(hkv):
    """Odd start slots split V token pairs across launches; a shuffled page
    table scatters pages. Contents must equal one contiguous quantisation."""
    B, H, T = 2, 2, 700
    x = ko.make_input(5, (B, H, T, 128), "fp16")
    npages = 2 * B * H * 3
    store = hkv.Int4KVStore(B, H, 768, fmt="ref", group=32, page_tokens=256, num_pages=npages)
    perm = np.random.default_rng(0).permutation(npages)[: B * H * 3].reshape(B * H, 3)
    store.page_table.copy_(torch.from_numpy(perm.astype(np.int32)))
    xt = t16(x)
    for a, b in ((0, 1), (1, 130), (130, 131), (131, 700)):
        hkv.quantize_pack(xt[:, :, a:b], store, K, a)
        hkv.quantize_pack(xt[:, :, a:b], store, V, a)
    qc, qs, qz = ko.quantize_ref(x, 32)
    for role in (K, V):
        codes, sc, zp = read_side(store, role)
        assert np.array_equal(codes[:, :, :T], qc)
        assert np.array_equal(sc[:, :, :T].reshape(-1), qs)
        assert np.array_equal(zp[:, :, :T].reshape(-1), qz)


@pytest.mark.parametrize("fmt,dt", [("ref", "fp16"), ("fp16min", "bf16"), ("fp16min", "fp16")])
def test_quantize_pack_kv_one_launch(hkv, fmt, dt):
    """K and V quantised in one launch (hkv_quantize_pack_kv), at odd start slots
    and through a shuffled page table: the same pages, byte for byte, as one
    hkv_quantize_pack launch per side."""
    B, H, T = 2, 2, 700
    k = _torch_input(ko.make_input(6, (B, H, T, 128), dt), dt)
    v = _torch_input(ko.make_input(7, (B, H, T, 128), dt), dt)
    npages = 2 * B * H * 3
    perm = torch.from_numpy(np.random.default_rng(1).permutation(npages)[: B * H * 3].reshape(B * H, 3)
                            .astype(np.int32))
    one, two = [hkv.Int4KVStore(B, H, 768, fmt=fmt, group=32, page_tokens=256, num_pages=npages)
                for _ in range(2)]
    for st in (one, two):
        st.pool.zero_()
        st.page_table.copy_(perm)
    for a, b in ((0, 1), (1, 130), (130, 131), (131, 700)):
        hkv.quantize_pack_kv(k[:, :, a:b], v[:, :, a:b], one, a)
        hkv.quantize_pack(k[:, :, a:b], two, K, a)
        hkv.quantize_pack(v[:, :, a:b], two, V, a)
    torch.cuda.synchronize()
    assert torch.equal(one.pool, two.pool)
    for role in (K, V):
        assert np.array_equal(dequant_side(one, role, T), dequant_side(two, role, T))


@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_quantize_pack_special_values(hkv, group, dt):
    """Groups the random sweeps never hit, written at an odd start slot (partial
    64-position tiles, V pairs split across the chunk edge): constant groups
    (zero range: ref scale clamps to 1e-8, fp16min scale 0 -> codes 0), all
    zeros, a range whose fp16 scale is subnormal with quotients exactly on .5
    (ties to even), values at the fp16 extremes, negative-only groups, and for
    ref with bf16 inputs values near 1e30. Bit-exact with the oracle."""
    B, H, T, start = 1, 2, 100, 37
    base = ko.make_input(91 + group, (B, H, T, 128), dt).astype(np.float32)
    x = base.copy()
    x[0, 0, 0, :] = 3.0
    x[0, 0, 1, :] = 0.0
    x[0, 1, 2, :] = np.arange(128, dtype=np.float32) % 32 * np.float32(2.0 ** -24)
    # fp16 extremes that bf16 also holds (fp16min keeps the group min as fp16,
    # so inputs beyond the fp16 range are outside that format)
    x[0, 0, 3, :] = np.where(np.arange(128) % 2 == 0, 65280.0, -65280.0)
    x[0, 1, 4, :] = -1.0 - np.arange(128, dtype=np.float32) / 16
    x[0, 0, 5, :64] = 60000.0
    big = x.copy()
    big[0, 1, 6, :] = np.where(np.arange(128) % 3 == 0, 1e30, -3e29)
    for fmt in ("ref", "fp16min"):
        xin = big if (fmt == "ref" and dt == "bf16") else x
        xin = (xin.astype(np.float16) if dt == "fp16" else ko.round_bf16(xin))
        store = hkv.Int4KVStore(B, H, 256, fmt=fmt, group=group, page_tokens=256)
        store.pool.zero_()
        xt = _torch_input(xin.astype(np.float32), dt)
        hkv.quantize_pack_kv(xt, xt, store, start)
        for role in (K, V):
            codes, a, z = read_side(store, role)
            if fmt == "ref":
                qc, qs, qz = ko.quantize_ref(xin.astype(np.float32), group)
                assert np.array_equal(codes[:, :, start:start + T], qc), (fmt, role)
                assert np.array_equal(a[:, :, start:start + T].reshape(-1), qs), (fmt, role)
                assert np.array_equal(z[:, :, start:start + T].reshape(-1), qz), (fmt, role)
            else:
                qc, qs, qm = ko.quantize_fp16min(xin.astype(np.float32), group)
                assert np.array_equal(codes[:, :, start:start + T], qc), (fmt, role)
                assert np.array_equal(a[:, :, start:start + T].view(np.uint16), qs.view(np.uint16)), (fmt, role)
                assert np.array_equal(z[:, :, start:start + T].view(np.uint16), qm.view(np.uint16)), (fmt, role)
            # slots outside [start, start + T) untouched
            assert not codes[:, :, :start].any() and not codes[:, :, start + T:].any(), (fmt, role)


def test_quantize_pack_per_batch_start(hkv):
    B, H, T = 3, 2, 5
    x = ko.make_input(9, (B, H, T, 128), "bf16")
    store = hkv.Int4KVStore(B, H, 256, fmt="fp16min", group=32)
    starts = torch.tensor([0, 7, 250], dtype=torch.int32, device="cuda")
    hkv.quantize_pack(_torch_input(x, "bf16"), store, V, starts)
    codes, s, m = read_side(store, V)
    qc, qs, qm = ko.quantize_fp16min(x, 32)
    for b, st in enumerate([0, 7, 250]):
        assert np.array_equal(codes[b, :, st:st + T], qc[b])
        assert np.array_equal(s[b, :, st:st + T].view(np.uint16), qs[b].view(np.uint16))


def test_quantize_capacity_error(hkv):
    store = hkv.Int4KVStore(1, 1, 256, fmt="ref", group=32)
    x = torch.zeros(1, 1, 10, 128, dtype=torch.float16, device="cuda")
    with pytest.raises(RuntimeError, match="CAPACITY"):
        hkv.quantize_pack(x, store, K, 250)


def test_append_state_machine(hkv):
    """Sink + recent-ring eviction into the INT4 body, as
    HeteroKVManager._decode_update slides its tail (manager.py:621-664)."""
    B, H, sink, ring = 2, 3, 2, 5
    cap = sink + ring
    steps = 14
    toks_k = ko.make_input(31, (steps, B, H, 128), "fp16")
    toks_v = ko.make_input(32, (steps, B, H, 128), "fp16")
    dense = hkv.DenseKV(B, H, cap, dtype=torch.float16)
    store = hkv.Int4KVStore(B, H, 256, fmt="ref", group=32)
    for s in range(steps):
        hkv.append_kv(t16(toks_k[s]), t16(toks_v[s]), dense, sink, store)
    torch.cuda.synchronize()
    n_ev = steps - cap
    assert dense.lengths.tolist() == [cap] * B
    assert store.lengths.tolist() == [n_ev] * B
    assert dense.ring_head.tolist() == [n_ev % ring] * B
    # sink rows hold the first tokens; the ring holds the last `ring` tokens
    dk = dense.k.float().cpu().numpy()
    assert np.array_equal(dk[:, :, :sink], np.moveaxis(toks_k[:sink].astype(np.float32), 0, 2))
    for t in range(steps - ring, steps):
        slot = sink + (t - sink) % ring
        assert np.array_equal(dk[:, :, slot], toks_k[t].astype(np.float32))
    # evicted tokens sink..sink+n_ev-1, quantised bit-exactly in order
    ev_k = np.moveaxis(toks_k[sink:sink + n_ev], 0, 2)
    ev_v = np.moveaxis(toks_v[sink:sink + n_ev], 0, 2)
    for role, ev in ((K, ev_k), (V, ev_v)):
        codes, sc, zp = read_side(store, role)
        qc, qs, qz = ko.quantize_ref(ev, 32)
        assert np.array_equal(codes[:, :, :n_ev], qc)
        assert np.array_equal(sc[:, :, :n_ev].reshape(-1), qs)
        assert np.array_equal(zp[:, :, :n_ev].reshape(-1), qz)


def test_dequantize_pack_and_repack(hkv):
    B, H, T = 2, 2, 333
    x = ko.make_input(41, (B, H, T, 128), "fp16")
    store = hkv.Int4KVStore(B, H, 512, fmt="ref", group=32)
    hkv.prefill(store, t16(x), t16(x))
    for role in (K, V):
        got = hkv.dequantize_pack(store, role, 0, T, dtype=torch.float32).cpu().numpy()
        assert np.array_equal(got, dequant_side(store, role, T))
    # the reference's unpacked triple, repacked, gives identical pages
    q, s, z = hkv.quantize_flat(t16(x), 32)
    st2 = hkv.Int4KVStore(B, H, 512, fmt="ref", group=32)
    hkv.repack_ref(q, s, z, 32, st2, K)
    hkv.repack_ref(q, s, z, 32, st2, V)
    torch.cuda.synchronize()
    for role in (K, V):
        a = read_side(store, role)
        b = read_side(st2, role)
        for u, w in zip(a, b):
            assert np.array_equal(u[:, :, :T], w[:, :, :T])


def test_no_device_errors(hkv):
    from hetero_kvcache_optimizer_b200 import _lib
    _lib.device_error(clear=True)
    store = hkv.Int4KVStore(1, 1, 256, fmt="ref", group=32)
    hkv.prefill(store, torch.randn(1, 1, 256, 128, device="cuda", dtype=torch.float16),
                torch.randn(1, 1, 256, 128, device="cuda", dtype=torch.float16))
    assert _lib.device_error(clear=True) == 0
