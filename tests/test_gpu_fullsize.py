"""Configuration 2 at full size (Qwen2-VL-7B-shaped long multimodal decode):
B1, Hq 28 / Hkv 4 (GQA 7), a 131,072-token context whose positions below
100,000 are 'vision' tokens K/V ~ N(0, 0.5^2) and whose text tokens are
N(0, 1) with 4 seeded K channels per KV head scaled x10; 64 sink + 1,024
recent tokens stay fp16, the 129,984 in between are quantised by the chunked
prefill in 4,096-token chunks.

* the chunked quantise is bit-exact with the oracle (codes, scales,
  zero-points / mins) on the chunks that hold the start, the vision -> text
  boundary and the ragged end of the body;
* the decode attention over [sink ; INT4 body ; recent] is within the
  north-star tolerance, max |out - ref| <= 2e-3 * ||ref||_2 per (b, head), of
  an fp32 softmax(q K^T / sqrt(128)) V over the same dequantised cache
  (dequantize_pack is itself pinned bit-exact to the oracle in
  test_gpu_quantize.py).
"""
import math

import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko

pytestmark = pytest.mark.gpu

TOL = 2e-3
K, V = 0, 1
B, HQ, HKV, CTX, SINK, RECENT, CHUNK, VISION = 1, 28, 4, 131072, 64, 1024, 4096, 100000
BODY = CTX - SINK - RECENT


@pytest.fixture(scope="module")
def hkv():
    from hetero_kvcache_optimizer_b200 import kvstore
    return kvstore


@pytest.fixture(scope="module")
def cfg2_kv():
    """fp16 K/V [1, 4, 131072, 128] on the device (seeded, configuration 2's mix)."""
    gen = torch.Generator(device="cuda").manual_seed(2)
    k = torch.randn(B, HKV, CTX, 128, device="cuda", generator=gen)
    v = torch.randn(B, HKV, CTX, 128, device="cuda", generator=gen)
    k[:, :, :VISION] *= 0.5
    v[:, :, :VISION] *= 0.5
    for h in range(HKV):
        ch = torch.randperm(128, device="cuda", generator=gen)[:4]
        k[:, h, VISION:, ch] *= 10.0
    return k.half(), v.half()


def _chunked_store(hkv, k, v, fmt):
    store = hkv.Int4KVStore(B, HKV, BODY, fmt=fmt, group=32, page_tokens=CHUNK)
    for t0 in range(0, BODY, CHUNK):
        n = min(CHUNK, BODY - t0)
        hkv.quantize_pack_kv(k[:, :, SINK + t0:SINK + t0 + n], v[:, :, SINK + t0:SINK + t0 + n], store, t0)
    store.set_lengths(BODY)
    return store


def _read_chunk(store, role, c):
    """Codes and the two metadata arrays of body chunk c (= page c, 4,096-token
    pages) of every unit, unpacked by the oracle's layout spec."""
    torch.cuda.synchronize()
    fmt = 0 if store.fmt == "ref" else 1
    out = []
    for u in range(B * HKV):
        page = store.pool[u * store.max_pages + c].cpu().numpy()
        cd, a, z = ko.split_page(page, CHUNK, fmt, store.group, role)
        out.append((ko.unpack_k(cd) if role == K else ko.unpack_v(cd, CHUNK), a, z))
    return out


@pytest.mark.parametrize("fmt", ["fp16min", "ref"])
def test_cfg2_chunked_quantize_bit_exact(hkv, cfg2_kv, fmt):
    k, v = cfg2_kv
    store = _chunked_store(hkv, k, v, fmt)
    last = (BODY - 1) // CHUNK
    boundary = (VISION - SINK) // CHUNK  # the chunk where vision tokens end and text begins
    for c in (0, boundary, last):
        n = min(CHUNK, BODY - c * CHUNK)
        for role, x in ((K, k), (V, v)):
            src = x[:, :, SINK + c * CHUNK:SINK + c * CHUNK + n].float().cpu().numpy()
            got = _read_chunk(store, role, c)
            for u in range(B * HKV):
                xs = src[0, u]
                codes, a, z = got[u]
                if fmt == "ref":
                    qc, qs, qz = ko.quantize_ref(xs, 32)
                    assert np.array_equal(codes[:n], qc), (fmt, c, role, u)
                    assert np.array_equal(a[:n].reshape(-1), qs), (fmt, c, role, u)
                    assert np.array_equal(z[:n].reshape(-1), qz), (fmt, c, role, u)
                else:
                    qc, qs, qm = ko.quantize_fp16min(xs, 32)
                    assert np.array_equal(codes[:n], qc), (fmt, c, role, u)
                    assert np.array_equal(a[:n].view(np.uint16), qs.view(np.uint16)), (fmt, c, role, u)
                    assert np.array_equal(z[:n].view(np.uint16), qm.view(np.uint16)), (fmt, c, role, u)


@pytest.mark.parametrize("fmt", ["fp16min", "ref"])
def test_cfg2_full_size_decode_vs_fp32(hkv, cfg2_kv, fmt):
    k, v = cfg2_kv
    store = _chunked_store(hkv, k, v, fmt)
    dense = hkv.DenseKV(B, HKV, SINK + RECENT)
    dense.k[:, :, :SINK] = k[:, :, :SINK]
    dense.v[:, :, :SINK] = v[:, :, :SINK]
    dense.k[:, :, SINK:] = k[:, :, CTX - RECENT:]
    dense.v[:, :, SINK:] = v[:, :, CTX - RECENT:]
    dense.set_lengths(SINK + RECENT)
    gen = torch.Generator(device="cuda").manual_seed(22)
    q = torch.randn(B, HQ, 128, device="cuda", generator=gen).to(torch.bfloat16)
    out = hkv.decode(q, store, dense)
    from hetero_kvcache_optimizer_b200 import _lib
    assert _lib.device_error() == 0
    kd = torch.cat([hkv.dequantize_pack(store, K, 0, BODY, torch.float32), dense.k.float()], dim=2)
    vd = torch.cat([hkv.dequantize_pack(store, V, 0, BODY, torch.float32), dense.v.float()], dim=2)
    G = HQ // HKV
    qg = q.float().reshape(B, HKV, G, 128)
    s = torch.einsum("bhgd,bhsd->bhgs", qg, kd) / math.sqrt(128)
    ref = torch.einsum("bhgs,bhsd->bhgd", torch.softmax(s, dim=-1), vd).reshape(B, HQ, 128)
    err = ((out - ref).abs().amax(-1) / ref.norm(dim=-1)).max().item()
    assert err < TOL, err
