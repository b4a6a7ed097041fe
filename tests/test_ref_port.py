"""Pins oracle/ref_port.py, the CPU port of the reference's decode-step path
that bench.py times as the CPU baseline and as the ``--impl reference`` arm,
against golden fixtures produced by the reference package itself
(tests/golden/make_golden.py): the compressor bit for bit, the decompressor,
the dequant-then-SDPA attention, and the decode-step state machine of
``RefLayer.step`` (src/memory/manager.py:621-664 eviction of the oldest tail
token into INT4) against the numpy oracle.
"""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from oracle import ref_port as rp


def _t(x: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "fp16":
        return torch.from_numpy(x.astype(np.float16))
    return torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16)


def test_compress_sweep_bit_exact(golden):
    """Codes, scales, zero-points and fp32 decompression of every compressor
    case the goldens hold (7 shapes x 3 groups x fp16/bf16)."""
    digests, arrays = golden
    names = sorted(k for k in digests if k.startswith("compress_"))
    assert len(names) == 42
    for name in names:
        d = digests[name]
        x = ko.make_input(d["seed"], tuple(d["shape"]), d["dtype"])
        q, s, z = rp.compress(_t(x, d["dtype"]), d["group"])
        assert ko.sha256(q.numpy()) == d["codes"], name
        assert ko.sha256(s.numpy()) == d["scales"], name
        assert ko.sha256(z.numpy()) == d["zps"], name
        assert np.array_equal(q.numpy().reshape(-1)[:256], arrays[name + "_codes_head"]), name
        deq = rp.decompress(q, s, z, d["group"], torch.float32)
        assert ko.sha256(deq.numpy()) == d["decompress_f32"], name


def test_cfg0_compress_and_attention(golden):
    digests, arrays = golden
    d = digests["cfg0"]
    k, v = ko.make_kv(d["seed"], d["B"], d["Hkv"], d["S"])
    parts = {}
    for name, x in (("k", k), ("v", v)):
        q, s, z = rp.compress(torch.from_numpy(x), d["group"])
        assert ko.sha256(q.numpy()) == d[name + "_codes"]
        assert ko.sha256(s.numpy()) == d[name + "_scales"]
        assert ko.sha256(z.numpy()) == d[name + "_zps"]
        parts[name] = rp.decompress(q, s, z, d["group"])
    qq = torch.from_numpy(arrays["cfg0_q"])[:, :, None, :]
    out = rp.decode_attention(qq, parts["k"], parts["v"])[:, :, 0].numpy()
    assert ko.rel_err(out, arrays["cfg0_out"]) < 1e-5


def test_segmented_attention(golden):
    """[sink fp16 ; INT4 body ; recent fp16] with GQA 4, as RefLayer concatenates."""
    digests, arrays = golden
    d = digests["seg"]
    B, Hkv, sink, body, recent = d["B"], d["Hkv"], d["sink"], d["body"], d["recent"]
    k, v = ko.make_kv(d["seed"], B, Hkv, sink + body + recent)
    kq, ks, kz = rp.compress(torch.from_numpy(k[:, :, sink:sink + body].copy()), 32)
    vq, vs, vz = rp.compress(torch.from_numpy(v[:, :, sink:sink + body].copy()), 32)
    kf = torch.cat([torch.from_numpy(k[:, :, :sink]).float(), rp.decompress(kq, ks, kz, 32),
                    torch.from_numpy(k[:, :, sink + body:]).float()], dim=2)
    vf = torch.cat([torch.from_numpy(v[:, :, :sink]).float(), rp.decompress(vq, vs, vz, 32),
                    torch.from_numpy(v[:, :, sink + body:]).float()], dim=2)
    out = rp.decode_attention(torch.from_numpy(arrays["seg_q"])[:, :, None, :], kf, vf)[:, :, 0].numpy()
    assert ko.rel_err(out, arrays["seg_out"]) < 1e-5


def test_legacy_per_token_attention(golden):
    """Group 128 == head_dim, MHA: the reference's benchmark representation."""
    digests, arrays = golden
    d = digests["legacy"]
    k, v = ko.make_kv(d["seed"], d["B"], d["H"], d["S"], outlier_channels=0)
    kq, ks, kz = rp.compress(torch.from_numpy(k), 128)
    vq, vs, vz = rp.compress(torch.from_numpy(v), 128)
    q = torch.from_numpy(arrays["legacy_q"].astype(np.float32))[:, :, None, :]
    out = rp.decode_attention(q, rp.decompress(kq, ks, kz, 128), rp.decompress(vq, vs, vz, 128))
    assert ko.rel_err(out[:, :, 0].numpy(), arrays["legacy_out"]) < 1e-5


@pytest.mark.parametrize("steps", [1, 3])
def test_reflayer_step_matches_oracle(steps):
    """RefLayer.step = evict the oldest recent token into the INT4 body
    (reference quantiser), append the new token, attend over
    [body ; sink ; recent]: checked against the numpy oracle on the same data."""
    B, Hkv, G, body, sink, recent = 2, 2, 4, 200, 8, 16
    layer = rp.RefLayer(B, Hkv, body, sink, recent, group=32, seed=5)
    # the layer's own fp16 inputs, regenerated with the same generator order
    g = torch.Generator().manual_seed(5)
    kb = torch.randn(B, Hkv, body, 128, generator=g).half().numpy()
    vb = torch.randn(B, Hkv, body, 128, generator=g).half().numpy()
    sk = torch.randn(B, Hkv, sink, 128, generator=g).half().numpy()
    sv = torch.randn(B, Hkv, sink, 128, generator=g).half().numpy()
    tk = torch.randn(B, Hkv, recent, 128, generator=g).half().numpy()
    tv = torch.randn(B, Hkv, recent, 128, generator=g).half().numpy()
    rng = ko.rng_for(77)
    for _ in range(steps):
        q = rng.standard_normal((B, Hkv * G, 128), dtype=np.float32)
        kn = rng.standard_normal((B, Hkv, 128), dtype=np.float32).astype(np.float16)
        vn = rng.standard_normal((B, Hkv, 128), dtype=np.float32).astype(np.float16)
        out = layer.step(torch.from_numpy(q), torch.from_numpy(kn), torch.from_numpy(vn)).numpy()
        # oracle: the evicted token joins the body, the tail slides
        kb = np.concatenate([kb, tk[:, :, :1]], axis=2)
        vb = np.concatenate([vb, tv[:, :, :1]], axis=2)
        tk = np.concatenate([tk[:, :, 1:], kn[:, :, None]], axis=2)
        tv = np.concatenate([tv[:, :, 1:], vn[:, :, None]], axis=2)
        kq, ks, kz = ko.quantize_ref(kb, 32)
        vq, vs, vz = ko.quantize_ref(vb, 32)
        kd = np.concatenate([ko.dequantize_ref(kq, ks, kz, 32), sk.astype(np.float32),
                             tk.astype(np.float32)], axis=2)
        vd = np.concatenate([ko.dequantize_ref(vq, vs, vz, 32), sv.astype(np.float32),
                             tv.astype(np.float32)], axis=2)
        ref = ko.decode_attention(q, kd, vd)
        assert ko.rel_err(out, ref) < 1e-5
