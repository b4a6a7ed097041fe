"""Generate golden fixtures from the REFERENCE implementation itself.

Run in the build container, where the reference package is importable:

    python tests/golden/make_golden.py <path-to-reference-checkout>
    (or HKV_REFERENCE=<path-to-reference-checkout> python tests/golden/make_golden.py)

It imports ``src.quantization.kv_compressor.KVCompressor`` and the PyTorch
fallbacks of ``src.quantization.fused_dequant_attn.fused_dequant_attn_decode``
and ``fused_dequant_attn_forward`` (what runs on CPU tensors,
fused_dequant_attn.py:326-331 and :241-246) from the
reference checkout, feeds them seeded inputs from ``oracle.kv_oracle`` and
writes ``tests/golden/golden.npz`` (small arrays) and ``golden.json`` (SHA-256
digests of full-size outputs, so configuration-0-sized results are pinned
without committing megabytes). The GPU box never runs this script; tests only
read its outputs.
"""
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle import kv_oracle as ko  # noqa: E402

REF = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("HKV_REFERENCE")
if not REF:
    sys.exit("usage: make_golden.py <reference checkout> (or set HKV_REFERENCE)")
sys.path.insert(0, REF)
from src.quantization.kv_compressor import KVCompressor  # noqa: E402
from src.quantization.fused_dequant_attn import fused_dequant_attn_decode, fused_dequant_attn_forward  # noqa: E402

torch.set_num_threads(max(1, os.cpu_count() or 1))

# Shapes the reference's own compressor regression test sweeps
# (test_kv_compressor_fix.py:46-58), plus group 32 (the build's group size).
COMPRESS_SHAPES = [(1, 32, 16, 128), (1, 4, 1984, 64), (1, 8, 512, 64), (1, 8, 123, 128),
                   (1, 8, 1, 128), (1, 8, 1999, 64), (1, 3, 7, 11)]
GROUPS = [32, 64, 128]
DTYPES = ["fp16", "bf16"]


def to_torch(x, dtype):
    if dtype == "fp16":
        return torch.from_numpy(x.astype(np.float16))
    return torch.from_numpy(x.astype(np.float32)).to(torch.bfloat16)


def ref_attention(q, kdeq, vdeq, G):
    """The reference's dequant->SDPA fallback, with K/V expanded for GQA by
    repeat_interleave (HF repeat_kv). Dequantised K/V are passed as the
    "quantised" operand with unit scale and zero zero-point, so the reference's
    own _dequant_tensor (fused_dequant_attn.py:388-390) is the identity and its
    matmul/softmax/matmul lines (:327-331) compute the attention."""
    k = torch.from_numpy(kdeq).repeat_interleave(G, dim=1)
    v = torch.from_numpy(vdeq).repeat_interleave(G, dim=1)
    B, H, S, _ = k.shape
    ones = torch.ones(B, H, S)
    zeros = torch.zeros(B, H, S)
    qt = torch.from_numpy(q)[:, :, None, :]
    out = fused_dequant_attn_decode(qt, k, ones, zeros, v, ones, zeros)
    return out[:, :, 0, :].numpy()


def main():
    arrays = {}
    digests = {}

    # 1. Compressor sweep: bit-exact codes/scales/zps.
    for si, shape in enumerate(COMPRESS_SHAPES):
        for g in GROUPS:
            for dt in DTYPES:
                seed = 1000 + si
                x = ko.make_input(seed, shape, dt)
                comp = KVCompressor(group_size=g)
                q, s, z = comp.compress(to_torch(x, dt))
                name = f"compress_s{si}_g{g}_{dt}"
                digests[name] = {"seed": seed, "shape": list(shape), "group": g, "dtype": dt,
                                 "codes": ko.sha256(q.numpy()), "scales": ko.sha256(s.numpy()),
                                 "zps": ko.sha256(z.numpy())}
                arrays[name + "_codes_head"] = q.numpy().reshape(-1)[:256]
                arrays[name + "_scales_head"] = s.numpy()[:64]
                arrays[name + "_zps_head"] = z.numpy()[:64]
                deq = comp.decompress(q, s, z, target_dtype=torch.float32).numpy()
                digests[name]["decompress_f32"] = ko.sha256(deq)

    # 2. Configuration 0: K/V [1,8,4096,128] fp16 with outlier channels, group 32.
    k, v = ko.make_kv(0, 1, 8, 4096)
    comp = KVCompressor(group_size=32)
    kq, ks, kz = comp.compress(torch.from_numpy(k))
    vq, vs, vz = comp.compress(torch.from_numpy(v))
    digests["cfg0"] = {"seed": 0, "B": 1, "Hkv": 8, "S": 4096, "group": 32,
                       "k_codes": ko.sha256(kq.numpy()), "k_scales": ko.sha256(ks.numpy()),
                       "k_zps": ko.sha256(kz.numpy()), "v_codes": ko.sha256(vq.numpy()),
                       "v_scales": ko.sha256(vs.numpy()), "v_zps": ko.sha256(vz.numpy())}
    kdeq = comp.decompress(kq, ks, kz, target_dtype=torch.float32).numpy()
    vdeq = comp.decompress(vq, vs, vz, target_dtype=torch.float32).numpy()
    q = ko.make_q(0, 1, 32).astype(np.float16).astype(np.float32)
    arrays["cfg0_q"] = q
    arrays["cfg0_out"] = ref_attention(q, kdeq, vdeq, 4)

    # 3. Segmented decode (sink fp16 | INT4 body | recent fp16), GQA 4, small S.
    B, Hkv, G, sink, body, recent = 2, 8, 4, 64, 1000, 96
    S = sink + body + recent
    k, v = ko.make_kv(11, B, Hkv, S)
    q = ko.make_q(11, B, Hkv * G).astype(np.float16).astype(np.float32)
    kq, ks, kz = comp.compress(torch.from_numpy(k[:, :, sink:sink + body].copy()))
    vq, vs, vz = comp.compress(torch.from_numpy(v[:, :, sink:sink + body].copy()))
    kb = comp.decompress(kq, ks, kz, target_dtype=torch.float32).numpy()
    vb = comp.decompress(vq, vs, vz, target_dtype=torch.float32).numpy()
    kfull = np.concatenate([k[:, :, :sink].astype(np.float32), kb,
                            k[:, :, sink + body:].astype(np.float32)], axis=2)
    vfull = np.concatenate([v[:, :, :sink].astype(np.float32), vb,
                            v[:, :, sink + body:].astype(np.float32)], axis=2)
    arrays["seg_q"] = q
    arrays["seg_out"] = ref_attention(q, kfull, vfull, G)
    digests["seg"] = {"seed": 11, "B": B, "Hkv": Hkv, "G": G, "sink": sink, "body": body,
                      "recent": recent, "group": 32}

    # 4. Legacy per-token path exactly as the reference's callers build it
    #    (unified_benchmark.py:151-162): group 128 == head_dim, MHA.
    B, H, S = 2, 4, 300
    k, v = ko.make_kv(21, B, H, S, outlier_channels=0)
    comp128 = KVCompressor(group_size=128)
    kq, ks, kz = comp128.compress(torch.from_numpy(k))
    vq, vs, vz = comp128.compress(torch.from_numpy(v))
    q = ko.make_q(21, B, H).astype(np.float16)
    out = fused_dequant_attn_decode(torch.from_numpy(q)[:, :, None, :],
                                    kq, ks.reshape(B, H, S), kz.reshape(B, H, S).float(),
                                    vq, vs.reshape(B, H, S), vz.reshape(B, H, S).float())
    arrays["legacy_q"] = q
    arrays["legacy_out"] = out[:, :, 0, :].numpy()
    digests["legacy"] = {"seed": 21, "B": B, "H": H, "S": S, "group": 128}

    # 5. Legacy multi-query forward (prefill), same per-token metadata, Sq = 24.
    B, H, S, Sq = 1, 4, 300, 24
    k, v = ko.make_kv(22, B, H, S, outlier_channels=0)
    kq, ks, kz = comp128.compress(torch.from_numpy(k))
    vq, vs, vz = comp128.compress(torch.from_numpy(v))
    q = ko.rng_for(22).standard_normal((B, H, Sq, 128), dtype=np.float32).astype(np.float16)
    out = fused_dequant_attn_forward(torch.from_numpy(q), kq, ks.reshape(B, H, S), kz.reshape(B, H, S).float(),
                                     vq, vs.reshape(B, H, S), vz.reshape(B, H, S).float())
    arrays["legacy_fwd_q"] = q
    arrays["legacy_fwd_out"] = out.numpy()
    digests["legacy_fwd"] = {"seed": 22, "B": B, "H": H, "S": S, "Sq": Sq, "group": 128}

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(digests, f, indent=1, sort_keys=True)
    print("wrote", len(arrays), "arrays and", len(digests), "digest records")


if __name__ == "__main__":
    main()
