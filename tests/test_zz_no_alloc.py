"""hkv_decode_attn_static: decode attention served from the library's own
per-device scratch array instead of a caller workspace. Collected last, so it
also runs after every other test has used the library in the same process."""
import ctypes

import numpy as np
import pytest
import torch

from hetero_kvcache_optimizer_b200 import _lib as L


def test_static_rejects_oversized_request_on_host():
    """A request whose workspace exceeds the scratch fails before any CUDA call
    (the pointers below are never dereferenced)."""
    lib = L.load()
    st = L.HkvInt4Store()
    st.pages, st.page_stride = 0x100000, lib.hkv_page_bytes(L.FMT_FP16MIN, 32, 256)
    st.format, st.group, st.page_tokens, st.max_pages = L.FMT_FP16MIN, 32, 256, 4
    st.page_table, st.lengths, st.len = None, None, 1024
    B, Hq, Hkv = 8192, 64, 8  # 65536 units: the merge partials alone need ~1 GiB
    need = lib.hkv_decode_workspace_bytes(ctypes.byref(st), None, B, Hq, Hkv, 128, 148)
    assert need > L.STATIC_SCRATCH_BYTES
    rc = lib.hkv_decode_attn_static(0x300000, L.DT_F16, Hq * 128, 128, ctypes.byref(st), None, B, Hq, Hkv,
                                    128, 0.088, 148, 0x400000, L.DT_F32, Hq * 128, 128, None)
    assert rc == L.HKV_ERR_CAPACITY


def _case(seed, B, Hkv, G, nbody, ndense, fmt):
    from hetero_kvcache_optimizer_b200 import kvstore as kv
    g = torch.Generator(device="cuda").manual_seed(seed)
    dev = torch.device("cuda", 0)
    st = kv.Int4KVStore(B, Hkv, 1024, fmt=fmt, group=32, device=dev)
    k = torch.randn(B, Hkv, nbody, 128, device=dev, generator=g).half()
    v = torch.randn(B, Hkv, nbody, 128, device=dev, generator=g).half()
    kv.prefill(st, k, v)
    d = kv.DenseKV(B, Hkv, 256, device=dev)
    d.k.normal_(generator=g)
    d.v.normal_(generator=g)
    d.set_lengths(ndense)
    q = torch.randn(B, Hkv * G, 128, device=dev, generator=g).bfloat16()
    return st, d, q


@pytest.mark.gpu
def test_static_matches_workspace_entry_point_twice():
    from hetero_kvcache_optimizer_b200 import kvstore as kv
    cases = [_case(1, 2, 8, 4, 700, 200, "fp16min"), _case(2, 3, 4, 8, 333, 65, "ref")]
    refs = [kv.decode(q, st, d) for st, d, q in cases]
    for _ in range(2):  # two rounds in a row: the scratch keeps the last call's contents
        for (st, d, q), ref in zip(cases, refs):
            out = torch.full_like(ref, float("nan"))
            kv.decode_static(q, st, d, out=out)
            torch.cuda.synchronize()
            err = (out - ref).abs().max().item()
            assert np.isfinite(err) and err <= 1e-6 * max(1.0, ref.abs().max().item()), err
            # and directly against the CPU oracle (dequant-then-softmax over the
            # same cache), at the tolerance every decode parity test uses
            from oracle import kv_oracle as ko
            from tests.hkv_testutil import dequant_side
            nb, nd = int(st.lengths[0]), int(d.lengths[0])
            kd = np.concatenate([dequant_side(st, 0, nb), d.k[:, :, :nd].float().cpu().numpy()], axis=2)
            vd = np.concatenate([dequant_side(st, 1, nb), d.v[:, :, :nd].float().cpu().numpy()], axis=2)
            oracle = ko.decode_attention(q.float().cpu().numpy(), kd, vd)
            assert ko.rel_err(out.cpu().numpy(), oracle) < 2e-3
    assert L.device_error() == 0
