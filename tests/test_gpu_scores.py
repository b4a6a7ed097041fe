"""GPU: where the attention fell (kvstore.decode_scored / hkv_tile_scores).
For every (sequence, KV head) unit, the mass on each 128-token INT4 tile must
equal the oracle's softmax probability on those tokens, averaged over the
unit's query heads; the attention output must equal plain decode's."""
import numpy as np
import pytest
import torch

from oracle import kv_oracle as ko
from tests.hkv_testutil import dequant_side, t16

pytestmark = pytest.mark.gpu
K, V = 0, 1


def _probs(q, k, scale):
    """softmax over the last axis of q.k (fp64): q [B,Hq,D], k [B,Hkv,S,D] -> [B,Hq,S]."""
    G = q.shape[1] // k.shape[1]
    s = np.einsum("bhd,bhsd->bhs", q.astype(np.float64), np.repeat(k, G, axis=1).astype(np.float64)) * scale
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    return p / p.sum(-1, keepdims=True)


@pytest.mark.parametrize("fmt,group,G", [("fp16min", 32, 4), ("ref", 32, 7), ("fp16min", 64, 1)])
@pytest.mark.parametrize("lens", [(700, 700), (513, 129)])
def test_tile_mass_matches_oracle(fmt, group, G, lens):
    from hetero_kvcache_optimizer_b200 import kvstore as kv
    B, Hkv, Sd = 2, 2, 40
    S = max(lens)
    k, v = ko.make_kv(len(lens) + G, B, Hkv, S + Sd)
    store = kv.Int4KVStore(B, Hkv, S, fmt=fmt, group=group)
    kv.prefill(store, t16(k[:, :, :S]), t16(v[:, :, :S]))
    store.set_lengths(torch.tensor(lens, dtype=torch.int32, device="cuda"))
    dense = kv.DenseKV(B, Hkv, 64)
    dense.k[:, :, :Sd] = t16(k[:, :, S:])
    dense.v[:, :, :Sd] = t16(v[:, :, S:])
    dense.set_lengths(Sd)
    q = ko.make_q(G, B, Hkv * G).astype(np.float16).astype(np.float32)
    qt = t16(q)
    out, mass = kv.decode_scored(qt, store, dense, ctas=5)
    plain = kv.decode(qt, store, dense, ctas=5)
    torch.testing.assert_close(out, plain, rtol=0, atol=1e-6)
    mass = mass.cpu().numpy()
    kd, dk = dequant_side(store, K, S), dense.k[:, :, :Sd].float().cpu().numpy()
    T = mass.shape[2]
    for b, n in enumerate(lens):
        p = _probs(q[b:b + 1], np.concatenate([kd[b:b + 1, :, :n], dk[b:b + 1]], axis=2), 1 / np.sqrt(128))[0]
        for h in range(Hkv):
            ph = p[h * G:(h + 1) * G, :n].mean(axis=0)          # mean over the unit's query heads
            want = np.zeros(T)
            for t in range(0, n, 128):
                want[t // 128] = ph[t:t + 128].sum()
            np.testing.assert_allclose(mass[b, h], want, atol=2e-3, err_msg=f"b={b} h={h}")
