"""Shared adapter for the reference's fused_dequant_attn_* signatures.

The reference's callers pass either per-token metadata ([B, H, S] scales and
zero-points, group = head_dim; unified_benchmark.py:151-162) or the flat 1-D
arrays KVCompressor.compress returns (group = any divisor of 128). Both are
repacked on the GPU into the nibble-packed store (hkv_repack_ref), then the
split-KV kernel runs. A packed ``Int4KVStore`` may be passed directly as
``k_quant`` (then the other K/V arguments are ignored).
"""
from __future__ import annotations

import collections
import math
import weakref
from typing import Optional

import torch

from .. import _lib as L
from .. import kvstore as kv


def _as_4d(t: torch.Tensor, meta: bool = False) -> torch.Tensor:
    # kernels/fused_dequant_attn.py:327-340 accepts 2-D [S, D] / 3-D [H, S, D] K/V
    need = 3 if meta else 4
    while t.dim() < need:
        t = t.unsqueeze(0)
    return t


# Packed stores of recent calls, keyed by the identity and version counter of
# the six argument tensors: a caller that decodes step after step with the same
# (unchanged) INT4 tensors pays the repack once, not O(S) per call. Entries hold
# weak references, so a freed tensor (whose address may be reused) never hits.
_STORE_CACHE: "collections.OrderedDict" = collections.OrderedDict()
_STORE_CACHE_SIZE = 4


def _cache_key(ts):
    return tuple((id(t), t._version) for t in ts)


def _cache_get(ts):
    key = _cache_key(ts)
    hit = _STORE_CACHE.get(key)
    if hit is None:
        return None
    refs, store = hit
    if any(r() is not t for r, t in zip(refs, ts)):
        del _STORE_CACHE[key]
        return None
    _STORE_CACHE.move_to_end(key)
    return store


def _cache_put(ts, store) -> None:
    _STORE_CACHE[_cache_key(ts)] = (tuple(weakref.ref(t) for t in ts), store)
    while len(_STORE_CACHE) > _STORE_CACHE_SIZE:
        _STORE_CACHE.popitem(last=False)


def build_store(k_quant, k_scales, k_zps, v_quant, v_scales, v_zps) -> kv.Int4KVStore:
    if isinstance(k_quant, kv.Int4KVStore):
        return k_quant
    args = (k_quant, k_scales, k_zps, v_quant, v_scales, v_zps)
    cached = _cache_get(args)
    if cached is not None:
        return cached
    store = _repack(*args)
    _cache_put(args, store)
    return store


def _repack(k_quant, k_scales, k_zps, v_quant, v_scales, v_zps) -> kv.Int4KVStore:
    kq = _as_4d(k_quant)
    vq = _as_4d(v_quant)
    B, H, S, D = kq.shape
    if D != 128:
        raise ValueError("fused INT4 decode needs head_dim 128")
    n = kq.numel()
    ng = k_scales.numel()
    if ng == 0 or n % ng:
        raise ValueError("scales do not tile the K tensor into equal groups")
    group = n // ng
    if group not in (32, 64, 128):
        raise ValueError(f"group size {group} unsupported (32, 64 or 128)")
    store = kv.Int4KVStore(B, H, max(S, 1), fmt="ref", group=group, device=kq.device)
    kv.repack_ref(kq, k_scales.reshape(-1), k_zps.reshape(-1), group, store, L.ROLE_K)
    kv.repack_ref(vq, v_scales.reshape(-1), v_zps.reshape(-1), group, store, L.ROLE_V)
    store.set_lengths(S)
    return store


def decode(q, store: kv.Int4KVStore, sm_scale: Optional[float], out_dtype) -> torch.Tensor:
    """q [B, Hq, 1, D] -> [B, Hq, 1, D]."""
    if q.dim() != 4 or q.shape[2] != 1:
        raise ValueError(f"Decode expects [B,H,1,D], got {tuple(q.shape)}")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(q.shape[-1])
    return kv.decode(q, store, None, sm_scale=sm_scale, out_dtype=out_dtype)


# (query, head) rows per KV head from which the tensor-core prefill kernel
# takes over from the split-KV decode kernel
PREFILL_MIN_ROWS = 16


def forward(q, store: kv.Int4KVStore, sm_scale: Optional[float], out_dtype) -> torch.Tensor:
    """Multi-query (prefill-shaped) attention without a causal mask, as the
    reference computes it (fused_dequant_attn.py:158-247). f16/bf16 queries
    with at least PREFILL_MIN_ROWS (query, head) rows per KV head run the
    tcgen05 prefill kernel (kvstore.prefill_attn); otherwise the Sq query rows
    of each head are folded into GQA query heads (at most 8 per KV head per
    launch) of the split-KV decode kernel."""
    if q.dim() != 4:
        raise ValueError(f"Forward expects [B,H,S,D], got {tuple(q.shape)}")
    B, Hq, Sq, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    Hkv = store.kv_heads
    G = Hq // Hkv
    if q.dtype in (torch.float16, torch.bfloat16) and Sq * G >= PREFILL_MIN_ROWS:
        return kv.prefill_attn(q, store, sm_scale=sm_scale, out_dtype=out_dtype)
    out = torch.empty(B, Hq, Sq, D, dtype=out_dtype, device=q.device)
    step = max(1, 8 // G)
    for s0 in range(0, Sq, step):
        s1 = min(Sq, s0 + step)
        n = s1 - s0
        # [B, Hq, n, D] -> [B, Hkv, G, n, D] -> [B, Hkv*G*n, D]: KV head of row = row // (G*n)
        qq = q[:, :, s0:s1].reshape(B, Hkv, G * n, D).reshape(B, Hkv * G * n, D).contiguous()
        o = kv.decode(qq, store, None, sm_scale=sm_scale, out_dtype=out_dtype)
        out[:, :, s0:s1] = o.reshape(B, Hkv, G, n, D).reshape(B, Hq, n, D)
    return out
