"""Drop-in for src/quantization/kernels/fused_dequant_attn.py (returns q.dtype).

Same wrappers as the reference (:283-435): decode/forward accept 2-D, 3-D or
4-D K/V and return ``q.dtype``. The reference's decode kernel in this file
computes wrong offsets and ignores sm_scale; this one is the same validated
split-KV CUDA kernel as quantization.fused_dequant_attn.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _legacy
from ... import kvstore as kv


def fused_dequant_attention(q, k_q, k_s, k_z):
    """Legacy single-head scores (reference :283-298): [seq_len] in q.dtype."""
    qf = q.reshape(-1)
    S, D = k_q.shape[0], qf.shape[0]
    return kv.qk_scores_flat(qf, k_q.reshape(S, D), k_s.reshape(-1), k_z.reshape(-1), D).to(q.dtype)


def fused_dequant_attn_decode(q: torch.Tensor, k_data, k_scales, k_zps, v_data, v_scales, v_zps,
                              sm_scale: Optional[float] = None) -> torch.Tensor:
    assert q.dim() == 4 and q.shape[2] == 1, f"Decode expects [B,H,1,D], got {q.shape}"
    store = _legacy.build_store(k_data, k_scales, k_zps, v_data, v_scales, v_zps)
    return _legacy.decode(q, store, sm_scale, torch.float32).to(q.dtype)


def fused_dequant_attn_forward(q: torch.Tensor, k_data, k_scales, k_zps, v_data, v_scales, v_zps,
                               sm_scale: Optional[float] = None) -> torch.Tensor:
    assert q.dim() == 4, f"Forward expects [B,H,S,D], got {q.shape}"
    store = _legacy.build_store(k_data, k_scales, k_zps, v_data, v_scales, v_zps)
    return _legacy.forward(q, store, sm_scale, torch.float32).to(q.dtype)
