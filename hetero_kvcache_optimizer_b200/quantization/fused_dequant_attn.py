"""Drop-in for src/quantization/fused_dequant_attn.py (returns fp32).

``fused_dequant_attn_decode`` (reference :254-331) and
``fused_dequant_attn_forward`` (:158-247) keep their signatures; both run the
split-KV INT4 CUDA kernel of libhetero_kv (GQA when q has more heads than
K/V). Unlike the reference (:239-240, :323-324) nothing falls back to a
PyTorch path on error: failures raise.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _legacy
from .. import kvstore as kv


def fused_dequant_attn_forward(Q: torch.Tensor, K_quant, K_scales: torch.Tensor, K_zps: torch.Tensor,
                               V_quant: torch.Tensor, V_scales: torch.Tensor, V_zps: torch.Tensor,
                               sm_scale: Optional[float] = None) -> torch.Tensor:
    """[B, H, Sq, D] queries against INT4 K/V, no causal mask -> fp32 [B, H, Sq, D]."""
    store = _legacy.build_store(K_quant, K_scales, K_zps, V_quant, V_scales, V_zps)
    return _legacy.forward(Q, store, sm_scale, torch.float32)


def fused_dequant_attn_decode(q: torch.Tensor, k_quant, k_scales: torch.Tensor, k_zps: torch.Tensor,
                              v_quant: torch.Tensor, v_scales: torch.Tensor, v_zps: torch.Tensor,
                              sm_scale: Optional[float] = None) -> torch.Tensor:
    """q [B, Hq, 1, D] against INT4 K/V -> fp32 [B, Hq, 1, D]."""
    store = _legacy.build_store(k_quant, k_scales, k_zps, v_quant, v_scales, v_zps)
    return _legacy.decode(q, store, sm_scale, torch.float32)


def fused_dequant_attention(q: torch.Tensor, k_quant: torch.Tensor, k_scales: torch.Tensor,
                            k_zps: torch.Tensor, group_size: int = 128) -> torch.Tensor:
    """Legacy single-head scores q . dequant(K)^T (reference :338-381): [S] fp32.
    The reference reads one scale and zero-point per key (k_scales.reshape(seq_k),
    :354-355), i.e. groups of head_dim values; so does this call."""
    q_flat = q.reshape(-1)
    D = q_flat.shape[0]
    S = k_quant.shape[0] if k_quant.dim() >= 1 else 1
    return kv.qk_scores_flat(q_flat, k_quant.reshape(S, D), k_scales.reshape(S), k_zps.reshape(S), D)
