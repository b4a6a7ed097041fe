"""Drop-in ``KVCompressor`` (reference: src/quantization/kv_compressor.py:24-171).

Same constructor, methods, argument meaning and return contract; the
arithmetic runs in libhetero_kv's CUDA kernels and is bit-identical to the
reference's fp32 torch code (codes, scales and zero-points). CUDA tensors
only: a CPU tensor raises instead of falling back.

Added: ``compress_packed`` returns the nibble-packed page format consumed by
the fused decode kernel (half the bytes of the reference's one-code-per-byte
layout).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import kvstore as kv


class KVCompressor:
    """4-bit group-wise asymmetric quantiser (kv_compressor.py:24-35):
    scale = (max - min) / 15, zero_point = clamp(round(-min / scale), 0, 15),
    Q = clamp(round(X / scale + zero_point), 0, 15); X' = (Q - zero_point) * scale."""

    def __init__(self, group_size: int = 128, bits: int = 4):
        assert bits == 4, "Current implementation only supports 4-bit quantization"
        self.group_size = group_size
        self.bits = bits
        self.qmax = (1 << bits) - 1
        self.qmin = 0
        print(f"[KVCompressor] init | bits={bits} group_size={group_size}")

    def compress(self, tensor: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(quantized uint8 shaped like ``tensor``, scales f32 [num_groups],
        zero_points uint8 [num_groups]) over the flattened tensor, last group
        zero-padded (kv_compressor.py:50-98)."""
        return kv.quantize_flat(tensor, self.group_size)

    def decompress(self, quantized: torch.Tensor, scales: torch.Tensor, zero_points: torch.Tensor,
                   target_dtype: torch.dtype = torch.float16) -> torch.Tensor:
        """(Q - zero_point) * scale in fp32, cast to ``target_dtype`` (kv_compressor.py:100-132)."""
        return kv.dequantize_flat(quantized, scales, zero_points, self.group_size, dtype=target_dtype)

    def mse_error(self, original: torch.Tensor, quantized: torch.Tensor, scales: torch.Tensor,
                  zero_points: torch.Tensor) -> float:
        restored = self.decompress(quantized, scales, zero_points, target_dtype=original.dtype)
        return torch.nn.functional.mse_loss(restored, original.float()).item()

    def relative_error(self, original: torch.Tensor, quantized: torch.Tensor, scales: torch.Tensor,
                       zero_points: torch.Tensor) -> float:
        restored = self.decompress(quantized, scales, zero_points, target_dtype=original.dtype)
        orig_f = original.float()
        rel = (restored.float() - orig_f).abs().mean() / (orig_f.abs().mean() + 1e-8)
        return rel.item() * 100.0

    def compression_ratio(self, tensor: torch.Tensor) -> float:
        """Theoretical ratio (kv_compressor.py:160-171): 4 bits/value + 40 bits/group vs fp16."""
        n = tensor.numel()
        bits_orig = n * 16
        num_groups = (n + self.group_size - 1) // self.group_size
        bits_quant = n * 4 + num_groups * (32 + 8)
        return 1.0 - bits_quant / bits_orig

    # ------------------------------------------------------------------ packed format
    def compress_packed(self, k: torch.Tensor, v: torch.Tensor, fmt: str = "ref",
                        page_tokens: int = 256, capacity: Optional[int] = None) -> kv.Int4KVStore:
        """Quantise K and V [B, H, T, 128] into a nibble-packed INT4 store
        (group = this compressor's group size). With fmt="ref" the codes,
        scales and zero-points are those ``compress`` returns, just packed."""
        B, H, T, D = k.shape
        if D != 128:
            raise ValueError("the packed format needs head_dim 128")
        store = kv.Int4KVStore(B, H, capacity or max(T, 1), fmt=fmt, group=self.group_size,
                               page_tokens=page_tokens, device=k.device)
        kv.prefill(store, k, v)
        return store


PackedKV = kv.Int4KVStore

__all__ = ["KVCompressor", "PackedKV"]
