"""Drop-in ``FusedHeteroCache`` (reference: src/core/engine_wrapper.py:32-404).

A HuggingFace ``DynamicCache`` subclass backed by ``HeteroKVManager``, with the
reference's constructor keywords and methods (``update``, ``get_seq_length``,
``seen_tokens``, ``get_mask_sizes``, ``allocate``, ``compress``,
``memory_summary``, ``dram_table``, ``schedule_prefetch``, ``swap_in_chunk``,
``swap_in_quantized``, ``fused_attn_on_swapped``).

What ``update`` returns follows the reference: the full K/V during prefill, the
HBM-resident [sink ; tail] during decode, and, with ``self_healing`` (its full
retrieval path, engine_wrapper.py:236-245), the INT4 body dequantised to bf16
in front of them, so a stock attention layer sees the whole context. The fast
path does not materialise anything: ``attend(q, layer_idx)`` runs the fused
INT4 decode kernel over [sink ; INT4 body ; tail] of that layer.

With ``adaptive_self_healing`` the decode step follows the reference's paths A
(``enable_triton``: the top-w_t DRAM chunks stay INT4 on the device in
``_dram_quant_kv``) and B (they are dequantised to bf16 in front of [sink ;
tail]), w_t from the manager's window controller. Method D (query-aware
retrieval) is accepted as a keyword and rejected when enabled, rather than
silently ignored.
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch
from transformers.cache_utils import DynamicCache

from ..memory.manager import HeteroKVManager
from ..quantization.kernels.fused_dequant_attn import fused_dequant_attn_decode, fused_dequant_attn_forward


class FusedHeteroCache(DynamicCache):
    def __init__(self, num_layers: Optional[int] = None, sink_tokens: int = 64, keep_tail: int = 8192,
                 chunk_size: int = 2048, device: str = "cuda:0", group_size: int = 128,
                 enable_quant: bool = True, enable_prefetch: bool = True, enable_triton: bool = True,
                 bandwidth_limiter=None, self_healing: bool = True, adaptive_self_healing: bool = False,
                 enable_method_d: bool = False, method_d_alpha: float = 1.0, **manager_kwargs):
        super().__init__()
        if enable_method_d:
            raise NotImplementedError("Method D (query-aware retrieval) is a policy feature outside this "
                                      "build's INT4 hot path")
        self.sink_tokens = sink_tokens
        self.keep_tail = keep_tail
        self.chunk_size = chunk_size
        self.device = device
        self.enable_quant = enable_quant
        self.enable_prefetch = enable_prefetch
        self.enable_triton = enable_triton
        self.group_size = group_size
        self._bandwidth_limiter = bandwidth_limiter
        self.self_healing = self_healing
        self.adaptive_self_healing = adaptive_self_healing
        self.enable_method_d = enable_method_d
        self.method_d_alpha = method_d_alpha
        self._num_layers = num_layers
        self._manager_kwargs = manager_kwargs
        self._manager: Optional[HeteroKVManager] = None
        self.real_seq_len = 0
        self._swap_in_tokens = 0
        self._pending_attention_weights: Optional[torch.Tensor] = None
        self._dram_quant_kv: Optional[Dict[str, torch.Tensor]] = None  # path A's INT4 chunks
        self._dram_quant_layer = -1

    def _ensure_manager(self, layer_idx: int) -> HeteroKVManager:
        if self._manager is None:
            n = self._num_layers if self._num_layers is not None else layer_idx + 1
            self._manager = HeteroKVManager(num_layers=n, sink_tokens=self.sink_tokens,
                                            hbm_budget_tokens=self.keep_tail, device=self.device,
                                            enable_quant=self.enable_quant, enable_prefetch=self.enable_prefetch,
                                            group_size=self.group_size, bandwidth_limiter=self._bandwidth_limiter,
                                            **self._manager_kwargs)
        return self._manager

    # ------------------------------------------------------------------ DynamicCache interface
    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[Dict[str, Any]] = None, *args, **kwargs) -> Tuple[torch.Tensor, torch.Tensor]:
        m = self._ensure_manager(layer_idx)
        new_len = key_states.shape[-2]
        mode = "prefill" if new_len > 1 else "decode"
        out_k, out_v = m.update(layer_idx=layer_idx, key_states=key_states, value_states=value_states, mode=mode,
                                seq_offset=self.real_seq_len)
        last = self._num_layers is not None and layer_idx == self._num_layers - 1
        if mode == "decode" and last and self._pending_attention_weights is not None:
            m.update_attention_scores(self._pending_attention_weights)
            self._pending_attention_weights = None
        adaptive_count = None
        if mode == "decode" and self.self_healing and self.adaptive_self_healing and self.enable_triton:
            # path A (reference engine_wrapper.py:205-221): the top-w_t chunks stay
            # INT4 on the device for a fused consumer; nothing is concatenated
            self._dram_quant_kv = m.get_dram_chunks_quantized_adaptive(layer_idx)
            self._dram_quant_layer = layer_idx
        elif mode == "decode" and self.self_healing and self.adaptive_self_healing:
            # path B (:223-234): the top-w_t chunks dequantised to bf16 in front
            dk, dv, n = m.decompress_dram_chunks_adaptive(layer_idx)
            adaptive_count = n
            if dk is not None and n > 0:
                out_k = torch.cat([dk.to(out_k.dtype), out_k], dim=-2)
                out_v = torch.cat([dv.to(out_v.dtype), out_v], dim=-2)
        elif mode == "decode" and self.self_healing and self._swap_in_tokens > 0:
            # path C (:236-245): the whole INT4 body dequantised to bf16 in front
            dk, dv, n = m.decompress_dram_chunks(layer_idx)
            if dk is not None and n > 0:
                out_k = torch.cat([dk.to(out_k.dtype), out_k], dim=-2)
                out_v = torch.cat([dv.to(out_v.dtype), out_v], dim=-2)
        if layer_idx == 0:
            self.real_seq_len += new_len
            if mode == "decode" and self.self_healing:
                self._swap_in_tokens = (adaptive_count if adaptive_count is not None
                                        else 0 if self.adaptive_self_healing and self.enable_triton
                                        else m.count_dram_tokens(layer_idx=0))
        return out_k, out_v

    def attend(self, q: torch.Tensor, layer_idx: int, sm_scale: Optional[float] = None,
               out_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
        """Fused decode attention of q [B, Hq, 1, 128] over the layer's whole
        context ([sink ; INT4 body ; tail]); returns [B, Hq, 1, 128]."""
        m = self._ensure_manager(layer_idx)
        out = m.attend(layer_idx, q, sm_scale=sm_scale, out_dtype=out_dtype or q.dtype)
        return out if out.dim() == 4 else out[:, :, None, :]

    def holds_layer(self, layer_idx: int) -> bool:
        """Whether ``attend`` can serve this layer (it holds cached tokens)."""
        m = self._manager
        return (m is not None and layer_idx < len(m._dense) and m._dense[layer_idx] is not None
                and m._dense_len[layer_idx] > 0)

    def get_seq_length(self, layer_idx: int = 0) -> int:
        if self._manager is None or self._manager._dense[layer_idx] is None:
            return 0
        return self._manager._dense_len[layer_idx] + (self._swap_in_tokens if self.self_healing else 0)

    @property
    def seen_tokens(self) -> int:
        return self.real_seq_len

    def get_mask_sizes(self, cache_position, layer_idx: int = 0, *args, **kwargs) -> Tuple[int, int]:
        # transformers >= 5 passes the query length, earlier versions the cache positions
        q = cache_position if isinstance(cache_position, int) else cache_position.shape[0]
        if self._manager is None or self._manager._dense[layer_idx] is None:
            return q, 0
        m = self._manager
        phys = m._dense_len[layer_idx]
        if q > 1:
            return phys + q, 0
        swap = self._swap_in_tokens if self.self_healing else 0
        full = phys >= m.sink_tokens + m.tail_budget
        return phys + swap + (0 if full else 1), 0

    # ------------------------------------------------------------------ tiered storage passthrough
    def allocate(self, layer_idx: int, seq_len: int = 0, budget_tokens: Optional[int] = None) -> bool:
        return self._ensure_manager(layer_idx).allocate(layer_idx, budget_tokens)

    def compress(self, layer_idx: int, device: str = "DRAM") -> int:
        return self._ensure_manager(layer_idx).compress(layer_idx, device)

    def memory_summary(self) -> Dict[str, Any]:
        if self._manager is None:
            return {"hbm_tokens": 0, "dram_entries": 0, "dram_bytes": 0,
                    "max_hbm_tokens": self.sink_tokens + self.keep_tail}
        return self._manager.memory_summary()

    @property
    def dram_table(self) -> Dict[str, Dict[str, torch.Tensor]]:
        return {} if self._manager is None else self._manager._dram_table

    def schedule_prefetch(self, chunk_key: str) -> None:
        if self._manager is not None:
            self._manager.schedule_prefetch(chunk_key)

    def swap_in_chunk(self, chunk_key: str) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        return None if self._manager is None else self._manager.swap_in(0, chunk_key)

    def swap_in_quantized(self, chunk_key: str) -> Optional[Dict[str, torch.Tensor]]:
        return None if self._manager is None else self._manager.swap_in_quantized(0, chunk_key)

    def fused_attn_on_swapped(self, q: torch.Tensor, chunk_key: str,
                              sm_scale: Optional[float] = None) -> Optional[torch.Tensor]:
        """Fused INT4 attention of q [B, H, Sq, D] over one DRAM chunk (the
        reference's engine_wrapper.py:357-404; errors raise, no torch fallback)."""
        qd = self.swap_in_quantized(chunk_key)
        if qd is None:
            return None
        fn = fused_dequant_attn_decode if q.shape[2] == 1 else fused_dequant_attn_forward
        return fn(q, qd["k_data"], qd["k_scales"], qd["k_zps"], qd["v_data"], qd["v_scales"], qd["v_zps"],
                  sm_scale=sm_scale)
