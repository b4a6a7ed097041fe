"""Drop-in ``HeteroKVManager`` (reference: src/memory/manager.py:30-1319).

Same constructor, public methods and return contracts for the INT4 hot path:
``allocate``, ``update`` (prefill / incremental prefill / decode), ``compress``,
``swap_in_quantized``, ``swap_in``, ``get_hbm_kv``, ``get_seq_offset``,
``schedule_prefetch``, ``memory_summary``, ``max_hbm_tokens``,
``count_dram_tokens``, ``decompress_dram_chunks``, ``update_attention_scores``,
``get_oracle_scores``, ``_dram_table``.

Storage per layer (all on the device, sizes fixed at the first prefill):
  * sink + tail ("recent") tokens in fp16/bf16: one ``DenseKV`` of
    ``sink + (hbm_budget_tokens - sink)`` rows, the tail kept as a ring;
  * every token evicted from sink + tail as packed INT4 pages in an
    ``Int4KVStore`` (format ``ref``: bit-exact with KVCompressor at the
    manager's group size), written by the quantise-pack / append kernels.
Decode attention runs over [sink ; INT4 body ; tail] in one fused kernel
(``attend``): nothing is decompressed, concatenated or synchronised per step.

With ``hbm_body_pages`` set, the INT4 body gets a host (DRAM) tier
(``host_tier.HostTier``): the last ``hbm_body_pages`` pages per (layer,
sequence x KV head) stay in HBM, older pages move to pinned host memory as the
body grows, and ``attend`` stages a layer's host pages into a shared staging
area (copied while the previous layer's attention runs) and reads them through
the page table, as the reference's eviction to DRAM and swap-in do
(manager.py:1231-1299, :779-821).

Prefill evictions are also kept as the reference's DRAM entries
(``l{layer}_e{n}``: unpacked u8 codes, f32 scales, u8 zero-points in pinned
host memory, bit-exact with ``KVCompressor.compress``) when ``legacy_dram`` is
set, so ``_dram_table``, ``swap_in_quantized``, ``schedule_prefetch`` and the
adaptive self-healing retrievals (``get_dram_chunks_quantized_adaptive``,
``decompress_dram_chunks_adaptive``: the top-w_t chunks by attention score,
w_t from the window controller) keep working for callers of the old API.

Not rebuilt (policy, outside the INT4 hot path): the HeavyHitter zone and its
attention-competition queue (decode evictions go straight to the INT4 body),
Method D query-aware retrieval, the predictive prefetch scheduler
(``predictive_prefetch_step`` returns no keys). ``get_oracle_scores`` returns
the attention mass accumulated per token by ``update_attention_scores``.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import torch

from .. import kvstore as kv
from ..policy.chunk_scores import DeviceWindowController
from ..policy.prefetcher import AsyncPrefetcher
from ..quantization.kv_compressor import KVCompressor
from .dram_storage import DRAMStorageManager
from .host_tier import HostTier


class HeteroKVManager:
    def __init__(self, num_layers: int, sink_tokens: int = 64, hbm_budget_tokens: int = 8192,
                 device: str = "cuda", enable_quant: bool = True, enable_prefetch: bool = True,
                 group_size: int = 128, bits: int = 4, bandwidth_limiter=None,
                 enable_method_d: bool = False, method_d_alpha: float = 1.0, *,
                 body_capacity: Optional[int] = None, legacy_dram: bool = True,
                 page_tokens: int = 256, kv_format: str = "ref", hbm_body_pages: Optional[int] = None):
        if not enable_quant:
            raise ValueError("the INT4 body is the point of this build: enable_quant=False is not supported")
        if bits != 4:
            raise ValueError("only 4-bit quantisation is supported")
        self.num_layers = num_layers
        self.sink_tokens = sink_tokens
        self.hbm_budget_tokens = hbm_budget_tokens
        self.device = device
        self.enable_quant = enable_quant
        self.group_size = group_size
        self.bits = bits
        self.kv_format = kv_format
        self.page_tokens = page_tokens
        self.legacy_dram = legacy_dram
        self._bandwidth_limiter = bandwidth_limiter
        self._body_capacity = body_capacity
        self._compressor = KVCompressor(group_size=group_size, bits=bits)
        self._dram = DRAMStorageManager()
        self._prefetcher: Optional[AsyncPrefetcher] = (
            AsyncPrefetcher(device=torch.device(device)) if enable_prefetch and torch.cuda.is_available() else None)
        self._dense: List[Optional[kv.DenseKV]] = [None] * num_layers
        self._body: List[Optional[kv.Int4KVStore]] = [None] * num_layers
        self._seq_offsets: List[int] = [0] * num_layers
        self._dense_len: List[int] = [0] * num_layers   # host mirror of the device lengths
        self._body_len: List[int] = [0] * num_layers
        self._ring_head: List[int] = [0] * num_layers
        self._eviction_counter = 0
        self._chunk_eviction_order: List[str] = []
        self._chunk_tokens: Dict[str, int] = {}
        self._token_scores: Optional[torch.Tensor] = None
        self._last_attention_weights: Optional[torch.Tensor] = None
        # host (DRAM) tier of the INT4 body: the last hbm_body_pages pages per
        # (layer, sequence x KV head) stay in HBM, older ones in pinned host
        # memory, staged layer-ahead for the attention (None: all in HBM)
        self.hbm_body_pages = hbm_body_pages
        self._tier: Optional[HostTier] = None
        # reference bookkeeping for the adaptive self-healing retrieval
        # (manager.py:138, :1261-1272): score of every legacy DRAM chunk, and the
        # window controller (adaptive_prefetch_controller.py:77-133)
        self._chunk_attention_scores: Dict[str, float] = {}
        self._adaptive_controller = DeviceWindowController(device=device) if torch.cuda.is_available() else None

    # ------------------------------------------------------------------ geometry
    @property
    def tail_budget(self) -> int:
        return max(0, self.hbm_budget_tokens - self.sink_tokens)

    @property
    def _dram_table(self) -> Dict[str, Dict[str, torch.Tensor]]:
        return self._dram.table

    def allocate(self, layer: int, budget: Optional[int] = None) -> bool:
        if layer < 0 or layer >= self.num_layers:
            raise ValueError(f"Invalid layer {layer}, num_layers={self.num_layers}")
        if budget is not None:
            self.hbm_budget_tokens = budget
        return True

    def _ensure_layer(self, layer: int, ref: torch.Tensor, total_tokens: int) -> None:
        if self._dense[layer] is not None:
            return
        B, H, _, D = ref.shape
        if D != 128:
            raise ValueError("head_dim must be 128")
        dtype = ref.dtype if ref.dtype in (torch.float16, torch.bfloat16) else torch.float16
        self._dense[layer] = kv.DenseKV(B, H, self.sink_tokens + self.tail_budget, dtype=dtype, device=ref.device)
        self._dense[layer].set_lengths(0)
        self._dense[layer].ring_head.zero_()
        cap = self._body_capacity or max(total_tokens, 1) * 2 + 4096
        if self.hbm_body_pages is not None:
            if self._tier is None:
                self._tier = HostTier(self.num_layers, B, H, cap, resident_pages=self.hbm_body_pages,
                                      fmt=self.kv_format, group=self.group_size, page_tokens=self.page_tokens,
                                      device=ref.device)
            self._body[layer] = self._tier.views[layer]
        else:
            self._body[layer] = kv.Int4KVStore(B, H, cap, fmt=self.kv_format, group=self.group_size,
                                               page_tokens=self.page_tokens, device=ref.device)
        self._body[layer].set_lengths(0)

    # ------------------------------------------------------------------ update
    def update(self, layer_idx: int, key_states: torch.Tensor, value_states: torch.Tensor,
               mode: str = "prefill", seq_offset: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
        if mode == "prefill":
            if self._dense[layer_idx] is not None and self._dense_len[layer_idx] > 0:
                return self._incremental_prefill_update(layer_idx, key_states, value_states, seq_offset)
            return self._prefill_update(layer_idx, key_states, value_states, seq_offset)
        if mode == "decode":
            return self._decode_update(layer_idx, key_states, value_states, seq_offset)
        raise ValueError(f"Unknown mode: {mode}")

    def _evict(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantise tokens into the INT4 body (and keep the legacy DRAM entry)."""
        n = k.shape[-2]
        if n == 0:
            return
        st = self._body[layer]
        start = self._body_len[layer]
        if start + n > st.capacity:
            raise RuntimeError(f"INT4 body of layer {layer} is full ({st.capacity} tokens); "
                               "raise body_capacity")
        if self._tier is not None:
            self._tier.write(layer, start, k, v)
        else:
            kv.quantize_pack_kv(k, v, st, start)
        self._body_len[layer] = start + n
        st.set_lengths(start + n)
        if self.legacy_dram:
            key = f"l{layer}_e{self._eviction_counter}"
            qk, sk, zk = self._compressor.compress(k)
            qv, sv, zv = self._compressor.compress(v)
            self._dram.store_entry(key, {"k_data": qk, "k_scales": sk, "k_zps": zk,
                                         "v_data": qv, "v_scales": sv, "v_zps": zv})
            self._chunk_eviction_order.append(key)
            self._chunk_tokens[key] = n
            self._chunk_attention_scores[key] = self._chunk_score(layer, start, n)
        if layer == 0:  # chunk keys advance with layer 0, as the reference's (manager.py:1311-1313)
            self._eviction_counter += 1

    def _write_tail(self, layer: int, tail_k: torch.Tensor, tail_v: torch.Tensor) -> None:
        d = self._dense[layer]
        n = tail_k.shape[-2]
        s = self.sink_tokens
        d.k[:, :, s:s + n] = tail_k
        d.v[:, :, s:s + n] = tail_v
        self._ring_head[layer] = 0
        d.ring_head.zero_()

    def _prefill_update(self, layer: int, k: torch.Tensor, v: torch.Tensor, seq_offset: int):
        S = k.shape[-2]
        self._ensure_layer(layer, k, S)
        d = self._dense[layer]
        sink_amt = min(S, self.sink_tokens)
        tail_amt = min(S - sink_amt, self.tail_budget)
        d.k[:, :, :sink_amt] = k[:, :, :sink_amt]
        d.v[:, :, :sink_amt] = v[:, :, :sink_amt]
        if sink_amt < self.sink_tokens:
            # a short first chunk: there is no tail yet, the sink is still filling
            self._dense_len[layer] = sink_amt
        else:
            self._write_tail(layer, k[:, :, S - tail_amt:], v[:, :, S - tail_amt:])
            self._dense_len[layer] = sink_amt + tail_amt
        d.set_lengths(self._dense_len[layer])
        self._evict(layer, k[:, :, sink_amt:S - tail_amt], v[:, :, sink_amt:S - tail_amt])
        self._seq_offsets[layer] = seq_offset + S
        return k, v

    def _incremental_prefill_update(self, layer: int, k: torch.Tensor, v: torch.Tensor, seq_offset: int):
        S = k.shape[-2]
        d = self._dense[layer]
        sink_k, sink_v = d.k[:, :, :self.sink_tokens], d.v[:, :, :self.sink_tokens]
        old_k, old_v = self._tail_logical(layer)
        comb_k = torch.cat([old_k, k.to(d.dtype)], dim=-2)
        comb_v = torch.cat([old_v, v.to(d.dtype)], dim=-2)
        ret_k = torch.cat([sink_k[:, :, :min(self._dense_len[layer], self.sink_tokens)], comb_k], dim=-2)
        ret_v = torch.cat([sink_v[:, :, :min(self._dense_len[layer], self.sink_tokens)], comb_v], dim=-2)
        n = comb_k.shape[-2]
        ev = max(0, n - self.tail_budget)
        self._evict(layer, comb_k[:, :, :ev], comb_v[:, :, :ev])
        self._write_tail(layer, comb_k[:, :, ev:].clone(), comb_v[:, :, ev:].clone())
        self._dense_len[layer] = self.sink_tokens + (n - ev)
        d.set_lengths(self._dense_len[layer])
        self._seq_offsets[layer] = seq_offset + S
        return ret_k, ret_v

    def _decode_update(self, layer: int, k: torch.Tensor, v: torch.Tensor, seq_offset: int):
        if self._dense[layer] is None:
            self._ensure_layer(layer, k, 1)
        d, st = self._dense[layer], self._body[layer]
        if self._tier is not None and self._dense_len[layer] >= d.capacity:
            self._tier.prepare_write(layer, self._body_len[layer] + 1)  # the step adds a body token
        kv.append_kv(k.to(d.dtype), v.to(d.dtype), d, self.sink_tokens, st)
        cap = d.capacity
        if self._dense_len[layer] < cap:
            self._dense_len[layer] += 1
        else:
            self._body_len[layer] += 1
            self._ring_head[layer] = (self._ring_head[layer] + 1) % max(1, self.tail_budget)
        st.len_hint = self._body_len[layer]
        self._seq_offsets[layer] = seq_offset + 1
        return self.get_hbm_kv(layer)

    def _tail_logical(self, layer: int) -> Tuple[torch.Tensor, torch.Tensor]:
        d = self._dense[layer]
        s, n = self.sink_tokens, max(0, self._dense_len[layer] - self.sink_tokens)
        h = self._ring_head[layer] if n == self.tail_budget else 0
        idx = (torch.arange(n, device=d.k.device) + h) % max(1, n) + s
        return d.k[:, :, idx], d.v[:, :, idx]

    # ------------------------------------------------------------------ fused decode attention
    def attend(self, layer_idx: int, q: torch.Tensor, sm_scale: Optional[float] = None,
               out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
        """softmax(q K^T) V over [sink ; INT4 body ; tail] of the layer, in one
        launch of the fused decode kernel. q: [B, Hq, 128] or [B, Hq, 1, 128]."""
        st, d = self._body[layer_idx], self._dense[layer_idx]
        if d is None:
            raise RuntimeError(f"Layer {layer_idx} has not been allocated yet.")
        tier = self._tier
        if tier is not None:
            tier.gate(layer_idx)  # this layer's host pages are in its staging area
            nxt = layer_idx + 1
            if nxt < self.num_layers and self._body[nxt] is not None:
                tier.stage(nxt)  # layer-ahead: copied while this layer's attention runs
        o = kv.decode(q, st if self._body_len[layer_idx] > 0 else None, d, sm_scale=sm_scale,
                      out=out, out_dtype=out_dtype, body_len=self._body_len[layer_idx],
                      dense_len=self._dense_len[layer_idx])
        if tier is not None:
            tier.release(layer_idx)
        return o

    # ------------------------------------------------------------------ reference API
    def compress(self, layer: int, device: str = "DRAM") -> int:
        """Move every HBM tail token beyond the sink into the INT4 body."""
        if device.upper() != "DRAM":
            raise NotImplementedError("Only DRAM compression is currently supported.")
        if self._dense[layer] is None or self._dense_len[layer] <= self.sink_tokens:
            return 0
        tk, tv = self._tail_logical(layer)
        n = tk.shape[-2]
        self._evict(layer, tk.contiguous(), tv.contiguous())
        self._dense_len[layer] = self.sink_tokens
        self._ring_head[layer] = 0
        self._dense[layer].set_lengths(self.sink_tokens)
        self._dense[layer].ring_head.zero_()
        return n

    def swap_in_quantized(self, layer_idx: int, chunk_key: str) -> Optional[Dict[str, torch.Tensor]]:
        entry = self._dram.retrieve(chunk_key) if chunk_key in self._dram else None
        if entry is None:
            return None
        return {key: entry[key].to(self.device, non_blocking=True)
                for key in ("k_data", "k_scales", "k_zps", "v_data", "v_scales", "v_zps")}

    def swap_in(self, layer_idx: int, chunk_key: str) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        if not self._dram.contains(chunk_key):
            return None
        if self._prefetcher is not None:
            hit = self._prefetcher.fetch_if_ready(chunk_key)
            if hit is not None:
                self._dram.remove(chunk_key)
                return hit
        q = self.swap_in_quantized(layer_idx, chunk_key)
        self._dram.remove(chunk_key)
        k = self._compressor.decompress(q["k_data"], q["k_scales"], q["k_zps"]).to(torch.bfloat16)
        v = self._compressor.decompress(q["v_data"], q["v_scales"], q["v_zps"]).to(torch.bfloat16)
        return k, v

    def get_hbm_kv(self, layer_idx: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """[sink ; tail] in logical order (the HBM-resident fp16/bf16 tokens)."""
        d = self._dense[layer_idx]
        if d is None:
            raise RuntimeError(f"Layer {layer_idx} has not been allocated yet.")
        ns = min(self._dense_len[layer_idx], self.sink_tokens)
        tk, tv = self._tail_logical(layer_idx)
        return (torch.cat([d.k[:, :, :ns], tk], dim=-2), torch.cat([d.v[:, :, :ns], tv], dim=-2))

    def get_seq_offset(self, layer_idx: int) -> int:
        return self._seq_offsets[layer_idx]

    def update_attention_scores(self, attention_weights: torch.Tensor) -> None:
        w = attention_weights.detach().float()
        mass = w.reshape(-1, w.shape[-1]).sum(0)
        if self._token_scores is None or self._token_scores.numel() < mass.numel():
            old = self._token_scores
            self._token_scores = torch.zeros(mass.numel(), device=mass.device)
            if old is not None:
                self._token_scores[:old.numel()] += old
        self._token_scores[:mass.numel()] += mass
        self._last_attention_weights = attention_weights.detach().clone()

    def get_oracle_scores(self) -> Optional[torch.Tensor]:
        return self._token_scores

    def schedule_prefetch(self, chunk_key: str) -> None:
        if self._prefetcher is None or not self._dram.contains(chunk_key):
            return
        self._prefetcher.submit_prefetch_task(chunk_key, self._dram.retrieve(chunk_key), self._compressor)

    def predictive_prefetch_step(self, current_chunk: Optional[str] = None,
                                 attention_weights: Optional[torch.Tensor] = None,
                                 cache_miss: bool = False) -> List[str]:
        return []

    def count_dram_tokens(self, layer_idx: int = 0) -> int:
        """Tokens of the layer held outside the fp16 zones (the INT4 body)."""
        return self._body_len[layer_idx]

    def decompress_dram_chunks(self, layer_idx: int):
        """(k, v, count): the whole INT4 body of the layer dequantised to bf16
        (the reference's full-retrieval path), or (None, None, 0)."""
        n = self._body_len[layer_idx]
        if n == 0:
            return None, None, 0
        st = self._body[layer_idx]
        if self._tier is not None:
            self._tier.gate(layer_idx)
        k = kv.dequantize_pack(st, 0, 0, n, dtype=torch.bfloat16)
        v = kv.dequantize_pack(st, 1, 0, n, dtype=torch.bfloat16)
        if self._tier is not None:
            self._tier.release(layer_idx)
        return k, v, n

    # ------------------------------------------------------------------ adaptive retrieval (legacy entries)
    def _chunk_score(self, layer: int, start: int, n: int) -> float:
        """Score of a chunk at eviction (reference manager.py:1261-1272): the mean
        accumulated attention score of its tokens when scores exist, else the
        FIFO fallback 1 / (eviction counter + 1). The chunk's tokens are body
        slots [start, start + n), absolute positions sink + start onwards."""
        ts = self._token_scores
        if ts is not None:
            a = self.sink_tokens + start
            seg = ts[a:a + n]
            return float(seg.mean().item()) if seg.numel() else 0.0
        return 1.0 / (self._eviction_counter + 1)

    def _layer_chunk_keys(self, layer_idx: int) -> List[str]:
        prefix = f"l{layer_idx}_"
        return [k for k in self._chunk_eviction_order if k.startswith(prefix) and k in self._dram]

    def _window(self, n_keys: int, window_size: Optional[int]) -> int:
        if window_size is None:
            w = (int(self._adaptive_controller.compute_window(attention_weights=self._last_attention_weights))
                 if self._adaptive_controller is not None else 2)
            window_size = w
        return max(1, min(int(window_size), n_keys))

    def _select_chunks(self, layer_idx: int, window_size: Optional[int]) -> List[str]:
        """Top-w chunks of the layer by score, returned in eviction order
        (reference manager.py:859-872, :904-906)."""
        keys = self._layer_chunk_keys(layer_idx)
        if not keys:
            return []
        w = self._window(len(keys), window_size)
        ranked = sorted(keys, key=lambda k: self._chunk_attention_scores.get(k, 0.0), reverse=True)[:w]
        order = {k: i for i, k in enumerate(self._chunk_eviction_order)}
        return sorted(ranked, key=lambda k: order[k])

    @staticmethod
    def _per_token_meta(entry: Dict[str, torch.Tensor], name: str) -> torch.Tensor:
        """A chunk's flat scales / zero-points as [..., tokens, groups] so that
        chunks concatenate along the token axis like their codes do."""
        data = entry["k_data" if name.startswith("k") else "v_data"]
        t = entry[name]
        ng = t.numel() // max(1, data.numel() // data.shape[-1])
        return t.reshape(*data.shape[:-1], ng)

    def get_dram_chunks_quantized_adaptive(self, layer_idx: int,
                                           window_size: Optional[int] = None) -> Optional[Dict[str, torch.Tensor]]:
        """The top-w_t DRAM chunks of the layer by attention score, still INT4,
        on the device and concatenated in eviction order (reference
        manager.py:931-1056): k_data / v_data along the token axis; scales and
        zero-points flat, in the order of the concatenated codes (the
        reference concatenates 1-D metadata chunk after chunk, which matches
        the codes only for one sequence and one head). None without chunks."""
        keys = self._select_chunks(layer_idx, window_size)
        if not keys:
            return None
        parts: Dict[str, List[torch.Tensor]] = {k: [] for k in ("k_data", "k_scales", "k_zps", "v_data",
                                                                 "v_scales", "v_zps")}
        for key in keys:
            e = self._dram.transfer_to_device(key, torch.device(self.device))
            for name in parts:
                parts[name].append(e[name] if name.endswith("data") else self._per_token_meta(e, name))
        out = {name: torch.cat(ts, dim=-2) for name, ts in parts.items()}
        for name in ("k_scales", "k_zps", "v_scales", "v_zps"):
            out[name] = out[name].reshape(-1)
        return out

    def decompress_dram_chunks_adaptive(self, layer_idx: int, window_size: Optional[int] = None):
        """(k, v, tokens): the top-w_t DRAM chunks of the layer dequantised to
        bf16 and concatenated in eviction order (reference manager.py:823-929),
        or (None, None, 0)."""
        q = self.get_dram_chunks_quantized_adaptive(layer_idx, window_size)
        if q is None:
            return None, None, 0
        k = self._compressor.decompress(q["k_data"], q["k_scales"], q["k_zps"], target_dtype=torch.bfloat16)
        v = self._compressor.decompress(q["v_data"], q["v_scales"], q["v_zps"], target_dtype=torch.bfloat16)
        return k, v, int(k.shape[-2])

    def _get_dram_kv_quantized(self, layer_idx: int) -> Optional[Dict[str, torch.Tensor]]:
        """Every DRAM chunk of the layer, INT4, concatenated in eviction order
        (reference manager.py:1160-1216; here on the device)."""
        keys = self._layer_chunk_keys(layer_idx)
        return self.get_dram_chunks_quantized_adaptive(layer_idx, len(keys)) if keys else None

    def memory_summary(self) -> Dict[str, Any]:
        hbm = sum(self._dense_len)
        dram = self._dram.memory_summary()
        int4_bytes = sum(st.page_bytes * st.num_pages for st in self._body if st is not None)
        if self._tier is not None:
            int4_bytes = self._tier.summary()["device_pool_bytes"]
        out = {"hbm_tokens": hbm, "dram_entries": dram["num_entries"], "dram_bytes": dram["total_bytes"],
               "max_hbm_tokens": self.max_hbm_tokens(), "int4_tokens": sum(self._body_len),
               "int4_bytes": int4_bytes}
        if self._tier is not None:
            out["host_tier"] = self._tier.summary()
        return out

    def max_hbm_tokens(self) -> int:
        return self.sink_tokens + self.tail_budget
