"""Tiered offload decode (config 3): most INT4 pages live in pinned host DRAM
and are copied into HBM one layer ahead of the layer that attends to them.

Per layer and (sequence, KV head) unit, ``resident_pages`` INT4 pages stay in
HBM with the fp16/bf16 sink + recent tokens; ``cold_pages`` pages live in a
pinned host arena. Before layer l's attention, layer l+1's cold pages (all of
them, or a window of the last ``window_pages``) are copied host -> device on a
side stream into one of two staging areas of the device pool (``PagePrefetcher``,
one cudaMemcpyAsync per run of consecutive pages); an event gates layer l+1's
attention, and a second event tells the side stream when a staging area is free
again. Every layer's page table points at its resident pages and at the
staging slots of its parity, so the decode kernel reads the prefetched pages in
place: nothing is concatenated or dequantised.

This replaces the reference's per-chunk swap-in (HeteroKVManager.swap_in /
AsyncPrefetcher, src/memory/manager.py:233-307, src/policy/prefetcher.py:47-111):
six small copies and a BF16 decompression per chunk, joined by a device-wide
synchronisation.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import _lib as L
from . import kvstore as kv
from .policy.prefetcher import PagePrefetcher


class _LayerStore:
    """One layer's view of the shared device page pool (what kv.decode reads)."""

    def __init__(self, pool: torch.Tensor, page_bytes: int, page_table: torch.Tensor, lengths: torch.Tensor,
                 batch: int, kv_heads: int, fmt: str, group: int, page_tokens: int, len_tokens: int):
        self.pool, self.page_bytes, self.page_table, self.lengths = pool, page_bytes, page_table, lengths
        self.batch, self.kv_heads, self.fmt, self.group = batch, kv_heads, fmt, group
        self.page_tokens, self.len_tokens = page_tokens, len_tokens

    def struct(self, len_hint: Optional[int] = None) -> L.HkvInt4Store:
        s = L.HkvInt4Store()
        s.pages = self.pool.data_ptr()
        s.page_stride = self.page_bytes
        s.format = kv.FORMATS[self.fmt]
        s.group = self.group
        s.page_tokens = self.page_tokens
        s.max_pages = int(self.page_table.shape[1])
        s.page_table = self.page_table.data_ptr()
        s.lengths = self.lengths.data_ptr()
        s.len = int(self.len_tokens if len_hint is None else len_hint)
        s.num_pages = int(self.pool.shape[0])
        return s


class TieredOffloadDecoder:
    def __init__(self, num_layers: int, batch: int, q_heads: int, kv_heads: int, *, resident_pages: int,
                 cold_pages: int, window_pages: Optional[int] = None, sink: int = 64, recent: int = 1024,
                 fmt: str = "fp16min", group: int = 32, page_tokens: int = 256,
                 kv_dtype: torch.dtype = torch.float16, device="cuda"):
        self.L, self.B, self.Hq, self.Hkv = num_layers, batch, q_heads, kv_heads
        self.units = batch * kv_heads
        self.resident, self.cold = resident_pages, cold_pages
        self.window = cold_pages if window_pages is None else min(window_pages, cold_pages)
        self.fmt, self.group, self.P = fmt, group, page_tokens
        self.device = torch.device(device)
        self.page_bytes = kv.page_bytes(fmt, group, page_tokens)
        U = self.units
        self.stage_pages = U * self.window
        n_res = num_layers * U * resident_pages
        # device pool: [resident pages of every layer | staging area 0 | staging area 1]
        self.pool = torch.empty(n_res + 2 * self.stage_pages, self.page_bytes, dtype=torch.uint8,
                                device=self.device)
        self.stage_base = [n_res, n_res + self.stage_pages]
        # host arena: the cold pages of every unit, shared by all layers (one layer's worth)
        self.host = torch.empty(U * cold_pages, self.page_bytes, dtype=torch.uint8).pin_memory()
        self.prefetcher = PagePrefetcher(self.host, self.pool)
        attended = resident_pages + self.window
        self.tokens = attended * page_tokens
        self.dense = [kv.DenseKV(batch, kv_heads, sink + recent, dtype=kv_dtype, device=self.device)
                      for _ in range(num_layers)]
        for d in self.dense:
            d.set_lengths(sink + recent)
        self.stores: List[_LayerStore] = []
        for l in range(num_layers):
            table = torch.empty(U, attended, dtype=torch.int32)
            for u in range(U):
                table[u, :resident_pages] = torch.arange(resident_pages) + (l * U + u) * resident_pages
                table[u, resident_pages:] = torch.arange(self.window) + self.stage_base[l % 2] + u * self.window
            lengths = torch.full((batch,), self.tokens, dtype=torch.int32, device=self.device)
            self.stores.append(_LayerStore(self.pool, self.page_bytes, table.to(self.device), lengths, batch,
                                           kv_heads, fmt, group, page_tokens, self.tokens))
        # host pages copied per layer: the last `window` cold pages of each unit
        self.src_pages = [u * cold_pages + (cold_pages - self.window) + i for u in range(U) for i in range(self.window)]
        self.dst_slots = [[self.stage_base[p] + i for i in range(self.stage_pages)] for p in range(2)]
        self.free = [torch.cuda.Event() for _ in range(2)]
        self.ready: List[Optional[torch.cuda.Event]] = [None] * num_layers

    # ------------------------------------------------------------------ data
    def fill(self, gen: torch.Generator, outlier_channels: int = 4) -> None:
        """Seeded synthetic K/V: quantise every unit's resident + cold pages, keep the
        resident ones in the pool and the cold ones in the host arena."""
        U, P = self.units, self.P
        ntok = (self.resident + self.cold) * P
        for l in range(self.L):
            tmp = kv.Int4KVStore(self.B, self.Hkv, ntok, fmt=self.fmt, group=self.group, page_tokens=P,
                                 device=self.device)
            chunk = 8192
            for t0 in range(0, ntok, chunk):
                n = min(chunk, ntok - t0)
                k = torch.randn(self.B, self.Hkv, n, 128, device=self.device, generator=gen)
                for h in range(self.Hkv):
                    ch = torch.randperm(128, device=self.device, generator=gen)[:outlier_channels]
                    k[:, h, :, ch] *= 10.0
                v = torch.randn(self.B, self.Hkv, n, 128, device=self.device, generator=gen)
                kv.quantize_pack_kv(k.half(), v.half(), tmp, t0)
            pages = tmp.pool.view(U, tmp.max_pages, self.page_bytes)
            self.pool[l * U * self.resident:(l + 1) * U * self.resident] = \
                pages[:, :self.resident].reshape(-1, self.page_bytes)
            if l == 0:
                self.host.copy_(pages[:, self.resident:self.resident + self.cold].reshape(-1, self.page_bytes))
            d = self.dense[l]
            d.k.normal_(generator=gen)
            d.v.normal_(generator=gen)
            del tmp
        torch.cuda.synchronize(self.device)

    # ------------------------------------------------------------------ step
    def prefetch(self, layer: int) -> None:
        """Side stream: wait until the staging area of `layer`'s parity is free,
        copy the layer's cold pages into it, record its ready event."""
        par = layer % 2
        self.prefetcher.stream.wait_event(self.free[par])
        self.ready[layer] = self.prefetcher.submit(self.src_pages, self.dst_slots[par])

    def step(self, q: torch.Tensor, out: torch.Tensor, transfer: bool = True) -> None:
        """Attention of every layer (q [L, B, Hq, 128] -> out [L, B, Hq, 128]) with
        the next layer's pages copied during the current layer's attention."""
        cs = torch.cuda.current_stream(self.device)
        if transfer and self.ready[0] is None:
            self.prefetch(0)
        for l in range(self.L):
            if transfer:
                if l + 1 < self.L:
                    self.prefetch(l + 1)
                cs.wait_event(self.ready[l])
            st, d = self.stores[l], self.dense[l]
            kv.decode(q[l], st, d, out=out[l], body_len=self.tokens, dense_len=d.len_hint)
            self.free[l % 2].record(cs)
            self.ready[l] = None
        if transfer:
            self.prefetch(0)  # the next step's first layer, behind this step's last attention

    def h2d_bytes_per_step(self) -> int:
        return self.L * self.stage_pages * self.page_bytes

    def attn_bytes_per_step(self) -> int:
        per_tok = 2 * (64 + 4 * (128 // self.group) + (128 // self.group if self.fmt == "ref" else 0))
        dense = self.dense[0].len_hint * 2 * 128 * 2
        return self.L * self.units * (self.tokens * per_tok + dense)
