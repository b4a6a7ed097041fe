"""Host (DRAM) tier for the INT4 body of a multi-layer KV cache.

The reference keeps every evicted chunk in pinned DRAM and copies chunks back
to the GPU when attention needs them (src/memory/manager.py:1231-1299 evicts,
:779-821 and :931-1056 bring them back, :335-348 prefetches through
AsyncPrefetcher). Here the body of every layer is a paged INT4 store over one
device pool, and the page table decides where each page is read from:

* per (layer, unit = sequence x KV head) the last ``resident`` pages of the body
  stay in HBM, in a ring of ``resident`` device slots, so the decode step's
  append always writes a resident page;
* older pages live in a pinned host arena; a page leaves the ring (a
  device->host copy per unit, on the compute stream, after the kernels that
  wrote it) when the body grows into the slot it occupies;
* before a layer's attention its host pages are copied into one of two staging
  areas (even / odd layers) by the page prefetcher (``hkv_prefetch_submit``:
  one cudaMemcpyAsync per unit's run of pages, on a side stream), and the
  layer's page table points there. ``stage(l + 1)`` issued before layer l's
  attention is the layer-ahead prefetch; ``gate`` makes the compute stream wait
  for the copy and ``release`` marks the staging area free again.

HBM holds L*U*resident + 2*U*(max_pages - resident) pages instead of
L*U*max_pages. Lengths are uniform over the batch (the manager's usage).
"""
from __future__ import annotations

import math
from typing import List, Optional

import torch

from .. import _lib as L
from .. import kvstore as kv
from ..policy.prefetcher import PagePrefetcher


class _LayerView:
    """One layer's body as the kernels see it: a paged store over the shared pool."""

    def __init__(self, tier: "HostTier", layer: int):
        self.tier, self.layer = tier, layer
        self.batch, self.kv_heads = tier.batch, tier.kv_heads
        self.fmt, self.group, self.page_tokens = tier.fmt, tier.group, tier.P
        self.max_pages = tier.max_pages
        self.capacity = tier.max_pages * tier.P
        self.paged = True
        self.num_pages = int(tier.pool.shape[0])
        self.pool = tier.pool
        self.page_bytes = tier.page_bytes
        self.device = tier.device
        U, mp, R, S = tier.U, tier.max_pages, tier.R, tier.S
        u = torch.arange(U, dtype=torch.int32, device=tier.device)[:, None]
        p = torch.arange(mp, dtype=torch.int32, device=tier.device)[None, :]
        # slot of page p of unit u when resident (ring) / when staged
        self._res = (layer * U + u) * R + p % R
        self._stage = tier.stage_base[layer % 2] + u * S + p.clamp(max=max(S - 1, 0))
        self._p = p.expand(U, mp)
        self.page_table = self._res.clone()
        self.lengths = torch.zeros(tier.batch, dtype=torch.int32, device=tier.device)
        self.len_hint = 0

    def refresh(self, n_host: int) -> None:
        """Pages [0, n_host) read from the staging area, the rest from the ring
        (stream-ordered on the current stream)."""
        torch.where(self._p < n_host, self._stage, self._res, out=self.page_table)

    def struct(self, len_hint: Optional[int] = None) -> L.HkvInt4Store:
        s = L.HkvInt4Store()
        s.pages = self.pool.data_ptr()
        s.page_stride = self.page_bytes
        s.format = kv.FORMATS[self.fmt]
        s.group = self.group
        s.page_tokens = self.page_tokens
        s.max_pages = self.max_pages
        s.page_table = self.page_table.data_ptr()
        s.lengths = self.lengths.data_ptr()
        s.len = int(self.len_hint if len_hint is None else len_hint)
        s.num_pages = self.num_pages
        return s

    def set_lengths(self, n: int) -> None:
        self.lengths.fill_(int(n))
        self.len_hint = int(n)


class HostTier:
    def __init__(self, num_layers: int, batch: int, kv_heads: int, capacity: int, *, resident_pages: int,
                 fmt: str = "ref", group: int = 32, page_tokens: int = 256,
                 device: torch.device = torch.device("cuda")):
        if resident_pages < 1:
            raise ValueError("resident_pages must be >= 1 (the page the append writes)")
        self.L, self.batch, self.kv_heads = num_layers, batch, kv_heads
        self.U = batch * kv_heads
        self.fmt, self.group, self.P = fmt, group, page_tokens
        self.device = torch.device(device)
        self.page_bytes = kv.page_bytes(fmt, group, page_tokens)
        self.max_pages = max(1, math.ceil(capacity / page_tokens))
        self.R = min(resident_pages, self.max_pages)
        self.S = self.max_pages - self.R  # host pages per unit at most (staging slots per unit)
        n_res = num_layers * self.U * self.R
        self.stage_base = [n_res, n_res + self.U * self.S]
        self.pool = torch.empty(n_res + 2 * self.U * self.S, self.page_bytes, dtype=torch.uint8,
                                device=self.device)
        self.host = torch.empty(num_layers * self.U * self.max_pages, self.page_bytes,
                                dtype=torch.uint8).pin_memory()
        self.prefetcher = PagePrefetcher(self.host, self.pool)
        self.stream = self.prefetcher.stream
        self.views: List[_LayerView] = [_LayerView(self, l) for l in range(num_layers)]
        self.n_pages = [0] * num_layers  # body pages per unit in use
        self.n_host = [0] * num_layers   # of which on the host (pages [0, n_host))
        self.ready: List[Optional[torch.cuda.Event]] = [None] * num_layers
        self.evicted: List[Optional[torch.cuda.Event]] = [None] * num_layers
        self.free: List[Optional[torch.cuda.Event]] = [None, None]
        self.h2d_bytes = 0
        self.d2h_bytes = 0

    # ------------------------------------------------------------------ geometry
    def _host_page(self, l: int, u: int, p: int) -> int:
        return (l * self.U + u) * self.max_pages + p

    def _res_slot(self, l: int, u: int, p: int) -> int:
        return (l * self.U + u) * self.R + p % self.R

    # ------------------------------------------------------------------ writes
    def prepare_write(self, l: int, t_end: int) -> None:
        """Make body slots [0, t_end) of layer l writable: pages beyond the ring
        displace the oldest resident pages, which first go to the host (a copy
        per unit on the current stream, so after every kernel that wrote them
        and before any that reuses their slot)."""
        need = math.ceil(t_end / self.P)
        if need > self.max_pages:
            raise RuntimeError(f"layer {l}: body of {t_end} tokens exceeds the capacity "
                               f"({self.max_pages * self.P})")
        if need <= self.n_pages[l]:
            return
        new_host = max(self.n_host[l], need - self.R)
        for p in range(self.n_host[l], new_host):  # page p leaves the ring (its slot holds page p + R next)
            for u in range(self.U):
                self.host[self._host_page(l, u, p)].copy_(self.pool[self._res_slot(l, u, p)], non_blocking=True)
            self.d2h_bytes += self.U * self.page_bytes
        if new_host != self.n_host[l]:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            self.evicted[l] = ev
            self.n_host[l] = new_host
            self.views[l].refresh(new_host)
            self.ready[l] = None  # a prefetch issued before misses the new host pages: stage again
        self.n_pages[l] = need

    def write(self, l: int, start: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantise K/V [B, H, n, 128] into body slots [start, start + n) of layer l,
        at most a ring's worth of pages per launch."""
        n = k.shape[2]
        t = start
        while t < start + n:
            t1 = min(start + n, (t // self.P + self.R) * self.P)  # the pages one launch writes are resident together
            self.prepare_write(l, t1)
            kv.quantize_pack_kv(k[:, :, t - start:t1 - start], v[:, :, t - start:t1 - start], self.views[l], t)
            t = t1

    # ------------------------------------------------------------------ reads
    def stage(self, l: int) -> None:
        """Side stream: after the layer's device->host copies and once the staging
        area of its parity is free, copy layer l's host pages into it and record
        the event ``gate`` waits on. Issue it before the launch of the attention
        it should overlap (layer-ahead prefetch)."""
        nh = self.n_host[l]
        self.ready[l] = None
        if nh == 0:
            return
        if self.evicted[l] is not None:
            self.stream.wait_event(self.evicted[l])
        if self.free[l % 2] is not None:
            self.stream.wait_event(self.free[l % 2])
        src = [self._host_page(l, u, p) for u in range(self.U) for p in range(nh)]
        dst = [self.stage_base[l % 2] + u * self.S + p for u in range(self.U) for p in range(nh)]
        self.ready[l] = self.prefetcher.submit(src, dst)
        self.h2d_bytes += nh * self.U * self.page_bytes

    def gate(self, l: int) -> None:
        """The current stream waits for layer l's staged pages (staging them now
        if no prefetch was issued). The staging area of a parity is shared, so a
        layer's pages are staged again before each of its attentions."""
        if self.n_host[l] == 0:
            return
        if self.ready[l] is None:
            self.stage(l)
        torch.cuda.current_stream(self.device).wait_event(self.ready[l])
        self.ready[l] = None

    def release(self, l: int) -> None:
        """Call after the launches that read layer l's staged pages."""
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.device))
        self.free[l % 2] = ev

    # ------------------------------------------------------------------ accounting
    def summary(self) -> dict:
        return {"resident_pages_per_unit": self.R,
                "host_pages": [self.n_host[l] * self.U for l in range(self.L)],
                "device_body_pages": [(self.n_pages[l] - self.n_host[l]) * self.U for l in range(self.L)],
                "device_pool_bytes": int(self.pool.numel()), "h2d_bytes": self.h2d_bytes,
                "d2h_bytes": self.d2h_bytes}
