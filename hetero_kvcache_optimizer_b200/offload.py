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

import ctypes
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


class SlidingWindowOffload:
    """Tiered offload with pages that stay in HBM across steps: each layer and
    unit attends its ``resident_pages`` plus a window of ``window_pages`` cold
    pages, and the window slides by ``delta`` pages per step (the pages the
    window policy picks change slowly: the reference's adaptive window is
    w_t in [2, 8] chunks, src/policy/adaptive_prefetch_controller.py:44-45, and
    its ranking follows accumulated attention scores). Cold pages that are in
    the window stay in a per-(layer, unit) cache ring of window + delta device
    slots, so a step copies only the ``delta`` pages entering the window, one
    layer ahead of their attention, on the page prefetcher's side stream. The
    ring never overwrites a page the current or previous step attends: the
    pages leaving it (p - window - delta) left the window a step earlier.

    Host arena and ring are page-major ([page][unit]): the pages entering the
    window of every unit of a layer are one contiguous run on both sides, so a
    layer's fetch is one cudaMemcpyAsync (two when the ring or the cold set
    wraps) instead of one per unit; per-copy overhead (a few µs) would
    otherwise dominate copies of single 40 KB pages.

    The page table of step s maps window entry i to slot (s * delta + i) mod
    (window + delta); the distinct tables of a layer (the ring's period) are
    built once, so a step passes a pointer and writes no table.

    As in ``TieredOffloadDecoder`` one layer's cold pages (``cold_pages`` per
    unit) live in the pinned host arena and every layer reads them (a
    benchmark harness: the attention differs per layer through its queries)."""

    def __init__(self, num_layers: int, batch: int, q_heads: int, kv_heads: int, *, resident_pages: int,
                 cold_pages: int, window_pages: int, delta: int, sink: int = 64, recent: int = 1024,
                 fmt: str = "fp16min", group: int = 32, page_tokens: int = 256,
                 kv_dtype: torch.dtype = torch.float16, device="cuda", gather_ctas: int = 0):
        if not 0 <= delta <= window_pages <= cold_pages:
            raise ValueError("need 0 <= delta <= window_pages <= cold_pages")
        self.L, self.B, self.Hq, self.Hkv = num_layers, batch, q_heads, kv_heads
        self.units = U = batch * kv_heads
        self.resident, self.cold, self.window, self.delta = resident_pages, cold_pages, window_pages, delta
        self.C = window_pages + delta  # cache ring slots per (layer, unit)
        self.fmt, self.group, self.P = fmt, group, page_tokens
        self.device = torch.device(device)
        self.page_bytes = kv.page_bytes(fmt, group, page_tokens)
        n_res = num_layers * U * resident_pages
        self.cache_base = n_res
        self.pool = torch.empty(n_res + num_layers * U * self.C, self.page_bytes, dtype=torch.uint8,
                                device=self.device)
        self.host = torch.empty(U * cold_pages, self.page_bytes, dtype=torch.uint8).pin_memory()
        self.prefetcher = PagePrefetcher(self.host, self.pool)
        attended = resident_pages + window_pages
        self.tokens = attended * page_tokens
        self.dense = [kv.DenseKV(batch, kv_heads, sink + recent, dtype=kv_dtype, device=self.device)
                      for _ in range(num_layers)]
        for d in self.dense:
            d.set_lengths(sink + recent)
        # the ring's period: window start s * delta mod C repeats after C / gcd(C, delta) steps
        import math
        self.period = self.C // math.gcd(self.C, delta) if delta else 1
        self.tables = []  # [layer][phase] -> [U, attended] int32 on the device
        for l in range(num_layers):
            per = []
            for ph in range(self.period):
                t = torch.empty(U, attended, dtype=torch.int32)
                for u in range(U):
                    t[u, :resident_pages] = torch.arange(resident_pages) + (l * U + u) * resident_pages
                    t[u, resident_pages:] = self._slot(l, u, torch.arange(window_pages) + ph * delta)
                per.append(t.to(self.device))
            self.tables.append(per)
        self.lengths = torch.full((batch,), self.tokens, dtype=torch.int32, device=self.device)
        self.step_idx = 0
        self.done: List[Optional[torch.cuda.Event]] = [None] * num_layers  # layer's last attention
        self.ready: List[Optional[torch.cuda.Event]] = [None] * num_layers
        self.fetched_pages = 0
        # device-side form of a step's fetch, for the zero-copy gather kernel
        # (graph replays): entry (i, u) of the pages entering the window reads
        # host page (src + step * delta * U) mod (cold * U), i.e. page
        # (step * delta + window - delta + i) mod cold of unit u, and writes ring
        # slot dst[layer][phase]; step_dev counts steps on the device.
        enter = range(window_pages - delta, window_pages)
        self.g_src = torch.tensor([j * U + u for j in enter for u in range(U)], dtype=torch.int32,
                                  device=self.device)
        self.g_dst = [[torch.tensor([self._slot(l, u, ph * delta + j) for j in enter for u in range(U)],
                                    dtype=torch.int32, device=self.device) for ph in range(self.period)]
                      for l in range(num_layers)]
        self.step_dev = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.gather_ctas = gather_ctas  # grid of the captured gathers (0: the library's default)
        self._graphs = None
        self.transport = "copy"
        self._copy_nodes: list = []

    def _slot(self, l: int, u: int, p):
        """Ring slot of window page p (any integer) of layer l, unit u."""
        return self.cache_base + (l * self.C + p % self.C) * self.units + u

    def _store(self, l: int, phase: int) -> _LayerStore:
        return _LayerStore(self.pool, self.page_bytes, self.tables[l][phase], self.lengths, self.B, self.Hkv,
                           self.fmt, self.group, self.P, self.tokens)

    def fill(self, gen: torch.Generator, outlier_channels: int = 4) -> None:
        """Seeded synthetic K/V as TieredOffloadDecoder.fill: resident pages in the
        pool, cold pages in the host arena; the window of step 0 copied into
        every layer's ring."""
        U, P = self.units, self.P
        ntok = (self.resident + self.cold) * P
        for l in range(self.L):
            tmp = kv.Int4KVStore(self.B, self.Hkv, ntok, fmt=self.fmt, group=self.group, page_tokens=P,
                                 device=self.device)
            for t0 in range(0, ntok, 8192):
                n = min(8192, ntok - t0)
                k = torch.randn(self.B, self.Hkv, n, 128, device=self.device, generator=gen)
                for h in range(self.Hkv):
                    ch = torch.randperm(128, device=self.device, generator=gen)[:outlier_channels]
                    k[:, h, :, ch] *= 10.0
                v = torch.randn(self.B, self.Hkv, n, 128, device=self.device, generator=gen)
                kv.quantize_pack_kv(k.half(), v.half(), tmp, t0)
            pages = tmp.pool.view(U, tmp.max_pages, self.page_bytes)
            self.pool[l * U * self.resident:(l + 1) * U * self.resident] = \
                pages[:, :self.resident].reshape(-1, self.page_bytes)
            if l == 0:  # host page p of unit u at p * U + u
                self.host.copy_(pages[:, self.resident:self.resident + self.cold].transpose(0, 1)
                                .reshape(-1, self.page_bytes))
            d = self.dense[l]
            d.k.normal_(generator=gen)
            d.v.normal_(generator=gen)
            del tmp
        torch.cuda.synchronize(self.device)
        for l in range(self.L):  # step 0's window, before the first step
            self._fetch(l, 0, range(self.window))
        torch.cuda.synchronize(self.device)

    def _fetch(self, l: int, step: int, idx) -> None:
        """Copy window pages ``idx`` (positions in step ``step``'s window) of layer
        l into their ring slots on the side stream."""
        first = step * self.delta
        src, dst = [], []
        for i in idx:  # page-major: consecutive units are consecutive on both sides
            p = (first + i) % self.cold
            for u in range(self.units):
                src.append(p * self.units + u)
                dst.append(self._slot(l, u, first + i))
        if self.done[l] is not None:  # the ring slots' previous readers
            self.prefetcher.stream.wait_event(self.done[l])
        self.ready[l] = self.prefetcher.submit(src, dst)
        self.fetched_pages += len(src)

    def prefetch(self, l: int, step: int) -> None:
        """The pages entering layer l's window at ``step`` (its last ``delta``)."""
        if self.delta:
            self._fetch(l, step, range(self.window - self.delta, self.window))
        else:
            self.ready[l] = None

    def step(self, q: torch.Tensor, out: torch.Tensor, transfer: bool = True) -> None:
        """Attention of every layer over its resident pages + the current window,
        the next layer's new window pages copied during the current layer (step
        0's window is in the ring since ``fill``). transfer=False skips the
        copies, for timing: the step then attends whatever the ring holds."""
        s = self.step_idx
        cs = torch.cuda.current_stream(self.device)
        phase = s % self.period
        if transfer and s > 0 and self.ready[0] is None:
            self.prefetch(0, s)
        for l in range(self.L):
            if transfer:
                if l + 1 < self.L and s > 0:
                    self.prefetch(l + 1, s)
                if self.ready[l] is not None:
                    cs.wait_event(self.ready[l])
            d = self.dense[l]
            kv.decode(q[l], self._store(l, phase), d, out=out[l], body_len=self.tokens, dense_len=d.len_hint)
            ev = torch.cuda.Event()
            ev.record(cs)
            self.done[l] = ev
            self.ready[l] = None
        self.step_idx += 1
        self.step_dev.add_(1)
        if transfer:
            self.prefetch(0, self.step_idx)  # the next step's first layer, behind this step's last attention

    # ------------------------------------------------------------------ graphs
    def capture(self, q: torch.Tensor, out: torch.Tensor, transport: str = "copy", copy_streams: int = 1) -> None:
        """Capture one step per phase of the ring as CUDA graphs over the static
        q [L, B, Hq, 128] / out, with and without the transfer, so a step is one
        graph launch with no host work per layer. A transfer graph forks the page
        prefetcher's side stream, which moves layer l+1's entering pages while
        layer l attends, each layer's attention waiting for its own pages; the
        next step's layer-0 pages move behind the last layers and are joined
        before the graph ends.

        transport "copy": one host -> device copy per entering page row (the
        row of all U units, contiguous on both sides), on the copy engines; the
        host rows move with the step, so ``replay`` points the graph's copy
        nodes at the step's rows first (``hkv_graph_exec_set_copy_srcs``, one
        library call per step). "gather": one zero-copy gather kernel per layer
        (``hkv_prefetch_gather``) whose host rows follow the device step
        counter, so nothing changes between replays (SM loads over the host
        link: ~42 GB/s measured here against ~45-48 for the copy engines); needs
        a mapped pinned arena. ``copy_streams`` > 1 side streams take the layers
        in turn, so one layer's copy may start while the previous one is in
        flight (measured: no gain, the host link is the bound)."""
        if transport not in ("copy", "gather"):
            raise ValueError("transport: 'copy' or 'gather'")
        U, cs = self.units, torch.cuda.Stream(device=self.device)
        sides = [self.prefetcher.stream] + [torch.cuda.Stream(device=self.device)
                                            for _ in range(max(1, copy_streams) - 1)]
        W, dl, pb = self.window, self.delta, self.page_bytes
        cs.wait_stream(torch.cuda.current_stream(self.device))
        torch.cuda.synchronize(self.device)
        self.step_dev.fill_(self.step_idx)
        self.transport = transport

        def fetch(l: int, ph: int, add: int, side: torch.cuda.Stream) -> None:
            if transport == "gather":
                self.prefetcher.gather(self.g_src, self.g_dst[l][ph], self.step_dev, dl * U, add,
                                       ctas=self.gather_ctas, stream=side)
                return
            for i in range(dl):  # one copy node per page row; its source is retargeted per replay
                j = W - dl + i
                p = ((ph + add) * dl + j) % self.cold
                self.prefetcher.submit([p * U + u for u in range(U)],
                                       [self._slot(l, u, ph * dl + j) for u in range(U)], stream=side)

        def body(ph: int, transfer: bool) -> None:
            ready: List[Optional[torch.cuda.Event]] = [None] * self.L
            move = transfer and dl > 0
            if move:
                fork = torch.cuda.Event()
                fork.record(cs)
                for side in sides:
                    side.wait_event(fork)
            for l in range(self.L):
                if move:
                    if l + 1 < self.L:
                        side = sides[(l + 1) % len(sides)]
                        fetch(l + 1, ph, 0, side)
                        ready[l + 1] = torch.cuda.Event()
                        ready[l + 1].record(side)
                    if l > 0:
                        cs.wait_event(ready[l])
                d = self.dense[l]
                kv.decode(q[l], self._store(l, ph), d, out=out[l], body_len=self.tokens, dense_len=d.len_hint)
            if move:
                fetch(0, (ph + 1) % self.period, 1, sides[0])
                for side in sides:  # join every side stream
                    join = torch.cuda.Event()
                    join.record(side)
                    cs.wait_event(join)
            self.step_dev.add_(1)

        with torch.cuda.stream(cs):  # warm: the decode workspace of the capture stream
            for l in range(self.L):
                d = self.dense[l]
                kv.decode(q[l], self._store(l, 0), d, out=out[l], body_len=self.tokens, dense_len=d.len_hint)
        cs.synchronize()
        graphs = {True: [], False: []}
        self._copy_nodes = []  # per phase: (nodes, dsts, row, step offset) of its copy nodes
        for transfer in (True, False):
            for ph in range(self.period):
                g = torch.cuda.CUDAGraph(keep_graph=True)
                with torch.cuda.graph(g, stream=cs):
                    body(ph, transfer)
                g.instantiate()
                graphs[transfer].append(g)
                if transfer and transport == "copy" and dl:
                    self._copy_nodes.append(self._map_copy_nodes(g, ph))
        torch.cuda.current_stream(self.device).wait_stream(cs)
        self._graphs = graphs

    def _map_copy_nodes(self, g: "torch.cuda.CUDAGraph", ph: int):
        """The copy nodes of phase ph's transfer graph, matched to (layer, row)
        through their destinations: layers 1..L-1 copy step s's rows, layer 0
        step s+1's rows (into phase ph+1's ring slots)."""
        import numpy as np
        lib = L.load()
        cap = self.L * self.delta
        nodes = (ctypes.c_void_p * cap)()
        dsts = (ctypes.c_void_p * cap)()
        n = ctypes.c_int32(0)
        L.check(lib.hkv_graph_copy_nodes(ctypes.c_void_p(int(g.raw_cuda_graph())), cap, nodes, dsts,
                                         ctypes.byref(n)), "hkv_graph_copy_nodes")
        by_dst = {int(dsts[k]): int(nodes[k]) for k in range(n.value)}
        base, U, W, dl, pb = self.pool.data_ptr(), self.units, self.window, self.delta, self.page_bytes
        ent_nodes, ent_dsts, layer, row, add = [], [], [], [], []
        for l in range(self.L):
            a, ph_dst = (1, (ph + 1) % self.period) if l == 0 else (0, ph)
            for i in range(dl):
                dst = base + self._slot(l, 0, ph_dst * dl + W - dl + i) * pb
                if dst not in by_dst:
                    raise RuntimeError("captured copy node not found for a window row")
                ent_nodes.append(by_dst[dst])
                ent_dsts.append(dst)
                layer.append(l)
                row.append(W - dl + i)
                add.append(a)
        return (np.array(ent_nodes, np.uint64), np.array(ent_dsts, np.uint64), np.array(row, np.int64),
                np.array(add, np.int64))

    def _retarget(self, s: int) -> None:
        """Point phase (s mod period)'s copy nodes at step s's host rows."""
        import numpy as np
        nodes, dsts, row, add = self._copy_nodes[s % self.period]
        p = ((s + add) * self.delta + row) % self.cold
        srcs = (self.host.data_ptr() + p * (self.units * self.page_bytes)).astype(np.uint64)
        nbytes = np.full(len(nodes), self.units * self.page_bytes, np.int64)
        g = self._graphs[True][s % self.period]
        L.check(L.load().hkv_graph_exec_set_copy_srcs(
            ctypes.c_void_p(int(g.raw_cuda_graph_exec())), len(nodes), nodes.ctypes.data, dsts.ctypes.data,
            srcs.ctypes.data, nbytes.ctypes.data), "hkv_graph_exec_set_copy_srcs")

    def replay(self, transfer: bool = True) -> None:
        """One captured step (``capture``) on the current stream."""
        if self._graphs is None:
            raise RuntimeError("SlidingWindowOffload.replay: call capture() first")
        if self.ready[0] is not None:  # layer 0's pages of an eager prefetch
            torch.cuda.current_stream(self.device).wait_event(self.ready[0])
            self.ready[0] = None
        if transfer and self.delta and self.transport == "copy":
            self._retarget(self.step_idx)
        self._graphs[transfer][self.step_idx % self.period].replay()
        if transfer:
            self.fetched_pages += self.L * self.units * self.delta
        self.step_idx += 1

    def h2d_bytes_per_step(self) -> int:
        return self.L * self.units * self.delta * self.page_bytes

    def attn_bytes_per_step(self) -> int:
        per_tok = 2 * (64 + 4 * (128 // self.group) + (128 // self.group if self.fmt == "ref" else 0))
        dense = self.dense[0].len_hint * 2 * 128 * 2
        return self.L * self.units * (self.tokens * per_tok + dense)
