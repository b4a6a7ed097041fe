"""Multi-layer tiered INT4 KV cache for decoding, built on libhetero_kv.

Per layer it keeps the three zones of HeteroKVManager (src/memory/manager.py:
sink + recent tail in fp16/bf16 HBM, the evicted body as packed INT4 pages)
and runs one decode step as ONE launch (``fused_append``, the default for the
fp16min format):

    decode_append  (new token -> recent ring; oldest ring row -> INT4 body;
                    split-KV GQA attention over body + sink/recent, LSE merge)

or, with ``fused_append=False`` (the default for the ref format), as the two
launches it fuses (append_kv, then decode). In the ref format the fused launch's
append job shares a warp with the metadata expansion of the CTA's first tiles
and holds the CTA back: 107.4 us per layer against 95.4 us for the two launches
(config 1); in fp16min the append has a warp of its own and the fused step is
the faster one (2.485 against 2.569 ms per 32-layer step). All state (lengths, ring heads) lives on the device, so a whole
multi-layer step can be captured once into a CUDA graph and replayed every token.
"""
from __future__ import annotations

from typing import List, Optional

import torch

from . import _lib as L
from . import kvstore as kv


class TieredKVDecoder:
    def __init__(self, num_layers: int, batch: int, q_heads: int, kv_heads: int, *,
                 sink: int = 64, recent: int = 1024, body_capacity: int = 32768,
                 fmt: str = "fp16min", group: int = 32, page_tokens: int = 256,
                 kv_dtype: torch.dtype = torch.float16, out_dtype: torch.dtype = torch.float32,
                 device="cuda", ctas: int = 0, fused_append: Optional[bool] = None,
                 early: Optional[bool] = None):
        # the fused launch takes at most 8 query heads per KV head; more run as
        # the two launches (the attention split in groups of at most 8)
        fused_ok = q_heads // kv_heads <= 8
        self.fused_append = (fmt != "ref" and fused_ok) if fused_append is None else fused_append
        if self.fused_append and not fused_ok:
            raise ValueError("fused_append needs at most 8 query heads per KV head")
        self.early = early
        self.num_layers, self.batch = num_layers, batch
        self.q_heads, self.kv_heads = q_heads, kv_heads
        self.sink, self.recent = sink, recent
        self.fmt, self.group = fmt, group
        self.kv_dtype, self.out_dtype = kv_dtype, out_dtype
        self.device = torch.device(device)
        self.ctas = ctas
        self.stores: List[kv.Int4KVStore] = []
        self.dense: List[kv.DenseKV] = []
        for _ in range(num_layers):
            self.stores.append(kv.Int4KVStore(batch, kv_heads, body_capacity, fmt=fmt, group=group,
                                              page_tokens=page_tokens, device=self.device))
            self.dense.append(kv.DenseKV(batch, kv_heads, sink + recent, dtype=kv_dtype,
                                         device=self.device))
        self.body_len = 0
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.host_graph: Optional[torch.cuda.CUDAGraph] = None
        self._static = None
        self._host = None

    # ------------------------------------------------------------------ prefill
    def prefill_layer(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """k, v [B, Hkv, S, 128]: the first ``sink`` tokens and the last
        ``recent`` stay dense, the rest is quantised into the INT4 body."""
        S = k.shape[2]
        d, st = self.dense[layer], self.stores[layer]
        ns = min(self.sink, S)
        nr = min(self.recent, S - ns)
        d.k[:, :, :ns] = k[:, :, :ns]
        d.v[:, :, :ns] = v[:, :, :ns]
        if nr:
            d.k[:, :, self.sink:self.sink + nr] = k[:, :, S - nr:]
            d.v[:, :, self.sink:self.sink + nr] = v[:, :, S - nr:]
        nb = S - ns - nr
        if nb:
            kv.prefill(st, k[:, :, ns:ns + nb], v[:, :, ns:ns + nb])
        else:
            st.set_lengths(0)
        d.set_lengths(ns + nr if ns == self.sink else ns)
        d.ring_head.zero_()
        self.body_len = nb

    def set_state(self, body_len: int) -> None:
        """Declare that every layer holds ``body_len`` INT4 tokens and a full sink + ring."""
        for st, d in zip(self.stores, self.dense):
            st.set_lengths(body_len)
            d.set_lengths(self.sink + self.recent)
            d.ring_head.zero_()
        self.body_len = body_len

    # ------------------------------------------------------------------ decode
    def step_layer(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                   out: Optional[torch.Tensor] = None, len_hint: Optional[int] = None,
                   early: bool = False) -> torch.Tensor:
        """One layer's decode step. ``early``: the launch just before this one on
        the stream does not write this layer's cache (another layer's step), so
        the fused launch may stream the cache while that one finishes."""
        st, d = self.stores[layer], self.dense[layer]
        hint = len_hint if len_hint is not None else self.body_len + 1
        if self.fused_append:
            return kv.decode_append(q, k_new, v_new, d, self.sink, st, out_dtype=self.out_dtype, out=out,
                                    ctas=self.ctas, body_len=hint, dense_len=self.sink + self.recent,
                                    early=early)
        kv.append_kv(k_new, v_new, d, self.sink, st)
        return kv.decode(q, st, d, out_dtype=self.out_dtype, out=out, ctas=self.ctas,
                         body_len=hint, dense_len=self.sink + self.recent)

    @property
    def launches_per_layer(self) -> int:
        """Kernel launches of one layer's decode step."""
        return 1 if self.fused_append else 2

    @property
    def _early(self) -> bool:
        # a step runs the layers in order, so with two or more layers the launch
        # before a layer's is always another layer's (which never writes its cache)
        return self.num_layers >= 2 if self.early is None else (self.early and self.num_layers >= 2)

    def step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
             out: Optional[torch.Tensor] = None, len_hint: Optional[int] = None) -> torch.Tensor:
        """q [L, B, Hq, 128], k_new/v_new [L, B, Hkv, 128] -> out [L, B, Hq, 128]."""
        if out is None:
            out = torch.empty(self.num_layers, self.batch, self.q_heads, 128, dtype=self.out_dtype,
                              device=self.device)
        for l in range(self.num_layers):
            self.step_layer(l, q[l], k_new[l], v_new[l], out=out[l], len_hint=len_hint, early=self._early)
        self.body_len += 1
        return out

    def decode_only(self, q: torch.Tensor, out: torch.Tensor, len_hint: Optional[int] = None) -> None:
        """Attention of every layer without appending (cache unchanged)."""
        hint = len_hint if len_hint is not None else self.body_len
        for l in range(self.num_layers):
            kv.decode(q[l], self.stores[l], self.dense[l], out_dtype=self.out_dtype, out=out[l],
                      ctas=self.ctas, body_len=hint, dense_len=self.sink + self.recent)

    # ------------------------------------------------------------------ CUDA graph
    def capture(self, max_steps: int) -> None:
        """Capture one decode step over static input/output buffers. The split
        grid is sized for a body of ``body_len + max_steps`` tokens; device-side
        lengths keep replays exact as the body grows."""
        Lyr, B = self.num_layers, self.batch
        q = torch.zeros(Lyr, B, self.q_heads, 128, dtype=torch.bfloat16, device=self.device)
        kn = torch.zeros(Lyr, B, self.kv_heads, 128, dtype=self.kv_dtype, device=self.device)
        vn = torch.zeros_like(kn)
        out = torch.empty(Lyr, B, self.q_heads, 128, dtype=self.out_dtype, device=self.device)
        hint = self.body_len + max_steps
        self._hint = hint
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        g = torch.cuda.CUDAGraph()
        # warm the library (function attributes, workspace) outside capture, on a
        # throwaway copy of the state, then restore it
        snap = self._snapshot()
        with torch.cuda.stream(s):
            for l in range(Lyr):
                self.step_layer(l, q[l], kn[l], vn[l], out=out[l], len_hint=hint, early=self._early)
        s.synchronize()
        self._restore(snap)
        with torch.cuda.graph(g, stream=s):
            for l in range(Lyr):
                self.step_layer(l, q[l], kn[l], vn[l], out=out[l], len_hint=hint, early=self._early)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = g
        self._static = (q, kn, vn, out)

    def capture_host(self) -> None:
        """Capture the end-to-end step over engine-owned pinned host buffers
        (``host_buffers``: q, new K, new V in; out back), after ``capture``.
        Inputs go in on a side stream as three copies, each gating the first
        layer that reads it: layer 0's, layers 1-3's (small, lands while layer 0
        computes) and the rest (lands while layers 0-3 compute; the host link
        moves ~26 GB/s, so one copy of all later layers would hold layer 1 up).
        Outputs go back on another side stream
        as two copies: layers [0, L-2) once layer L-3 is done, and the last two
        layers at the end. Every dependency of a kernel on a copy, and every
        copy, costs microseconds of the step even when the data is ready, hence
        as few of them as the overlap allows (measured on the 32-layer config-1
        step: per-layer copies +138 us over the device-only step, this ~+55 us)."""
        assert self._static is not None, "capture() first"
        q, kn, vn, out = self._static
        hq = torch.empty(q.shape, dtype=q.dtype, pin_memory=True)
        hk = torch.empty(kn.shape, dtype=kn.dtype, pin_memory=True)
        hv = torch.empty(vn.shape, dtype=vn.dtype, pin_memory=True)
        ho = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        hint = self._hint
        Lyr = self.num_layers
        cuts = sorted({c for c in (Lyr - 2,) if 0 < c < Lyr}) + [Lyr]
        chunks = list(zip([0] + cuts[:-1], cuts))
        s = torch.cuda.Stream(device=self.device)
        s_in = torch.cuda.Stream(device=self.device)
        s_out = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        bounds = sorted({b for b in (1, 4) if b < Lyr}) + [Lyr]
        in_chunks = list(zip([0] + bounds[:-1], bounds))  # [0,1), [1,4), [4,L)
        ev_in = [torch.cuda.Event() for _ in in_chunks]
        ev_out = [torch.cuda.Event() for _ in chunks]
        # warm the capture stream's decode workspace outside capture (state restored)
        snap = self._snapshot()
        with torch.cuda.stream(s):
            for l in range(Lyr):
                self.step_layer(l, q[l], kn[l], vn[l], out=out[l], len_hint=hint, early=self._early)
        s.synchronize()
        self._restore(snap)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            s_in.wait_stream(s)
            s_out.wait_stream(s)
            with torch.cuda.stream(s_in):
                for i, (a, b) in enumerate(in_chunks):
                    q[a:b].copy_(hq[a:b], non_blocking=True)
                    kn[a:b].copy_(hk[a:b], non_blocking=True)
                    vn[a:b].copy_(hv[a:b], non_blocking=True)
                    ev_in[i].record(s_in)
            ci = 0
            for l in range(Lyr):
                for i, (a, _) in enumerate(in_chunks):
                    if l == a:  # the first layer that reads input copy i
                        s.wait_event(ev_in[i])
                self.step_layer(l, q[l], kn[l], vn[l], out=out[l], len_hint=hint, early=self._early)
                a, b = chunks[ci]
                if l == b - 1:
                    ev_out[ci].record(s)
                    with torch.cuda.stream(s_out):
                        s_out.wait_event(ev_out[ci])
                        ho[a:b].copy_(out[a:b], non_blocking=True)
                    ci += 1
            s.wait_stream(s_in)
            s.wait_stream(s_out)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.host_graph = g
        self._host = (hq, hk, hv, ho)

    @property
    def host_buffers(self):
        """Pinned host (q, new K, new V, out) of the pipelined end-to-end step.
        The step's copies read and write them asynchronously: write the next
        step's inputs, and read ``out``, only after the step has finished on
        the device (e.g. after a stream or event synchronisation)."""
        return self._host

    def _snapshot(self):
        return [(st.lengths.clone(), d.lengths.clone(), d.ring_head.clone(),
                 d.k.clone(), d.v.clone()) for st, d in zip(self.stores, self.dense)]

    def _restore(self, snap) -> None:
        for (bl, dl, rh, k, v), st, d in zip(snap, self.stores, self.dense):
            st.lengths.copy_(bl)
            d.lengths.copy_(dl)
            d.ring_head.copy_(rh)
            d.k.copy_(k)
            d.v.copy_(v)

    @property
    def static_buffers(self):
        return self._static

    def replay(self) -> None:
        self.graph.replay()
        self.body_len += 1

    def step_host(self, q_host: torch.Tensor, k_host: torch.Tensor, v_host: torch.Tensor,
                  out_host: torch.Tensor) -> None:
        """End-to-end step from (pinned) host buffers: H2D of the step's queries
        and new K/V, the captured step, D2H of the attention outputs. Given the
        engine's own ``host_buffers`` (after ``capture_host``) it replays the
        pipelined graph (per-layer copies overlapping the kernels); otherwise it
        copies everything in, replays the step and copies everything out."""
        if self._host is not None and all(a.data_ptr() == b.data_ptr() for a, b in
                                          zip((q_host, k_host, v_host, out_host), self._host)):
            self.host_graph.replay()
            self.body_len += 1
            return
        q, kn, vn, out = self._static
        q.copy_(q_host, non_blocking=True)
        kn.copy_(k_host, non_blocking=True)
        vn.copy_(v_host, non_blocking=True)
        self.replay()
        out_host.copy_(out, non_blocking=True)

    # ------------------------------------------------------------------ accounting
    def step_bytes(self, body_len: Optional[int] = None) -> int:
        """Algorithmic HBM bytes of one decode step (all layers): each INT4 code,
        meta, dense K/V byte, query and output read or written once, plus the
        append (new token in, evicted row in, packed row out, ring row out)."""
        nb = self.body_len if body_len is None else body_len
        return self.num_layers * (self.layer_attn_bytes(nb + 1) + self.layer_append_bytes())

    def layer_attn_bytes(self, body_tokens: int) -> int:
        ng = 128 // self.group
        meta = 4 * ng + (ng if self.fmt == "ref" else 0)
        per_tok_body = 2 * (64 + meta)
        esz = torch.tensor([], dtype=self.kv_dtype).element_size()
        per_tok_dense = 2 * 128 * esz
        units = self.batch * self.kv_heads
        qo = self.batch * self.q_heads * 128 * (2 + torch.tensor([], dtype=self.out_dtype).element_size())
        return units * (body_tokens * per_tok_body + (self.sink + self.recent) * per_tok_dense) + qo

    def layer_append_bytes(self) -> int:
        ng = 128 // self.group
        meta = 4 * ng + (ng if self.fmt == "ref" else 0)
        esz = torch.tensor([], dtype=self.kv_dtype).element_size()
        units = self.batch * self.kv_heads
        return units * 2 * (128 * esz * 3 + 64 + meta)
