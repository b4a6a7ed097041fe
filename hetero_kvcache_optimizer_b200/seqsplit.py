"""Sequence-split decode attention across GPUs (config 4, variant B).

Every rank holds a contiguous, page-aligned slice of each sequence's INT4 body
and any share of its fp16/bf16 sink + recent rows (attention does not depend on
the order of the keys, so ``shard_range`` over the rows balances them too), computes the
un-normalised partial (o, m, l) of the attention over its slice with
``hkv_decode_attn_partial``, and one NCCL all-gather of those partials
(B*Hq*130 floats per rank) feeds ``hkv_lse_merge``, which every rank runs to get
the full output. No other collective; the data path itself never crosses
NVLink.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib as L
from . import kvstore as kv


def shard_range(total_pages: int, world: int, rank: int) -> Tuple[int, int]:
    """Pages [p0, p1) of a body of ``total_pages`` pages held by ``rank``:
    contiguous slices whose sizes differ by at most one page."""
    base, extra = divmod(total_pages, world)
    p0 = rank * base + min(rank, extra)
    return p0, p0 + base + (1 if rank < extra else 0)


def shard_spans(body_pages: int, dense_rows: int, world: int, rank: int, page_bytes: int,
                row_bytes: int) -> Tuple[Tuple[int, int], Tuple[int, int]]:
    """Body pages [p0, p1) and dense rows [r0, r1) held by ``rank`` when the
    byte line [every body page | every dense row] of a unit is cut into ``world``
    slices of equal bytes (a page or row goes to the rank whose slice holds its
    middle byte). Most ranks then hold one segment per unit, not two: the decode
    kernel pays a fixed start cost per segment of a unit, which weighs on the
    small per-rank shares of short contexts. The spans of consecutive ranks
    tile both segments."""
    if world < 1 or not 0 <= rank < world or page_bytes <= 0 or row_bytes <= 0:
        raise ValueError("bad shard geometry")
    body = body_pages * page_bytes
    total = body + dense_rows * row_bytes

    def cut(x: int) -> Tuple[int, int]:  # pages, rows whose middle byte lies before byte x
        p = min(body_pages, max(0, -(-(2 * x - page_bytes) // (2 * page_bytes))))
        r = min(dense_rows, max(0, -(-(2 * (x - body) - row_bytes) // (2 * row_bytes))))
        return p, r

    (p0, r0), (p1, r1) = cut(total * rank // world), cut(total * (rank + 1) // world)
    return (p0, p1), (r0, r1)


def all_gather_partials(o: torch.Tensor, ml: torch.Tensor,
                        group: Optional[dist.ProcessGroup] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """One all-gather of this rank's partials o [B, Hq, D] and ml [B, Hq, 2]:
    returns [n, B, Hq, D] and [n, B, Hq, 2] (rank order)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return o.unsqueeze(0), ml.unsqueeze(0)
    n = dist.get_world_size(group)
    B, Hq, D = o.shape
    flat = torch.cat([o.reshape(-1), ml.reshape(-1)])
    out = torch.empty(n * flat.numel(), dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(out, flat, group=group)
    out = out.view(n, -1)
    parts_o = out[:, :B * Hq * D].reshape(n, B, Hq, D)
    parts_ml = out[:, B * Hq * D:].reshape(n, B, Hq, 2)
    return parts_o, parts_ml


def decode(q: torch.Tensor, store: Optional[kv.Int4KVStore], dense: Optional[kv.DenseKV],
           sm_scale: Optional[float] = None, out_dtype: torch.dtype = torch.float32,
           out: Optional[torch.Tensor] = None, group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """Attention of q [B, Hq, 128] over the union of every rank's (store, dense)
    slice; every rank returns the full [B, Hq, 128] output."""
    o, ml = kv.decode_partial(q, store, dense, sm_scale=sm_scale)
    parts_o, parts_ml = all_gather_partials(o, ml, group)
    return kv.lse_merge(parts_o, parts_ml, out_dtype=out_dtype, out=out)


class SeqSplitDecoder:
    """The sequence-split decode of a multi-layer step without host work per
    layer: every layer's partial is written straight into its all-gather send
    buffer ([o | (m, l)] of B*Hq*130 floats), one NCCL ``all_gather_into_tensor``
    per layer gathers the ranks' buffers, and ``hkv_lse_merge_strided`` merges
    from the gathered buffer in place (no concatenation, no copy). ``capture``
    records the whole step, NCCL calls included, as one CUDA graph; ``close``
    releases it (before the process group is destroyed).

    ``chunks`` > 1 pipelines each layer over batch slices: slice c's all-gather
    runs on a side stream while slice c+1's partial runs on the compute stream,
    and each slice is merged as soon as its own gather has landed (one
    all-gather of [o | (m, l)] of that slice's sequences per slice). A rank whose
    store and dense segment are both None contributes the empty partial
    (o = 0, m = -inf, l = 0)."""

    def __init__(self, stores: List[Optional[kv.Int4KVStore]], denses: List[Optional[kv.DenseKV]],
                 batch: int, q_heads: int, group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None, chunks: int = 1):
        if len(stores) != len(denses) or not stores:
            raise ValueError("one (store, dense) pair per layer")
        if not 1 <= chunks <= batch:
            raise ValueError(f"chunks={chunks} must lie in [1, batch={batch}]")
        self.stores, self.denses = stores, denses
        self.L, self.B, self.Hq = len(stores), batch, q_heads
        self.group = group
        self.n = dist.get_world_size(group) if dist.is_initialized() else 1
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        row = q_heads * (kv.HEAD_DIM + 2)  # floats of one sequence's partial
        self.F = batch * row
        # slice c: sequences [b0, b1); its send block starts at float b0*row,
        # its gathered block (n ranks x (b1-b0)*row floats) at n*b0*row
        self.slices = [shard_range(batch, chunks, c) for c in range(chunks)]
        self.row = row
        self.send = torch.empty(self.L, self.F, dtype=torch.float32, device=self.device)
        self.recv = (torch.empty(self.L, self.n * self.F, dtype=torch.float32, device=self.device)
                     if self.n > 1 else self.send)
        self.comm = torch.cuda.Stream(device=self.device) if (self.n > 1 and chunks > 1) else None
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def _partial(self, l: int, q: torch.Tensor, b0: int, b1: int) -> None:
        Bc, Hq, D = b1 - b0, self.Hq, kv.HEAD_DIM
        blk = self.send[l, b0 * self.row:b1 * self.row]
        o = blk[:Bc * Hq * D].view(Bc, Hq, D)
        ml = blk[Bc * Hq * D:].view(Bc, Hq, 2)
        if self.stores[l] is None and self.denses[l] is None:
            o.zero_()
            ml[..., 0].fill_(float("-inf"))
            ml[..., 1].zero_()
            return
        kv.decode_partial(q[b0:b1], self.stores[l], self.denses[l], out_o=o, out_ml=ml, b0=b0)

    def _gather(self, l: int, b0: int, b1: int) -> None:
        r = self.row
        dist.all_gather_into_tensor(self.recv[l, self.n * b0 * r:self.n * b1 * r],
                                    self.send[l, b0 * r:b1 * r], group=self.group)

    def _merge(self, l: int, out: torch.Tensor, b0: int, b1: int) -> None:
        Bc, Hq, D, r = b1 - b0, self.Hq, kv.HEAD_DIM, self.row
        src = self.recv[l, self.n * b0 * r:self.n * b1 * r]
        dst = out[b0:b1]
        L.check(L.load().hkv_lse_merge_strided(
            src.data_ptr(), src.data_ptr() + Bc * Hq * D * 4, self.n, Bc * r, Bc * r, Bc, Hq, D, dst.data_ptr(),
            kv.dtype_code(dst.dtype), dst.stride(0), dst.stride(1),
            ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)), "hkv_lse_merge_strided")

    def _layer(self, l: int, q: torch.Tensor, out: torch.Tensor) -> None:
        if self.comm is None:  # one slice, or one rank: everything on the compute stream
            for b0, b1 in self.slices:
                self._partial(l, q, b0, b1)
                if self.n > 1:
                    self._gather(l, b0, b1)
                self._merge(l, out, b0, b1)
            return
        cur = torch.cuda.current_stream(self.device)
        landed = []
        for b0, b1 in self.slices:
            self._partial(l, q, b0, b1)
            self.comm.wait_stream(cur)
            with torch.cuda.stream(self.comm):
                self._gather(l, b0, b1)
                ev = torch.cuda.Event()
                ev.record(self.comm)
            landed.append(ev)
        for (b0, b1), ev in zip(self.slices, landed):
            cur.wait_event(ev)
            self._merge(l, out, b0, b1)

    def step(self, q: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """q [L, B, Hq, 128] -> out [L, B, Hq, 128] (every rank gets the full output)."""
        for l in range(self.L):
            self._layer(l, q[l], out[l])
        return out

    def capture(self, q: torch.Tensor, out: torch.Tensor) -> None:
        """Record ``step(q, out)`` over these static buffers as one CUDA graph
        (run once eagerly first: NCCL's communicator and the decode workspace of
        the capture stream come up outside the capture)."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step(q, out)
        s.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self.step(q, out)
        torch.cuda.current_stream(self.device).wait_stream(s)
        self.graph = g

    def replay(self) -> None:
        if self.graph is None:
            raise RuntimeError("SeqSplitDecoder.replay: call capture() first (or it was closed)")
        self.graph.replay()

    def close(self) -> None:
        self.graph = None
