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
    releases it (before the process group is destroyed)."""

    def __init__(self, stores: List[Optional[kv.Int4KVStore]], denses: List[Optional[kv.DenseKV]],
                 batch: int, q_heads: int, group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None):
        if len(stores) != len(denses) or not stores:
            raise ValueError("one (store, dense) pair per layer")
        self.stores, self.denses = stores, denses
        self.L, self.B, self.Hq = len(stores), batch, q_heads
        self.group = group
        self.n = dist.get_world_size(group) if dist.is_initialized() else 1
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.F = batch * q_heads * (kv.HEAD_DIM + 2)
        self.send = torch.empty(self.L, self.F, dtype=torch.float32, device=self.device)
        self.recv = (torch.empty(self.L, self.n * self.F, dtype=torch.float32, device=self.device)
                     if self.n > 1 else self.send)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def _layer(self, l: int, q: torch.Tensor, out: torch.Tensor) -> None:
        B, Hq, D = self.B, self.Hq, kv.HEAD_DIM
        o = self.send[l, :B * Hq * D].view(B, Hq, D)
        ml = self.send[l, B * Hq * D:].view(B, Hq, 2)
        kv.decode_partial(q, self.stores[l], self.denses[l], out_o=o, out_ml=ml)
        if self.n > 1:
            dist.all_gather_into_tensor(self.recv[l], self.send[l], group=self.group)
        src = self.recv[l]
        L.check(L.load().hkv_lse_merge_strided(
            src.data_ptr(), src.data_ptr() + B * Hq * D * 4, self.n, self.F, self.F, B, Hq, D, out.data_ptr(),
            kv.dtype_code(out.dtype), out.stride(0), out.stride(1),
            ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)), "hkv_lse_merge_strided")

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
