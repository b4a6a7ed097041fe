"""Sequence-split decode attention across GPUs (config 4, variant B).

Every rank holds a contiguous, page-aligned slice of each sequence's INT4 body
(the last rank also holds the fp16/bf16 sink + recent segment), computes the
un-normalised partial (o, m, l) of the attention over its slice with
``hkv_decode_attn_partial``, and one NCCL all-gather of those partials
(B*Hq*130 floats per rank) feeds ``hkv_lse_merge``, which every rank runs to get
the full output. No other collective; the data path itself never crosses
NVLink.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist

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
