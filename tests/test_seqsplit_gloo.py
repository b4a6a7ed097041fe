"""Sequence-split decode (config 4, variant B), host side on CPU: the shard
ranges tile the body exactly, and the all-gather of partials (gloo, 2 ranks)
delivers them in rank order so that an LSE merge reproduces the attention over
the whole sequence. Partials and merge here are the oracle's (numpy); the GPU
path swaps in hkv_decode_attn_partial / hkv_lse_merge around the same exchange."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hetero_kvcache_optimizer_b200.seqsplit import all_gather_partials, shard_range, shard_spans
from oracle import kv_oracle as ko


@pytest.mark.parametrize("world", [1, 2, 3, 4, 7, 8])
def test_shard_ranges_tile_the_body(world):
    for total in range(0, 41):
        spans = [shard_range(total, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == total
        for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
            assert a1 == b0
        sizes = [b - a for a, b in spans]
        assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("world", [1, 2, 3, 4, 7, 8])
def test_shard_spans_tile_both_segments(world):
    """Byte-balanced spans: both segments tiled in rank order, every rank's
    bytes within one page (or row) of the equal share, and at most one rank
    that holds both a body slice and dense rows."""
    pb, rb = 40960, 512
    for pages in (0, 1, 3, 11, 59, 507):
        for rows in (0, 1, 100, 1088):
            if pages == rows == 0:
                continue
            spans = [shard_spans(pages, rows, world, r, pb, rb) for r in range(world)]
            assert spans[0][0][0] == 0 and spans[-1][0][1] == pages
            assert spans[0][1][0] == 0 and spans[-1][1][1] == rows
            for ((p0, p1), (r0, r1)), ((q0, q1), (s0, s1)) in zip(spans, spans[1:]):
                assert p1 == q0 and r1 == s0
            share = (pages * pb + rows * rb) / world
            for (p0, p1), (r0, r1) in spans:
                assert p1 >= p0 and r1 >= r0
                assert abs((p1 - p0) * pb + (r1 - r0) * rb - share) <= pb + rb
            both = sum(1 for (p0, p1), (r0, r1) in spans if p1 > p0 and r1 > r0)
            assert both <= 1, spans


def _partials(q, k, v, scale):
    """(o unnormalised, m, l) of one slice, natural-log domain. q [B,Hq,D], k/v [B,Hkv,S,D]."""
    G = q.shape[1] // k.shape[1]
    kk, vv = np.repeat(k, G, axis=1), np.repeat(v, G, axis=1)
    s = np.einsum("bhd,bhsd->bhs", q, kk) * scale
    m = s.max(axis=-1)
    p = np.exp(s - m[..., None])
    return np.einsum("bhs,bhsd->bhd", p, vv), m, p.sum(axis=-1)


def _rank(rank, world, port, q, k, v, result):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        S = k.shape[2]
        t0, t1 = shard_range(S, world, rank)
        o, m, l = _partials(q, k[:, :, t0:t1], v[:, :, t0:t1], 1 / np.sqrt(q.shape[-1]))
        ml = np.stack([m, l], axis=-1)
        po, pml = all_gather_partials(torch.from_numpy(o).float(), torch.from_numpy(ml).float())
        out = ko.lse_merge(po.numpy().astype(np.float64), pml[..., 0].numpy().astype(np.float64),
                           pml[..., 1].numpy().astype(np.float64))
        result[rank] = torch.from_numpy(out)
    finally:
        dist.destroy_process_group()


def test_all_gather_partials_merge_to_full_attention():
    world, port = 2, 29000 + os.getpid() % 1000
    rng = np.random.default_rng(4)
    B, Hq, Hkv, S, D = 2, 8, 2, 37, 128
    q = rng.standard_normal((B, Hq, D))
    k = rng.standard_normal((B, Hkv, S, D))
    v = rng.standard_normal((B, Hkv, S, D))
    ref = ko.decode_attention(q, k, v, dtype=np.float64)
    ctx = mp.get_context("spawn")
    with ctx.Manager() as man:
        result = man.dict()
        procs = [ctx.Process(target=_rank, args=(r, world, port, q, k, v, result)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
        assert all(p.exitcode == 0 for p in procs)
        for r in range(world):
            assert np.allclose(result[r].numpy(), ref, atol=1e-5), r
