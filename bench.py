#!/usr/bin/env python
"""Benchmark: INT4-KV decode attention HBM GB/s (% of 8 TB/s) and tokens/s.

Default workload (benchmark spec configuration 1, Llama-3.1-8B-shaped decode):
32 layers, batch 8, 32 query / 8 KV heads, head_dim 128, 32768-token context
per sequence: 64 sink + 1024 recent tokens in fp16, 31,680 INT4 tokens
(group 32, fp16 scale + fp16 zero = min). One step = for every layer, one fused
launch: append the new token (ring eviction -> INT4 quantise) + split-KV decode
attention over the whole context + LSE merge (--no-fused, and the default for
--fmt ref: two launches). Synthetic seeded data (K/V ~ N(0,1) with four x10
outlier K channels per head, bf16 queries); the per-step working set (12 GB)
is far larger than L2, so no flush is needed between steps. The 1-GPU line
also carries short config-2, config-3 and ref-format measurements.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
  python bench.py --workload cfg2                       # config 2: long multimodal context
  python bench.py --workload cfg3 [--window PAGES [--delta D]] [--sweep]   # config 3: tiered offload
  python bench.py --workload cfg4 | cfg4b               # config 4: B64 context sweep / sequence split
  python bench.py --workload prefill [--sq N]          # multi-query attention over the INT4 body

With N > 1 (torchrun, one rank per GPU) every rank decodes its own 8
sequences (batch x KV-head sharding, no collective on the data path): weak
scaling, value = all ranks' bytes / max-over-ranks time. The N > 1 line also
carries a short config-4 variant-B measurement (``seqsplit_cfg4b``: each
sequence split over the ranks, one NCCL all-gather of the partials per layer).
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from typing import Optional

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "INT4-KV decode attn HBM GB/s (% of 8 TB/s) & tokens/s at 32K ctx, 1–8 GPU"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0

CFG1 = dict(layers=32, batch=8, q_heads=32, kv_heads=8, ctx=32768, sink=64, recent=1024, group=32)


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--fmt", default="fp16min", choices=["fp16min", "ref"])
    ap.add_argument("--layers", type=int, default=None,
                    help="layers (default: the workload's own, 32 for cfg1/cfg3, 28 for cfg2)")
    ap.add_argument("--ctas", type=int, default=0, help="persistent decode grid (0 = one CTA per SM)")
    ap.add_argument("--workload", default="cfg1", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg4b", "prefill"],
                    help="cfg1: the headline decode benchmark (default); cfg2: long multimodal context "
                         "(chunked prefill quantise + decode); cfg3: tiered offload, layer-ahead "
                         "host->device page prefetch; cfg4: B64 context sweep 4K-128K, unit shard and "
                         "sequence split; cfg4b: sequence split across ranks + NCCL all-gather "
                         "of partials + LSE merge; prefill: tcgen05 multi-query attention over a "
                         "32K INT4 body (each prints its own line)")
    ap.add_argument("--sq", type=int, default=2048, help="prefill: query positions per sequence")
    ap.add_argument("--ctx", type=int, default=131072, help="cfg4b: context per sequence")
    ap.add_argument("--batch", type=int, default=64, help="cfg4b: sequences")
    ap.add_argument("--seq-chunks", type=int, default=1,
                    help="cfg4b: pipelined batch slices per layer (all-gather of one overlaps the next's partial)")
    ap.add_argument("--window", type=int, default=0,
                    help="cfg3: cold pages copied and attended per unit and layer (0 = all of them)")
    ap.add_argument("--delta", type=int, default=-1,
                    help="cfg3: with --window, keep the window cached in HBM and slide it by this many pages "
                         "per step (only those are copied); -1 = copy the whole window every step")
    ap.add_argument("--sweep", action="store_true",
                    help="cfg3: add the exposed-transfer curve over window slides of 0, 1, 2, 4, 8 pages")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--cpu-steps", type=int, default=2)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-offload", action="store_true",
                    help="cfg1: leave out the short config-2 and config-3 measurements on the 1-GPU line")
    ap.add_argument("--no-early", action="store_true",
                    help="cfg1/cfg2: fused launches wait for the previous launch before reading the cache "
                         "(default: stream it while the previous layer's launch finishes)")
    ap.add_argument("--no-fused", action="store_true",
                    help="cfg1/cfg2: run each layer's step as two launches (append, then decode) "
                         "instead of the fused decode-append launch")
    return ap.parse_args()


def measured_tensor_peak(sustained: bool = False):
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops_sustained" if sustained else "bf16_tflops"]), "measured"
    except Exception:
        return (1400.0 if sustained else 1590.0), "fallback"


def measured_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(bytes_per_launch: float, name: str = "decode_kernel_cfg1_traffic.json"):
    """DRAM bytes (read + write) per launch from a committed ncu capture
    (profiles/<name>), scaled to this launch's algorithmic bytes; None when no
    capture is recorded."""
    p = os.path.join(REPO, "profiles", name)
    try:
        with open(p) as f:
            t = json.load(f)
        return round((t["dram_bytes_read"] + t["dram_bytes_write"]) * bytes_per_launch / t["algorithmic_bytes"])
    except Exception:
        return None


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, interval_ms: int = 200):
        self.gpu = gpu_index
        self.interval = interval_ms
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", str(self.interval),
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sms, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sms.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, val in zip(names, f[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(n)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sms)}


# --------------------------------------------------------------------------- CPU reference path
def run_cpu_reference(steps: int, warmup: int, fmt_bytes_fn, sample_batch: int = 2):
    """Time the reference's CPU path (oracle/ref_port.py) on a bounded sample:
    one layer of configuration 1 with ``sample_batch`` of its 8 sequences."""
    import torch
    from oracle.ref_port import RefLayer
    torch.set_num_threads(os.cpu_count() or 1)
    c = CFG1
    body = c["ctx"] - c["sink"] - c["recent"]
    layer = RefLayer(sample_batch, c["kv_heads"], body, c["sink"], c["recent"], group=c["group"])
    g = torch.Generator().manual_seed(5)
    times = []
    for i in range(warmup + steps):
        q = torch.randn(sample_batch, c["q_heads"], 128, generator=g).bfloat16()
        kn = torch.randn(sample_batch, c["kv_heads"], 128, generator=g).half()
        vn = torch.randn(sample_batch, c["kv_heads"], 128, generator=g).half()
        t0 = time.perf_counter()
        layer.step(q, kn, vn)
        dt = time.perf_counter() - t0
        if i >= warmup:
            times.append(dt)
    sec = sum(times) / len(times)
    nbytes = fmt_bytes_fn(sample_batch, body + 1)
    return {"value": nbytes / sec / 1e9, "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"1 of 32 layers, {sample_batch} of 8 sequences, {len(times)} decode steps "
                      f"(append-compress + dequant + SDPA, reference torch CPU path, pinned to the "
                      f"reference's goldens by tests/test_ref_port.py); {sec * 1e3:.0f} ms per layer-step; "
                      f"GB/s = the GPU workload's algorithmic bytes for the same tokens "
                      f"({nbytes / (sample_batch * (body + 1)):.1f} B per body token, packed format) "
                      f"/ time, a normalisation, not the CPU's own traffic (it reads 1 B per code)",
            "ms_per_layer_step": sec * 1e3}


def layer_bytes(batch, body_tokens, fmt, kv_heads=8, q_heads=32, sink=64, recent=1024, group=32):
    ng = 128 // group
    meta = 4 * ng + (ng if fmt == "ref" else 0)
    units = batch * kv_heads
    attn = units * (body_tokens * 2 * (64 + meta) + (sink + recent) * 512) + batch * q_heads * 128 * (2 + 4)
    append = units * 2 * (128 * 2 * 3 + 64 + meta)
    return attn + append


# --------------------------------------------------------------------------- config 2
def cfg2_measure(layers: int, steps: int, warmup: int, fmt: str, dev, fused: Optional[bool] = None,
                 early: Optional[bool] = None) -> dict:
    """Qwen2-VL-7B-shaped long multimodal decode: 28 layers, B1, Hq28/Hkv4 (GQA 7),
    131,072-token context (positions < 100,000 'vision' K/V ~ N(0, 0.5^2), the rest
    'text' ~ N(0, 1) with 4 x10 outlier K channels per head); chunked prefill
    quantises the INT4 body in 4,096-token chunks, then decode steps (append +
    attention over 64 sink + 1,024 recent fp16 + 129,984 INT4 tokens)."""
    import torch
    from hetero_kvcache_optimizer_b200 import _lib, kvstore as kv
    from hetero_kvcache_optimizer_b200.decode_engine import TieredKVDecoder
    B, Hq, Hkv, ctx, sink, recent, chunk = 1, 28, 4, 131072, 64, 1024, 4096
    body = ctx - sink - recent
    total_steps = warmup + steps + 4
    eng = TieredKVDecoder(layers, B, Hq, Hkv, sink=sink, recent=recent, body_capacity=body + total_steps + 8,
                          fmt=fmt, group=32, kv_dtype=torch.float16, out_dtype=torch.float32, device=dev,
                          fused_append=fused, early=early)
    gen = torch.Generator(device=dev).manual_seed(2)
    st_ = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    q_ms = 0.0
    for l in range(layers):
        k = torch.randn(B, Hkv, ctx, 128, device=dev, generator=gen)
        v = torch.randn(B, Hkv, ctx, 128, device=dev, generator=gen)
        k[:, :, :100000] *= 0.5
        v[:, :, :100000] *= 0.5
        for h in range(Hkv):
            ch = torch.randperm(128, device=dev, generator=gen)[:4]
            k[:, h, 100000:, ch] *= 10.0
        k, v = k.half(), v.half()
        d = eng.dense[l]
        d.k[:, :, :sink] = k[:, :, :sink]
        d.v[:, :, :sink] = v[:, :, :sink]
        d.k[:, :, sink:] = k[:, :, ctx - recent:]
        d.v[:, :, sink:] = v[:, :, ctx - recent:]
        def chunked(store=eng.stores[l], k=k, v=v):
            for t0 in range(0, body, chunk):  # chunked prefill: the body in 4,096-token chunks
                n = min(chunk, body - t0)
                kv.quantize_pack_kv(k[:, :, sink + t0:sink + t0 + n], v[:, :, sink + t0:sink + t0 + n], store, t0)
        torch.cuda.synchronize()
        if l == 0:
            # device time of the chunk launches: captured once, replayed (the Python
            # dispatch of 64 small calls would otherwise be what is timed)
            gs = torch.cuda.Stream(device=dev)
            gs.wait_stream(st_)
            with torch.cuda.stream(gs):
                chunked()
            gs.synchronize()
            qg = torch.cuda.CUDAGraph()
            with torch.cuda.graph(qg, stream=gs):
                chunked()
            st_.wait_stream(gs)
            qg.replay()
            torch.cuda.synchronize()
            e0.record(st_)
            for _ in range(5):
                qg.replay()
            e1.record(st_)
            torch.cuda.synchronize()
            q_ms = layers * e0.elapsed_time(e1) / 5
            del qg
        else:
            chunked()
        del k, v
    eng.set_state(body)
    ng = 4
    q_bytes = layers * B * Hkv * body * 2 * (128 * 2 + 64 + 4 * ng + (ng if fmt == "ref" else 0))
    eng.capture(max_steps=total_steps)
    q, kn, vn, out = eng.static_buffers
    q.copy_(torch.randn(q.shape, device=dev, generator=gen))
    kn.copy_(torch.randn(kn.shape, device=dev, generator=gen))
    vn.copy_(torch.randn(vn.shape, device=dev, generator=gen))
    for _ in range(warmup):
        eng.replay()
    torch.cuda.synchronize()
    body0 = eng.body_len
    sampler = ClockSampler(dev.index, 50)
    sampler.start()
    e0.record(st_)
    for _ in range(steps):
        eng.replay()
    e1.record(st_)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / steps
    step_bytes = sum(eng.step_bytes(body0 + i) for i in range(steps)) / steps
    derr = _lib.device_error(clear=True)
    if derr:
        raise RuntimeError(f"device error bits {derr} during the benchmark")
    return {
        "metric": "config2 long-context decode: HBM GB/s and tokens/s; chunked prefill quantise GB/s",
        "value": round(step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "n_gpus": 1, "steps": steps,
        "warmup": warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 mma (int4 storage, fp32 accum)", "data": "synthetic",
        "config": {"workload": "config2: Qwen2-VL-7B-shaped, 28 layers, B1, Hq28/Hkv4 (GQA 7), ctx 131072 "
                               "(100,000 vision tokens N(0,0.5^2), text N(0,1) + outliers); 64 sink + 1024 "
                               "recent fp16 + 129,984 INT4 g32", "layers": layers, "kv_format": fmt},
        "tokens_per_s": round(B / (ms * 1e-3), 1),
        "prefill_quantize": {"chunk_tokens": chunk, "ms_all_layers": round(q_ms, 3),
                             "gbs": round(q_bytes / (q_ms * 1e-3) / 1e9, 1),
                             "tokens_per_s": round(layers * B * body / (q_ms * 1e-3), 0)},
        "gpu_launches": steps * layers * eng.launches_per_layer, "clocks": clocks}


def run_cfg2(args) -> None:
    import torch
    torch.cuda.set_device(0)
    print(json.dumps(cfg2_measure(args.layers, args.steps, args.warmup, args.fmt, torch.device("cuda", 0),
                                  fused=False if args.no_fused else None,
                                  early=False if args.no_early else None)))


# --------------------------------------------------------------------------- prefill
def run_prefill(args) -> None:
    """Chunked-prefill attention against an offloaded INT4 context: Sq query
    positions x 32 query heads (GQA 4 over 8 KV heads) of one sequence attend a
    32,768-token INT4 body (fp16min, group 32; Llama-3.1-8B attention shape),
    one launch of the tcgen05 prefill kernel per step (fused_dequant_attn_forward's
    path). FLOPs = 4 * Hq * Sq * S * 128 (QK^T and PV). The body (8 heads x
    32,768 tokens x 160 B = 42 MB) fits in L2, so L2 is flushed before every
    timed launch; the launch then reads it from HBM once and from L2 after."""
    import numpy as np
    import torch
    from hetero_kvcache_optimizer_b200 import _lib, kvstore as kv
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    B, Hq, Hkv, S, Sq = 1, 32, 8, 32768, args.sq
    gen = torch.Generator(device=dev).manual_seed(5)
    store = kv.Int4KVStore(B, Hkv, S, fmt=args.fmt, group=32, device=dev)
    k = torch.randn(B, Hkv, S, 128, device=dev, generator=gen)
    for h in range(Hkv):
        ch = torch.randperm(128, device=dev, generator=gen)[:4]
        k[:, h, :, ch] *= 10.0
    kv.prefill(store, k.half(), torch.randn(B, Hkv, S, 128, device=dev, generator=gen).half())
    del k
    q = torch.randn(B, Hq, Sq, 128, device=dev, generator=gen).to(torch.bfloat16)
    out = torch.empty(B, Hq, Sq, 128, device=dev, dtype=torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 256 MB > L2
    st_ = torch.cuda.current_stream()
    for _ in range(args.warmup):
        kv.prefill_attn(q, store, out=out)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    sampler = ClockSampler(0)
    sampler.start()
    time.sleep(0.2)
    for i in range(args.steps):
        flush.fill_(i & 255)
        starts[i].record(st_)
        kv.prefill_attn(q, store, out=out)
        ends[i].record(st_)
    torch.cuda.synchronize()
    clocks = sampler.stop()
    ms = sum(a.elapsed_time(b) for a, b in zip(starts, ends)) / args.steps
    flops = 4.0 * B * Hq * Sq * S * 128
    # launches per step: the attention kernel, plus the merge when the library splits the body
    import ctypes
    pst = store.struct()
    split = _lib.load().hkv_prefill_workspace_bytes(ctypes.byref(pst), B, Hq, Hkv, Sq, 128, 0) > 0
    kname = ("prefill2_kernel (two query tiles per CTA)" if Sq * (Hq // Hkv) > 128 else "prefill_kernel") + \
        (" + prefill_merge_kernel (body split)" if split else "")
    tflops = flops / (ms * 1e-3) / 1e12
    peak, kind = measured_tensor_peak(sustained=False)

    # end to end through the public API: q from pinned host, out back to pinned host
    qh = q.cpu().pin_memory()
    oh = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    qd = torch.empty_like(q)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(2):
        qd.copy_(qh, non_blocking=True)
        kv.prefill_attn(qd, store, out=out)
        oh.copy_(out, non_blocking=True)
    torch.cuda.synchronize()
    e0.record(st_)
    for _ in range(args.steps):
        qd.copy_(qh, non_blocking=True)
        kv.prefill_attn(qd, store, out=out)
        oh.copy_(out, non_blocking=True)
    e1.record(st_)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    derr = _lib.device_error(clear=True)
    if derr:
        raise RuntimeError(f"device error bits {derr} during the benchmark")

    cpu = None
    if not args.no_cpu:  # the oracle's numpy restatement on a bounded sample: one KV head, 64 query rows
        from oracle import kv_oracle as ko
        rng = ko.rng_for(5)
        kk = rng.standard_normal((1, 1, S, 128), dtype=np.float32)
        vv = rng.standard_normal((1, 1, S, 128), dtype=np.float32)
        qq = rng.standard_normal((1, 4, 16, 128), dtype=np.float32)
        t0 = time.perf_counter()
        reps = 0
        while reps < 3 or time.perf_counter() - t0 < 2.0:
            ko.prefill_attention(qq, kk, vv)
            reps += 1
        dt = (time.perf_counter() - t0) / reps
        cpu = {"value": round(4.0 * 64 * S * 128 / dt / 1e12, 5), "unit": "TFLOP/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"numpy restatement (dequantised fp32 K/V given), 1 KV head x 64 query rows x {S} keys"}
    line = {
        "metric": "INT4 prefill attention TFLOP/s (tcgen05, fused dequant)", "value": round(tflops, 1),
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16 tcgen05 mma (int4 storage, fp32 accum)", "data": "synthetic",
        "config": {"workload": f"prefill: B1, Hq32/Hkv8, D128, {Sq} query positions vs a {S}-token INT4 body "
                               f"({args.fmt}, g32), no mask", "kv_format": args.fmt, "sq": Sq, "body": S,
                   "l2": "flushed (256 MB write) before every timed launch"},
        "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tflops / peak, 4), "traffic": None,
                     "kernel": kname, "flops_per_launch": flops,
                     "peak_kind": f"{kind} (cuBLAS bf16 burst)"},
        "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                "h2d_bytes_per_step": qh.numel() * qh.element_size(),
                "d2h_bytes_per_step": oh.numel() * oh.element_size(), "ms_per_step": round(e2e_ms, 4),
                "api": "kvstore.prefill_attn (pinned host q in, bf16 out back to pinned host)"},
        "gpu_launches": args.steps * (2 if split else 1), "clocks": clocks,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line))


# --------------------------------------------------------------------------- config 3
def cfg3_measure(layers: int, window: int, delta: Optional[int], steps: int, warmup: int, fmt: str, dev,
                 clocks: bool = False, sweep_ctas: bool = False, transport: str = "copy",
                 copy_streams: int = 1) -> dict:
    """InternLM2-7B-shaped tiered offload: 32 layers, B4, Hq32/Hkv8, 131,072-token
    context of which 8,256 stay in HBM (64 sink + 1,024 recent fp16, 28 INT4 pages)
    and 480 INT4 pages of 256 tokens per (sequence, KV head) live in pinned host
    DRAM. delta None: every step copies the layer's cold pages (all 480, or the
    last `window`), one layer ahead of their attention; delta d: the window of
    `window` cold pages stays cached in HBM and slides by d pages per step, so a
    step copies only the d pages entering it (SlidingWindowOffload). Exposed
    transfer = step time with the copies - step time without them."""
    import torch
    from hetero_kvcache_optimizer_b200 import _lib
    from hetero_kvcache_optimizer_b200.offload import SlidingWindowOffload, TieredOffloadDecoder
    if delta is None:
        dec = TieredOffloadDecoder(layers, 4, 32, 8, resident_pages=28, cold_pages=480,
                                   window_pages=window or None, fmt=fmt, device=dev)
    else:
        dec = SlidingWindowOffload(layers, 4, 32, 8, resident_pages=28, cold_pages=480, window_pages=window,
                                   delta=delta, fmt=fmt, device=dev)
    gen = torch.Generator(device=dev).manual_seed(3)
    dec.fill(gen)
    q = torch.randn(layers, 4, 32, 128, device=dev, generator=gen).bfloat16()
    out = torch.empty(layers, 4, 32, 128, device=dev)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    graphs = delta is not None
    if graphs:  # one graph replay per step: page moves + attentions, no host work per layer
        dec.capture(q, out, transport=transport, copy_streams=copy_streams)

    def timed(transfer: bool) -> float:
        run = (lambda: dec.replay(transfer)) if graphs else (lambda: dec.step(q, out, transfer))
        for _ in range(warmup):
            run()
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(steps):
            run()
        e1.record(st)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    sampler = ClockSampler(dev.index, 50) if clocks else None
    if sampler:
        sampler.start()
    ms_with = timed(True)
    ms_without = timed(False)
    clk = sampler.stop() if sampler else None
    h2d = dec.h2d_bytes_per_step()
    copy_ms, ctas_gbs = None, None
    if h2d:
        # the host link alone: one step's copies back to back on the side stream
        ps = dec.prefetcher.stream
        c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        c0.record(ps)
        if delta is None:
            for l in range(layers):
                dec.prefetcher.submit(dec.src_pages, dec.dst_slots[l % 2])
        elif transport == "gather":  # the gathers a replayed step issues, back to back
            for l in range(layers):
                dec.prefetcher.gather(dec.g_src, dec.g_dst[l][0], dec.step_dev, delta * dec.units, 0,
                                      ctas=dec.gather_ctas)
        else:  # the copies a replayed step issues (one per page row of all units), back to back
            for l in range(layers):
                for i in range(delta):
                    p = (dec.window - delta + i) % dec.cold
                    dec.prefetcher.submit([p * dec.units + u for u in range(dec.units)],
                                          [dec._slot(l, u, dec.window - delta + i) for u in range(dec.units)])
        c1.record(ps)
        torch.cuda.synchronize()
        copy_ms = c0.elapsed_time(c1)
        if delta is not None and sweep_ctas:  # the gather alone at other grid sizes
            ctas_gbs = {}
            for ct in (16, 32, 64, 128, 148):
                torch.cuda.synchronize()
                c0.record(ps)
                for l in range(layers):
                    dec.prefetcher.gather(dec.g_src, dec.g_dst[l][0], dec.step_dev, delta * dec.units, 0, ctas=ct)
                c1.record(ps)
                torch.cuda.synchronize()
                ctas_gbs[ct] = round(h2d / (c0.elapsed_time(c1) * 1e-3) / 1e9, 2)
    derr = _lib.device_error(clear=True)
    if derr:
        raise RuntimeError(f"device error bits {derr} during the config-3 benchmark")
    r = {"mode": "full cold set" if delta is None and not window else
             f"window of the last {window} pages, copied every step" if delta is None else
             f"window of {window} pages cached in HBM, sliding {delta} page(s) per step "
             f"(CUDA graph per step, page moves by "
             f"{f'copy engines, {copy_streams} stream(s)' if transport == 'copy' else 'zero-copy gather kernel'})",
         "layers": layers, "window_pages": dec.window, "delta_pages": delta,
         "h2d_bytes_per_step": h2d, "ms_per_step": round(ms_with, 4),
         "decode_ms_per_step_without_transfer": round(ms_without, 4),
         "exposed_ms_per_step": round(ms_with - ms_without, 4),
         "exposed_pct_of_step": round(100 * (ms_with - ms_without) / ms_with, 2),
         "h2d_gbs_in_step": round(h2d / (ms_with * 1e-3) / 1e9, 2),
         "h2d_copy_only_ms_per_step": round(copy_ms, 4) if copy_ms else None,
         "h2d_copy_only_gbs": round(h2d / (copy_ms * 1e-3) / 1e9, 2) if copy_ms else None,
         "attn_gbs_without_transfer": round(dec.attn_bytes_per_step() / (ms_without * 1e-3) / 1e9, 1),
         "attended_tokens": dec.tokens + dec.dense[0].len_hint, "gpu_launches": steps * layers}
    if ctas_gbs is not None:
        r["gather_gbs_by_ctas"] = ctas_gbs
    if clk is not None:
        r["clocks"] = clk
    del dec
    return r


def run_cfg3(args) -> None:
    """Config 3 as its own line (see cfg3_measure); --delta d selects the
    residency-aware sliding window, --sweep the exposed-transfer curve over
    d = 0, 1, 2, 4, 8 with an 8-page window beside the full-cold-set figure."""
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    delta = None if args.delta < 0 else args.delta
    r = cfg3_measure(args.layers, args.window, delta, args.steps, args.warmup, args.fmt, dev, clocks=True,
                     sweep_ctas=True)
    line = {"metric": "config3 tiered offload: H2D GB/s and exposed transfer ms per decode step",
            "value": r["h2d_gbs_in_step"], "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 mma (int4 storage, fp32 accum)",
            "data": "synthetic",
            "config": {"workload": "config3: InternLM2-7B-shaped tiered offload, 32 layers, B4, Hq32/Hkv8, "
                                   "ctx 131072: 64 sink + 1024 recent fp16 + 28 INT4 pages in HBM, 480 INT4 "
                                   "pages of 256 tokens per unit in pinned host DRAM",
                       "layers": args.layers, "kv_format": args.fmt},
            **{k: v for k, v in r.items() if k not in ("clocks",)}, "clocks": r.get("clocks")}
    if args.sweep:
        line["sweep"] = [cfg3_measure(args.layers, 8, d, args.steps, args.warmup, args.fmt, dev)
                         for d in (0, 1, 2, 4, 8)]
        line["sweep_gather"] = [cfg3_measure(args.layers, 8, d, args.steps, args.warmup, args.fmt, dev,
                                             transport="gather") for d in (1, 2)]
        line["sweep_two_copy_streams"] = [cfg3_measure(args.layers, 8, d, args.steps, args.warmup, args.fmt, dev,
                                                       copy_streams=2) for d in (1, 2)]
    print(json.dumps(line))


# --------------------------------------------------------------------------- ref format
def ref_format_measure(args, dev, peak: float, layers: int = 4, steps: int = 20, warmup: int = 5) -> dict:
    """The decode step of config 1 in the reference-bit-exact format (codes,
    fp32 scales and u8 zero-points equal to KVCompressor.compress; the decode
    kernel expands the metadata in shared memory), as the engine runs it for
    that format (two launches per layer: append, then attention): time per
    layer and GB/s over a graph of `layers` layers, CUDA events on the
    replaying stream."""
    import torch
    from hetero_kvcache_optimizer_b200 import kvstore as kv
    from hetero_kvcache_optimizer_b200.decode_engine import TieredKVDecoder
    c = CFG1
    body = c["ctx"] - c["sink"] - c["recent"]
    eng = TieredKVDecoder(layers, c["batch"], c["q_heads"], c["kv_heads"], sink=c["sink"], recent=c["recent"],
                          body_capacity=body + warmup + steps + 8, fmt="ref", group=c["group"],
                          kv_dtype=torch.float16, out_dtype=torch.float32, device=dev)
    gen = torch.Generator(device=dev).manual_seed(11)
    for l in range(layers):
        k = torch.randn(c["batch"], c["kv_heads"], body, 128, device=dev, generator=gen).half()
        v = torch.randn(c["batch"], c["kv_heads"], body, 128, device=dev, generator=gen).half()
        kv.prefill(eng.stores[l], k, v)
        del k, v
        eng.dense[l].k.normal_(generator=gen)
        eng.dense[l].v.normal_(generator=gen)
    eng.set_state(body)
    eng.capture(max_steps=warmup + steps + 2)
    q, kn, vn, _ = eng.static_buffers
    q.copy_(torch.randn(q.shape, device=dev, generator=gen))
    kn.copy_(torch.randn(kn.shape, device=dev, generator=gen))
    vn.copy_(torch.randn(vn.shape, device=dev, generator=gen))
    for _ in range(warmup):
        eng.replay()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    body0 = eng.body_len
    e0.record(st)
    for _ in range(steps):
        eng.replay()
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / (steps * layers)
    nbytes = sum(eng.step_bytes(body0 + i) for i in range(steps)) / (steps * layers)
    gbs = nbytes / (us * 1e-6) / 1e9
    del eng
    return {"kernel": "append_kv_kernel + decode_kernel, HKV_FMT_REF group 32 (168 B per token), two launches "
                      "per layer", "layers_timed": layers,
            "us_per_layer": round(us, 2), "bytes_per_layer": round(nbytes), "achieved": round(gbs, 1),
            "frac": round(gbs / peak, 4), "unit": "GB/s"}


# --------------------------------------------------------------------------- config 4, variant B
def seqsplit_measure(B: int, ctx: int, layers: int, steps: int, warmup: int, fmt: str, world: int, rank: int,
                     dev, chunks: int = 1) -> dict:
    """Config 4 variant B on this process group: Llama-3.1-8B shape, B sequences
    of `ctx` tokens; each unit's byte line [INT4 body pages | 64 sink + 1024
    recent fp16 rows] cut into equal contiguous spans, one per rank
    (``seqsplit.shard_spans``: attention does not depend on the order of the
    keys, so any rank may hold any rows, and most ranks hold one segment); per
    layer: partial attention on every rank, one all-gather of the partials, LSE
    merge, in ``chunks`` pipelined batch slices. Returns the max-over-ranks step
    time and the aggregate figures (every rank gets the same dict)."""
    import torch
    import torch.distributed as dist
    from hetero_kvcache_optimizer_b200 import _lib, kvstore as kv, seqsplit
    Hq, Hkv = 32, 8
    sink, recent = 64, 1024
    body_pages = (ctx - sink - recent) // 256
    (p0, p1), (r0, r1) = seqsplit.shard_spans(body_pages, sink + recent, world, rank,
                                              kv.page_bytes(fmt, 32, 256), 2 * 128 * 2)
    ntok = (p1 - p0) * 256
    nrows = r1 - r0
    gen = torch.Generator(device=dev).manual_seed(40 + rank)
    stores, denses = [], []
    for l in range(layers):
        st = kv.Int4KVStore(B, Hkv, max(ntok, 256), fmt=fmt, group=32, device=dev)
        for t0 in range(0, ntok, 4096):
            n = min(4096, ntok - t0)
            x = torch.randn(B, Hkv, n, 128, device=dev, generator=gen).half()
            kv.quantize_pack(x, st, 0, t0)
            kv.quantize_pack(x, st, 1, t0)
        st.set_lengths(ntok)
        stores.append(st)
        if nrows:
            d = kv.DenseKV(B, Hkv, nrows, device=dev)
            d.k.normal_(generator=gen)
            d.v.normal_(generator=gen)
            d.set_lengths(nrows)
            denses.append(d)
        else:
            denses.append(None)
    q = torch.randn(layers, B, Hq, 128, device=dev, generator=gen).bfloat16()
    out = torch.empty(layers, B, Hq, 128, device=dev)
    # one CUDA graph per step: partial -> NCCL all-gather -> in-place merge per layer
    dec = seqsplit.SeqSplitDecoder([st if ntok else None for st in stores], denses, B, Hq, device=dev,
                                   chunks=chunks)
    dec.capture(q, out)

    def step():
        dec.replay()

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    st_ = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st_)
    for _ in range(steps):
        step()
    e1.record(st_)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    derr = _lib.device_error(clear=True)
    if derr:
        raise RuntimeError(f"device error bits {derr} during the sequence-split benchmark")
    per_tok = 2 * (64 + 4 * 4 + (4 if fmt == "ref" else 0))
    step_bytes = layers * (B * Hkv * (body_pages * 256 * per_tok + (sink + recent) * 512) + B * Hq * 128 * 6)
    peak, _ = measured_peak()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    dec.close()  # the graph holds NCCL calls: release it before the process group goes
    del dec, stores, denses, q, out
    return {"ms_per_step": round(ms, 4), "gbs": round(gbs, 2), "tokens_per_s": round(B / (ms * 1e-3), 1),
            "pct_of_aggregate_measured_peak": round(100 * gbs / (world * peak), 2),
            "workload": f"config4 B: Llama-3.1-8B shape, B{B}, ctx {ctx} ({body_pages} INT4 pages + 64 sink + "
                        f"1024 recent fp16 rows per unit, byte-balanced spans over the ranks), "
                        f"{layers} layers, sequence split over {world} GPU(s), one "
                        f"NCCL all-gather of the partials per layer and batch slice + LSE merge, "
                        f"{chunks} pipelined batch slice(s), one CUDA graph per step",
            "chunks": chunks, "gpu_launches": world * steps * layers * 2 * chunks}


def batchshard_measure(B: int, ctx: int, layers: int, steps: int, warmup: int, fmt: str, world: int, rank: int,
                       dev) -> dict:
    """Config 4 variant A on this process group: Llama-3.1-8B shape, B sequences
    of `ctx` tokens (64 sink + 1024 recent fp16, the rest INT4), the B x Hkv
    units sharded by sequence over the ranks (B / world each), every rank running
    the single-GPU decode on its shard: no collective. Max-over-ranks step time
    and aggregate figures (every rank gets the same dict)."""
    import torch
    import torch.distributed as dist
    from hetero_kvcache_optimizer_b200 import _lib, kvstore as kv
    Hq, Hkv, sink, recent = 32, 8, 64, 1024
    if B % world:
        raise ValueError("batch must divide over the ranks")
    Br = B // world
    ntok = ctx - sink - recent
    gen = torch.Generator(device=dev).manual_seed(50 + rank)
    stores, denses = [], []
    for l in range(layers):
        st = kv.Int4KVStore(Br, Hkv, ntok, fmt=fmt, group=32, device=dev)
        for t0 in range(0, ntok, 4096):
            n = min(4096, ntok - t0)
            x = torch.randn(Br, Hkv, n, 128, device=dev, generator=gen).half()
            kv.quantize_pack(x, st, 0, t0)
            kv.quantize_pack(x, st, 1, t0)
        st.set_lengths(ntok)
        d = kv.DenseKV(Br, Hkv, sink + recent, device=dev)
        d.k.normal_(generator=gen)
        d.v.normal_(generator=gen)
        d.set_lengths(sink + recent)
        stores.append(st)
        denses.append(d)
    q = torch.randn(layers, Br, Hq, 128, device=dev, generator=gen).bfloat16()
    out = torch.empty(layers, Br, Hq, 128, device=dev)

    def step():
        for l in range(layers):
            kv.decode(q[l], stores[l], denses[l], out=out[l])

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    st_ = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(st_)
    for _ in range(steps):
        step()
    e1.record(st_)
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    derr = _lib.device_error(clear=True)
    if derr:
        raise RuntimeError(f"device error bits {derr} during the batch-shard benchmark")
    per_tok = 2 * (64 + 4 * 4 + (4 if fmt == "ref" else 0))
    step_bytes = layers * (B * Hkv * (ntok * per_tok + (sink + recent) * 512) + B * Hq * 128 * 6)
    peak, _ = measured_peak()
    gbs = step_bytes / (ms * 1e-3) / 1e9
    del stores, denses, q, out
    return {"ms_per_step": round(ms, 4), "gbs": round(gbs, 2), "tokens_per_s": round(B / (ms * 1e-3), 1),
            "pct_of_aggregate_measured_peak": round(100 * gbs / (world * peak), 2),
            "pct_of_aggregate_8TBs": round(100 * gbs / (world * NOMINAL_HBM_GBS), 2),
            "gpu_launches": world * steps * layers}


def run_cfg4(args, world: int, rank: int, local: int) -> None:
    """Config 4: Llama-3.1-8B decode at B 64 over contexts of 4K, 16K, 64K and
    128K tokens, variant A (batch x KV-head units sharded over the ranks, no
    collective) and variant B (each sequence split over the ranks, one NCCL
    all-gather of the partials per layer, LSE merge): tokens/s and % of the
    aggregate HBM roofline, 2 layers per step (per-layer figures)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    rows = []
    for ctx in (4096, 16384, 65536, 131072):
        a = batchshard_measure(args.batch, ctx, 2, args.steps, args.warmup, args.fmt, world, rank, dev)
        b = seqsplit_measure(args.batch, ctx, 2, args.steps, args.warmup, args.fmt, world, rank, dev)
        row = {"ctx": ctx, "variant_a": a, "variant_b": {k: v for k, v in b.items() if k != "workload"}}
        if world > 1:  # the same step pipelined over two batch slices (gathers overlap partials)
            b2 = seqsplit_measure(args.batch, ctx, 2, args.steps, args.warmup, args.fmt, world, rank, dev, chunks=2)
            row["variant_b_pipelined"] = {k: v for k, v in b2.items() if k != "workload"}
        rows.append(row)
    if rank == 0:
        top = rows[-1]["variant_a"]
        print(json.dumps({
            "metric": "config4: Llama-3.1-8B INT4-KV decode attention at B64, tokens/s and % of aggregate HBM "
                      "roofline, contexts 4K-128K, variants A (unit shard) and B (sequence split)",
            "value": top["tokens_per_s"], "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": top["ms_per_step"], "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f16 mma (int4 storage, fp32 accum)",
            "data": "synthetic",
            "config": {"workload": "config4: Llama-3.1-8B shape (Hq32/Hkv8, D128), B64, 2 layers, contexts "
                                   "4096/16384/65536/131072 (64 sink + 1024 recent fp16, the rest INT4 g32); "
                                   "value = variant A at 131072", "kv_format": args.fmt,
                       "parallelism": f"A: shard{world} / B: seqsplit{world}"},
            "sweep": rows, "gpu_launches": sum(r["variant_a"]["gpu_launches"] + r["variant_b"]["gpu_launches"]
                                               + r.get("variant_b_pipelined", {}).get("gpu_launches", 0)
                                               for r in rows)}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_cfg4b(args, world: int, rank: int, local: int) -> None:
    """Config 4 variant B as its own line (see seqsplit_measure)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    r = seqsplit_measure(args.batch, args.ctx, args.layers, args.steps, args.warmup, args.fmt, world, rank, dev,
                         chunks=args.seq_chunks)
    if rank == 0:
        print(json.dumps({
            "metric": "config4 variant B: sequence-split INT4 decode attention, aggregate HBM GB/s and tokens/s",
            "value": r["gbs"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 mma (int4 storage, fp32 accum)", "data": "synthetic",
            "config": {"workload": r["workload"], "kv_format": args.fmt, "layers": args.layers,
                       "parallelism": f"seqsplit{world}"},
            "tokens_per_s": r["tokens_per_s"],
            "pct_of_aggregate_measured_peak": r["pct_of_aggregate_measured_peak"],
            "gpu_launches": r["gpu_launches"]}))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------- GPU arm
def main():
    args = parse_args()
    if args.layers is None:
        args.layers = 28 if args.workload == "cfg2" else CFG1["layers"]
    if args.workload == "cfg2" and args.impl == "ours":
        run_cfg2(args)
        return
    if args.workload == "cfg3" and args.impl == "ours":
        run_cfg3(args)
        return
    if args.workload == "prefill" and args.impl == "ours":
        run_prefill(args)
        return
    if args.workload == "cfg4" and args.impl == "ours":
        run_cfg4(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
                 int(os.environ.get("LOCAL_RANK", "0")))
        return
    if args.workload == "cfg4b" and args.impl == "ours":
        run_cfg4b(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
                  int(os.environ.get("LOCAL_RANK", "0")))
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        cpu = run_cpu_reference(args.steps, args.warmup, lambda b, n: layer_bytes(b, n, args.fmt))
        line = {"metric": METRIC, "value": round(cpu["value"], 4), "unit": "GB/s", "n_gpus": args.gpus,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(cpu["ms_per_layer_step"], 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic", "impl": "reference",
                "config": {"workload": "config1 sample: 1 layer, 2 of 8 sequences, Llama-3.1-8B-shaped decode "
                                       "at 32K ctx (64 sink + 1024 recent fp16, 31680 INT4 g32)",
                           "kv_format": "reference unpacked (u8 code per value, f32 scale, u8 zero)"},
                "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "e2e": {"value": round(cpu["value"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line))
        return

    import torch
    import torch.distributed as dist

    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())

    from hetero_kvcache_optimizer_b200 import _lib, kvstore as kv
    from hetero_kvcache_optimizer_b200.decode_engine import TieredKVDecoder

    c = CFG1
    body = c["ctx"] - c["sink"] - c["recent"]
    total_steps = args.warmup + args.steps + args.e2e_steps + 4
    eng = TieredKVDecoder(args.layers, c["batch"], c["q_heads"], c["kv_heads"], sink=c["sink"],
                          recent=c["recent"], body_capacity=body + total_steps + 8, fmt=args.fmt,
                          group=c["group"], kv_dtype=torch.float16, out_dtype=torch.float32, device=dev,
                          ctas=args.ctas, fused_append=False if args.no_fused else None,
                          early=False if args.no_early else None)
    gen = torch.Generator(device=dev).manual_seed(1 + rank)
    B, Hkv = c["batch"], c["kv_heads"]
    for l in range(args.layers):
        k = torch.randn(B, Hkv, body, 128, device=dev, generator=gen)
        for h in range(Hkv):
            ch = torch.randperm(128, device=dev, generator=gen)[:4]
            k[:, h, :, ch] *= 10.0
        v = torch.randn(B, Hkv, body, 128, device=dev, generator=gen)
        kv.prefill(eng.stores[l], k.half(), v.half())
        del k, v
        d = eng.dense[l]
        d.k.normal_(generator=gen)
        d.v.normal_(generator=gen)
    eng.set_state(body)
    torch.cuda.synchronize()
    _lib.device_error(clear=True)

    eng.capture(max_steps=total_steps)
    q, kn, vn, out = eng.static_buffers
    q.copy_(torch.randn(q.shape, device=dev, generator=gen))
    kn.copy_(torch.randn(kn.shape, device=dev, generator=gen))
    vn.copy_(torch.randn(vn.shape, device=dev, generator=gen))

    for _ in range(args.warmup):
        eng.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    body0 = eng.body_len
    sampler = ClockSampler(dev.index, 50)
    sampler.start()
    time.sleep(0.3)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda.profiler.start()  # lets `ncu --profile-from-start off` list exactly the timed launches
    e0.record(st)
    for _ in range(args.steps):
        eng.replay()
    e1.record(st)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    step_bytes = sum(eng.step_bytes(body0 + i) for i in range(args.steps)) / args.steps
    gbs = world * step_bytes / (ms * 1e-3) / 1e9
    tok_s = world * c["batch"] / (ms * 1e-3)

    # ---- roofline of the dominant kernel: decode (split-KV + merge) per layer, graph of all layers
    g2 = torch.cuda.CUDAGraph()
    s2 = torch.cuda.Stream(device=dev)
    s2.wait_stream(st)
    with torch.cuda.stream(s2):
        eng.decode_only(q, out)
    s2.synchronize()
    with torch.cuda.graph(g2, stream=s2):
        eng.decode_only(q, out)
    st.wait_stream(s2)
    for _ in range(3):
        g2.replay()
    R = 20
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(R):
        g2.replay()
    e1.record(st)
    torch.cuda.synchronize()
    dec_ms = e0.elapsed_time(e1) / (R * args.layers)
    dec_bytes = eng.layer_attn_bytes(eng.body_len)
    peak, peak_kind = measured_peak()
    dec_achieved = dec_bytes / (dec_ms * 1e-3) / 1e9
    if eng.fused_append:
        # the dominant (only) kernel of the timed step is the fused decode-append
        # launch: one per layer, back to back in the step graph, so its average
        # launch duration is the timed step / layers (CUDA events on the stream
        # that replays the graph; gaps between launches count against it)
        kern_us = ms * 1e3 / args.layers
        kern_bytes = step_bytes / args.layers
        kern_name = ("decode_kernel<APPEND> (fused decode-step append + split-KV attention + merge), "
                     "one launch per layer")
        traffic = profiled_traffic(kern_bytes, "decode_append_kernel_cfg1_traffic.json")
    else:
        kern_us, kern_bytes = dec_ms * 1e3, dec_bytes
        kern_name = "decode_kernel (split-KV + fused merge), one launch per layer"
        traffic = profiled_traffic(dec_bytes)
    achieved = kern_bytes / (kern_us * 1e-6) / 1e9

    # ---- e2e through the public API from pinned host buffers: the engine's own
    # pinned buffers, so step_host replays the pipelined graph (layer l's copies
    # overlap the kernels of the layers before / after it)
    eng.capture_host()
    qh, kh, vh, oh = eng.host_buffers
    qh.copy_(torch.randn(q.shape, generator=torch.Generator().manual_seed(3)).to(q.dtype))
    kh.copy_(torch.randn(kn.shape, generator=torch.Generator().manual_seed(4)).to(kn.dtype))
    vh.copy_(torch.randn(vn.shape, generator=torch.Generator().manual_seed(5)).to(vn.dtype))
    for _ in range(2):
        eng.step_host(qh, kh, vh, oh)
    torch.cuda.synchronize()
    body1 = eng.body_len
    e0.record(st)
    for _ in range(args.e2e_steps):
        eng.step_host(qh, kh, vh, oh)
    e1.record(st)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_bytes = sum(eng.step_bytes(body1 + i) for i in range(args.e2e_steps)) / args.e2e_steps
    e2e_gbs = world * e2e_bytes / (e2e_ms * 1e-3) / 1e9
    h2d = (qh.numel() * qh.element_size() + kh.numel() * kh.element_size() + vh.numel() * vh.element_size())
    d2h = oh.numel() * oh.element_size()

    derr = _lib.device_error(clear=True)
    if derr:
        raise RuntimeError(f"device error bits {derr} during the benchmark")

    # ---- the reference-bit-exact INT4 format (fp32 scale + u8 zero-point, 168 B
    # per token) on the same decode step: 4 layers of config 1 (the per-launch
    # figures do not depend on the layer count), one rank, after the main line
    ref_fmt = None
    if world == 1 and args.fmt != "ref":
        ref_fmt = ref_format_measure(args, dev, peak)

    # ---- config 3 in short (4 of its 32 layers, one rank): exposed host->device
    # transfer when every step copies the whole cold set, and when a window of
    # 8 cold pages stays cached in HBM and slides by one page per step
    offload = cfg2 = None
    if world == 1 and not args.no_offload:
        offload = {"layers": 4,
                   "full_cold_set": cfg3_measure(4, 0, None, 4, 3, args.fmt, dev),
                   "sliding_window": cfg3_measure(4, 8, 1, 10, 3, args.fmt, dev)}
        # config 2 in short: 4 of its 28 layers (the per-layer figures do not
        # depend on the layer count beyond the first)
        c2 = cfg2_measure(4, 30, 5, args.fmt, dev)
        cfg2 = {"layers": 4, "ms_per_step": c2["ms_per_step"], "ms_per_layer": round(c2["ms_per_step"] / 4, 4),
                "gbs": c2["value"], "tokens_per_s": c2["tokens_per_s"], "prefill_quantize": c2["prefill_quantize"],
                "workload": c2["config"]["workload"]}

    # ---- N > 1: variant B of config 4 as well (sequence split + one NCCL
    # all-gather of the partials per layer + LSE merge), short: 2 layers at
    # B 64, 131,072-token context, strong scaling over this run's ranks
    split = None
    if world > 1:
        split = seqsplit_measure(64, 131072, 2, 5, 3, args.fmt, world, rank, dev)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = run_cpu_reference(args.cpu_steps, 1, lambda b, n: layer_bytes(b, n, args.fmt))

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16 mma (int4 storage, fp32 accum)", "data": "synthetic",
            "config": {"workload": "config1: Llama-3.1-8B-shaped decode, 32 layers, B8/GPU, Hq32/Hkv8, "
                                   "D128, ctx 32768 = 64 sink + 1024 recent fp16 + 31680 INT4",
                       "kv_format": args.fmt, "group": c["group"], "layers": args.layers,
                       "global_batch": c["batch"] * world, "seq_len": c["ctx"], "parallelism": f"shard{world}",
                       "l2": "no flush: per-step working set ~12 GB >> 126 MB L2",
                       "decode_grid": eng.ctas or "1 CTA per SM"},
            "tokens_per_s": round(tok_s, 1),
            "pct_of_8TBs": round(100 * gbs / (NOMINAL_HBM_GBS * world), 2),
            "pct_of_measured_peak": round(100 * gbs / (peak * world), 2),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "kernel": kern_name,
                         "bytes_per_launch": round(kern_bytes), "us_per_launch": round(kern_us, 2),
                         "peak_kind": f"{peak_kind} (copy)"},
            # the attention alone (decode_kernel without the append, a graph of
            # `layers` launches over the same cache), for comparison
            "attention_only": {"achieved": round(dec_achieved, 1), "frac": round(dec_achieved / peak, 4),
                               "bytes_per_launch": dec_bytes, "us_per_launch": round(dec_ms * 1e3, 2),
                               "traffic": profiled_traffic(dec_bytes)},
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
                    "api": "TieredKVDecoder.step_host (pinned host q/k/v in, fp32 out; per-layer copies "
                           "pipelined with the kernels)"},
            # one fused decode-append launch per layer (two without fusion), all ranks
            "gpu_launches": world * args.steps * args.layers * eng.launches_per_layer,
            "clocks": clocks,
        }
        if split is not None:
            line["seqsplit_cfg4b"] = split
        if ref_fmt is not None:
            line["ref_format"] = ref_fmt
        if offload is not None:
            line["offload_cfg3"] = offload
        if cfg2 is not None:
            line["long_context_cfg2"] = cfg2
        if cpu is not None:
            line["cpu_baseline"] = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in cpu.items()
                                    if k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line))
    del eng, g2
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
