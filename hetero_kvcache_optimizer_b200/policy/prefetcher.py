"""DRAM -> HBM prefetch.

``AsyncPrefetcher`` is the drop-in for the reference's class
(src/policy/prefetcher.py:21-122): same constructor, ``submit_prefetch_task``,
``fetch_if_ready``, ``clear`` and ``pending_keys``, same two dict protocols and
the same BF16 (K, V) result. Differences, all invisible to callers:
  * each task records its own CUDA event and ``fetch_if_ready`` makes only the
    current stream wait on that event (the reference joins the whole side
    stream, :110), and hands the tensors to the consumer stream with
    ``record_stream`` so the caching allocator cannot recycle them early;
  * the dequantisation runs in libhetero_kv's kernel on the side stream.

``PagePrefetcher`` is the page-pool path the decode kernel consumes: whole
INT4 pages (K and V side by side) move from a pinned host arena into device
page slots with one cudaMemcpyAsync per run of consecutive page ids (C ABI
``hkv_prefetch_submit``), on a side stream, gated by events (layer-ahead:
submit layer l+1 while layer l decodes, then make the compute stream wait on
the event right before layer l+1's attention).
"""
from __future__ import annotations

import ctypes
from typing import Any, Dict, Optional, Sequence, Tuple

import numpy as np
import torch

from .. import _lib as L


class AsyncPrefetcher:
    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        if self.device.type == "cuda":
            self.prefetch_stream = torch.cuda.Stream(device=self.device)
        else:
            self.prefetch_stream = None
        self.buffer: Dict[str, Tuple[torch.Tensor, torch.Tensor, Optional[torch.cuda.Event]]] = {}

    def submit_prefetch_task(self, chunk_key: str, dram_data: Dict[str, Any], compressor) -> None:
        if chunk_key in self.buffer:
            return
        has_split_kv = "k_data" in dram_data and "v_data" in dram_data
        has_merged = "q_data" in dram_data
        if not has_split_kv and not has_merged:
            return
        if self.prefetch_stream is None:
            raise RuntimeError("AsyncPrefetcher needs a CUDA device (no CPU path)")
        ctx = torch.cuda.stream(self.prefetch_stream)
        with ctx:
            if has_split_kv:
                q_k = dram_data["k_data"].to(self.device, non_blocking=True)
                s_k = dram_data["k_scales"].to(self.device, non_blocking=True)
                z_k = dram_data["k_zps"].to(self.device, non_blocking=True)
                q_v = dram_data["v_data"].to(self.device, non_blocking=True)
                s_v = dram_data["v_scales"].to(self.device, non_blocking=True)
                z_v = dram_data["v_zps"].to(self.device, non_blocking=True)
                # as prefetcher.py:82-83: decompress (fp16 default) then cast to bf16
                restored_k = compressor.decompress(q_k, s_k, z_k).to(torch.bfloat16)
                restored_v = compressor.decompress(q_v, s_v, z_v).to(torch.bfloat16)
            else:
                q_d = dram_data["q_data"].to(self.device, non_blocking=True)
                s_d = dram_data["scales"].to(self.device, non_blocking=True)
                z_d = dram_data["zps"].to(self.device, non_blocking=True)
                restored_k = compressor.decompress(q_d, s_d, z_d).to(torch.bfloat16)
                restored_v = restored_k
            ev = torch.cuda.Event()
            ev.record(self.prefetch_stream)
        self.buffer[chunk_key] = (restored_k, restored_v, ev)

    def fetch_if_ready(self, chunk_key: str) -> Optional[Tuple[torch.Tensor, torch.Tensor]]:
        if chunk_key not in self.buffer:
            return None
        k, v, ev = self.buffer.pop(chunk_key)
        if ev is not None:
            cur = torch.cuda.current_stream(self.device)
            cur.wait_event(ev)
            k.record_stream(cur)
            if v is not k:
                v.record_stream(cur)
        return k, v

    def clear(self) -> None:
        self.buffer.clear()

    @property
    def pending_keys(self):
        return list(self.buffer.keys())


class PagePrefetcher:
    """Copies whole pages host arena -> device pool on a side stream.

    host_pool: pinned uint8 [host_pages, page_bytes]; dev_pool: uint8
    [dev_pages, page_bytes] on the device. Both stay owned by the caller.
    """

    def __init__(self, host_pool: torch.Tensor, dev_pool: torch.Tensor,
                 stream: Optional[torch.cuda.Stream] = None):
        if not host_pool.is_pinned():
            raise ValueError("host_pool must be pinned (page-locked) memory")
        if host_pool.shape[1] != dev_pool.shape[1] or not dev_pool.is_cuda:
            raise ValueError("host and device pools must have the same page size; device pool on CUDA")
        self.host_pool, self.dev_pool = host_pool, dev_pool
        self.page_bytes = int(host_pool.shape[1])
        self.stream = stream or torch.cuda.Stream(device=dev_pool.device)
        h = ctypes.c_void_p(0)
        L.check(L.load().hkv_prefetcher_create(host_pool.data_ptr(), host_pool.shape[0], dev_pool.data_ptr(),
                                               dev_pool.shape[0], self.page_bytes, ctypes.byref(h)),
                "hkv_prefetcher_create")
        self._h = h

    def submit(self, src_pages: Sequence[int], dst_slots: Sequence[int],
               event: Optional[torch.cuda.Event] = None,
               stream: Optional[torch.cuda.Stream] = None) -> torch.cuda.Event:
        """Issue the copies on ``stream`` (default: the side stream); returns an
        event recorded after them."""
        s = stream or self.stream
        src = np.ascontiguousarray(np.asarray(src_pages, dtype=np.int32))
        dst = np.ascontiguousarray(np.asarray(dst_slots, dtype=np.int32))
        if src.shape != dst.shape:
            raise ValueError("src_pages and dst_slots differ in length")
        L.check(L.load().hkv_prefetch_submit(self._h, src.ctypes.data, dst.ctypes.data, int(src.size),
                                             ctypes.c_void_p(s.cuda_stream), None),
                "hkv_prefetch_submit")
        ev = event or torch.cuda.Event()
        ev.record(s)
        return ev

    def gather(self, src_pages: torch.Tensor, dst_slots: torch.Tensor, step: Optional[torch.Tensor] = None,
               step_mul: int = 0, step_add: int = 0, ctas: int = 0, stream=None) -> None:
        """One zero-copy gather kernel (``hkv_prefetch_gather``) on ``stream``
        (default: the side stream): host page (src_pages[k] + (step + step_add) *
        step_mul) mod host_pages (just src_pages[k] without ``step``) -> device
        slot dst_slots[k]. The id tensors (int32) and the step counter (int64,
        one element) live on the device, so the call can be captured in a CUDA
        graph and the page set chosen by device code. Records no event."""
        if src_pages.dtype != torch.int32 or dst_slots.dtype != torch.int32:
            raise TypeError("page ids must be int32")
        if not (src_pages.is_cuda and dst_slots.is_cuda) or src_pages.numel() != dst_slots.numel():
            raise ValueError("src_pages / dst_slots: device tensors of one length")
        if step is not None and (step.dtype != torch.int64 or not step.is_cuda):
            raise TypeError("step must be a device int64 tensor")
        s = stream or self.stream
        L.check(L.load().hkv_prefetch_gather(
            self._h, src_pages.data_ptr(), dst_slots.data_ptr(), int(src_pages.numel()),
            step.data_ptr() if step is not None else None, int(step_mul), int(step_add), int(ctas),
            ctypes.c_void_p(s.cuda_stream)), "hkv_prefetch_gather")

    @staticmethod
    def gate(event: torch.cuda.Event, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Make ``stream`` (default: current) wait for the pages of ``event`` on the device."""
        (stream or torch.cuda.current_stream()).wait_event(event)

    @staticmethod
    def host_wait(event: torch.cuda.Event, timeout_us: int = 5_000_000) -> None:
        """Bounded host wait for an event (raises on timeout)."""
        L.check(L.load().hkv_event_wait(ctypes.c_void_p(event.cuda_event), int(timeout_us)), "hkv_event_wait")

    @property
    def bytes_submitted(self) -> int:
        return int(L.load().hkv_prefetch_bytes(self._h))

    def close(self) -> None:
        if self._h:
            L.load().hkv_prefetcher_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

