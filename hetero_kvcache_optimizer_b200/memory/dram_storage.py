"""Tier-2 DRAM storage in page-locked host memory.

``DRAMStorageManager`` is the drop-in for src/memory/dram_storage.py:20-255
(same methods, keys, byte accounting and capacity caps). The reference pins
every evicted tensor with ``.cpu().pin_memory()`` (:93-100), a synchronous
copy plus a page-lock per tensor. Here entries are carved out of large pinned
arenas allocated once; the device->host copy is asynchronous on a dedicated
stream and an event per entry makes ``retrieve`` / ``transfer_to_device``
wait (bounded) only for that entry.

``PinnedPageArena`` is the fixed-size page pool the page prefetcher reads:
[num_pages, page_bytes] pinned, with a free list of page ids.
"""
from __future__ import annotations

from typing import Any, Dict, List, Optional

import torch

from .. import _lib as L

_KEYS = ("k_data", "k_scales", "k_zps", "v_data", "v_scales", "v_zps")
_ARENA_BYTES = 256 << 20


class _PinnedArena:
    """Bump allocator over pinned chunks with a size-keyed free list (256-B aligned)."""

    def __init__(self, chunk_bytes: int = _ARENA_BYTES):
        self.chunk_bytes = chunk_bytes
        self.chunks: List[torch.Tensor] = []
        self.top = 0
        self.free: Dict[int, List[torch.Tensor]] = {}

    def alloc(self, nbytes: int) -> torch.Tensor:
        nb = max(256, (nbytes + 255) // 256 * 256)
        lst = self.free.get(nb)
        if lst:
            return lst.pop()
        if not self.chunks or self.top + nb > self.chunks[-1].numel():
            self.chunks.append(torch.empty(max(self.chunk_bytes, nb), dtype=torch.uint8).pin_memory())
            self.top = 0
        buf = self.chunks[-1][self.top:self.top + nb]
        self.top += nb
        return buf

    def release(self, buf: torch.Tensor) -> None:
        self.free.setdefault(buf.numel(), []).append(buf)


class DRAMStorageManager:
    def __init__(self, max_entries: Optional[int] = None, max_bytes: Optional[int] = None):
        self.max_entries = max_entries
        self.max_bytes = max_bytes
        self._table: Dict[str, Dict[str, torch.Tensor]] = {}
        self._raw: Dict[str, List[torch.Tensor]] = {}
        self._events: Dict[str, torch.cuda.Event] = {}
        self._total_bytes = 0
        self._arena = _PinnedArena()
        self._stream: Optional[torch.cuda.Stream] = None
        print(f"[DRAM] Storage Manager initialized | max_entries={max_entries or 'inf'} "
              f"max_bytes={max_bytes or 'inf'}")

    # ------------------------------------------------------------------ CRUD
    def store(self, chunk_key: str, q_k, k_scales, k_zps, q_v, v_scales, v_zps) -> bool:
        entry = {"k_data": q_k, "k_scales": k_scales, "k_zps": k_zps,
                 "v_data": q_v, "v_scales": v_scales, "v_zps": v_zps}
        if self.max_entries is not None and len(self._table) >= self.max_entries:
            print(f"[DRAM] Capacity exceeded: {len(self._table)}/{self.max_entries} entries")
            return False
        nbytes = sum(t.element_size() * t.nelement() for t in entry.values())
        if self.max_bytes is not None and self._total_bytes + nbytes > self.max_bytes:
            print(f"[DRAM] Memory cap exceeded: {self._total_bytes + nbytes}/{self.max_bytes} bytes")
            return False
        self._put(chunk_key, entry, nbytes)
        return True

    def store_entry(self, chunk_key: str, entry: Dict[str, torch.Tensor]) -> bool:
        if not all(k in entry for k in _KEYS):
            raise ValueError(f"Entry missing required keys. Need: {_KEYS}")
        nbytes = sum(entry[k].element_size() * entry[k].nelement() for k in _KEYS)
        if self.max_entries is not None and len(self._table) >= self.max_entries:
            return False
        if self.max_bytes is not None and self._total_bytes + nbytes > self.max_bytes:
            return False
        self._put(chunk_key, {k: entry[k] for k in _KEYS}, nbytes)
        return True

    def _put(self, chunk_key: str, entry: Dict[str, torch.Tensor], nbytes: int) -> None:
        # page-locked space for every tensor first: if an allocation fails the
        # exception leaves the table (and an entry being replaced) untouched
        raw_of: Dict[str, torch.Tensor] = {}
        try:
            for k, t in entry.items():
                if not (t.device.type == "cpu" and t.is_pinned()):
                    raw_of[k] = self._arena.alloc(t.element_size() * t.nelement())
        except BaseException:
            for r in raw_of.values():
                self._arena.release(r)
            raise
        if chunk_key in self._table:
            self._drop(chunk_key)
        pinned: Dict[str, torch.Tensor] = {}
        raws: List[torch.Tensor] = list(raw_of.values())
        ev = None
        on_gpu = any(t.is_cuda for t in entry.values())
        if on_gpu and self._stream is None:
            dev = next(t.device for t in entry.values() if t.is_cuda)
            self._stream = torch.cuda.Stream(device=dev)
        for k, t in entry.items():
            if k not in raw_of:
                pinned[k] = t
                continue
            raw = raw_of[k]
            dst = raw[: t.element_size() * t.nelement()].view(t.dtype).view(t.shape)
            if t.is_cuda:
                self._stream.wait_stream(torch.cuda.current_stream(t.device))
                with torch.cuda.stream(self._stream):
                    dst.copy_(t, non_blocking=True)
                    t.record_stream(self._stream)
            else:
                dst.copy_(t)
            pinned[k] = dst
        if on_gpu:
            ev = torch.cuda.Event()
            ev.record(self._stream)
            self._events[chunk_key] = ev
        self._table[chunk_key] = pinned
        self._raw[chunk_key] = raws
        self._total_bytes += nbytes

    def _ready(self, chunk_key: str) -> None:
        ev = self._events.pop(chunk_key, None)
        if ev is not None:
            L.check(L.load().hkv_event_wait(ev.cuda_event, 10_000_000), "DRAM entry copy")

    def retrieve(self, chunk_key: str) -> Optional[Dict[str, torch.Tensor]]:
        if chunk_key not in self._table:
            return None
        self._ready(chunk_key)
        return self._table[chunk_key]

    def remove(self, chunk_key: str) -> Optional[Dict[str, torch.Tensor]]:
        if chunk_key not in self._table:
            return None
        self._ready(chunk_key)
        entry = self._table[chunk_key]
        self._drop(chunk_key, keep_raw=True)
        return entry

    def _drop(self, chunk_key: str, keep_raw: bool = False) -> None:
        entry = self._table.pop(chunk_key)
        self._events.pop(chunk_key, None)
        self._total_bytes -= sum(t.element_size() * t.nelement() for t in entry.values())
        raws = self._raw.pop(chunk_key, [])
        if not keep_raw:
            for r in raws:
                self._arena.release(r)

    def contains(self, chunk_key: str) -> bool:
        return chunk_key in self._table

    def __contains__(self, chunk_key: str) -> bool:
        return chunk_key in self._table

    # ------------------------------------------------------------------ transfer
    def transfer_to_device(self, chunk_key: str, device: torch.device,
                           non_blocking: bool = True) -> Optional[Dict[str, torch.Tensor]]:
        entry = self.retrieve(chunk_key)
        if entry is None:
            return None
        return {k: entry[k].to(device, non_blocking=non_blocking) for k in _KEYS}

    # ------------------------------------------------------------------ stats
    @property
    def table(self) -> Dict[str, Dict[str, torch.Tensor]]:
        for k in list(self._events):
            self._ready(k)
        return self._table

    @property
    def total_bytes(self) -> int:
        return self._total_bytes

    @property
    def num_entries(self) -> int:
        return len(self._table)

    @property
    def keys(self) -> List[str]:
        return list(self._table.keys())

    def memory_summary(self) -> Dict[str, Any]:
        return {"num_entries": len(self._table), "total_bytes": self._total_bytes,
                "total_mb": self._total_bytes / (1024 * 1024)}


class PinnedPageArena:
    """[num_pages, page_bytes] pinned host pages with a free list of page ids."""

    def __init__(self, num_pages: int, page_bytes: int):
        self.pages = torch.empty(num_pages, page_bytes, dtype=torch.uint8).pin_memory()
        self.page_bytes = page_bytes
        self._free = list(range(num_pages - 1, -1, -1))

    def alloc(self, n: int) -> List[int]:
        if n > len(self._free):
            raise MemoryError(f"page arena full: {n} requested, {len(self._free)} free")
        return [self._free.pop() for _ in range(n)]

    def release(self, ids) -> None:
        self._free.extend(int(i) for i in ids)

    @property
    def free_pages(self) -> int:
        return len(self._free)
