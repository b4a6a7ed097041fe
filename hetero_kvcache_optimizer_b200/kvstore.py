"""PyTorch-facing wrappers over libhetero_kv: the packed INT4 page pool, the
dense (sink + recent) segment, and the hot-path operations.

Torch is plumbing here: it owns device memory and streams. Every computation
runs in the CUDA kernels of libhetero_kv.so through its C ABI; tensors are
passed as raw pointers plus sizes.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Tuple, Union

import torch

from . import _lib as L

_DT = {torch.float16: L.DT_F16, torch.bfloat16: L.DT_BF16, torch.float32: L.DT_F32}
FORMATS = {"ref": L.FMT_REF, "fp16min": L.FMT_FP16MIN}
HEAD_DIM = 128


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def _stream(stream: Optional[torch.cuda.Stream] = None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError(
                "hetero_kv kernels need CUDA tensors (HKV_ERR_UNSUPPORTED for CPU tensors: "
                "there is no CPU fallback)")


def page_bytes(fmt: str, group: int, page_tokens: int) -> int:
    n = L.load().hkv_page_bytes(FORMATS[fmt], group, page_tokens)
    if n <= 0:
        raise ValueError(f"bad store geometry fmt={fmt} group={group} page_tokens={page_tokens}")
    return int(n)


class Int4KVStore:
    """Packed INT4 body of a KV cache for B sequences x H KV heads.

    Memory: one pool of pages; a page is page_tokens/128 contiguous blocks of
    128 tokens, each holding K and V codes and metadata together (21,504 B per
    block for the reference format at group 32; 20,480 B for fp16min), so that
    one copy moves a decode tile and one host->device copy moves a whole page.

    Dense mode (``num_pages=None``): unit u = b*H + h owns pages
    [u*max_pages, (u+1)*max_pages) and no page table is used. Paged mode: the
    caller provides ``num_pages`` and fills ``page_table`` [B*H, max_pages].
    ``lengths`` [B] int32 on the device holds the tokens per sequence.
    """

    def __init__(self, batch: int, kv_heads: int, capacity: int, *, fmt: str = "ref",
                 group: int = 32, page_tokens: int = 256, num_pages: Optional[int] = None,
                 device: Union[str, torch.device] = "cuda"):
        if fmt not in FORMATS:
            raise ValueError(f"fmt must be one of {list(FORMATS)}")
        if page_tokens % 128:
            raise ValueError("page_tokens must be a multiple of 128")
        self.batch, self.kv_heads, self.fmt, self.group = batch, kv_heads, fmt, group
        self.page_tokens = page_tokens
        self.max_pages = max(1, math.ceil(capacity / page_tokens))
        self.capacity = self.max_pages * page_tokens
        self.page_bytes = page_bytes(fmt, group, page_tokens)
        units = batch * kv_heads
        self.paged = num_pages is not None
        self.num_pages = num_pages if self.paged else units * self.max_pages
        self.device = torch.device(device)
        self.pool = torch.empty(self.num_pages, self.page_bytes, dtype=torch.uint8, device=self.device)
        self.page_table = (torch.full((units, self.max_pages), -1, dtype=torch.int32, device=self.device)
                           if self.paged else None)
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=self.device)
        self.len_hint = 0  # host-side upper bound of lengths (sizes the split-KV grid)

    def struct(self, len_hint: Optional[int] = None, b0: int = 0) -> L.HkvInt4Store:
        """The C view of this store; ``b0`` > 0 views sequences [b0, batch)
        only (a launch over a batch slice starting at sequence b0)."""
        if not 0 <= b0 < self.batch:
            raise ValueError(f"b0={b0} outside the batch of {self.batch}")
        skip = b0 * self.kv_heads * self.max_pages  # page slots of the skipped units
        s = L.HkvInt4Store()
        s.format = FORMATS[self.fmt]
        s.group = self.group
        s.page_tokens = self.page_tokens
        s.max_pages = self.max_pages
        if self.paged:
            s.pages = self.pool.data_ptr()
            s.page_table = self.page_table.data_ptr() + skip * 4
            s.num_pages = self.num_pages
        else:
            s.pages = self.pool.data_ptr() + skip * self.page_bytes
            s.page_table = None
            s.num_pages = self.num_pages - skip
        s.page_stride = self.page_bytes
        s.lengths = self.lengths.data_ptr() + b0 * 4
        s.len = int(self.len_hint if len_hint is None else len_hint)
        return s

    def set_lengths(self, n: Union[int, torch.Tensor]) -> None:
        if isinstance(n, int):
            self.lengths.fill_(n)
            self.len_hint = n
        else:
            self.lengths.copy_(n.to(torch.int32))
            self.len_hint = int(n.max().item())


class DenseKV:
    """Dense fp16/bf16 K/V segment [B, H, capacity, 128] (e.g. sink + recent ring)."""

    def __init__(self, batch: int, kv_heads: int, capacity: int, dtype=torch.float16,
                 device: Union[str, torch.device] = "cuda", k: Optional[torch.Tensor] = None,
                 v: Optional[torch.Tensor] = None):
        self.batch, self.kv_heads, self.capacity, self.dtype = batch, kv_heads, capacity, dtype
        shape = (batch, kv_heads, capacity, HEAD_DIM)
        self.k = k if k is not None else torch.zeros(shape, dtype=dtype, device=device)
        self.v = v if v is not None else torch.zeros(shape, dtype=dtype, device=device)
        assert self.k.shape == shape and self.v.shape == shape and self.k.stride() == self.v.stride()
        assert self.k.stride(-1) == 1
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=self.k.device)
        self.ring_head = torch.zeros(batch, dtype=torch.int32, device=self.k.device)
        self.len_hint = 0

    def struct(self, len_hint: Optional[int] = None, b0: int = 0) -> L.HkvDenseKV:
        """The C view of this segment; ``b0`` > 0 views sequences [b0, batch)."""
        if not 0 <= b0 < self.batch:
            raise ValueError(f"b0={b0} outside the batch of {self.batch}")
        es = self.k.element_size()
        d = L.HkvDenseKV()
        d.k = self.k.data_ptr() + b0 * self.k.stride(0) * es
        d.v = self.v.data_ptr() + b0 * self.v.stride(0) * es
        d.dtype = dtype_code(self.dtype)
        d.capacity = self.capacity
        d.stride_b, d.stride_h, d.stride_t = self.k.stride(0), self.k.stride(1), self.k.stride(2)
        d.lengths = self.lengths.data_ptr() + b0 * 4
        d.len = int(self.len_hint if len_hint is None else len_hint)
        return d

    def set_lengths(self, n: int) -> None:
        self.lengths.fill_(n)
        self.len_hint = n


# ----------------------------------------------------------------------------- workspace
_ws_cache: dict = {}


def workspace(nbytes: int, device: torch.device, stream=None, kind: str = "decode") -> torch.Tensor:
    """A per-(device, stream, kind) scratch buffer for split partials, grown on
    demand. Zeroed at allocation: a decode workspace holds the per-unit merge
    counters, which the decode kernel leaves at zero after every call, so the
    prefill's partials (kind "prefill") live in a buffer of their own."""
    key = (device.index, (stream or torch.cuda.current_stream(device)).cuda_stream, kind)
    buf = _ws_cache.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws_cache[key] = buf
    return buf


def reset_workspaces() -> None:
    """Zero every cached workspace. A decode kernel whose bounded wait expired
    stops early and leaves some merge counters non-zero, which would make the
    next call on that workspace merge too soon; ``_lib.device_error`` runs this
    whenever it reports a timeout. Synchronises the device."""
    for buf in _ws_cache.values():
        buf.zero_()
    if _ws_cache:
        torch.cuda.synchronize()


L.on_device_timeout(reset_workspaces)


# ----------------------------------------------------------------------------- operations
def quantize_pack(x: torch.Tensor, store: Int4KVStore, role: int,
                  start: Union[int, torch.Tensor] = 0, stream=None) -> None:
    """Quantise x [B, H, T, 128] into side ``role`` of ``store`` at body slots
    start + t (start: int, or [B] int32 device tensor). Does not touch lengths."""
    _require_cuda(x)
    B, H, T, D = x.shape
    if x.stride(-1) != 1:
        x = x.contiguous()
    st = store.struct()
    dst_start = start.data_ptr() if isinstance(start, torch.Tensor) else None
    s0 = 0 if isinstance(start, torch.Tensor) else int(start)
    L.check(L.load().hkv_quantize_pack(
        x.data_ptr(), dtype_code(x.dtype), B, H, T, D, x.stride(0), x.stride(1), x.stride(2), role,
        ctypes.byref(st), dst_start, s0, _stream(stream)), "hkv_quantize_pack")


def quantize_pack_kv(k: torch.Tensor, v: torch.Tensor, store: Int4KVStore,
                     start: Union[int, torch.Tensor] = 0, stream=None) -> None:
    """quantize_pack of a K chunk and its V chunk in one launch (both [B, H, T,
    128] of one dtype; laid out alike, else two launches). Does not touch lengths."""
    _require_cuda(k, v)
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    if k.shape != v.shape or k.dtype != v.dtype or k.stride() != v.stride():
        quantize_pack(k, store, L.ROLE_K, start, stream)
        quantize_pack(v, store, L.ROLE_V, start, stream)
        return
    B, H, T, D = k.shape
    st = store.struct()
    dst_start = start.data_ptr() if isinstance(start, torch.Tensor) else None
    s0 = 0 if isinstance(start, torch.Tensor) else int(start)
    L.check(L.load().hkv_quantize_pack_kv(
        k.data_ptr(), v.data_ptr(), dtype_code(k.dtype), B, H, T, D, k.stride(0), k.stride(1), k.stride(2),
        ctypes.byref(st), dst_start, s0, _stream(stream)), "hkv_quantize_pack_kv")


def prefill(store: Int4KVStore, k: torch.Tensor, v: torch.Tensor, start: int = 0, stream=None) -> None:
    """Quantise a [B, H, T, 128] K/V chunk into body slots [start, start+T) and
    set the (uniform) lengths to start + T."""
    quantize_pack_kv(k, v, store, start, stream)
    store.set_lengths(start + k.shape[2])


def append_kv(k_new: torch.Tensor, v_new: torch.Tensor, dense: DenseKV, sink: int,
              store: Int4KVStore, stream=None) -> None:
    """One decode step of the cache: the new token enters the recent ring of
    ``dense``; when the ring is full its oldest row is quantised into ``store``.
    All state lives on the device (dense.lengths, dense.ring_head, store.lengths)."""
    _require_cuda(k_new, v_new)
    if k_new.dim() == 4:
        k_new, v_new = k_new[:, :, 0], v_new[:, :, 0]
    B, H, D = k_new.shape
    ds, st = dense.struct(), store.struct()
    L.check(L.load().hkv_append_kv(
        k_new.data_ptr(), v_new.data_ptr(), dtype_code(k_new.dtype), B, H, D, k_new.stride(0),
        k_new.stride(1), ctypes.byref(ds), sink, dense.lengths.data_ptr(),
        dense.ring_head.data_ptr(), ctypes.byref(st), store.lengths.data_ptr(), _stream(stream)),
        "hkv_append_kv")


def decode(q: torch.Tensor, store: Optional[Int4KVStore], dense: Optional[DenseKV],
           sm_scale: Optional[float] = None, out_dtype: torch.dtype = torch.float32,
           ctas: int = 0, out: Optional[torch.Tensor] = None,
           body_len: Optional[int] = None, dense_len: Optional[int] = None,
           stream=None) -> torch.Tensor:
    """Decode attention of q [B, Hq, 128] (or [B, Hq, 1, 128]) over the INT4
    body and/or the dense segment. Returns [B, Hq, 128] in ``out_dtype``.
    ``ctas`` sets the persistent grid (0: one CTA per SM); ``body_len`` /
    ``dense_len`` override the host-side length hints that size the schedule.
    More than 8 query heads per KV head (the kernel's limit) run as several
    launches over groups of at most 8 of them, each reading the cache again."""
    _require_cuda(q)
    squeeze = q.dim() == 4
    if squeeze:
        q = q[:, :, 0]
    B, Hq, D = q.shape
    Hkv = (store or dense).kv_heads
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, D, dtype=out_dtype, device=q.device)
    G = Hq // Hkv if Hkv else 0
    if G > 8 and Hq % Hkv == 0:
        # heads [k*gs, (k+1)*gs) of every KV head's group, as a [B, Hkv*gs, D] copy
        gs = max(d for d in range(1, 9) if G % d == 0)
        with torch.cuda.stream(stream if stream is not None else torch.cuda.current_stream()):
            qg = q.reshape(B, Hkv, G // gs, gs, D)
            og = torch.empty(B, Hkv, G // gs, gs, D, dtype=out.dtype, device=q.device)
            for k in range(G // gs):
                part = decode(qg[:, :, k].reshape(B, Hkv * gs, D), store, dense, sm_scale, out.dtype, ctas,
                              None, body_len, dense_len)
                og[:, :, k] = part.view(B, Hkv, gs, D)
            out.copy_(og.view(B, Hq, D))
        return out[:, :, None, :] if squeeze else out
    st = store.struct(body_len) if store is not None else None
    ds = dense.struct(dense_len) if dense is not None else None
    pst = ctypes.byref(st) if st is not None else None
    pds = ctypes.byref(ds) if ds is not None else None
    lib = L.load()
    nbytes = lib.hkv_decode_workspace_bytes(pst, pds, B, Hq, Hkv, D, ctas)
    if nbytes == 0:
        raise RuntimeError("hkv_decode_workspace_bytes: unsupported decode configuration")
    ws = workspace(nbytes, q.device, stream)
    L.check(lib.hkv_decode_attn(
        q.data_ptr(), dtype_code(q.dtype), q.stride(0), q.stride(1), pst, pds,
        B, Hq, Hkv, D, float(sm_scale), ctas, ws.data_ptr(), ws.numel(), out.data_ptr(),
        dtype_code(out.dtype), out.stride(0), out.stride(1), _stream(stream)), "hkv_decode_attn")
    return out[:, :, None, :] if squeeze else out


def decode_append(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, dense: DenseKV, sink: int,
                  store: Int4KVStore, sm_scale: Optional[float] = None, out_dtype: torch.dtype = torch.float32,
                  ctas: int = 0, out: Optional[torch.Tensor] = None, body_len: Optional[int] = None,
                  dense_len: Optional[int] = None, early: bool = False, stream=None) -> torch.Tensor:
    """One decode step in one launch: ``append_kv(k_new, v_new, dense, sink,
    store)`` then ``decode(q, store, dense)``, with the same cache contents and
    state afterwards and the attention over the cache after the append.
    ``body_len`` / ``dense_len``: host-side length hints sizing the schedule
    (upper bounds of the lengths after the step). ``early``: the kernel launched
    just before this one on the stream does not write this cache (e.g. another
    layer's step), so the launch may stream the cache while it finishes."""
    _require_cuda(q, k_new, v_new)
    if q.dim() == 4:
        q = q[:, :, 0]
    if k_new.dim() == 4:
        k_new, v_new = k_new[:, :, 0], v_new[:, :, 0]
    if k_new.dtype != dense.dtype or v_new.dtype != dense.dtype:
        raise TypeError("k_new / v_new must have the dense segment's dtype")
    if k_new.stride(-1) != 1 or k_new.stride() != v_new.stride():
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    B, Hq, D = q.shape
    Hkv = store.kv_heads
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, D, dtype=out_dtype, device=q.device)
    st = store.struct(body_len)
    ds = dense.struct(dense_len)
    lib = L.load()
    nbytes = lib.hkv_decode_workspace_bytes(ctypes.byref(st), ctypes.byref(ds), B, Hq, Hkv, D, ctas)
    if nbytes == 0:
        raise RuntimeError("hkv_decode_workspace_bytes: unsupported decode configuration")
    ws = workspace(nbytes, q.device, stream)
    L.check(lib.hkv_decode_append(
        q.data_ptr(), dtype_code(q.dtype), q.stride(0), q.stride(1), k_new.data_ptr(), v_new.data_ptr(),
        k_new.stride(0), k_new.stride(1), ctypes.byref(st), ctypes.byref(ds), sink, dense.lengths.data_ptr(),
        dense.ring_head.data_ptr(), store.lengths.data_ptr(), B, Hq, Hkv, D, float(sm_scale), ctas,
        ws.data_ptr(), ws.numel(), out.data_ptr(), dtype_code(out.dtype), out.stride(0), out.stride(1),
        L.APPEND_EARLY if early else 0, _stream(stream)), "hkv_decode_append")
    return out


def decode_scored(q: torch.Tensor, store: Int4KVStore, dense: Optional[DenseKV],
                  sm_scale: Optional[float] = None, out_dtype: torch.dtype = torch.float32,
                  ctas: int = 0, out: Optional[torch.Tensor] = None,
                  body_len: Optional[int] = None, dense_len: Optional[int] = None,
                  stat_tiles: Optional[int] = None, stream=None):
    """``decode`` plus where the attention fell: returns (out, mass) with mass
    [B, Hkv, stat_tiles] f32 the mean over each KV head's query heads of the
    softmax probability on every 128-token INT4 body tile (0 past the body
    length). Stays on the device (no host sync). ``stat_tiles`` defaults to the
    store's capacity in tiles."""
    _require_cuda(q)
    squeeze = q.dim() == 4
    if squeeze:
        q = q[:, :, 0]
    B, Hq, D = q.shape
    Hkv = store.kv_heads
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, D, dtype=out_dtype, device=q.device)
    if stat_tiles is None:
        stat_tiles = store.max_pages * store.page_tokens // 128
    st = store.struct(body_len)
    ds = dense.struct(dense_len) if dense is not None else None
    pds = ctypes.byref(ds) if ds is not None else None
    lib = L.load()
    nbytes = lib.hkv_decode_workspace_bytes(ctypes.byref(st), pds, B, Hq, Hkv, D, ctas)
    if nbytes == 0:
        raise RuntimeError("hkv_decode_workspace_bytes: unsupported decode configuration")
    ws = workspace(nbytes, q.device, stream)
    stats = torch.empty(B * Hkv * stat_tiles * 4 * 8 * 2, dtype=torch.float32, device=q.device)
    unit_ml = torch.empty(B * Hkv * 8 * 2, dtype=torch.float32, device=q.device)
    mass = torch.empty(B, Hkv, stat_tiles, dtype=torch.float32, device=q.device)
    L.check(lib.hkv_decode_attn_scored(
        q.data_ptr(), dtype_code(q.dtype), q.stride(0), q.stride(1), ctypes.byref(st), pds,
        B, Hq, Hkv, D, float(sm_scale), ctas, ws.data_ptr(), ws.numel(), out.data_ptr(),
        dtype_code(out.dtype), out.stride(0), out.stride(1), stats.data_ptr(), stat_tiles,
        unit_ml.data_ptr(), _stream(stream)), "hkv_decode_attn_scored")
    L.check(lib.hkv_tile_scores(stats.data_ptr(), unit_ml.data_ptr(), ctypes.byref(st), B, Hkv, Hq // Hkv,
                                stat_tiles, mass.data_ptr(), _stream(stream)), "hkv_tile_scores")
    return (out[:, :, None, :] if squeeze else out), mass


def prefill_attn(q: torch.Tensor, store: Int4KVStore, sm_scale: Optional[float] = None,
                 out_dtype: torch.dtype = torch.float32, out: Optional[torch.Tensor] = None,
                 body_len: Optional[int] = None, causal: bool = False, lse: Optional[torch.Tensor] = None,
                 splits: int = 0, stream=None) -> torch.Tensor:
    """Multi-query attention of q [B, Hq, Sq, 128] over the INT4 body of each
    sequence on the tcgen05 tensor cores. Returns [B, Hq, Sq, 128].

    causal: the queries are the last Sq positions of the body, so query s sees
    tokens t <= len - Sq + s. lse: optional contiguous f32 [B, Hq, Sq] that
    receives ln sum_t exp(sm_scale q.k_t) per row (-inf for a row that sees no
    token), for merging with attention over other segments. splits: CTAs per
    query tile sharing its body (0: chosen to fill the SMs; partials merged by
    a second launch)."""
    _require_cuda(q)
    B, Hq, Sq, D = q.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, Sq, D, dtype=out_dtype, device=q.device)
    if out.stride(3) != 1 or q.stride(3) != 1:
        raise ValueError("q and out need a contiguous head dimension")
    lse_ptr = None
    if lse is not None:
        if lse.dtype != torch.float32 or tuple(lse.shape) != (B, Hq, Sq) or not lse.is_contiguous():
            raise ValueError("lse must be a contiguous float32 [B, Hq, Sq] tensor")
        lse_ptr = lse.data_ptr()
    st = store.struct(body_len)
    lib = L.load()
    nbytes = lib.hkv_prefill_workspace_bytes(ctypes.byref(st), B, Hq, store.kv_heads, Sq, D, int(splits)) \
        if Sq > 0 else 0
    ws = workspace(nbytes, q.device, stream, kind="prefill") if nbytes else None
    L.check(lib.hkv_prefill_attn(
        q.data_ptr(), dtype_code(q.dtype), q.stride(0), q.stride(1), q.stride(2), ctypes.byref(st), B, Hq,
        store.kv_heads, Sq, D, float(sm_scale), int(bool(causal)), out.data_ptr(), dtype_code(out.dtype),
        out.stride(0), out.stride(1), out.stride(2), lse_ptr, int(splits),
        ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0, _stream(stream)),
        "hkv_prefill_attn")
    return out


def decode_static(q: torch.Tensor, store: Optional[Int4KVStore], dense: Optional[DenseKV],
                  sm_scale: Optional[float] = None, out_dtype: torch.dtype = torch.float32,
                  ctas: int = 0, out: Optional[torch.Tensor] = None,
                  body_len: Optional[int] = None, dense_len: Optional[int] = None,
                  stream=None) -> torch.Tensor:
    """``decode`` through hkv_decode_attn_static: no workspace is allocated, the
    library's per-device scratch array serves the merge (so calls on one device
    must not overlap). Pass ``out`` to keep the call free of allocations."""
    _require_cuda(q)
    squeeze = q.dim() == 4
    if squeeze:
        q = q[:, :, 0]
    B, Hq, D = q.shape
    Hkv = (store or dense).kv_heads
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty(B, Hq, D, dtype=out_dtype, device=q.device)
    st = store.struct(body_len) if store is not None else None
    ds = dense.struct(dense_len) if dense is not None else None
    L.check(L.load().hkv_decode_attn_static(
        q.data_ptr(), dtype_code(q.dtype), q.stride(0), q.stride(1),
        ctypes.byref(st) if st is not None else None, ctypes.byref(ds) if ds is not None else None,
        B, Hq, Hkv, D, float(sm_scale), ctas, out.data_ptr(), dtype_code(out.dtype), out.stride(0),
        out.stride(1), _stream(stream)), "hkv_decode_attn_static")
    return out[:, :, None, :] if squeeze else out


def decode_plan(store: Optional[Int4KVStore], dense: Optional[DenseKV], batch: int, q_heads: int,
                ctas: int = 0) -> Tuple[int, int]:
    """(grid, partial slots per unit) the decode kernel would use."""
    st = store.struct() if store is not None else None
    ds = dense.struct() if dense is not None else None
    Hkv = (store or dense).kv_heads
    g, s_ = ctypes.c_int32(0), ctypes.c_int32(0)
    L.check(L.load().hkv_decode_plan(ctypes.byref(st) if st is not None else None,
                                     ctypes.byref(ds) if ds is not None else None, batch, q_heads, Hkv,
                                     ctas, ctypes.byref(g), ctypes.byref(s_)), "hkv_decode_plan")
    return g.value, s_.value


def decode_partial(q: torch.Tensor, store: Optional[Int4KVStore], dense: Optional[DenseKV],
                   sm_scale: Optional[float] = None, ctas: int = 0,
                   out_o: Optional[torch.Tensor] = None, out_ml: Optional[torch.Tensor] = None,
                   stream=None, b0: int = 0) -> Tuple[torch.Tensor, torch.Tensor]:
    """Un-normalised partial (o [B,Hq,128], (m, l) [B,Hq,2], base-2 logits) of the
    attention over this GPU's share of the context; merge with ``lse_merge``.
    ``b0`` > 0: q holds sequences [b0, b0 + B) of the store's batch."""
    _require_cuda(q)
    if q.dim() == 4:
        q = q[:, :, 0]
    B, Hq, D = q.shape
    Hkv = (store or dense).kv_heads
    for seg in (store, dense):
        if seg is not None and b0 + B > seg.batch:
            raise ValueError(f"sequences [{b0}, {b0 + B}) outside the batch of {seg.batch}")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    out_o = out_o if out_o is not None else torch.empty(B, Hq, D, dtype=torch.float32, device=q.device)
    out_ml = out_ml if out_ml is not None else torch.empty(B, Hq, 2, dtype=torch.float32, device=q.device)
    st = store.struct(b0=b0) if store is not None else None
    ds = dense.struct(b0=b0) if dense is not None else None
    pst = ctypes.byref(st) if st is not None else None
    pds = ctypes.byref(ds) if ds is not None else None
    lib = L.load()
    nbytes = lib.hkv_decode_workspace_bytes(pst, pds, B, Hq, Hkv, D, ctas)
    if nbytes == 0:
        raise RuntimeError("hkv_decode_workspace_bytes: unsupported decode configuration")
    ws = workspace(nbytes, q.device, stream)
    L.check(lib.hkv_decode_attn_partial(
        q.data_ptr(), dtype_code(q.dtype), q.stride(0), q.stride(1), pst, pds,
        B, Hq, Hkv, D, float(sm_scale), ctas, ws.data_ptr(), ws.numel(), out_o.data_ptr(),
        out_ml.data_ptr(), _stream(stream)), "hkv_decode_attn_partial")
    return out_o, out_ml


def lse_merge(parts_o: torch.Tensor, parts_ml: torch.Tensor, out_dtype=torch.float32,
              out: Optional[torch.Tensor] = None, stream=None) -> torch.Tensor:
    """Merge [n, B, Hq, 128] / [n, B, Hq, 2] partials into [B, Hq, 128]."""
    _require_cuda(parts_o, parts_ml)
    n, B, Hq, D = parts_o.shape
    parts_o, parts_ml = parts_o.contiguous(), parts_ml.contiguous()
    if out is None:
        out = torch.empty(B, Hq, D, dtype=out_dtype, device=parts_o.device)
    L.check(L.load().hkv_lse_merge(parts_o.data_ptr(), parts_ml.data_ptr(), n, B, Hq, D,
                                   out.data_ptr(), dtype_code(out.dtype), out.stride(0),
                                   out.stride(1), _stream(stream)), "hkv_lse_merge")
    return out


def dequantize_pack(store: Int4KVStore, role: int, t0: int, T: int,
                    dtype=torch.bfloat16, stream=None) -> torch.Tensor:
    """Dense [B, H, T, 128] copy of body tokens [t0, t0+T) of one side."""
    out = torch.empty(store.batch, store.kv_heads, T, HEAD_DIM, dtype=dtype, device=store.device)
    st = store.struct()
    L.check(L.load().hkv_dequantize_pack(ctypes.byref(st), role, store.batch, store.kv_heads, t0, T,
                                         out.data_ptr(), dtype_code(dtype), _stream(stream)),
            "hkv_dequantize_pack")
    return out


def quantize_flat(x: torch.Tensor, group: int, stream=None):
    """KVCompressor.compress contract: (codes u8 like x, scales f32 [ngroups], zps u8 [ngroups])."""
    _require_cuda(x)
    xc = x.contiguous()
    n = xc.numel()
    ng = (n + group - 1) // group
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    scales = torch.empty(ng, dtype=torch.float32, device=x.device)
    zps = torch.empty(ng, dtype=torch.uint8, device=x.device)
    if n == 0:
        return codes, scales, zps
    L.check(L.load().hkv_quantize_flat(xc.data_ptr(), dtype_code(xc.dtype), n, group,
                                       codes.data_ptr(), scales.data_ptr(), zps.data_ptr(),
                                       _stream(stream)), "hkv_quantize_flat")
    return codes, scales, zps


def dequantize_flat(codes: torch.Tensor, scales: torch.Tensor, zps: torch.Tensor, group: int,
                    dtype=torch.float16, stream=None) -> torch.Tensor:
    _require_cuda(codes, scales, zps)
    c = codes.contiguous()
    s = scales.contiguous().to(torch.float32)
    z = zps.contiguous()
    if z.dtype != torch.uint8:
        z = z.round().clamp(0, 255).to(torch.uint8)
    out = torch.empty(codes.shape, dtype=dtype, device=codes.device)
    if c.numel() == 0:
        return out
    L.check(L.load().hkv_dequantize_flat(c.data_ptr(), s.data_ptr(), z.data_ptr(), c.numel(), group,
                                         out.data_ptr(), dtype_code(dtype), _stream(stream)),
            "hkv_dequantize_flat")
    return out


def qk_scores_flat(q: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, zps: torch.Tensor,
                   group: int, stream=None) -> torch.Tensor:
    """Scores q . dequant(K)^T of one query row q [D] against codes [S, D] in the
    reference's unpacked layout (flat f32 scales / zero-points over groups of
    ``group`` values): [S] fp32."""
    _require_cuda(q, codes, scales, zps)
    S, D = codes.shape
    qc = q.reshape(-1).contiguous()
    c = codes.contiguous()
    s = scales.contiguous().to(torch.float32)
    z = zps.contiguous()
    if z.dtype != torch.uint8:
        z = z.round().clamp(0, 255).to(torch.uint8)
    out = torch.empty(S, dtype=torch.float32, device=q.device)
    L.check(L.load().hkv_qk_scores_flat(qc.data_ptr(), dtype_code(qc.dtype), c.data_ptr(), s.data_ptr(),
                                        z.data_ptr(), S, D, group, out.data_ptr(), _stream(stream)),
            "hkv_qk_scores_flat")
    return out


def selftest_bounded_wait(limit_ns: int, arrive: bool, stream=None) -> int:
    """Run the bounded device wait self-test; returns the library status
    (HKV_OK when the phase completed, HKV_ERR_DEVICE when the wait ran out)."""
    return int(L.load().hkv_selftest_bounded_wait(int(limit_ns), 1 if arrive else 0, _stream(stream)))


def repack_ref(codes: torch.Tensor, scales: torch.Tensor, zps: torch.Tensor, group: int,
               store: Int4KVStore, role: int, stream=None) -> None:
    """Load the reference's unpacked representation (codes [B,H,S,128] u8,
    flat f32 scales / u8 zps over groups) into body slots [0, S) of ``store``."""
    _require_cuda(codes, scales, zps)
    B, H, S_, D = codes.shape
    c = codes.contiguous()
    s = scales.contiguous().to(torch.float32)
    z = zps.contiguous()
    if z.dtype != torch.uint8:
        z = z.round().clamp(0, 15).to(torch.uint8)
    st = store.struct()
    L.check(L.load().hkv_repack_ref(c.data_ptr(), s.data_ptr(), z.data_ptr(), B, H, S_, group, role,
                                    ctypes.byref(st), _stream(stream)), "hkv_repack_ref")
