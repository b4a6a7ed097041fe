"""ctypes binding of libhetero_kv.so (the C ABI in include/hetero_kv.h).

The library is loaded from the package's ``lib/`` directory. There is no
fallback: if the shared object is missing or fails to load, every entry point
raises, so a run can never silently take a CPU or PyTorch path.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libhetero_kv.so")

HKV_OK = 0
HKV_ERR_ARG = 1
HKV_ERR_CUDA = 2
HKV_ERR_TIMEOUT = 3
HKV_ERR_UNSUPPORTED = 4
HKV_ERR_CAPACITY = 5
HKV_ERR_DEVICE = 6

STATIC_SCRATCH_BYTES = 8 << 20  # HKV_STATIC_SCRATCH_BYTES

DT_F16, DT_BF16, DT_F32 = 0, 1, 2
FMT_REF, FMT_FP16MIN = 0, 1
ROLE_K, ROLE_V = 0, 1

DEVERR_TIMEOUT, DEVERR_BAD_PAGE, DEVERR_CAPACITY = 1, 2, 4
APPEND_EARLY = 1  # HKV_APPEND_EARLY

c_i32, c_i64, c_u32, c_f32, c_vp, c_sz = (ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32,
                                          ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t)
P_i32 = ctypes.POINTER(ctypes.c_int32)


class HkvInt4Store(ctypes.Structure):
    _fields_ = [("pages", c_vp), ("page_stride", c_i64), ("format", c_i32), ("group", c_i32),
                ("page_tokens", c_i32), ("max_pages", c_i32), ("page_table", c_vp),
                ("lengths", c_vp), ("len", c_i32), ("num_pages", c_i32)]


class HkvDenseKV(ctypes.Structure):
    _fields_ = [("k", c_vp), ("v", c_vp), ("dtype", c_i32), ("capacity", c_i32),
                ("stride_b", c_i64), ("stride_h", c_i64), ("stride_t", c_i64),
                ("lengths", c_vp), ("len", c_i32), ("reserved", c_i32)]


P_store = ctypes.POINTER(HkvInt4Store)
P_dense = ctypes.POINTER(HkvDenseKV)

# name -> (restype, argtypes); must match include/hetero_kv.h exactly.
SIGNATURES = {
    "hkv_status_str": (ctypes.c_char_p, [c_i32]),
    "hkv_version": (c_i32, []),
    "hkv_device_error": (c_i32, [ctypes.POINTER(c_u32), c_i32]),
    "hkv_last_cuda_error": (c_i32, []),
    "hkv_page_bytes": (c_i64, [c_i32, c_i32, c_i32]),
    "hkv_quantize_flat": (c_i32, [c_vp, c_i32, c_i64, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "hkv_dequantize_flat": (c_i32, [c_vp, c_vp, c_vp, c_i64, c_i32, c_vp, c_i32, c_vp]),
    "hkv_quantize_pack": (c_i32, [c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, c_i64,
                                  c_i32, P_store, c_vp, c_i32, c_vp]),
    "hkv_quantize_pack_kv": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, c_i64,
                                     P_store, c_vp, c_i32, c_vp]),
    "hkv_append_kv": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i64, c_i64, P_dense, c_i32,
                              c_vp, c_vp, P_store, c_vp, c_vp]),
    "hkv_dequantize_pack": (c_i32, [P_store, c_i32, c_i32, c_i32, c_i32, c_i32, c_vp, c_i32, c_vp]),
    "hkv_repack_ref": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_i32, P_store, c_vp]),
    "hkv_decode_workspace_bytes": (c_sz, [P_store, P_dense, c_i32, c_i32, c_i32, c_i32, c_i32]),
    "hkv_decode_plan": (c_i32, [P_store, P_dense, c_i32, c_i32, c_i32, c_i32, P_i32, P_i32]),
    "hkv_decode_attn": (c_i32, [c_vp, c_i32, c_i64, c_i64, P_store, P_dense, c_i32, c_i32, c_i32,
                                c_i32, c_f32, c_i32, c_vp, c_sz, c_vp, c_i32, c_i64, c_i64, c_vp]),
    "hkv_decode_append": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_vp, c_vp, c_i64, c_i64, P_store, P_dense, c_i32,
                                  c_vp, c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_f32, c_i32, c_vp, c_sz, c_vp,
                                  c_i32, c_i64, c_i64, c_i32, c_vp]),
    "hkv_decode_attn_scored": (c_i32, [c_vp, c_i32, c_i64, c_i64, P_store, P_dense, c_i32, c_i32, c_i32,
                                       c_i32, c_f32, c_i32, c_vp, c_sz, c_vp, c_i32, c_i64, c_i64, c_vp,
                                       c_i32, c_vp, c_vp]),
    "hkv_tile_scores": (c_i32, [c_vp, c_vp, P_store, c_i32, c_i32, c_i32, c_i32, c_vp, c_vp]),
    "hkv_prefill_workspace_bytes": (c_sz, [P_store, c_i32, c_i32, c_i32, c_i32, c_i32, c_i32]),
    "hkv_prefill_attn": (c_i32, [c_vp, c_i32, c_i64, c_i64, c_i64, P_store, c_i32, c_i32, c_i32, c_i32, c_i32,
                                 c_f32, c_i32, c_vp, c_i32, c_i64, c_i64, c_i64, c_vp, c_i32, c_vp, c_sz, c_vp]),
    "hkv_decode_attn_partial": (c_i32, [c_vp, c_i32, c_i64, c_i64, P_store, P_dense, c_i32, c_i32,
                                        c_i32, c_i32, c_f32, c_i32, c_vp, c_sz, c_vp, c_vp, c_vp]),
    "hkv_decode_attn_static": (c_i32, [c_vp, c_i32, c_i64, c_i64, P_store, P_dense, c_i32, c_i32, c_i32,
                                       c_i32, c_f32, c_i32, c_vp, c_i32, c_i64, c_i64, c_vp]),
    "hkv_lse_merge": (c_i32, [c_vp, c_vp, c_i32, c_i32, c_i32, c_i32, c_vp, c_i32, c_i64, c_i64,
                              c_vp]),
    "hkv_lse_merge_strided": (c_i32, [c_vp, c_vp, c_i32, c_i64, c_i64, c_i32, c_i32, c_i32, c_vp, c_i32, c_i64,
                                      c_i64, c_vp]),
    "hkv_prefetcher_create": (c_i32, [c_vp, c_i64, c_vp, c_i64, c_i64, ctypes.POINTER(c_vp)]),
    "hkv_prefetcher_destroy": (c_i32, [c_vp]),
    "hkv_prefetch_submit": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_vp, c_vp]),
    "hkv_prefetch_bytes": (c_i64, [c_vp]),
    "hkv_prefetch_gather": (c_i32, [c_vp, c_vp, c_vp, c_i32, c_vp, c_i64, c_i32, c_i32, c_vp]),
    "hkv_graph_copy_nodes": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp]),
    "hkv_graph_exec_set_copy_srcs": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_vp]),
    "hkv_event_wait": (c_i32, [c_vp, c_i64]),
    "hkv_qk_scores_flat": (c_i32, [c_vp, c_i32, c_vp, c_vp, c_vp, c_i64, c_i32, c_i32, c_vp, c_vp]),
    "hkv_selftest_bounded_wait": (c_i32, [c_i64, c_i32, c_vp]),
}

_lib = None
_lock = threading.Lock()


class HkvError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = status_str(status) if _lib is not None else f"status {status}"
        if status == HKV_ERR_CUDA and _lib is not None:
            msg += f" (cudaError {_lib.hkv_last_cuda_error()})"
        super().__init__(f"{what}: {msg}" if what else msg)


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raises if it is missing."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libhetero_kv.so not found at {LIB_PATH}; build it with "
                "`python -m hetero_kvcache_optimizer_b200.csrc.build` (no CPU fallback exists)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def status_str(status: int) -> str:
    return load().hkv_status_str(status).decode()


def check(status: int, what: str = "") -> None:
    if status != HKV_OK:
        raise HkvError(status, what)


# Called with the error bits whenever device_error() sees a bounded wait that
# expired: a decode kernel that gave up leaves merge counters non-zero in its
# workspace, so the owners of cached workspaces re-zero them here.
_timeout_hooks = []


def on_device_timeout(fn) -> None:
    if fn not in _timeout_hooks:
        _timeout_hooks.append(fn)


def device_error(clear: bool = True) -> int:
    """Sticky device error bits (synchronises the device). A timeout bit also
    runs the registered workspace-reset hooks."""
    bits = c_u32(0)
    check(load().hkv_device_error(ctypes.byref(bits), 1 if clear else 0), "hkv_device_error")
    if bits.value & DEVERR_TIMEOUT:
        for fn in _timeout_hooks:
            fn()
    return int(bits.value)
