"""CPU checks of the C ABI boundary: the in-tree library loads, exports every
function include/hetero_kv.h declares, and the ctypes table matches the header.
Only host-only entry points are called (no GPU here)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "hetero_kv.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(hkv_\w+)\s*\(", src, flags=re.M)
    return sorted(set(names))


@pytest.fixture(scope="module")
def lib():
    from hetero_kvcache_optimizer_b200.csrc import build
    build.build()
    from hetero_kvcache_optimizer_b200 import _lib
    return _lib


def test_header_parses():
    names = header_functions()
    assert "hkv_decode_attn" in names and "hkv_quantize_pack" in names
    assert len(names) >= 20


def test_every_declared_symbol_is_exported(lib):
    so = lib.load()
    for name in header_functions():
        assert hasattr(so, name), name
    assert set(header_functions()) == set(lib.SIGNATURES)


def test_struct_layouts_match_header(lib):
    assert ctypes.sizeof(lib.HkvInt4Store) == 8 + 8 + 4 * 4 + 8 + 8 + 4 + 4
    assert ctypes.sizeof(lib.HkvDenseKV) == 8 + 8 + 4 + 4 + 3 * 8 + 8 + 4 + 4


def test_host_only_entry_points(lib):
    so = lib.load()
    assert so.hkv_version() >= 100
    assert lib.status_str(0) == "HKV_OK"
    assert "CAPACITY" in lib.status_str(5)
    # page geometry (K and V): 168 B/token (ref, group 32), 160 B/token (fp16min, group 32)
    assert so.hkv_page_bytes(0, 32, 256) == 256 * 168
    assert so.hkv_page_bytes(1, 32, 256) == 256 * 160
    assert so.hkv_page_bytes(0, 128, 256) == 256 * 138
    assert so.hkv_page_bytes(0, 48, 256) == -1
    assert so.hkv_page_bytes(0, 32, 200) == -1  # pages hold whole 128-token blocks
    # no body and no dense segment: nothing to plan
    assert so.hkv_decode_workspace_bytes(None, None, 8, 32, 8, 128, 0) == 0


def test_no_cpu_fallback(lib):
    """CPU tensors are rejected loudly by the product path."""
    import torch
    from hetero_kvcache_optimizer_b200 import kvstore
    with pytest.raises(RuntimeError, match="CUDA"):
        kvstore.quantize_flat(torch.zeros(4, 128), 32)
