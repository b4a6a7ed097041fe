"""Helpers shared by the GPU parity tests: move seeded oracle inputs onto the
device, read packed pages back and unpack them with the oracle's layout spec."""
from __future__ import annotations

import numpy as np
import torch

from oracle import kv_oracle as ko

HEAD_DIM = 128


def t16(x: np.ndarray, device="cuda", dtype=torch.float16) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x.astype(np.float32))).to(device=device, dtype=dtype)


def read_side(store, role: int):
    """Unpack the K (role 0) or V (role 1) half of a dense-mode or paged store
    into numpy arrays over body slots [0, capacity): codes [B,H,cap,128] and the
    two meta arrays [B,H,cap,ng] (scale/zp for ref, scale/min for fp16min)."""
    torch.cuda.synchronize()
    pool = store.pool.cpu().numpy()
    P = store.page_tokens
    fmt = 0 if store.fmt == "ref" else 1
    ng = HEAD_DIM // store.group
    B, H, mp = store.batch, store.kv_heads, store.max_pages
    table = store.page_table.cpu().numpy() if store.paged else None
    codes = np.zeros((B, H, mp * P, HEAD_DIM), np.uint8)
    m0 = np.zeros((B, H, mp * P, ng), np.float32 if fmt == 0 else np.float16)
    m1 = np.zeros((B, H, mp * P, ng), np.uint8 if fmt == 0 else np.float16)
    for u in range(B * H):
        b, h = divmod(u, H)
        for pi in range(mp):
            page = table[u, pi] if table is not None else u * mp + pi
            if page < 0:
                continue
            c, a, z = ko.split_page(pool[page], P, fmt, store.group, role)
            codes[b, h, pi * P:(pi + 1) * P] = ko.unpack_k(c) if role == 0 else ko.unpack_v(c, P)
            m0[b, h, pi * P:(pi + 1) * P] = a
            m1[b, h, pi * P:(pi + 1) * P] = z
    return codes, m0, m1


def dequant_side(store, role: int, T: int) -> np.ndarray:
    """fp32 dequantised body tokens [0, T) of one side, via the oracle formulas."""
    codes, a, z = read_side(store, role)
    codes, a, z = codes[:, :, :T], a[:, :, :T], z[:, :, :T]
    if store.fmt == "ref":
        return ko.dequantize_ref(codes, a.reshape(-1), z.reshape(-1), store.group)
    return ko.dequantize_fp16min(codes, a, z, store.group)
