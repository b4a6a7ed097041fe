"""CPU oracle for the INT4 KV hot path (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it. The product path (``hetero_kvcache_optimizer_b200``)
never imports anything under ``oracle/`` and fails loudly when its CUDA library
is missing.

Parity status: PINNED. ``quantize_ref`` / ``dequantize_ref`` / ``decode_attention``
are checked against the reference implementation itself (the Python package in
kldxg123/Hetero-KVCache-Optimizer, run on CPU in the build container) through the
fixtures under ``tests/golden/`` produced by ``tests/golden/make_golden.py``.
The ``fp16min`` format and the packed nibble layouts are this build's own
specification (the reference has neither); they are pinned by round-trip
properties and by the ref-format goldens after unpacking.

Everything is plain numpy.
"""
from __future__ import annotations

import hashlib
from typing import Tuple

import numpy as np

QMAX = 15  # 2**4 - 1, kv_compressor.py:41
HEAD_DIM = 128
CODE_BYTES = HEAD_DIM // 2  # 64 packed bytes per token per tensor

FMT_REF = 0       # fp32 scale + uint8 zero-point (the reference's own format)
FMT_FP16MIN = 1   # fp16 scale + fp16 zero = group minimum

ROLE_K = 0
ROLE_V = 1


# ---------------------------------------------------------------------------
# Reference quantizer, restated (src/quantization/kv_compressor.py:50-132)
# ---------------------------------------------------------------------------

def quantize_ref(x: np.ndarray, group: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Restates ``KVCompressor.compress`` (kv_compressor.py:66-98).

    Flattens ``x`` in logical (row-major) order, zero-pads to a multiple of
    ``group`` (:70-74), takes per-group min/max (:76-77), ``scale =
    clamp((max-min)/15, 1e-8)`` in fp32 (:79-80), ``zp = clamp(rint(-min/scale),
    0, 15)`` as uint8 (:82-84) and ``q = clamp(rint(x/scale + zp), 0, 15)``
    (:86-88), then crops the padding (:91). ``rint`` is round-half-to-even, like
    ``torch.round``. All arithmetic is IEEE fp32, which makes the result
    bit-identical to the reference.

    Returns (codes uint8 shaped like ``x``, scales fp32 [ngroups], zps uint8
    [ngroups]).
    """
    shape = x.shape
    n = x.size
    flat = np.ascontiguousarray(x).astype(np.float32).reshape(-1)
    pad = (group - n % group) % group
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, np.float32)])
    f = flat.reshape(-1, group)
    mn = f.min(axis=1, keepdims=True)
    mx = f.max(axis=1, keepdims=True)
    scale = np.maximum((mx - mn) / np.float32(QMAX), np.float32(1e-8)).astype(np.float32)
    zp = np.clip(np.rint(-mn / scale), 0, QMAX).astype(np.uint8)
    q = np.clip(np.rint(f / scale + zp.astype(np.float32)), 0, QMAX).astype(np.uint8)
    codes = q.reshape(-1)[:n].reshape(shape)
    return codes, scale.reshape(-1), zp.reshape(-1)


def dequantize_ref(codes: np.ndarray, scales: np.ndarray, zps: np.ndarray,
                   group: int) -> np.ndarray:
    """Restates ``KVCompressor.decompress`` (kv_compressor.py:119-132):
    ``(q - zp) * scale`` in fp32 over the zero-padded flat view. Returns fp32."""
    shape = codes.shape
    n = codes.size
    q = codes.reshape(-1).astype(np.float32)
    pad = (group - n % group) % group
    if pad:
        q = np.concatenate([q, np.zeros(pad, np.float32)])
    q = q.reshape(-1, group)
    s = scales.reshape(-1, 1).astype(np.float32)
    z = zps.reshape(-1, 1).astype(np.float32)
    return ((q - z) * s).reshape(-1)[:n].reshape(shape)


# ---------------------------------------------------------------------------
# fp16min format: fp16 scale = (max-min)/15, fp16 zero = min (configuration-0
# text of the benchmark spec; the reference has no such format)
# ---------------------------------------------------------------------------

def quantize_fp16min(x: np.ndarray, group: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Group-wise asymmetric INT4 with fp16 scale and fp16 zero (= group min).

    ``x`` is [..., D] with D % group == 0; groups run along the last axis.
    Exact definition (the CUDA quantizer implements the same IEEE steps):
      mn, mx = fp32 min/max of the group
      scale_h = fp16_rn(min((mx - mn) / 15, 65504))
      min_h   = fp16_rn(mn)
      q = 0                                                if scale_h == 0
          clamp(rint((x - f32(min_h)) / f32(scale_h)), 0, 15)  otherwise
    Returns (codes uint8 like ``x``, scale fp16 [..., D/group], min fp16 [..., D/group]).
    """
    shape = x.shape
    D = shape[-1]
    assert D % group == 0
    f = x.astype(np.float32).reshape(-1, D // group, group)
    mn = f.min(axis=2)
    mx = f.max(axis=2)
    scale_f = np.minimum((mx - mn) / np.float32(QMAX), np.float32(65504.0)).astype(np.float32)
    scale_h = scale_f.astype(np.float16)
    min_h = mn.astype(np.float16)
    sf = scale_h.astype(np.float32)[..., None]
    mf = min_h.astype(np.float32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore"):
        q = np.clip(np.rint((f - mf) / sf), 0, QMAX)
    q = np.where(sf > 0, q, 0).astype(np.uint8)
    mshape = shape[:-1] + (D // group,)
    return q.reshape(shape), scale_h.reshape(mshape), min_h.reshape(mshape)


def dequantize_fp16min(codes: np.ndarray, scale_h: np.ndarray, min_h: np.ndarray,
                       group: int) -> np.ndarray:
    """``q * scale + min`` in fp32 for the fp16min format. Returns fp32."""
    shape = codes.shape
    D = shape[-1]
    q = codes.astype(np.float32).reshape(-1, D // group, group)
    s = scale_h.astype(np.float32).reshape(-1, D // group, 1)
    m = min_h.astype(np.float32).reshape(-1, D // group, 1)
    return (q * s + m).reshape(shape)


# ---------------------------------------------------------------------------
# Packed nibble layouts (this build's HBM format, D = 128)
# ---------------------------------------------------------------------------
#
# K codes, per token: 64 bytes = 16 little-endian u32 words, word index
# 4*j + w (j = 0..3, w = 0..3). Nibble k (bits 4k..4k+3) of word (j, w) holds
#   dim = 16*(2w + (k%4)//2) + 8*((k%4)%2) + 2j + k//4
# so that one 16-byte chunk j holds exactly the 32 K values that mma lane
# (lane%4 == j) needs as its A fragment for one token row, and each word holds
# one 32-wide group.
#
# V codes, per token PAIR (tokens 2p, 2p+1): 128 bytes = 32 u32 words, word
# index 4*i + k (i = 0..7, k = 0..3). Bits 4m..4m+3 (m = 0..3) hold token 2p and
# bits 16+4m.. hold token 2p+1, both at
#   dim = 16*(e//2) + 8*(e%2) + i,  e = 4k + m
# so that one 16-byte chunk i holds the V^T A fragment rows of lane (lane/4 == i)
# for two adjacent tokens, already paired as (token, token+1) half2 lanes.


def _k_dim_table() -> np.ndarray:
    """[64 bytes, 2 nibbles] -> dim, for one K token."""
    t = np.zeros((64, 2), np.int64)
    for j in range(4):
        for w in range(4):
            for k in range(8):
                dim = 16 * (2 * w + (k % 4) // 2) + 8 * ((k % 4) % 2) + 2 * j + k // 4
                word = 4 * j + w
                byte = word * 4 + k // 2
                t[byte, k % 2] = dim
    return t


def _v_dim_table() -> np.ndarray:
    """[128 bytes, 2 nibbles] -> (token-in-pair, dim), for one V token pair."""
    t = np.zeros((128, 2, 2), np.int64)
    for i in range(8):
        for k in range(4):
            for nib in range(8):
                tok = nib // 4
                m = nib % 4
                e = 4 * k + m
                dim = 16 * (e // 2) + 8 * (e % 2) + i
                word = 4 * i + k
                byte = word * 4 + nib // 2
                t[byte, nib % 2] = (tok, dim)
    return t


_KT = _k_dim_table()
_VT = _v_dim_table()


def pack_k(codes: np.ndarray) -> np.ndarray:
    """[..., T, 128] uint8 codes (0..15) -> [..., T, 64] packed K bytes."""
    assert codes.shape[-1] == HEAD_DIM
    lo = codes[..., _KT[:, 0]].astype(np.uint8)
    hi = codes[..., _KT[:, 1]].astype(np.uint8)
    return np.ascontiguousarray(lo | (hi << 4), dtype=np.uint8)


def unpack_k(packed: np.ndarray) -> np.ndarray:
    """[..., T, 64] packed K bytes -> [..., T, 128] codes."""
    out = np.zeros(packed.shape[:-1] + (HEAD_DIM,), np.uint8)
    out[..., _KT[:, 0]] = packed & 0xF
    out[..., _KT[:, 1]] = packed >> 4
    return out


def pack_v(codes: np.ndarray) -> np.ndarray:
    """[..., T, 128] codes -> [..., T + T%2, 64] packed V bytes (token pairs
    interleaved; an odd trailing token is paired with a zero token, so the
    result always covers a whole number of pairs)."""
    T = codes.shape[-2]
    Tp = T + (T % 2)
    if Tp != T:
        pad = np.zeros(codes.shape[:-2] + (1, HEAD_DIM), np.uint8)
        codes = np.concatenate([codes, pad], axis=-2)
    pairs = codes.reshape(codes.shape[:-2] + (Tp // 2, 2, HEAD_DIM))
    lo = pairs[..., _VT[:, 0, 0], _VT[:, 0, 1]]
    hi = pairs[..., _VT[:, 1, 0], _VT[:, 1, 1]]
    packed = np.ascontiguousarray(lo | (hi << 4), dtype=np.uint8)  # [..., Tp/2, 128]
    return packed.reshape(codes.shape[:-2] + (Tp, 64))


def unpack_v(packed: np.ndarray, T: int | None = None) -> np.ndarray:
    """[..., Tp, 64] packed V bytes (Tp even) -> [..., T, 128] codes."""
    if T is None:
        T = packed.shape[-2]
    Tp = packed.shape[-2]
    assert Tp % 2 == 0 and T <= Tp
    pb = packed.reshape(packed.shape[:-2] + (Tp // 2, 128))
    out = np.zeros(pb.shape[:-1] + (2, HEAD_DIM), np.uint8)
    out[..., _VT[:, 0, 0], _VT[:, 0, 1]] = pb & 0xF
    out[..., _VT[:, 1, 0], _VT[:, 1, 1]] = pb >> 4
    return out.reshape(packed.shape[:-2] + (Tp, HEAD_DIM))[..., :T, :]


BLOCK_TOKENS = 128


def block_bytes(fmt: int, group: int) -> int:
    """Bytes of one 128-token page block: K codes | V codes | K meta | V meta
    (| K zps | V zps for FMT_REF)."""
    ng = HEAD_DIM // group
    return BLOCK_TOKENS * (2 * CODE_BYTES + 8 * ng + (2 * ng if fmt == FMT_REF else 0))


def page_bytes(page_tokens: int, fmt: int, group: int) -> int:
    assert page_tokens % BLOCK_TOKENS == 0
    return page_tokens // BLOCK_TOKENS * block_bytes(fmt, group)


def v_chunk_pos(pair: int, chunk: int) -> int:
    """Stored 16-byte chunk position of logical chunk `chunk` of token pair `pair`
    inside the pair's 128 bytes of a block (rotated by 2*pair)."""
    return (chunk + 2 * pair) % 8


def _v_perm() -> np.ndarray:
    """[64 pairs * 128 bytes] stored byte index -> logical byte index for one block."""
    perm = np.zeros(64 * 128, np.int64)
    for q in range(64):
        for c in range(8):
            pos = v_chunk_pos(q, c)
            perm[q * 128 + pos * 16: q * 128 + pos * 16 + 16] = np.arange(q * 128 + c * 16, q * 128 + c * 16 + 16)
    return perm


_VPERM = _v_perm()


def split_page(page: np.ndarray, page_tokens: int, fmt: int, group: int, role: int):
    """Split one raw page (uint8 bytes) into the K (role 0) or V (role 1) half:
    (codes [P, 64] in the pack_k / pack_v byte order, meta0 [P, ng], meta1 [P, ng]).
    For FMT_REF the meta are (scales fp32, zps u8); for FMT_FP16MIN (scale fp16,
    min fp16), stored as four f16 arrays: K scales [128][ng], K mins, V scales
    [64 token pairs][ng][2], V mins."""
    ng = HEAD_DIM // group
    bb = block_bytes(fmt, group)
    codes, m0, m1 = [], [], []
    for blk in range(page_tokens // BLOCK_TOKENS):
        b = page[blk * bb:(blk + 1) * bb]
        if role == 0:
            codes.append(b[:8192].reshape(BLOCK_TOKENS, 64))
        else:
            logical = np.empty(8192, np.uint8)
            logical[_VPERM] = b[8192:16384]
            codes.append(logical.reshape(BLOCK_TOKENS, 64))
        meta = b[16384 + role * 512 * ng: 16384 + (role + 1) * 512 * ng]
        if fmt == FMT_REF:
            m0.append(meta.view(np.float32).reshape(BLOCK_TOKENS, ng))
            zo = 16384 + 1024 * ng + role * 128 * ng
            m1.append(b[zo: zo + 128 * ng].reshape(BLOCK_TOKENS, ng))
        else:
            hm = meta.view(np.float16).reshape(2, BLOCK_TOKENS * ng)   # scales | mins
            if role == 0:
                m0.append(hm[0].reshape(BLOCK_TOKENS, ng))
                m1.append(hm[1].reshape(BLOCK_TOKENS, ng))
            else:  # [pair][group][token parity] -> [token][group]
                m0.append(hm[0].reshape(BLOCK_TOKENS // 2, ng, 2).transpose(0, 2, 1).reshape(BLOCK_TOKENS, ng))
                m1.append(hm[1].reshape(BLOCK_TOKENS // 2, ng, 2).transpose(0, 2, 1).reshape(BLOCK_TOKENS, ng))
    return np.concatenate(codes), np.concatenate(m0), np.concatenate(m1)


# ---------------------------------------------------------------------------
# Attention (src/quantization/fused_dequant_attn.py:326-331, plus GQA)
# ---------------------------------------------------------------------------

def decode_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                     sm_scale: float | None = None, dtype=np.float32) -> np.ndarray:
    """Single-query attention, restating the reference's dequant-then-SDPA
    fallback (fused_dequant_attn.py:327-331): ``softmax(q @ K^T * sm_scale) @ V``
    with ``sm_scale = 1/sqrt(D)`` by default (:271-272).

    Extended with GQA the way HF ``repeat_kv`` expands heads: query head ``hq``
    reads KV head ``hq // (Hq // Hkv)``.

    q: [B, Hq, D]; k, v: [B, Hkv, S, D] (already dequantised). Returns
    [B, Hq, D] in ``dtype`` arithmetic (fp32 by default, like the reference).
    """
    B, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    if sm_scale is None:
        sm_scale = 1.0 / (D ** 0.5)
    kk = np.repeat(k.astype(dtype), G, axis=1)
    vv = np.repeat(v.astype(dtype), G, axis=1)
    qq = q.astype(dtype)[:, :, None, :]
    s = np.matmul(qq, np.swapaxes(kk, -1, -2))[:, :, 0, :] * dtype(sm_scale)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    return np.matmul(p[:, :, None, :], vv)[:, :, 0, :]


def prefill_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray,
                      sm_scale: float | None = None, causal: bool = False,
                      lengths=None, return_lse: bool = False):
    """Multi-query attention, restating the reference's decompress-then-matmul
    path of fused_dequant_attn_forward (src/quantization/fused_dequant_attn.py:
    241-246): ``softmax(Q K^T * sm_scale) V`` in fp32, for q [B, Hq, Sq, D]
    against dequantised k, v [B, Hkv, S, D] (GQA as in ``decode_attention``).

    Extensions of this build (the reference has no mask): ``lengths`` [B] keys
    per sequence (default S); ``causal`` lets query s see keys t <= len - Sq + s
    (the queries are the last Sq positions); a query that sees no key gets
    zeros and an lse of -inf. ``return_lse`` also returns ln sum exp(scores)."""
    B, Hq, Sq, D = q.shape
    S = k.shape[2]
    G = Hq // k.shape[1]
    if sm_scale is None:
        sm_scale = 1.0 / (D ** 0.5)
    kk = np.repeat(k.astype(np.float32), G, axis=1)
    vv = np.repeat(v.astype(np.float32), G, axis=1)
    s = np.matmul(q.astype(np.float32), np.swapaxes(kk, -1, -2)) * np.float32(sm_scale)
    lens = np.full(B, S) if lengths is None else np.asarray(lengths)
    tok = np.arange(S)[None, None, :]
    lim = lens[:, None, None] - Sq + 1 + np.arange(Sq)[None, :, None] if causal else lens[:, None, None]
    vis = np.broadcast_to(tok < np.minimum(lim, lens[:, None, None]), (B, Sq, S))[:, None]  # [B,1,Sq,S]
    s = np.where(vis, s, -np.inf)
    mx = s.max(axis=-1, keepdims=True)
    mx = np.where(np.isfinite(mx), mx, 0.0)
    e = np.where(vis, np.exp(s - mx), 0.0)
    den = e.sum(axis=-1, keepdims=True)
    out = np.matmul(e / np.where(den > 0, den, 1.0), vv)
    if not return_lse:
        return out
    with np.errstate(divide="ignore"):
        lse = np.where(den[..., 0] > 0, np.log(den[..., 0]) + mx[..., 0], -np.inf)
    return out, lse


def lse_merge(parts_o: np.ndarray, parts_m: np.ndarray, parts_l: np.ndarray) -> np.ndarray:
    """Merge split-KV partials: parts_o [n, ..., D] (unnormalised), parts_m /
    parts_l [n, ...] in the natural-log domain. Returns the normalised output."""
    M = parts_m.max(axis=0)
    w = np.exp(parts_m - M)
    w = np.where(np.isfinite(parts_m), w, 0.0)
    num = (w[..., None] * parts_o).sum(axis=0)
    den = (w * parts_l).sum(axis=0)
    return num / den[..., None]


def rel_err(out: np.ndarray, ref: np.ndarray) -> float:
    """max over heads of max|out - ref| / ||ref||_2 (norm over the head dim):
    the benchmark spec's attention tolerance metric (bound 2e-3)."""
    diff = np.abs(out.astype(np.float64) - ref.astype(np.float64)).max(axis=-1)
    nrm = np.linalg.norm(ref.astype(np.float64), axis=-1)
    return float((diff / np.maximum(nrm, 1e-30)).max())


# ---------------------------------------------------------------------------
# Seeded synthetic inputs (benchmark spec configurations; no dataset involved)
# ---------------------------------------------------------------------------

def rng_for(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def make_kv(seed: int, B: int, Hkv: int, S: int, D: int = HEAD_DIM,
            outlier_channels: int = 4, outlier_scale: float = 10.0,
            vision_tokens: int = 0, vision_std: float = 0.5):
    """K, V ~ N(0,1) fp16 with ``outlier_channels`` seeded K channels per KV head
    scaled by ``outlier_scale``. The first ``vision_tokens`` positions are
    N(0, vision_std^2) without outliers (configuration 2's multimodal prefix)."""
    rng = rng_for(seed)
    k = rng.standard_normal((B, Hkv, S, D), dtype=np.float32)
    v = rng.standard_normal((B, Hkv, S, D), dtype=np.float32)
    for h in range(Hkv):
        ch = rng.choice(D, outlier_channels, replace=False)
        k[:, h, vision_tokens:, ch] *= outlier_scale
    if vision_tokens:
        k[:, :, :vision_tokens] *= vision_std
        v[:, :, :vision_tokens] *= vision_std
    return k.astype(np.float16), v.astype(np.float16)


def make_q(seed: int, B: int, Hq: int, D: int = HEAD_DIM) -> np.ndarray:
    rng = rng_for(seed + 7919)
    return rng.standard_normal((B, Hq, D), dtype=np.float32)


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16 value, returned as fp32 (exactly representable)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
    return b.astype(np.uint32).view(np.float32)


def make_input(seed: int, shape, dtype: str) -> np.ndarray:
    """Seeded N(0,1) tensor rounded to ``dtype`` ('fp16' or 'bf16'); returned as
    float16 for fp16 and as the fp32 image of the bf16 values for bf16."""
    x = rng_for(seed).standard_normal(shape, dtype=np.float32)
    if dtype == "fp16":
        return x.astype(np.float16)
    return round_bf16(x)
