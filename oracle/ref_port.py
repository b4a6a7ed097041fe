"""CPU port of the reference's own decode-step path, for TIMING ONLY.

Test/benchmark infrastructure: ``bench.py`` times this as the CPU baseline
(``cpu_baseline.kind = "port"``) and as the ``--impl reference`` arm; nothing in
the product imports it. The reference package itself cannot travel to the GPU
box, so this restates, with the same PyTorch calls on the same layouts, what
the reference executes on CPU tensors for one layer of one decode step:

  * ``KVCompressor.compress`` of the evicted token, K and V
    (src/quantization/kv_compressor.py:66-98): fp32 flatten, per-group min/max,
    scale/zero-point, round/clamp to one uint8 code per value;
  * ``KVCompressor.decompress`` of the INT4 body (kv_compressor.py:119-132);
  * the body is concatenated with the fp16 sink/recent tokens the way the
    engine prepends swapped-in DRAM tokens (src/core/engine_wrapper.py:241-244),
    heads are expanded for GQA (HF ``repeat_kv``), and the attention is the
    fallback of ``fused_dequant_attn_decode``
    (src/quantization/fused_dequant_attn.py:327-331).

Its outputs are checked against the golden fixtures in tests/test_ref_port.py.
"""
from __future__ import annotations

import torch


def compress(t: torch.Tensor, group: int):
    shape, n = t.shape, t.numel()
    flat = t.to(torch.float32).reshape(-1)
    pad = (group - n % group) % group
    if pad:
        flat = torch.nn.functional.pad(flat, (0, pad))
    flat = flat.reshape(-1, group)
    mn = flat.min(dim=-1, keepdim=True).values
    mx = flat.max(dim=-1, keepdim=True).values
    scales = torch.clamp((mx - mn) / 15, min=1e-8)
    zps = torch.clamp(torch.round(-mn / scales), 0, 15).to(torch.uint8)
    q = torch.clamp(torch.round(flat / scales + zps.float()), 0, 15).to(torch.uint8)
    return q.reshape(-1)[:n].view(shape), scales.reshape(-1), zps.reshape(-1)


def decompress(q: torch.Tensor, scales: torch.Tensor, zps: torch.Tensor, group: int,
               dtype=torch.float32) -> torch.Tensor:
    shape, n = q.shape, q.numel()
    fq = q.reshape(-1)
    pad = (group - n % group) % group
    if pad:
        fq = torch.nn.functional.pad(fq, (0, pad))
    fq = fq.reshape(-1, group).to(torch.float32)
    out = (fq - zps.reshape(-1, 1).float()) * scales.reshape(-1, 1).float()
    return out.reshape(-1)[:n].view(shape).to(dtype)


def decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale=None) -> torch.Tensor:
    """q [B,Hq,1,D]; k, v [B,Hkv,S,D] (fp32) -> [B,Hq,1,D] fp32."""
    G = q.shape[1] // k.shape[1]
    if G > 1:
        k = k.repeat_interleave(G, dim=1)
        v = v.repeat_interleave(G, dim=1)
    if sm_scale is None:
        sm_scale = 1.0 / (q.shape[-1] ** 0.5)
    scores = torch.matmul(q.float(), k.transpose(-2, -1)) * sm_scale
    attn = torch.softmax(scores, dim=-1)
    return torch.matmul(attn, v)


class RefLayer:
    """One layer of the reference's cache in its own representation: unpacked
    uint8 codes + fp32 scales + uint8 zero-points for the body, fp16 sink and
    recent tail. The groups lie inside a token (group divides 128), so the flat
    scale/zero-point arrays are kept per token, [B, Hkv, T, 128/group], and
    grow along the token axis exactly like the codes."""

    def __init__(self, B, Hkv, body, sink, recent, group=32, seed=0):
        g = torch.Generator().manual_seed(seed)
        kb = torch.randn(B, Hkv, body, 128, generator=g).half()
        vb = torch.randn(B, Hkv, body, 128, generator=g).half()
        self.group = group
        self.kq, self.ks, self.kz = self._compress(kb)
        self.vq, self.vs, self.vz = self._compress(vb)
        self.sink_k = torch.randn(B, Hkv, sink, 128, generator=g).half()
        self.sink_v = torch.randn(B, Hkv, sink, 128, generator=g).half()
        self.tail_k = torch.randn(B, Hkv, recent, 128, generator=g).half()
        self.tail_v = torch.randn(B, Hkv, recent, 128, generator=g).half()

    def _compress(self, x: torch.Tensor):
        q, s, z = compress(x, self.group)
        meta = (*x.shape[:3], x.shape[3] // self.group)
        return q, s.reshape(meta), z.reshape(meta)

    def step(self, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor) -> torch.Tensor:
        """Evict the oldest tail token into INT4 (compress), slide the tail,
        dequantise the body and attend over [body ; sink ; tail]."""
        ek, ev = self.tail_k[:, :, :1], self.tail_v[:, :, :1]
        qk, sk, zk = self._compress(ek)
        qv, sv, zv = self._compress(ev)
        self.kq = torch.cat([self.kq, qk], dim=2)
        self.ks = torch.cat([self.ks, sk], dim=2)
        self.kz = torch.cat([self.kz, zk], dim=2)
        self.vq = torch.cat([self.vq, qv], dim=2)
        self.vs = torch.cat([self.vs, sv], dim=2)
        self.vz = torch.cat([self.vz, zv], dim=2)
        self.tail_k = torch.cat([self.tail_k[:, :, 1:], k_new[:, :, None]], dim=2)
        self.tail_v = torch.cat([self.tail_v[:, :, 1:], v_new[:, :, None]], dim=2)
        kd = decompress(self.kq, self.ks, self.kz, self.group)
        vd = decompress(self.vq, self.vs, self.vz, self.group)
        k = torch.cat([kd, self.sink_k.float(), self.tail_k.float()], dim=2)
        v = torch.cat([vd, self.sink_v.float(), self.tail_v.float()], dim=2)
        return decode_attention(q[:, :, None, :], k, v)[:, :, 0]
