"""Device-side chunk scoring for the prefetch policy: which INT4 pages deserve
prefetching, decided without a host synchronisation.

* ``compute_block_scores`` — the reference's block means of accumulated token
  scores (src/kernels/oracle_triton.py:53-79), in torch on the tensor's device.
* ``page_scores`` — attention mass per page, from the per-tile mass that
  ``kvstore.decode_scored`` returns next to the attention output.
* ``DeviceWindowController`` — the window formula of AdaptivePrefetchController
  (src/policy/adaptive_prefetch_controller.py:58-127) with its state on the
  device: the spread of the attention vector, the EMA reference, the miss-rate
  history, the clamp and the one-step smoothing stay tensors, so the window
  never has to reach the host (the reference calls ``.cpu()`` on the attention
  vector every step, adaptive_prefetch_controller.py:104).
* ``select_pages`` — the top-w pages per (sequence, KV head), as the top-w_max
  ranking plus a device mask of the first w.
"""
from __future__ import annotations

from typing import Optional, Tuple, Union

import torch


def compute_block_scores(token_scores: torch.Tensor, current_seq_len: int, block_size: int) -> torch.Tensor:
    """Mean score of each block of ``block_size`` consecutive tokens over the first
    ``current_seq_len`` entries of ``token_scores`` (the last block may be
    partial). Same contract as the reference (oracle_triton.py:53-79)."""
    n = int(current_seq_len)
    nblocks = (n + block_size - 1) // block_size
    if block_size == 1:
        return token_scores[:n].clone()
    x = token_scores[:n]
    pad = nblocks * block_size - n
    if pad:
        x = torch.cat([x, x.new_zeros(pad)])
    sums = x.view(nblocks, block_size).sum(dim=1)
    counts = torch.full((nblocks,), float(block_size), dtype=sums.dtype, device=sums.device)
    if pad:
        counts[-1] = block_size - pad
    return sums / counts


def page_scores(tile_mass: torch.Tensor, tiles_per_page: int) -> torch.Tensor:
    """[B, Hkv, tiles] attention mass per 128-token tile -> [B, Hkv, pages] per page."""
    B, H, T = tile_mass.shape
    P = (T + tiles_per_page - 1) // tiles_per_page
    pad = P * tiles_per_page - T
    if pad:
        tile_mass = torch.cat([tile_mass, tile_mass.new_zeros(B, H, pad)], dim=2)
    return tile_mass.view(B, H, P, tiles_per_page).sum(dim=3)


def select_pages(scores: torch.Tensor, w_max: int, w: Union[int, torch.Tensor]) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top ``w_max`` pages of ``scores`` [..., pages] (indices, by descending score)
    and a mask of the first ``w`` of them (``w`` may be a device tensor)."""
    k = min(w_max, scores.shape[-1])
    idx = torch.topk(scores, k, dim=-1).indices
    rank = torch.arange(k, device=scores.device)
    mask = rank < (w if isinstance(w, torch.Tensor) else torch.tensor(w, device=scores.device))
    return idx, mask.expand_as(idx)


class DeviceWindowController:
    """Prefetch window w_t = w_min + clip((sigma_t / sigma_ref - 1) alpha, -d_max, d_max)
    + beta * miss_rate * w_max, rounded, clamped to [w_min, w_max], moved by at
    most one per step; sigma_t is the standard deviation of the latest attention
    vector and sigma_ref its EMA (the first sigma seeds it). Same parameters and
    arithmetic as the reference controller; every quantity that depends on
    device data stays on the device."""

    def __init__(self, w_min: int = 2, w_max: int = 8, alpha: float = 1.5, beta: float = 0.5,
                 delta_max: float = 2.0, ema_decay: float = 0.9, miss_window_size: int = 16,
                 device: Union[str, torch.device] = "cuda"):
        self.w_min, self.w_max = w_min, w_max
        self.alpha, self.beta = alpha, beta
        self.delta_max, self.ema_decay = delta_max, ema_decay
        self.miss_window_size = miss_window_size
        self.device = torch.device(device)
        self._w = torch.tensor(float(w_min), dtype=torch.float32, device=self.device)
        self._sigma_ref = torch.zeros((), dtype=torch.float32, device=self.device)
        self._sigma_ref_initialized = False
        self._misses = torch.zeros(miss_window_size, dtype=torch.float32, device=self.device)
        self._n_miss = 0  # entries in the history (host-known: one per step)
        self._step = 0

    def compute_window(self, attention_weights: Optional[torch.Tensor] = None,
                       cache_miss: Union[bool, torch.Tensor] = False) -> torch.Tensor:
        """The window for this step, as a 0-d int64 tensor on the device."""
        # the last miss_window_size misses in a ring (their mean does not depend on order)
        miss = cache_miss.to(self.device, torch.float32) if isinstance(cache_miss, torch.Tensor) else float(cache_miss)
        self._misses[self._step % self.miss_window_size] = miss
        self._step += 1
        self._n_miss = min(self._step, self.miss_window_size)
        miss_rate = self._misses[:self._n_miss].mean()

        delta = torch.zeros((), dtype=torch.float32, device=self.device)
        if attention_weights is not None and attention_weights.numel() > 1:
            sigma_t = attention_weights.detach().float().std()
            if not self._sigma_ref_initialized:
                self._sigma_ref = sigma_t.clone()
                self._sigma_ref_initialized = True
            else:
                self._sigma_ref = self.ema_decay * self._sigma_ref + (1 - self.ema_decay) * sigma_t
            dev = torch.where(self._sigma_ref > 1e-8, sigma_t / self._sigma_ref.clamp_min(1e-30) - 1.0,
                              torch.zeros_like(sigma_t))
            delta = (dev * self.alpha).clamp(-self.delta_max, self.delta_max)

        raw = self.w_min + delta + self.beta * miss_rate * self.w_max
        w_new = torch.round(raw).clamp(self.w_min, self.w_max)
        step = w_new - self._w
        w_new = torch.where(step.abs() > 1, self._w + torch.sign(step), w_new)
        self._w = w_new
        return w_new.to(torch.int64)

    @property
    def current_w(self) -> torch.Tensor:
        return self._w
