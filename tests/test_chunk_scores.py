"""Device-side prefetch-policy pieces (policy/chunk_scores.py) on CPU tensors:
block means against a loop, page sums, the top-w selection mask, and the
device-state window controller against a scalar restatement of the window
formula (w_t = w_min + clip((sigma_t/sigma_ref - 1) alpha, -d, d) + beta
miss_rate w_max, rounded half-even, clamped, moved at most one per step)."""
import math
import random

import numpy as np
import pytest
import torch

from hetero_kvcache_optimizer_b200.policy.chunk_scores import (DeviceWindowController, compute_block_scores,
                                                               page_scores, select_pages)


@pytest.mark.parametrize("n,bs", [(1, 1), (7, 1), (100, 16), (128, 32), (129, 32), (1000, 256)])
def test_block_means(n, bs):
    x = torch.rand(1024, dtype=torch.float32, generator=torch.Generator().manual_seed(n))
    got = compute_block_scores(x, n, bs)
    want = [float(x[i:min(i + bs, n)].mean()) for i in range(0, n, bs)]
    assert got.shape == (len(want),)
    np.testing.assert_allclose(got.numpy(), want, rtol=1e-6)


def test_page_scores_and_selection():
    m = torch.rand(2, 3, 7, generator=torch.Generator().manual_seed(1))
    p = page_scores(m, 2)
    assert p.shape == (2, 3, 4)
    torch.testing.assert_close(p[..., :3], m[..., :6].view(2, 3, 3, 2).sum(-1))
    torch.testing.assert_close(p[..., 3], m[..., 6])
    idx, mask = select_pages(p, 3, torch.tensor(2))
    assert idx.shape == (2, 3, 3) and mask.shape == (2, 3, 3)
    assert mask[..., :2].all() and not mask[..., 2].any()
    top = torch.sort(p, dim=-1, descending=True).values[..., :3]
    torch.testing.assert_close(torch.gather(p, -1, idx), top)


class _ScalarWindow:
    """The window formula with Python floats (test oracle)."""

    def __init__(self, w_min, w_max, alpha, beta, delta_max, ema_decay, miss_window):
        self.a = (w_min, w_max, alpha, beta, delta_max, ema_decay, miss_window)
        self.w, self.ref, self.init, self.hist = float(w_min), 0.0, False, []

    def step(self, att, miss):
        w_min, w_max, alpha, beta, dmax, decay, nwin = self.a
        self.hist = (self.hist + [miss])[-nwin:]
        rate = sum(self.hist) / len(self.hist)
        delta = 0.0
        if att is not None and len(att) > 1:
            s = float(np.std(att, ddof=1))
            self.ref = s if not self.init else decay * self.ref + (1 - decay) * s
            self.init = True
            dev = s / self.ref - 1.0 if self.ref > 1e-8 else 0.0
            delta = max(-dmax, min(dmax, dev * alpha))
        w = max(w_min, min(w_max, round(w_min + delta + beta * rate * w_max)))
        if abs(w - self.w) > 1:
            w = int(self.w + math.copysign(1, w - self.w))
        self.w = float(w)
        return int(w)


def test_device_window_controller_matches_formula():
    rnd = random.Random(5)
    args = (2, 8, 1.5, 0.5, 2.0, 0.9, 4)
    ctl = DeviceWindowController(*args, device="cpu")
    ref = _ScalarWindow(*args)
    for t in range(60):
        scale = 10 ** rnd.uniform(-3, 0)
        att = None if t % 11 == 5 else np.abs(np.random.default_rng(t).standard_normal(257)) * scale
        miss = rnd.random() < 0.3
        got = ctl.compute_window(None if att is None else torch.from_numpy(att).float(), miss)
        assert got.dtype == torch.int64 and got.dim() == 0
        assert int(got) == ref.step(None if att is None else att.astype(np.float32).astype(np.float64), miss), t
