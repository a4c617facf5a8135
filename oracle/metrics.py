"""Parity metrics — TEST INFRASTRUCTURE ONLY (imported by tests/, smoke() and bench.py's
baseline legs; never by the product path).

`ssim_uniform` restates the reference's noise_pred / VAE SSIM (src/tests/test_unet.cu:161-200):
7x7 uniform windows centred every 3 pixels (stride = half window) in each channel plane,
C1 = (0.01 L)^2, C2 = (0.03 L)^2 with L the joint value range of both tensors, fp64 statistics,
mean over all windows of all planes.
"""
from __future__ import annotations

import numpy as np


def ssim_uniform(a, b) -> float:
    """a, b: arrays [..., H, W] (leading dims are flattened into planes)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    H, W = a.shape[-2:]
    a = a.reshape(-1, H, W)
    b = b.reshape(-1, H, W)
    lo = min(a.min(), b.min())
    hi = max(a.max(), b.max())
    L = hi - lo
    C1 = (0.01 * L) ** 2
    C2 = (0.03 * L) ** 2
    win, half = 7, 3
    ys = np.arange(half, H - half, half)
    xs = np.arange(half, W - half, half)
    if len(ys) == 0 or len(xs) == 0:
        return 0.0
    inv = 1.0 / (win * win)

    def box(x):
        # window sums at every (y, x) centre via a 2D cumulative sum
        c = np.cumsum(np.cumsum(np.pad(x, ((0, 0), (1, 0), (1, 0))), axis=1), axis=2)
        y0, y1 = ys - half, ys + half + 1
        x0, x1 = xs - half, xs + half + 1
        return (c[:, y1][:, :, x1] - c[:, y0][:, :, x1] - c[:, y1][:, :, x0] + c[:, y0][:, :, x0])

    sa, sb = box(a), box(b)
    saa, sbb, sab = box(a * a), box(b * b), box(a * b)
    mu_a, mu_b = sa * inv, sb * inv
    va = saa * inv - mu_a * mu_a
    vb = sbb * inv - mu_b * mu_b
    cov = sab * inv - mu_a * mu_b
    s = ((2 * mu_a * mu_b + C1) * (2 * cov + C2)) / ((mu_a * mu_a + mu_b * mu_b + C1) * (va + vb + C2))
    return float(s.mean())


def max_rel_err(got, ref) -> float:
    """max |got - ref| / max |ref| (the per-layer parity metric)."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    d = np.abs(ref).max()
    e = np.abs(got - ref).max()
    return float(e / d) if d > 0 else float(e)
