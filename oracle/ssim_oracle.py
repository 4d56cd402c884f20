"""numpy restatement of SSIM and the reference's L1 + SSIM training loss.

TEST INFRASTRUCTURE ONLY: the checker for the SSIM kernels
(3dgs_from_scratch_b200/csrc/ssim.cu). The shipped package never imports it.

The reference computes SSIM with the external fused_ssim package
(environment.yml:56 pins fused-ssim==0.0.0; not vendored, not installed
here), called at scripts/train.py:193-197 with padding="valid". This file
restates the published SSIM definition (Wang et al. 2004) that package
implements, in float64, as direct 11x11 window sums (not separable, so it
is an independent formulation of the kernels' separable passes):
Gaussian window w(i, j) = g(i) g(j), g(k) = exp(-(k-5)^2 / 4.5) / sum,
zero padding, C1 = 0.01^2, C2 = 0.03^2. Parity with fused_ssim itself is
unpinned: no test or fixture of the reference pins fused_ssim values.

The gradient is the analytic one: with A1 = 2 mx my + C1, A2 = 2 sxy + C2,
B1 = mx^2 + my^2 + C1, B2 = sxx + syy + C2, S = A1 A2 / (B1 B2):
  dS/dE[xy] = 2 A1 / (B1 B2),  dS/dE[x^2] = -S / B2,
  dS/dmu_x  = 2 my A2 / (B1 B2) - 2 mx S / B1 - 2 mx dS/dE[x^2] - my dS/dE[xy],
  dL/dx(p)  = sum_q w(q - p) (dL/dS_q) (dS/dmu_x(q) + 2 x(p) dS/dE[x^2](q) + y(p) dS/dE[xy](q)).
tests/test_ssim.py checks it against Torch autograd of a conv2d restatement.
"""
from __future__ import annotations

import numpy as np

C1 = 0.01 ** 2
C2 = 0.03 ** 2
R = 5


def window_1d() -> np.ndarray:
    k = np.arange(2 * R + 1, dtype=np.float64) - R
    g = np.exp(-(k * k) / (2 * 1.5 * 1.5))
    return g / g.sum()


_SEPARABLE = False


def _filter(img: np.ndarray) -> np.ndarray:
    """11x11 window sum with zero padding over the last two axes: direct 2D
    sums by default; row then column passes when _SEPARABLE is set (the
    faster form the CPU baseline of bench.py times)."""
    g = window_1d()
    h, w = img.shape[-2:]
    pad = np.zeros(img.shape[:-2] + (h + 2 * R, w + 2 * R))
    pad[..., R:R + h, R:R + w] = img
    out = np.zeros(img.shape)
    if _SEPARABLE:
        rows = np.zeros(img.shape[:-2] + (h + 2 * R, w))
        for j in range(2 * R + 1):
            rows += g[j] * pad[..., :, j:j + w]
        for i in range(2 * R + 1):
            out += g[i] * rows[..., i:i + h, :]
        return out
    w2 = np.outer(g, g)
    for i in range(2 * R + 1):
        for j in range(2 * R + 1):
            out += w2[i, j] * pad[..., i:i + h, j:j + w]
    return out


def set_separable(on: bool) -> None:
    global _SEPARABLE
    _SEPARABLE = bool(on)


def _mask(shape, valid: bool) -> np.ndarray:
    m = np.zeros(shape, dtype=bool)
    if valid:
        m[..., R:-R, R:-R] = True
    else:
        m[...] = True
    return m


def ssim(img1: np.ndarray, img2: np.ndarray, valid: bool = False, need_grad: bool = False):
    """Mean SSIM of (..., H, W) arrays; with need_grad also d mean / d img1."""
    x = np.asarray(img1, dtype=np.float64)
    y = np.asarray(img2, dtype=np.float64)
    mx, my = _filter(x), _filter(y)
    exx, eyy, exy = _filter(x * x), _filter(y * y), _filter(x * y)
    sxx, syy, sxy = exx - mx * mx, eyy - my * my, exy - mx * my
    a1, a2 = 2 * mx * my + C1, 2 * sxy + C2
    b1, b2 = mx * mx + my * my + C1, sxx + syy + C2
    s = a1 * a2 / (b1 * b2)
    m = _mask(s.shape, valid)
    count = int(m.sum())
    value = float(s[m].sum() / count)
    if not need_grad:
        return value
    wq = m / count
    d_xy = 2 * a1 / (b1 * b2)
    d_xx = -s / b2
    d_mu = 2 * my * a2 / (b1 * b2) - 2 * mx * s / b1 - 2 * mx * d_xx - my * d_xy
    grad = _filter(d_mu * wq) + 2 * x * _filter(d_xx * wq) + y * _filter(d_xy * wq)
    return value, grad


def l1_ssim_loss(raw_hwc: np.ndarray, target_hwc: np.ndarray, ssim_lambda: float):
    """The reference's loss (scripts/train.py:183-203) on a raw blended
    (H, W, 3) image: rendered = clamp(raw, 0, 1) * 255 / 255, target / 255,
    (1 - lambda) L1 + lambda (1 - SSIM_valid). Returns (loss, d loss / d raw)."""
    raw = np.asarray(raw_hwc, dtype=np.float32)
    x = ((np.clip(raw, 0.0, 1.0) * np.float32(255)) / np.float32(255)).astype(np.float64)
    y = np.asarray(target_hwc, dtype=np.float32).astype(np.float64) / 255.0
    d = x - y
    l1 = float(np.abs(d).mean())
    sv, sg = ssim(x.transpose(2, 0, 1), y.transpose(2, 0, 1), valid=True, need_grad=True)
    loss = (1 - ssim_lambda) * l1 + ssim_lambda * (1 - sv)
    gn = (1 - ssim_lambda) * np.sign(d) / d.size - ssim_lambda * sg.transpose(1, 2, 0)
    grad = np.where((raw >= 0) & (raw <= 1), gn, 0.0)
    return loss, grad
