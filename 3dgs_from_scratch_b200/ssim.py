"""SSIM with its gradient on this library's kernels (fused_ssim's interface).

The reference trains and evaluates with `fused_ssim(img1, img2,
padding="valid")` from the external fused_ssim package
(scripts/train.py:193-197, scripts/evaluate.py:57-61), on (1, C, H, W)
images in [0, 1]. `fused_ssim` here takes the same arguments and returns the
same quantity: the mean SSIM map (11x11 Gaussian window, sigma 1.5,
C1 = 0.01^2, C2 = 0.03^2, zero padding) over every pixel ("same") or over
the pixels at least 5 from every border ("valid"), differentiable w.r.t.
img1. Both kernels (gs_ssim_forward / gs_ssim_backward) run on the current
stream with no host synchronisation.
"""
from __future__ import annotations

import torch

from . import _native as nat


def _check(img1, img2):
    if img1.dim() != 4 or img1.shape != img2.shape:
        raise ValueError("fused_ssim expects two (N, C, H, W) tensors of the same shape")
    if not img1.is_cuda or img1.device != img2.device:
        raise ValueError("fused_ssim runs on CUDA tensors of one device")


class _FusedSSIM(torch.autograd.Function):
    @staticmethod
    def forward(ctx, img1, img2, valid):
        _check(img1, img2)
        a = img1.detach().to(torch.float32).contiguous()
        b = img2.detach().to(torch.float32).contiguous()
        n, c, h, w = a.shape
        planes = n * c
        dev = a.device
        scratch = torch.empty(nat.query("gs_ssim_scratch_bytes", planes, h, w) // 4,
                              dtype=torch.float32, device=dev)
        total = torch.zeros(1, dtype=torch.float64, device=dev)
        nat.call("gs_ssim_forward", planes, h, w, a.data_ptr(), b.data_ptr(), int(valid),
                 scratch.data_ptr(), scratch.numel() * 4, total.data_ptr(), nat.stream_ptr(dev))
        count = planes * ((h - 10) * (w - 10) if valid else h * w)
        ctx.save_for_backward(a, b, scratch)
        ctx.dtype = img1.dtype
        return (total / count).to(torch.float32).reshape(())

    @staticmethod
    def backward(ctx, grad_out):
        a, b, scratch = ctx.saved_tensors
        n, c, h, w = a.shape
        g = grad_out.detach().to(device=a.device, dtype=torch.float32).reshape(1).contiguous()
        grad = torch.empty_like(a)
        nat.call("gs_ssim_backward", n * c, h, w, a.data_ptr(), b.data_ptr(), scratch.data_ptr(),
                 g.data_ptr(), grad.data_ptr(), nat.stream_ptr(a.device))
        return grad.to(ctx.dtype), None, None


def fused_ssim(img1: torch.Tensor, img2: torch.Tensor, padding: str = "same",
               train: bool = True) -> torch.Tensor:
    """Mean SSIM of img1 against img2, both (N, C, H, W); gradient w.r.t.
    img1. padding is "same" or "valid"; `train` is accepted for interface
    compatibility (the forward always keeps what the backward needs)."""
    if padding not in ("same", "valid"):
        raise ValueError("padding must be 'same' or 'valid'")
    return _FusedSSIM.apply(img1, img2, padding == "valid")
