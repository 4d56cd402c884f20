"""SSIM and the L1 + SSIM training loss.

The reference takes SSIM from the external fused_ssim package, which is not
in this image and has no golden values in the reference's tests, so parity
with fused_ssim itself is unpinned. The chain checked here:
  * CPU: the numpy oracle (direct 11x11 window sums, analytic gradient)
    against Torch autograd of an independent conv2d restatement, in float64;
  * GPU: the kernels (separable, fp32) against the oracle on small ragged
    images, and against a Torch fp32 conv2d restatement at config 2's
    1600x1064 view size.
"""
import importlib

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from conftest import assert_close_metric, torch_ssim
from oracle import ssim_oracle


def torch_loss(raw, target, lam):
    """scripts/train.py:183-203 on a raw (H, W, 3) image (wrapper.py:294)."""
    rendered = raw.clamp(0, 1) * 255
    rn = rendered / 255.0
    tn = target / 255.0
    l1 = F.l1_loss(rn, tn)
    ss = torch_ssim(rn.permute(2, 0, 1).unsqueeze(0), tn.permute(2, 0, 1).unsqueeze(0), True)
    return (1 - lam) * l1 + lam * (1 - ss)


# ---- CPU: the oracle pinned against Torch autograd -------------------------

@pytest.mark.parametrize("valid", [False, True])
def test_oracle_ssim_matches_torch_autograd(valid):
    rng = np.random.default_rng(3)
    x = rng.uniform(0, 1, (2, 3, 23, 30))
    y = np.clip(x + rng.normal(0, 0.1, x.shape), 0, 1)
    val, grad = ssim_oracle.ssim(x, y, valid=valid, need_grad=True)
    xt = torch.tensor(x, requires_grad=True)
    ref = torch_ssim(xt, torch.tensor(y), valid)
    ref.backward()
    assert abs(val - ref.item()) < 1e-12
    np.testing.assert_allclose(grad, xt.grad.numpy(), rtol=1e-9, atol=1e-14)


def test_oracle_ssim_identity():
    x = np.random.default_rng(4).uniform(0, 1, (1, 3, 20, 20))
    val, grad = ssim_oracle.ssim(x, x, valid=True, need_grad=True)
    assert abs(val - 1.0) < 1e-12
    assert np.abs(grad).max() < 1e-10


@pytest.mark.parametrize("lam", [0.0, 0.2, 1.0])
def test_oracle_loss_matches_torch_autograd(lam):
    rng = np.random.default_rng(5)
    raw = rng.uniform(-0.2, 1.2, (19, 27, 3)).astype(np.float32)
    tgt = rng.integers(0, 256, (19, 27, 3)).astype(np.float32)
    loss, grad = ssim_oracle.l1_ssim_loss(raw, tgt, lam)
    rt = torch.tensor(raw.astype(np.float64), requires_grad=True)
    ref = torch_loss(rt, torch.tensor(tgt, dtype=torch.float64), lam)
    ref.backward()
    assert abs(loss - ref.item()) < 1e-9
    np.testing.assert_allclose(grad, rt.grad.numpy(), rtol=1e-6, atol=1e-12)


# ---- GPU: the kernels ---------------------------------------------------------

@pytest.fixture(scope="module")
def ssim_mod():
    return importlib.import_module("3dgs_from_scratch_b200.ssim")


@pytest.mark.gpu
@pytest.mark.parametrize("shape", [(1, 3, 64, 80), (2, 3, 37, 45), (1, 1, 11, 11), (1, 2, 16, 33)])
@pytest.mark.parametrize("padding", ["same", "valid"])
def test_fused_ssim_vs_oracle(ssim_mod, shape, padding):
    rng = np.random.default_rng(sum(shape))
    x = rng.uniform(0, 1, shape).astype(np.float32)
    y = np.clip(x + rng.normal(0, 0.15, shape), 0, 1).astype(np.float32)
    val, grad = ssim_oracle.ssim(x, y, valid=padding == "valid", need_grad=True)
    xt = torch.tensor(x, device="cuda", requires_grad=True)
    out = ssim_mod.fused_ssim(xt, torch.tensor(y, device="cuda"), padding=padding)
    (out * 2.0).backward()
    assert abs(out.item() - val) < 2e-6
    assert_close_metric("ssim grad", xt.grad.cpu().numpy(), 2.0 * grad, min_cos=0.99999,
                        max_rel=1e-4)


@pytest.mark.gpu
def test_fused_ssim_identity_and_rejects_small_valid(ssim_mod):
    x = torch.rand(1, 3, 50, 70, device="cuda", requires_grad=True)
    out = ssim_mod.fused_ssim(x, x.detach().clone(), padding="valid")
    out.backward()
    assert abs(out.item() - 1.0) < 1e-5
    assert x.grad.abs().max().item() < 1e-6
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    with pytest.raises(nat.NativeError):
        ssim_mod.fused_ssim(torch.rand(1, 3, 10, 40, device="cuda"),
                            torch.rand(1, 3, 10, 40, device="cuda"), padding="valid")


def _loss_native(raw, target, lam):
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    H, W, _ = raw.shape
    dev = raw.device
    scratch = torch.empty(nat.query("gs_ssim_scratch_bytes", 3, H, W) // 4, device=dev)
    sums = torch.zeros(2, dtype=torch.float64, device=dev)
    grad = torch.empty_like(raw)
    nat.call("gs_l1_ssim_loss_grad", H, W, raw.data_ptr(), target.data_ptr(),
             int(target.dtype == torch.uint8), lam, grad.data_ptr(), sums.data_ptr(),
             scratch.data_ptr(), scratch.numel() * 4, nat.stream_ptr(dev))
    s = sums.cpu().numpy()
    loss = (1 - lam) * s[0] / raw.numel() + lam * (1 - s[1] / (3 * (H - 10) * (W - 10)))
    return loss, grad


@pytest.mark.gpu
@pytest.mark.parametrize("u8", [True, False])
@pytest.mark.parametrize("lam", [0.0, 0.2, 1.0])
def test_l1_ssim_loss_grad_vs_oracle(u8, lam):
    rng = np.random.default_rng(int(u8) * 10 + int(lam * 10))
    H, W = 45, 67
    raw = rng.uniform(-0.2, 1.2, (H, W, 3)).astype(np.float32)
    tgt = rng.integers(0, 256, (H, W, 3)).astype(np.uint8)
    loss_o, grad_o = ssim_oracle.l1_ssim_loss(raw, tgt.astype(np.float32), lam)
    t = torch.tensor(tgt if u8 else tgt.astype(np.float32), device="cuda")
    loss, grad = _loss_native(torch.tensor(raw, device="cuda"), t, lam)
    assert abs(loss - loss_o) < 2e-6
    assert_close_metric("loss grad", grad.cpu().numpy(), grad_o, min_cos=0.99999, max_rel=1e-4)


@pytest.mark.gpu
def test_l1_ssim_loss_grad_config2_size():
    """Config 2's view size (1600 x 1064) against Torch fp32 autograd of the
    reference's loss expression (conv2d restatement of SSIM)."""
    g = torch.Generator(device="cuda").manual_seed(11)
    H, W = 1064, 1600
    raw = torch.rand((H, W, 3), device="cuda", generator=g) * 1.2 - 0.1
    tgt = (torch.rand((H, W, 3), device="cuda", generator=g) * 255).round().to(torch.uint8)
    loss, grad = _loss_native(raw, tgt, 0.2)
    rt = raw.clone().requires_grad_(True)
    ref = torch_loss(rt, tgt.float(), 0.2)
    ref.backward()
    assert abs(loss - ref.item()) < 1e-5
    assert_close_metric("loss grad", grad.cpu().numpy(), rt.grad.cpu().numpy(),
                        min_cos=0.9999, max_rel=1e-3)
