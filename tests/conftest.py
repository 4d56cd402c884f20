import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200); run with -m gpu")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def gs():
    return importlib.import_module("3dgs_from_scratch_b200")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle

    oracle.build()
    return oracle


def golden(name):
    with np.load(os.path.join(GOLDEN, name)) as z:
        return {k: z[k] for k in z.files}


def metric(a, b):
    """cosine similarity and relative L2 error of flattened tensors, as
    scripts/check_cuda_gradients.py:37-44 of the reference computes them."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    cos = float(a @ b) / max(na * nb, 1e-12)
    rel = float(np.linalg.norm(a - b)) / max(nb, 1e-12)
    return cos, rel


def assert_close_metric(name, a, b, min_cos=0.999, max_rel=1e-3):
    """The reference's pass rule (check_cuda_gradients.py:27-30,52)."""
    cos, rel = metric(a, b)
    assert cos >= min_cos and rel <= max_rel, f"{name}: cos={cos:.7f} rel={rel:.3e}"


def torch_ssim(x, y, valid):
    """SSIM of (N, C, H, W) tensors, restated with Torch conv2d (grouped,
    11x11 Gaussian window sigma 1.5, zero padding 5, C1 = 0.01^2,
    C2 = 0.03^2; "valid" crops 5 pixels per border) -- the test-side
    restatement of what scripts/train.py:193-197 gets from fused_ssim."""
    import torch
    import torch.nn.functional as F

    k = torch.arange(11, dtype=torch.float64) - 5
    g = torch.exp(-(k * k) / (2 * 1.5 * 1.5))
    g = (g / g.sum()).to(dtype=x.dtype, device=x.device)
    c = x.shape[1]
    win = torch.outer(g, g).expand(c, 1, 11, 11).contiguous()

    def f(t):
        return F.conv2d(t, win, padding=5, groups=c)

    c1, c2 = 0.01 ** 2, 0.03 ** 2
    mx, my = f(x), f(y)
    sxx = f(x * x) - mx * mx
    syy = f(y * y) - my * my
    sxy = f(x * y) - mx * my
    s = ((2 * mx * my + c1) * (2 * sxy + c2)) / ((mx * mx + my * my + c1) * (sxx + syy + c2))
    if valid:
        s = s[:, :, 5:-5, 5:-5]
    return s.mean()
