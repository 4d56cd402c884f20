"""Golden vectors for the device densification (DeviceStrategy) from the
reference's own Strategy (src/strategy.py), run on the CPU.

Run where the reference checkout is present (its path in $GS_REFERENCE_ROOT,
or a directory named "reference" beside the repository); the .npz files it
writes are committed and the tests never read the reference at run time.

Each case: a seeded set of Gaussians with torch.optim.Adam states after two
optimizer steps (the per-group learning rates and eps of
scripts/train.py:17-44), a few views' points_img gradients and radii fed
through Strategy.adjust at non-refining steps, then one adjust call at a
refining step. Recorded: the inputs, every view, the parameters and Adam
moments after the call, and the normal samples the reference drew for the
splits (its torch.randn call is intercepted), so a test can hand the same
samples to the device kernels.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("GS_REFERENCE_ROOT") or os.path.join(os.path.dirname(REPO), "reference")
GROUPS = ("means", "scales", "quaternions", "opacities", "sh_coeffs_dc", "sh_coeffs_rest")
LRS = {"means": 1.6e-4, "scales": 5e-3, "quaternions": 1e-3, "opacities": 5e-2,
       "sh_coeffs_dc": 2.5e-3, "sh_coeffs_rest": 2.5e-3 / 20}


def load_strategy():
    sys.path.insert(0, REF)
    from src.strategy import Strategy  # noqa: E402

    return Strategy


def make_case(seed, n, step, max_gaussians=None):
    Strategy = load_strategy()
    g = torch.Generator().manual_seed(seed)
    params = {
        "means": torch.rand(n, 3, generator=g) * 2 - 1,
        # log-scales around the split threshold log(0.01), some above log(0.1)
        "scales": torch.randn(n, 3, generator=g) * 1.2 + np.log(0.01),
        "quaternions": torch.randn(n, 4, generator=g),
        # opacity logits, some below logit(0.005)
        "opacities": torch.randn(n, generator=g) * 2.5,
        "sh_coeffs_dc": torch.randn(n, 3, generator=g) * 0.3,
        "sh_coeffs_rest": torch.randn(n, 15, 3, generator=g) * 0.05,
    }
    learnable = {k: torch.nn.Parameter(v.clone()) for k, v in params.items()}
    opts = {k: torch.optim.Adam([learnable[k]], lr=LRS[k], eps=1e-15) for k in GROUPS}
    for _ in range(2):
        for k in GROUPS:
            learnable[k].grad = torch.randn(learnable[k].shape, generator=g) * 0.01
            opts[k].step()
            opts[k].zero_grad()
    before = {k: learnable[k].detach().clone() for k in GROUPS}
    m0 = {k: opts[k].state[learnable[k]]["exp_avg"].clone() for k in GROUPS}
    v0 = {k: opts[k].state[learnable[k]]["exp_avg_sq"].clone() for k in GROUPS}

    strat = Strategy()
    if max_gaussians is not None:
        strat.max_gaussians = max_gaussians
    W, H = 160, 120
    views = []
    draws = []
    real_randn = torch.randn

    def randn(*a, **k):
        out = real_randn(*a, **k)
        draws.append(out.clone())
        return out

    for s in range(step - 3, step + 1):
        pts = torch.zeros(n, 2, requires_grad=True)
        pts.grad = torch.randn(n, 2, generator=g) * 2e-6 * torch.rand(n, 1, generator=g) * 3
        radii = torch.rand(n, 2, generator=g) * 5
        radii[torch.rand(n, generator=g) < 0.2] = 0.0
        views.append((pts.grad.clone(), radii.clone()))
        torch.randn = randn
        try:
            strat.adjust(learnable, opts, pts, radii, W, H, s)
        finally:
            torch.randn = real_randn
    after = {k: learnable[k].detach().clone() for k in GROUPS}
    m1 = {k: opts[k].state[learnable[k]]["exp_avg"].clone() for k in GROUPS}
    v1 = {k: opts[k].state[learnable[k]]["exp_avg_sq"].clone() for k in GROUPS}
    out = {"n": n, "step": step, "width": W, "height": H,
           "max_gaussians": strat.max_gaussians,
           "view_grads": np.stack([v[0].numpy() for v in views]),
           "view_radii": np.stack([v[1].numpy() for v in views]),
           "probe": draws[-1].numpy() if draws else np.zeros((2, 0, 3), np.float32)}
    for k in GROUPS:
        out["before_" + k] = before[k].numpy()
        out["m_before_" + k] = m0[k].numpy()
        out["v_before_" + k] = v0[k].numpy()
        out["after_" + k] = after[k].numpy()
        out["m_after_" + k] = m1[k].numpy()
        out["v_after_" + k] = v1[k].numpy()
    return out


def main():
    cases = {"densify_step600.npz": (11, 500, 600, None),
             "densify_step3000.npz": (12, 500, 3000, None),
             "densify_step3100.npz": (13, 500, 3100, None)}
    for name, (seed, n, step, cap) in cases.items():
        out = make_case(seed, n, step, cap)
        np.savez_compressed(os.path.join(HERE, name), **out)
        print(name, {k: out["after_" + k].shape for k in ("means",)}, "splits",
              out["probe"].shape[1])


if __name__ == "__main__":
    main()
