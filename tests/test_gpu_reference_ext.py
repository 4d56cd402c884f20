"""Parity with the reference's own CUDA extension (src/cuda/rasterizer.cpp +
kernel.cu compiled by oracle/build_ref.py into oracle/_ref/). Skipped when
that build is absent. Same seeded inputs go to both; integer results must be
identical, float results within the stated tolerances."""
import numpy as np
import pytest
import torch

from conftest import assert_close_metric, metric

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def ref():
    from oracle import build_ref

    mod = build_ref.load_module()
    if mod is None:
        pytest.skip("reference extension not built (oracle/_ref)")
    return mod


def np_(t):
    return t.detach().cpu().numpy()


def scene(gs, cfg_id, n=None, seed=0, W=None, H=None):
    cfg = gs.scenes.CONFIGS[cfg_id]
    raw = gs.scenes.make_gaussians(cfg, seed=seed, n=n)
    act = gs.scenes.activate({k: v.to(DEV) for k, v in raw.items()})
    W = cfg.width if W is None else W
    H = cfg.height if H is None else H
    w2c = gs.scenes.primary_camera(cfg).to(DEV)
    K = gs.scenes.intrinsic_for(cfg, W, H).to(DEV)
    return raw, act, w2c, K, W, H


ARGS = (0.01, 100.0, 1 / 255, 0.5, 128.0)


@pytest.mark.parametrize("cfg_id", [0, 1])
def test_project_points_vs_reference(gs, ref, cfg_id):
    _, a, w2c, K, W, H = scene(gs, cfg_id, n=200_000 if cfg_id == 1 else None)
    inp = (a["means"], a["scales"], a["quaternions"], a["opacities"], w2c, K) + ARGS + (W, H)
    r = ref.project_points(*inp)
    o = gs.cuda_rasterizer.project_points(*inp)
    assert torch.equal(r[5], o[5])  # mask
    exact = {}
    for name, x, y in zip(("points", "depths", "cov", "conic", "radii"), o[:5], r[:5]):
        exact[name] = float((x == y).float().mean())
        assert torch.allclose(x, y, rtol=1e-5, atol=1e-6), name
    print("bit-exact fraction vs reference:", exact)
    assert exact["depths"] == 1.0


@pytest.mark.parametrize("cfg_id", [0, 1])
def test_tile_layout_vs_reference_bit_exact(gs, ref, cfg_id):
    _, a, w2c, K, W, H = scene(gs, cfg_id)
    r = ref.project_points(a["means"], a["scales"], a["quaternions"], a["opacities"], w2c, K, *ARGS,
                           W, H)
    pts, depths, radii, mask = r[0], r[1], r[4], r[5]
    r_off, r_ids = ref.compute_tile_intersection(pts, radii, depths, mask, W, H, 16)
    off, ids = gs.cuda_rasterizer.compute_tile_intersection(pts, radii, depths, mask, W, H, 16)
    assert torch.equal(off, r_off)
    assert torch.equal(ids, r_ids)


def test_rasterize_vs_reference(gs, ref):
    _, a, w2c, K, W, H = scene(gs, 0)
    r = ref.project_points(a["means"], a["scales"], a["quaternions"], a["opacities"], w2c, K, *ARGS,
                           W, H)
    pts, depths, conic, radii, mask = r[0], r[1], r[3], r[4], r[5]
    campos = -w2c[:3, :3].t() @ w2c[:3, 3]
    colors = torch.clamp_min(ref.evaluate_spherical_harmonics(
        campos, a["means"], a["sh_coeffs_dc"], a["sh_coeffs_rest"], mask, False) + 0.5, 0.0)
    off, ids = ref.compute_tile_intersection(pts, radii, depths, mask, W, H, 16)
    args = (off, ids, pts, conic, a["opacities"], colors, W, H, 16, 1e-4, 1e-4, 9.21)
    ri = ref.rasterize(*args)
    oi = gs.cuda_rasterizer.rasterize(*args)
    d = (ri - oi).abs()
    print("rasterize: max |diff|", float(d.max()), "bit-exact fraction", float((d == 0).float().mean()))
    assert float(d.max()) <= 1e-4
    up = torch.randn((H, W, 3), device=DEV, generator=torch.Generator(DEV).manual_seed(2))
    rg = ref.rasterize_backward(up, *args)
    og = gs.cuda_rasterizer.rasterize_backward(up, *args)
    for name, x, y in zip(("points", "conic", "opac", "colors"), og, rg):
        assert_close_metric(name, np_(x), np_(y), 0.99999, 1e-4)


def make_ref_render(ref):
    """The reference composition (src/cuda/wrapper.py:244-294) over the
    reference extension: project_points, SH, +0.5/clamp, tile intersection,
    rasterize, clamp * 255, as three autograd Functions."""

    def ref_render(w2c, K, W, H, means, scales, quats, opac, dc, rest):
        class PP(torch.autograd.Function):
            @staticmethod
            def forward(ctx, means, scales, quats):
                o = ref.project_points(means, scales, quats, opac.detach(), w2c, K, *ARGS, W, H)
                ctx.save_for_backward(means, scales, quats, o[2], o[5])
                return o[0], o[1], o[3], o[4], o[5]

            @staticmethod
            def backward(ctx, gp, gd, gc, gr, gm):
                m, s, q, cov, mask = ctx.saved_tensors
                return ref.project_points_backward(gp.contiguous(), gc.contiguous(), m, s, q,
                                                   opac.detach(), w2c, K, W, H, cov, mask)

        class SH(torch.autograd.Function):
            @staticmethod
            def forward(ctx, campos, means, dc, rest, mask):
                c = ref.evaluate_spherical_harmonics(campos, means, dc, rest, mask, False)
                ctx.save_for_backward(campos, means, dc, rest, c, mask)
                return c

            @staticmethod
            def backward(ctx, g):
                campos, means, dc, rest, c, mask = ctx.saved_tensors
                gm, gdc, grest = ref.evaluate_spherical_harmonics_backward(
                    g.contiguous(), campos, means, dc, rest, c, mask, False)
                return None, gm, gdc, grest, None

        class RS(torch.autograd.Function):
            @staticmethod
            def forward(ctx, off, ids, pts, conic, opac_, colors):
                ctx.save_for_backward(off, ids, pts, conic, opac_, colors)
                return ref.rasterize(off, ids, pts, conic, opac_, colors, W, H, 16, 1e-4, 1e-4,
                                     9.21)

            @staticmethod
            def backward(ctx, g):
                off, ids, pts, conic, opac_, colors = ctx.saved_tensors
                gp, gc, go, gcol = ref.rasterize_backward(g.contiguous(), off, ids, pts, conic,
                                                          opac_, colors, W, H, 16, 1e-4, 1e-4,
                                                          9.21)
                return None, None, gp, gc, go, gcol

        pts, depths, conic, radii, mask = PP.apply(means, scales, quats)
        campos = -w2c[:3, :3].t() @ w2c[:3, 3]
        colors = torch.clamp_min(SH.apply(campos, means, dc, rest, mask) + 0.5, 0.0)
        off, ids = ref.compute_tile_intersection(pts.detach(), radii, depths, mask, W, H, 16)
        img = RS.apply(off, ids, pts, conic, opac, colors)
        return img.clamp(0, 1) * 255, pts, radii

    return ref_render


def l1_loss(img, target):
    return torch.nn.functional.l1_loss(img, target)


def l1_ssim_loss(img, target, lam=0.2):
    """scripts/train.py:187-205 after its SSIM warm-up: (1 - lam) L1 +
    lam (1 - SSIM "valid") on the [0, 1] images. fused_ssim is absent here;
    both renderers get the same SSIM (the Torch conv2d restatement), so the
    comparison isolates the rasterizers' gradients."""
    from conftest import torch_ssim

    rn, tn = img / 255.0, target / 255.0
    l1 = torch.nn.functional.l1_loss(rn, tn)
    ss = torch_ssim(rn.permute(2, 0, 1).unsqueeze(0), tn.permute(2, 0, 1).unsqueeze(0), True)
    return (1 - lam) * l1 + lam * (1 - ss)


def compare_fwd_bwd(gs, ref, raw, w2c, K, W, H, loss_fn=l1_loss, seed=3, image_tol=1e-4,
                    max_frac_over=0.0):
    """render() against the reference composition on identical inputs:
    activations in Torch, forward, the loss against a seeded uniform target,
    backward through both. The image must agree within image_tol on [0, 1]
    (with at most max_frac_over of its values above it), radii > 0 must
    agree, and every raw-parameter gradient plus points_img.grad must pass the
    reference's rule (cos >= 0.999, rel <= 1e-3;
    scripts/check_cuda_gradients.py:27-44). Returns the metrics."""
    target = torch.rand((H, W, 3), device=DEV, generator=torch.Generator(DEV).manual_seed(seed))
    target = target * 255

    def run(render):
        p = {k: v.to(DEV).clone().requires_grad_(True) for k, v in raw.items()}
        act = gs.scenes.activate(p)
        img, pts, radii = render(w2c, K, W, H, act["means"], act["scales"], act["quaternions"],
                                 act["opacities"], act["sh_coeffs_dc"], act["sh_coeffs_rest"])
        pts.retain_grad()
        loss_fn(img, target).backward()
        torch.cuda.synchronize()
        out = (img.detach() / 255.0, {k: np_(v.grad) for k, v in p.items()}, np_(pts.grad),
               radii.detach())
        del p, act, img, pts
        return out

    ri, rg, rp, rr = run(make_ref_render(ref))
    oi, og, op, orr = run(gs.render)
    d = (ri - oi).abs()
    over = float((d > image_tol).float().mean())
    print(f"render {W}x{H}: max |diff| on [0,1] {float(d.max()):.3e}, fraction > {image_tol}: "
          f"{over:.2e}")
    assert over <= max_frac_over and float(d.max()) < 1e-2
    assert torch.equal(rr > 0, orr > 0)
    res = {}
    for k in rg:
        res[k] = metric(og[k], rg[k])
        assert_close_metric(k, og[k], rg[k], 0.999, 1e-3)
    res["points_img"] = metric(op, rp)
    assert_close_metric("points_img.grad", op, rp, 0.999, 1e-3)
    print({k: (round(c, 7), f"{r:.2e}") for k, (c, r) in res.items()})
    return res


@pytest.mark.parametrize("cfg_id,n,W,H", [(0, None, None, None), (1, 300_000, 640, 360)])
def test_render_end_to_end_vs_reference(gs, ref, cfg_id, n, W, H):
    raw, _, w2c, K, W, H = scene(gs, cfg_id, n=n, W=W, H=H)
    compare_fwd_bwd(gs, ref, raw, w2c, K, W, H, max_frac_over=1e-5)


def test_cfg1_full_size_fwd_bwd_vs_reference(gs, ref):
    """Configuration 1 at full size (1M SH3 Gaussians, 1920x1080, L1 against a
    uniform target): image, all six raw-parameter gradients and
    points_img.grad against the reference extension."""
    raw, _, w2c, K, W, H = scene(gs, 1)
    compare_fwd_bwd(gs, ref, raw, w2c, K, W, H)


def test_cfg2_view_fwd_bwd_with_ssim_vs_reference(gs, ref):
    """One view of configuration 2 (3M Gaussians in [-5, 5]^3, 1600x1064,
    f = 1200, a camera on the radius-10 sphere) with the training loss
    0.8 L1 + 0.2 (1 - SSIM)."""
    cfg = gs.scenes.CONFIGS[2]
    raw = gs.scenes.make_gaussians(cfg, seed=0)
    w2c = gs.scenes.orbit_cameras(cfg, 4, sphere=True)[1].to(DEV)
    K = gs.scenes.intrinsic_for(cfg).to(DEV)
    compare_fwd_bwd(gs, ref, raw, w2c, K, cfg.width, cfg.height, loss_fn=l1_ssim_loss)


def test_cfg3_fwd_bwd_vs_reference(gs, ref):
    """Configuration 3 (2M clustered Gaussians, ~50 tiles each, 3840x2160,
    ~10^8 pairs), forward and backward."""
    raw, _, w2c, K, W, H = scene(gs, 3)
    compare_fwd_bwd(gs, ref, raw, w2c, K, W, H)


def test_cfg3_stress_layout_and_image_vs_reference(gs, ref):
    """Configuration 3 (2M Gaussians in 64 clusters, ~50 tiles per Gaussian,
    3840x2160, ~10^8 pairs): the reference's layout and image, bit for bit."""
    _, a, w2c, K, W, H = scene(gs, 3)
    r = ref.project_points(a["means"], a["scales"], a["quaternions"], a["opacities"], w2c, K, *ARGS,
                           W, H)
    o = gs.cuda_rasterizer.project_points(a["means"], a["scales"], a["quaternions"],
                                          a["opacities"], w2c, K, *ARGS, W, H)
    assert torch.equal(r[5], o[5])
    for x, y in zip(o[:5], r[:5]):
        assert torch.equal(x, y)
    pts, depths, conic, radii, mask = r[0], r[1], r[3], r[4], r[5]
    r_off, r_ids = ref.compute_tile_intersection(pts, radii, depths, mask, W, H, 16)
    off, ids = gs.cuda_rasterizer.compute_tile_intersection(pts, radii, depths, mask, W, H, 16)
    print("cfg3 pairs:", ids.numel())
    assert ids.numel() > 50_000_000
    assert torch.equal(off, r_off)
    assert torch.equal(ids, r_ids)
    del r_ids
    colors = torch.rand((pts.shape[0], 3), device=DEV, generator=torch.Generator(DEV).manual_seed(4))
    args = (off, ids, pts, conic, a["opacities"], colors, W, H, 16, 1e-4, 1e-4, 9.21)
    ri = ref.rasterize(*args)
    oi = gs.cuda_rasterizer.rasterize(*args)
    assert torch.equal(ri, oi)


def test_cfg3_fused_render_forward_vs_reference(gs, ref):
    """render()'s fused path on configuration 3 against the reference
    composition (forward)."""
    raw, a, w2c, K, W, H = scene(gs, 3)
    with torch.no_grad():
        img, pts, radii = gs.render(w2c, K, W, H, a["means"], a["scales"], a["quaternions"],
                                    a["opacities"], a["sh_coeffs_dc"], a["sh_coeffs_rest"])
        r = ref.project_points(a["means"], a["scales"], a["quaternions"], a["opacities"], w2c, K,
                               *ARGS, W, H)
        campos = -w2c[:3, :3].t() @ w2c[:3, 3]
        colors = torch.clamp_min(ref.evaluate_spherical_harmonics(
            campos, a["means"], a["sh_coeffs_dc"], a["sh_coeffs_rest"], r[5], False) + 0.5, 0.0)
        off, ids = ref.compute_tile_intersection(r[0], r[4], r[1], r[5], W, H, 16)
        ri = ref.rasterize(off, ids, r[0], r[3], a["opacities"], colors, W, H, 16, 1e-4, 1e-4, 9.21)
        ri = ri.clamp(0, 1) * 255
    assert torch.equal(radii, r[4]) and torch.equal(pts, r[0])
    d = (img - ri).abs() / 255.0
    assert float(d.max()) <= 1e-4, float(d.max())
