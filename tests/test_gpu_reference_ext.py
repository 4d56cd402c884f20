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


@pytest.mark.parametrize("cfg_id,n,W,H", [(0, None, None, None), (1, 300_000, 640, 360)])
def test_render_end_to_end_vs_reference(gs, ref, cfg_id, n, W, H):
    raw, _, w2c, K, W, H = scene(gs, cfg_id, n=n, W=W, H=H)
    target = torch.rand((H, W, 3), device=DEV, generator=torch.Generator(DEV).manual_seed(3)) * 255

    def ref_render(w2c, K, W, H, means, scales, quats, opac, dc, rest):
        # the reference composition, wrapper.py:244-294, over the reference ext
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
                return ref.rasterize(off, ids, pts, conic, opac_, colors, W, H, 16, 1e-4, 1e-4, 9.21)

            @staticmethod
            def backward(ctx, g):
                off, ids, pts, conic, opac_, colors = ctx.saved_tensors
                gp, gc, go, gcol = ref.rasterize_backward(g.contiguous(), off, ids, pts, conic, opac_,
                                                          colors, W, H, 16, 1e-4, 1e-4, 9.21)
                return None, None, gp, gc, go, gcol

        pts, depths, conic, radii, mask = PP.apply(means, scales, quats)
        campos = -w2c[:3, :3].t() @ w2c[:3, 3]
        colors = torch.clamp_min(SH.apply(campos, means, dc, rest, mask) + 0.5, 0.0)
        off, ids = ref.compute_tile_intersection(pts.detach(), radii, depths, mask, W, H, 16)
        img = RS.apply(off, ids, pts, conic, opac, colors)
        return img.clamp(0, 1) * 255, pts, radii

    def run(render):
        p = {k: v.to(DEV).clone().requires_grad_(True) for k, v in raw.items()}
        act = gs.scenes.activate(p)
        img, pts, radii = render(w2c, K, W, H, act["means"], act["scales"], act["quaternions"],
                                 act["opacities"], act["sh_coeffs_dc"], act["sh_coeffs_rest"])
        pts.retain_grad()
        torch.nn.functional.l1_loss(img, target).backward()
        return img.detach() / 255.0, {k: np_(v.grad) for k, v in p.items()}, np_(pts.grad), radii

    ri, rg, rp, rr = run(ref_render)
    oi, og, op, orr = run(gs.render)
    d = (ri - oi).abs()
    print("render: max |diff| on [0,1]", float(d.max()), "values > 1e-4:", int((d > 1e-4).sum()))
    assert float((d > 1e-4).float().mean()) <= 1e-5 and float(d.max()) < 1e-2
    assert torch.equal(rr > 0, orr > 0)
    for k in rg:
        assert_close_metric(k, og[k], rg[k], 0.999, 1e-3)
    assert_close_metric("points_img.grad", op, rp, 0.999, 1e-3)


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
