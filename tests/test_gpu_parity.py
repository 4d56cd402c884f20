"""Parity of the CUDA path with the CPU oracle and with the reference's golden
vectors. Every call goes through the C ABI of lib3dgs_b200.so (via the
package's cuda_rasterizer / render). Tolerances are written per test:
integer work (masks, tile layout, sort) is compared bit-exactly; floats as
noted, with the reference's own cos/rel rule (check_cuda_gradients.py:37-44)
for gradients."""
import importlib

import numpy as np
import pytest
import torch

from conftest import assert_close_metric, golden, metric, torch_ssim

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def cu(x, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(x))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(DEV)


def np_(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def cr(gs):
    return gs.cuda_rasterizer


def random_gaussians(n, seed, spread=2.0, zmin=-1.0, zmax=6.0):
    """Projection inputs that exercise every cull: behind the camera, low
    opacity, tiny and huge radii, off-screen, clamped Jacobian."""
    rng = np.random.default_rng(seed)
    means = np.empty((n, 3), np.float32)
    means[:, :2] = rng.uniform(-spread, spread, (n, 2))
    means[:, 2] = rng.uniform(zmin, zmax, n)
    scales = np.exp(rng.normal(np.log(0.05), 0.8, (n, 3))).astype(np.float32)
    q = rng.normal(size=(n, 4)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    opac = rng.uniform(0.0, 1.0, n).astype(np.float32)
    opac[: n // 50] = 0.001  # below 1/255
    dc = rng.normal(0, 0.3, (n, 3)).astype(np.float32)
    rest = rng.normal(0, 0.05, (n, 15, 3)).astype(np.float32)
    return means, scales, q, opac, dc, rest


def camera(W, H, f, yaw=0.1, t=(0.1, -0.2, 3.0)):
    c, s = np.cos(yaw), np.sin(yaw)
    w2c = np.eye(4, dtype=np.float32)
    w2c[:3, :3] = [[c, 0, s], [0, 1, 0], [-s, 0, c]]
    w2c[:3, 3] = t
    K = np.array([[f, 0, W / 2], [0, f, H / 2], [0, 0, 1]], np.float32)
    return w2c, K


# ---------------------------------------------------------------------------
# projection and SH
# ---------------------------------------------------------------------------

def test_project_points_matches_oracle(cr, orc):
    W, H = 200, 150
    means, scales, q, opac, _, _ = random_gaussians(20000, 1)
    w2c, K = camera(W, H, 150.0)
    args = (0.01, 100.0, 1 / 255, 0.5, 128.0, W, H)
    ref = orc.project_points(means, scales, q, opac, w2c, K, *args)
    out = cr.project_points(cu(means), cu(scales), cu(q), cu(opac), cu(w2c), cu(K), *args)
    pts, dep, cov, conic, radii, mask = map(np_, out)
    assert mask.dtype == np.bool_
    mismatch = int((mask != ref[5]).sum())
    assert mismatch <= 2, mismatch  # cull decisions at float ties only
    both = mask & ref[5]
    assert both.sum() > 2000 and (~ref[5]).sum() > 1000
    np.testing.assert_allclose(pts[both], ref[0][both], rtol=1e-5, atol=1e-3)
    np.testing.assert_allclose(dep[both], ref[1][both], rtol=1e-6)
    np.testing.assert_allclose(cov[both], ref[2][both], rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(conic[both], ref[3][both], rtol=1e-3, atol=1e-7)
    np.testing.assert_allclose(radii[both], ref[4][both], rtol=1e-5)
    assert np.all(pts[~mask] == 0) and np.all(radii[~mask] == 0)


def test_project_points_backward_vs_autograd_golden(cr):
    g = golden("project_points_seed0.npz")
    W, H = int(g["width"]), int(g["height"])
    out = cr.project_points(cu(g["means"]), cu(g["scales"]), cu(g["quats"]), cu(g["opac"]),
                            cu(g["w2c"]), cu(g["K"]), float(g["near"]), float(g["far"]),
                            float(g["min_opac"]), float(g["min_rad"]), float(g["max_rad"]), W, H)
    gm, gs_, gq = cr.project_points_backward(cu(g["up_points"]), cu(g["up_conic"]), cu(g["means"]),
                                             cu(g["scales"]), cu(g["quats"]), cu(g["opac"]),
                                             cu(g["w2c"]), cu(g["K"]), W, H, out[2], out[5])
    m = np_(out[5]).astype(np.float32)[:, None]
    assert_close_metric("points", np_(gm) * m, g["ref_grad_means"] * m)
    assert_close_metric("scales", np_(gs_) * m, g["ref_grad_scales"] * m)
    assert_close_metric("quaternions", np_(gq) * m, g["ref_grad_quats"] * m)


def test_project_points_backward_matches_oracle(cr, orc):
    W, H = 200, 150
    means, scales, q, opac, _, _ = random_gaussians(8000, 2)
    w2c, K = camera(W, H, 150.0)
    args = (0.01, 100.0, 1 / 255, 0.5, 128.0, W, H)
    ref = orc.project_points(means, scales, q, opac, w2c, K, *args)
    rng = np.random.default_rng(3)
    gp = rng.normal(size=(8000, 2)).astype(np.float32)
    gc = (rng.normal(size=(8000, 3)) * 0.1).astype(np.float32)
    r = orc.project_points_backward(gp, gc, means, scales, q, opac, w2c, K, W, H, ref[2], ref[5])
    o = cr.project_points_backward(cu(gp), cu(gc), cu(means), cu(scales), cu(q), cu(opac), cu(w2c),
                                   cu(K), W, H, cu(ref[2]), cu(ref[5]))
    for name, a, b in zip(("means", "scales", "quats"), o, r):
        assert_close_metric(name, np_(a), b, 0.99999, 1e-5)


def test_sh_forward_backward_golden(cr):
    g = golden("sh_seed200.npz")
    n = g["means"].shape[0]
    mask = torch.ones(n, dtype=torch.bool, device=DEV)
    colors = cr.evaluate_spherical_harmonics(cu(g["camera_pos"]), cu(g["means"]), cu(g["dc"]),
                                             cu(g["rest"]), mask)
    up = (0.3 * ((colors + 0.5) >= 0)).float()
    gm, gdc, grest = cr.evaluate_spherical_harmonics_backward(
        up, cu(g["camera_pos"]), cu(g["means"]), cu(g["dc"]), cu(g["rest"]), colors, mask)
    assert_close_metric("means", np_(gm), g["ref_grad_means"])
    assert_close_metric("sh_dc", np_(gdc), g["ref_grad_dc"])
    assert_close_metric("sh_rest", np_(grest), g["ref_grad_rest"])


@pytest.mark.parametrize("sig", [False, True])
def test_sh_matches_oracle(cr, orc, sig):
    means, _, _, _, dc, rest = random_gaussians(5000, 4)
    campos = np.array([0.3, -0.1, -3.0], np.float32)
    mask = np.random.default_rng(5).uniform(size=5000) > 0.1
    ref = orc.evaluate_spherical_harmonics(campos, means, dc, rest, mask, sig)
    col = cr.evaluate_spherical_harmonics(cu(campos), cu(means), cu(dc), cu(rest), cu(mask), sig)
    np.testing.assert_allclose(np_(col), ref, rtol=1e-5, atol=1e-6)
    gcol = np.random.default_rng(6).normal(size=(5000, 3)).astype(np.float32)
    r = orc.evaluate_spherical_harmonics_backward(gcol, campos, means, dc, rest, ref, mask, sig)
    o = cr.evaluate_spherical_harmonics_backward(cu(gcol), cu(campos), cu(means), cu(dc), cu(rest),
                                                 col, cu(mask), sig)
    for name, a, b in zip(("means", "dc", "rest"), o, r):
        assert_close_metric(name, np_(a), b, 0.99999, 1e-5)


# ---------------------------------------------------------------------------
# tile layout and sort: bit-exact
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("name", ["multitile_seed150.npz", "truncated_seed175.npz"])
def test_tile_layout_golden_bit_exact(cr, name):
    g = golden(name)
    off, ids = cr.compute_tile_intersection(cu(g["points"]), cu(g["radii"]), cu(g["depths"]),
                                            cu(g["mask"]), int(g["width"]), int(g["height"]), 16)
    assert np.array_equal(np_(off), g["ref_offsets"])
    assert np.array_equal(np_(ids), g["ref_ids"])


@pytest.mark.parametrize("W,H,n,seed", [(48, 48, 50, 0), (300, 170, 4000, 1), (1000, 600, 30000, 2),
                                        (16, 16, 10, 3), (37, 530, 3000, 4)])
def test_tile_layout_matches_oracle_bit_exact(cr, orc, W, H, n, seed):
    rng = np.random.default_rng(seed)
    pts = np.stack([rng.uniform(-20, W + 20, n), rng.uniform(-20, H + 20, n)], 1).astype(np.float32)
    radii = rng.uniform(0.5, 60, (n, 2)).astype(np.float32)
    # few distinct depths -> many equal keys: the order must be the stable one
    depths = rng.choice(np.array([0.5, 1.0, 1.5, 7.25], np.float32), n)
    mask = rng.uniform(size=n) > 0.2
    r_off, r_ids, r_keys = orc.compute_tile_intersection(pts, radii, depths, mask, W, H,
                                                         return_keys=True)
    off, ids, keys = cr.compute_tile_intersection(cu(pts), cu(radii), cu(depths), cu(mask), W, H, 16,
                                                  return_keys=True)
    assert np.array_equal(np_(off), r_off)
    assert np.array_equal(np_(ids), r_ids)
    assert np.array_equal(np_(keys), r_keys)


def test_tile_layout_empty(cr):
    z = torch.zeros
    off, ids = cr.compute_tile_intersection(z((5, 2), device=DEV), z((5, 2), device=DEV),
                                            z(5, device=DEV), z(5, dtype=torch.bool, device=DEV),
                                            40, 40, 16)
    assert ids.numel() == 0 and np.all(np_(off) == 0) and off.numel() == 9


@pytest.mark.parametrize("n", [1, 17, 3840, 3841, 100_003, 2_000_000])
@pytest.mark.parametrize("end_bit", [8, 21, 45, 64])
def test_sort_pairs_stable_bit_exact(gs, n, end_bit):
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    rng = np.random.default_rng(n + end_bit)
    hi = rng.integers(0, 40, n).astype(np.uint64)  # heavy duplication
    lo = rng.integers(0, 1 << 20, n).astype(np.uint64)
    keys = (hi << np.uint64(37)) | (lo << np.uint64(3)) | rng.integers(0, 2, n).astype(np.uint64)
    vals = np.arange(n, dtype=np.int32)
    k = cu(keys.view(np.int64))
    v = cu(vals)
    k2 = torch.empty_like(k)
    v2 = torch.empty_like(v)
    nb = int(nat.query("gs_sort_scratch_bytes", n))
    scratch = torch.empty(nb, dtype=torch.uint8, device=DEV)
    nat.call("gs_sort_pairs", n, k.data_ptr(), v.data_ptr(), k2.data_ptr(), v2.data_ptr(), end_bit,
             scratch.data_ptr(), nb, nat.stream_ptr())
    torch.cuda.synchronize()
    mask = np.uint64((1 << end_bit) - 1) if end_bit < 64 else np.uint64(0xFFFFFFFFFFFFFFFF)
    order = np.argsort(keys & mask, kind="stable")
    assert np.array_equal(np_(v), vals[order])
    assert np.array_equal(np_(k).view(np.uint64), keys[order])


def test_bounded_wait_reports_timeout_and_context_survives(gs):
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = nat.query("gs_selftest_bounded_wait", flag.data_ptr(), nat.stream_ptr())
    assert rc == nat.GS_ERR_DEVICE_TIMEOUT
    assert nat.query("gs_check_status", nat.stream_ptr()) == 0  # cleared
    x = torch.arange(10, device=DEV).sum().item()  # the context is still usable
    assert x == 45


# ---------------------------------------------------------------------------
# blending
# ---------------------------------------------------------------------------

def test_rasterize_single_tile_golden(cr):
    g = golden("rasterize_seed100.npz")
    args = (cu(g["offsets"]), cu(g["ids"]), cu(g["points"]), cu(g["conic"]), cu(g["opac"]),
            cu(g["colors"]), int(g["width"]), int(g["height"]), 16, float(g["athr"]),
            float(g["tthr"]), float(g["chi"]))
    img = np_(cr.rasterize(*args))
    np.testing.assert_allclose(img, g["ref_image"], rtol=1e-5, atol=1e-6)
    gp, gc, go, gcol = map(np_, cr.rasterize_backward(cu(g["upstream"]), *args))
    assert_close_metric("points_img", gp, g["ref_grad_points"])
    assert_close_metric("cov_inv", gc, g["ref_grad_conic"])
    assert_close_metric("opacities", go, g["ref_grad_opac"])
    assert_close_metric("colors", gcol, g["ref_grad_colors"])


@pytest.mark.parametrize("name", ["multitile_seed150.npz", "truncated_seed175.npz"])
def test_rasterize_multitile_golden(cr, name):
    g = golden(name)
    W, H = int(g["width"]), int(g["height"])
    args = (cu(g["ref_offsets"]), cu(g["ref_ids"]), cu(g["points"]), cu(g["conic"]), cu(g["opac"]),
            cu(g["colors"]), W, H, 16, float(g["athr"]), float(g["tthr"]), float(g["chi"]))
    img = np_(cr.rasterize(*args))
    assert_close_metric("rendered", img, g["ref_image"], 0.999999, 1e-6)
    gp, gc, go, gcol = map(np_, cr.rasterize_backward(cu(g["upstream"]), *args))
    assert_close_metric("points_img", gp, g["ref_grad_points"], 0.999, 2e-3)
    assert_close_metric("cov_inv", gc, g["ref_grad_conic"], 0.999, 2e-3)
    assert_close_metric("opacities", go, g["ref_grad_opac"], 0.99999, 1e-5)
    assert_close_metric("colors", gcol, g["ref_grad_colors"], 0.99999, 1e-5)


@pytest.mark.parametrize("size", [(160, 120), (157, 150)])
@pytest.mark.parametrize("thr", [(1e-4, 1e-4, 9.21), (0.0, 0.0, 20.0), (0.01, 0.3, 4.0)])
def test_rasterize_matches_oracle(cr, orc, thr, size):
    """Blend forward and backward against the oracle. 157 x 150 leaves the
    bottom tile row 6 pixels high, so some threads have their upper pixel in
    the image and their lower pixel (4 rows down) outside it."""
    (W, H), n = size, 3000
    rng = np.random.default_rng(7)
    pts = np.stack([rng.uniform(-5, W + 5, n), rng.uniform(-5, H + 5, n)], 1).astype(np.float32)
    radii = rng.uniform(1, 25, (n, 2)).astype(np.float32)
    depths = rng.uniform(1, 5, n).astype(np.float32)
    mask = np.ones(n, bool)
    sig = radii / 3
    conic = np.stack([1 / sig[:, 0] ** 2, rng.uniform(-0.2, 0.2, n) / (sig[:, 0] * sig[:, 1]),
                      1 / sig[:, 1] ** 2], 1).astype(np.float32)
    opac = rng.uniform(0.05, 0.99, n).astype(np.float32)
    colors = rng.uniform(0, 1, (n, 3)).astype(np.float32)
    off, ids = orc.compute_tile_intersection(pts, radii, depths, mask, W, H)
    a_np = (off, ids, pts, conic, opac, colors, W, H, 16) + thr
    ref = orc.rasterize(*a_np)
    a_cu = (cu(off), cu(ids), cu(pts), cu(conic), cu(opac), cu(colors), W, H, 16) + thr
    img = np_(cr.rasterize(*a_cu))
    assert np.abs(img - ref).max() < 1e-4
    assert_close_metric("image", img, ref, 0.9999999, 1e-6)
    up = rng.normal(size=(H, W, 3)).astype(np.float32)
    up[::7] = 0.0  # all-zero upstream rows are skipped, as in the reference
    r = orc.rasterize_backward(up, *a_np)
    o = cr.rasterize_backward(cu(up), *a_cu)
    for name, a, b in zip(("points", "conic", "opac", "colors"), o, r):
        assert_close_metric(name, np_(a), b, 0.99999, 1e-4)


# ---------------------------------------------------------------------------
# fused render path
# ---------------------------------------------------------------------------

def _scene(gs, n, W, H, f, seed=1, cfg=0):
    c = gs.scenes.CONFIGS[cfg]
    raw = gs.scenes.make_gaussians(c, seed=seed, n=n)
    w2c = gs.scenes.primary_camera(c)
    K = torch.tensor([[f, 0, W / 2.0], [0, f, H / 2.0], [0, 0, 1]], dtype=torch.float32)
    return raw, w2c, K


def _render_grads(render, raw, w2c, K, W, H, target):
    params = {k: v.to(DEV).clone().requires_grad_(True) for k, v in raw.items()}
    scales = torch.exp(params["scales"])
    q = params["quaternions"]
    quats = q / torch.norm(q, dim=1, keepdim=True).clamp_min(1e-12)
    opac = torch.sigmoid(params["opacities"])
    img, pts, radii = render(w2c.to(DEV), K.to(DEV), W, H, params["means"], scales, quats, opac,
                             params["sh_coeffs_dc"], params["sh_coeffs_rest"])
    pts.retain_grad()
    loss = torch.nn.functional.l1_loss(img, target.to(DEV))
    loss.backward()
    grads = {k: np_(v.grad) for k, v in params.items()}
    return np_(img), grads, np_(pts.grad), np_(radii), np_(pts)


def test_render_matches_oracle(gs, orc):
    W, H, f = 128, 96, 150.0
    raw, w2c, K = _scene(gs, 2000, W, H, f)
    target = torch.rand((H, W, 3), generator=torch.Generator().manual_seed(5)) * 255.0
    img, grads, pgrad, radii, pts = _render_grads(gs.render, raw, w2c, K, W, H, target)
    # oracle: same composition on the CPU
    act = {k: v for k, v in gs.scenes.activate(raw).items()}
    a = {k: v.numpy() for k, v in act.items()}
    rimg, st = orc.render_forward(w2c, K, W, H, a["means"], a["scales"], a["quaternions"],
                                  a["opacities"], a["sh_coeffs_dc"], a["sh_coeffs_rest"])
    assert np.abs(img - rimg).max() / 255.0 < 1e-4
    g_img = (np.sign(rimg - target.numpy()) / rimg.size).astype(np.float32)
    rg = orc.render_backward(g_img, st, w2c, K, W, H, a["means"], a["scales"], a["quaternions"],
                             a["opacities"], a["sh_coeffs_dc"], a["sh_coeffs_rest"])
    assert np.array_equal(radii[:, 0] > 0, st["mask"])
    assert_close_metric("points_img.grad", pgrad, rg["points_img"], 0.9999, 1e-3)
    # raw-parameter gradients through Torch's activation backward
    p = {k: torch.from_numpy(v.numpy().copy()).requires_grad_(True) for k, v in raw.items()}
    act2 = gs.scenes.activate(p)
    torch.autograd.backward([act2[k] for k in ("means", "scales", "quaternions", "opacities",
                                               "sh_coeffs_dc", "sh_coeffs_rest")],
                            [torch.from_numpy(rg[k]) for k in ("means", "scales", "quaternions",
                                                               "opacities", "sh_coeffs_dc",
                                                               "sh_coeffs_rest")])
    for k in p:
        assert_close_metric(k, grads[k], p[k].grad.numpy(), 0.9999, 1e-3)


def test_render_matches_reference_composition(gs):
    """render()'s fused kernels against the reference's three-Function
    composition (wrapper.py:244-294) served by this package's per-function
    kernels."""
    W, H, f = 200, 136, 220.0
    raw, w2c, K = _scene(gs, 6000, W, H, f, seed=3)
    target = torch.rand((H, W, 3), generator=torch.Generator().manual_seed(9)) * 255.0
    wr = importlib.import_module("3dgs_from_scratch_b200.wrapper")

    def composed(w2c, K, W, H, means, scales, quats, opac, dc, rest):
        pts, depths, conic, radii, mask = wr.ProjectPointsFunction.apply(
            means, scales, quats, opac, w2c, K, 0.01, 100.0, 1 / 255, 0.5, 128.0, W, H)
        campos = -w2c[:3, :3].t() @ w2c[:3, 3]
        colors = wr.SphericalHarmonicsFunction.apply(campos, means, dc, rest, mask, False)
        colors = torch.clamp_min(colors + 0.5, 0.0)
        off, ids = gs.cuda_rasterizer.compute_tile_intersection(pts, radii, depths, mask, W, H, 16)
        img = wr.RasterizeFunction.apply(off, ids, pts, conic, opac, colors, W, H, 16, 1e-4, 1e-4,
                                         9.21)
        return img.clamp(0, 1) * 255, pts, radii

    a = _render_grads(gs.render, raw, w2c, K, W, H, target)
    b = _render_grads(composed, raw, w2c, K, W, H, target)
    assert np.abs(a[0] - b[0]).max() < 1e-3  # 0..255 scale
    assert np.array_equal(a[3], b[3])
    for k in a[1]:
        assert_close_metric(k, a[1][k], b[1][k], 0.99999, 1e-4)
    assert_close_metric("points_img.grad", a[2], b[2], 0.99999, 1e-4)


def test_end_to_end_golden(gs):
    g = golden("end_to_end_seed300.npz")
    t = {k: torch.from_numpy(g[k]).to(DEV).requires_grad_(True)
         for k in ("means", "scales_raw", "quats_raw", "opac_raw", "dc_raw", "rest_raw")}
    q = t["quats_raw"]
    img, _, _ = gs.render(cu(g["w2c"]), cu(g["K"]), 64, 64, t["means"], torch.exp(t["scales_raw"]),
                          q / torch.norm(q, dim=1, keepdim=True), torch.sigmoid(t["opac_raw"]),
                          t["dc_raw"], t["rest_raw"])
    loss = torch.nn.functional.l1_loss(img, torch.zeros_like(img) + 64.0)
    loss.backward()
    names = {"means": "means", "scales_raw": "scales_raw", "quats_raw": "quaternions_raw",
             "opac_raw": "opacities_raw", "dc_raw": "sh_dc_raw", "rest_raw": "sh_rest_raw"}
    for k, ref_name in names.items():
        got = np_(t[k].grad)
        mc, mr = (0.995, 0.11) if k == "means" else (0.999, 1e-3)
        assert_close_metric(k, got, g[f"torch_grad_{ref_name}"], mc, mr)
        assert_close_metric(k, got, g[f"oracle_grad_{ref_name}"], 0.9999, 1e-3)


def test_render_torch_twin_golden(gs):
    g = golden("torch_render_small.npz")
    W, H = int(g["width"]), int(g["height"])
    raw = gs.scenes.make_gaussians(gs.scenes.CONFIGS[0], seed=int(g["seed"]), n=int(g["n"]))
    img, grads, _, _, _ = _render_grads(gs.render, raw, torch.from_numpy(g["w2c"]),
                                        torch.from_numpy(g["K"]), W, H, torch.from_numpy(g["target"]))
    diff = np.abs(img - g["image"]) / 255.0
    assert (diff > 1e-4).mean() <= 1e-4 and diff.max() < 1e-2
    for k in grads:
        mc, mr = (0.995, 0.11) if k == "means" else (0.999, 1e-3)
        assert_close_metric(k, grads[k], g[f"grad_{k}"], mc, mr)


def test_render_empty_and_all_culled(gs):
    W, H = 64, 48
    raw, w2c, K = _scene(gs, 100, W, H, 60.0)
    w2c = w2c.clone()
    w2c[2, 3] = -50.0  # everything behind the camera
    act = gs.scenes.activate({k: v.to(DEV) for k, v in raw.items()})
    img, pts, radii = gs.render(w2c.to(DEV), K.to(DEV), W, H, act["means"], act["scales"],
                                act["quaternions"], act["opacities"], act["sh_coeffs_dc"],
                                act["sh_coeffs_rest"])
    assert float(img.abs().max()) == 0.0 and float(radii.abs().max()) == 0.0
    z = torch.zeros
    img, pts, radii = gs.render(w2c.to(DEV), K.to(DEV), W, H, z((0, 3), device=DEV),
                                z((0, 3), device=DEV), z((0, 4), device=DEV), z(0, device=DEV),
                                z((0, 3), device=DEV), z((0, 15, 3), device=DEV))
    assert img.shape == (H, W, 3) and float(img.abs().max()) == 0.0


# ---------------------------------------------------------------------------
# full-size (config 1) properties
# ---------------------------------------------------------------------------

def test_cfg1_layout_and_image_properties(gs, orc):
    cfg = gs.scenes.CONFIGS[1]
    raw = gs.scenes.make_gaussians(cfg, seed=0)
    act = gs.scenes.activate({k: v.to(DEV) for k, v in raw.items()})
    W, H = cfg.width, cfg.height
    w2c = gs.scenes.primary_camera(cfg).to(DEV)
    K = gs.scenes.intrinsic_for(cfg).to(DEV)
    cr = gs.cuda_rasterizer
    pts, depths, cov, conic, radii, mask = cr.project_points(
        act["means"], act["scales"], act["quaternions"], act["opacities"], w2c, K, 0.01, 100.0,
        1 / 255, 0.5, 128.0, W, H)
    off, ids, keys = cr.compute_tile_intersection(pts, radii, depths, mask, W, H, 16,
                                                  return_keys=True)
    k = np_(keys).view(np.uint64)
    assert k.size > 4_000_000
    assert np.all(np.diff(k) >= 0)  # sorted
    tiles = (k >> np.uint64(32)).astype(np.int64)
    T = off.numel()
    assert np.array_equal(np_(off), np.searchsorted(tiles, np.arange(T), side="left").astype(np.int32))
    # sum of counts equals K and ids are masked Gaussians
    counts = orc.count_tiles(np_(pts), np_(radii), np_(mask), W, H)
    assert int(counts.astype(np.int64).sum()) == k.size
    assert np_(mask)[np_(ids)].all()
    # the layout equals the oracle's on the same inputs (bit-exact)
    r_off, r_ids = orc.compute_tile_intersection(np_(pts), np_(radii), np_(depths), np_(mask), W, H)
    assert np.array_equal(np_(off), r_off) and np.array_equal(np_(ids), r_ids)
    # blend on identical inputs: the oracle's image within 1e-4 on [0, 1] except at
    # isolated threshold ties
    colors = torch.rand((pts.shape[0], 3), device=DEV, generator=torch.Generator(DEV).manual_seed(1))
    img = np_(cr.rasterize(off, ids, pts, conic, act["opacities"], colors, W, H, 16, 1e-4, 1e-4, 9.21))
    ref = orc.rasterize(r_off, r_ids, np_(pts), np_(conic), np_(act["opacities"]), np_(colors), W, H,
                        16, 1e-4, 1e-4, 9.21)
    d = np.abs(img - ref)
    assert (d > 1e-4).mean() < 1e-5 and d.max() < 1e-2, ((d > 1e-4).sum(), d.max())


@pytest.mark.parametrize("n", [1, 2047, 2048, 2049, 131_079, 1_000_000, 5_000_001])
def test_exclusive_scan_matches_cumsum(gs, n):
    """The look-back scan against torch.cumsum, at sizes whose look-back
    windows reach past 32 predecessors without finding a prefix."""
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    g = torch.Generator(DEV).manual_seed(n)
    c = torch.randint(0, 50, (n,), dtype=torch.int32, device=DEV, generator=g)
    out = torch.empty(n, dtype=torch.int32, device=DEV)
    tot = torch.zeros(1, dtype=torch.int64, device=DEV)
    nb = int(nat.query("gs_scan_scratch_bytes", n))
    sc = torch.empty(nb, dtype=torch.uint8, device=DEV)
    nat.call("gs_exclusive_scan", n, c.data_ptr(), out.data_ptr(), tot.data_ptr(), sc.data_ptr(), nb,
             nat.stream_ptr())
    ref = torch.cumsum(c.long(), 0) - c.long()
    assert torch.equal(out.long(), ref)
    assert int(tot.item()) == int(c.long().sum().item())
    assert nat.query("gs_check_status", nat.stream_ptr()) == 0


def test_flat_adam_matches_torch_adam(gs):
    """gs_adam_step over the six flat groups against torch.optim.Adam with the
    reference's per-group learning rates and eps (scripts/train.py:17-44)."""
    dp = importlib.import_module("3dgs_from_scratch_b200.dp")
    raw = gs.scenes.make_gaussians(gs.scenes.CONFIGS[0], seed=2, n=3001)
    fp = dp.FlatParams({k: v.to(DEV) for k, v in raw.items()})
    ref = {k: v.to(DEV).clone().requires_grad_(True) for k, v in raw.items()}
    opts = [torch.optim.Adam([ref[k]], lr=dp.DEFAULT_LRS[k], eps=1e-15) for k in dp.GROUPS]
    g = torch.Generator(DEV).manual_seed(0)
    for _ in range(5):
        for k in dp.GROUPS:
            grad = torch.randn(ref[k].shape, device=DEV, generator=g)
            ref[k].grad = grad.clone()
            fp[k].grad.copy_(grad)
        for o in opts:
            o.step()
        fp.adam_step()
    for k in dp.GROUPS:
        torch.testing.assert_close(fp[k].detach(), ref[k].detach(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("u8,lam", [(False, 0.0), (True, 0.0), (True, 0.2), (False, 1.0)])
def test_native_trainer_step_matches_autograd_path(gs, u8, lam):
    """One NativeTrainer step (fused activations, fused loss, gradients
    accumulated in the flat buffer) against render() + Torch activations +
    the reference's loss expression (scripts/train.py:186-203, SSIM as a
    Torch conv2d restatement) + autograd, on two views."""
    tr_mod = importlib.import_module("3dgs_from_scratch_b200.trainer")
    W, H, f = 160, 120, 170.0
    cfg = gs.scenes.CONFIGS[0]
    raw = gs.scenes.make_gaussians(cfg, seed=4, n=4000)
    w2cs = gs.scenes.orbit_cameras(cfg, 2)
    K = torch.tensor([[f, 0, W / 2], [0, f, H / 2], [0, 0, 1]], dtype=torch.float32)
    g = torch.Generator().manual_seed(3)
    targets = [(torch.rand((H, W, 3), generator=g) * 255).round() for _ in range(2)]
    if u8:
        targets = [t.to(torch.uint8) for t in targets]
    # autograd path
    p = {k: v.to(DEV).clone().requires_grad_(True) for k, v in raw.items()}
    act = gs.scenes.activate(p)
    losses = []
    imgs = []
    for v in range(2):
        img, _, _ = gs.render(w2cs[v].to(DEV), K.to(DEV), W, H, act["means"], act["scales"],
                              act["quaternions"], act["opacities"], act["sh_coeffs_dc"],
                              act["sh_coeffs_rest"])
        imgs.append(img.detach())
        rn, tn = img / 255.0, targets[v].to(DEV).float() / 255.0
        loss = torch.nn.functional.l1_loss(rn, tn)
        if lam > 0:
            ss = torch_ssim(rn.permute(2, 0, 1).unsqueeze(0), tn.permute(2, 0, 1).unsqueeze(0),
                            True)
            loss = (1 - lam) * loss + lam * (1 - ss)
        losses.append(loss)
    torch.stack(losses).sum().backward()
    # native path
    tr = tr_mod.NativeTrainer({k: v.to(DEV) for k, v in raw.items()}, W, H, ssim_lambda=lam)
    views = tr.forward_views(w2cs, K)
    nl = tr.loss_and_backward(views, [t.to(DEV) for t in targets])
    for v in range(2):
        native_img = views[v]["image"].clamp(0, 1) * 255
        assert float((native_img - imgs[v]).abs().max()) / 255.0 < 1e-4
    torch.testing.assert_close(nl.float(), torch.stack(losses).detach(), rtol=1e-5, atol=2e-7)
    for k in p:
        a, n = tr.fp.spans[k]
        assert_close_metric(k, np_(tr.fp.grad[a:a + n]), np_(p[k].grad).ravel(), 0.9999, 1e-3)


@pytest.mark.parametrize("n", [4000, 4000 + 37])
def test_multi_view_preprocess_matches_per_view(gs, n):
    """gs_preprocess_forward_views equals one gs_preprocess_forward per view
    (bit for bit), and gs_preprocess_backward_views equals the per-view
    backward calls accumulated (summation order aside); n not a multiple of
    the chunk size exercises the tail kernel."""
    nat = importlib.import_module("3dgs_from_scratch_b200._native")
    cfg = gs.scenes.CONFIGS[0]
    raw = {k: v.to(DEV) for k, v in gs.scenes.make_gaussians(cfg, seed=9, n=n).items()}
    V, W, H = 3, 200, 150
    w2c = gs.scenes.orbit_cameras(cfg, V).to(DEV).contiguous()
    K = torch.tensor([[180.0, 0, 100], [0, 180.0, 75], [0, 0, 1]], device=DEV)
    Ks = K.expand(V, 3, 3).contiguous()
    campos = (-(w2c[:, :3, :3].transpose(1, 2) @ w2c[:, :3, 3:4])).squeeze(-1).contiguous()
    st = nat.stream_ptr()
    p = [raw[k].data_ptr() for k in ("means", "scales", "quaternions", "opacities",
                                     "sh_coeffs_dc", "sh_coeffs_rest")]
    f = dict(device=DEV, dtype=torch.float32)

    def outs(shape_v):
        return dict(points=torch.empty(shape_v + (n, 2), **f), depths=torch.empty(shape_v + (n,), **f),
                    radii=torch.empty(shape_v + (n, 2), **f),
                    mask=torch.empty(shape_v + (n,), device=DEV, dtype=torch.uint8),
                    splat=torch.empty(shape_v + (n, 8), **f),
                    counts=torch.empty(shape_v + (n,), device=DEV, dtype=torch.int32))
    opts = (0.01, 100.0, 1 / 255, 0.5, 128.0, W, H, 0, 1)
    b = outs((V,))
    totals = torch.empty(V, dtype=torch.int64, device=DEV)
    nat.call("gs_preprocess_forward_views", n, V, *p, w2c.data_ptr(), Ks.data_ptr(),
             campos.data_ptr(), *opts, b["points"].data_ptr(), b["depths"].data_ptr(),
             b["radii"].data_ptr(), b["mask"].data_ptr(), b["splat"].data_ptr(),
             b["counts"].data_ptr(), totals.data_ptr(), st)
    for v in range(V):
        o = outs(())
        tot = torch.empty(1, dtype=torch.int64, device=DEV)
        nat.call("gs_preprocess_forward", n, *p, w2c[v].data_ptr(), Ks[v].data_ptr(),
                 campos[v].data_ptr(), *opts, o["points"].data_ptr(), o["depths"].data_ptr(),
                 o["radii"].data_ptr(), o["mask"].data_ptr(), o["splat"].data_ptr(),
                 o["counts"].data_ptr(), tot.data_ptr(), st)
        for k in o:
            assert torch.equal(o[k], b[k][v]), k
        assert int(tot) == int(totals[v])
    assert int(b["mask"].sum()) > 100
    # backward
    g = torch.Generator(device=DEV).manual_seed(2)
    gp = torch.randn((V, n, 2), device=DEV, generator=g) * 1e-3
    gsp = torch.randn((V, n, 8), device=DEV, generator=g) * 1e-3
    numel = sum(raw[k].numel() for k in raw)
    grads_multi = {k: torch.empty_like(raw[k]) for k in raw}
    grads_ref = {k: torch.zeros_like(raw[k]) for k in raw}
    order = ("means", "scales", "quaternions", "opacities", "sh_coeffs_dc", "sh_coeffs_rest")
    nat.call("gs_preprocess_backward_views", n, V, *p, w2c.data_ptr(), Ks.data_ptr(),
             campos.data_ptr(), W, H, 0, 1, 0, b["mask"].data_ptr(), gp.data_ptr(), 2,
             gsp.data_ptr(), 8, *[grads_multi[k].data_ptr() for k in order], st)
    for v in range(V):
        nat.call("gs_preprocess_backward", n, *p, w2c[v].data_ptr(), Ks[v].data_ptr(),
                 campos[v].data_ptr(), W, H, 0, 1, 1, b["mask"][v].data_ptr(),
                 gp[v].data_ptr(), 2, gsp[v].data_ptr(), 8,
                 *[grads_ref[k].data_ptr() for k in order], st)
    del numel
    for k in order:
        assert_close_metric(k, np_(grads_multi[k]), np_(grads_ref[k]), 0.999999, 1e-5)


def test_native_trainer_host_targets_match_device_targets(gs):
    """Targets in pinned host memory (copied on the trainer's copy stream
    while the views render) give the same step as targets on the device."""
    tr_mod = importlib.import_module("3dgs_from_scratch_b200.trainer")
    W, H, f = 160, 120, 170.0
    cfg = gs.scenes.CONFIGS[0]
    raw = gs.scenes.make_gaussians(cfg, seed=5, n=3000)
    w2cs = gs.scenes.orbit_cameras(cfg, 3)
    K = torch.tensor([[f, 0, W / 2], [0, f, H / 2], [0, 0, 1]], dtype=torch.float32)
    g = torch.Generator().manual_seed(8)
    host = [(torch.rand((H, W, 3), generator=g) * 255).round().to(torch.uint8).pin_memory()
            for _ in range(3)]
    out = []
    for targets in (host, [t.to(DEV) for t in host]):
        tr = tr_mod.NativeTrainer({k: v.to(DEV) for k, v in raw.items()}, W, H, ssim_lambda=0.2)
        losses = tr.step(w2cs, K, targets, optimizer_step=False)
        torch.cuda.synchronize()
        out.append((losses.cpu(), tr.fp.grad.cpu().clone()))
    assert torch.allclose(out[0][0], out[1][0], rtol=1e-6, atol=1e-9)
    # the gradients are sums of atomics: equal up to their order
    assert_close_metric("grad", np_(out[0][1]), np_(out[1][1]), 0.999999, 1e-5)
