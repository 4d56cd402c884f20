"""Autograd boundary of the rasterizer: the drop-in for src/cuda/wrapper.py.

Keeps the reference's public surface (ruguangyou/3dgs_from_scratch
src/cuda/wrapper.py):

* ProjectPointsFunction, SphericalHarmonicsFunction, RasterizeFunction with
  the reference's forward/backward arities (wrapper.py:12-220), served by the
  per-function kernels through `cuda_rasterizer` (this package's module);
* render(...) with the reference's signature, defaults and return value
  (wrapper.py:223-294): (image (H,W,3) in [0, 255], points_img (N,2) that
  receives .grad, radii (N,2)).

render() runs the fused B200 path: one preprocess kernel (projection, EWA
covariance, conic, radii, SH colour with the +0.5 shift and clamp, tile
counts and their scan), the tile layout (key duplication, onesweep sort,
ranges), one blend kernel; backward: one blend-backward kernel and one fused
preprocess-backward kernel. Same results as the reference composition.
"""
from __future__ import annotations

import torch

from . import _native as nat
from . import cuda_rasterizer

TILE = 16


# ---------------------------------------------------------------------------
# reference-compatible autograd Functions (per-function kernels)
# ---------------------------------------------------------------------------

class ProjectPointsFunction(torch.autograd.Function):
    """wrapper.py:12-85."""

    @staticmethod
    def forward(ctx, means, scales, quaternions, opacities, world_to_camera, intrinsic,
                near_plane, far_plane, min_opacity, min_radius, max_radius, width, height):
        points_img, depths, cov_img, cov_inv_img, radii, mask = cuda_rasterizer.project_points(
            means, scales, quaternions, opacities, world_to_camera, intrinsic, near_plane,
            far_plane, min_opacity, min_radius, max_radius, width, height)
        ctx.save_for_backward(means, scales, quaternions, opacities, world_to_camera, intrinsic,
                              cov_img, mask)
        ctx.width = width
        ctx.height = height
        ctx.mark_non_differentiable(depths, radii, mask)
        return points_img, depths, cov_inv_img, radii, mask

    @staticmethod
    def backward(ctx, grad_points_img, grad_depths, grad_cov_inv_img, grad_radii, grad_mask):
        means, scales, quaternions, opacities, world_to_camera, intrinsic, cov_img, mask = (
            ctx.saved_tensors)
        if grad_points_img is None:
            grad_points_img = torch.zeros((means.shape[0], 2), device=means.device)
        if grad_cov_inv_img is None:
            grad_cov_inv_img = torch.zeros((means.shape[0], 3), device=means.device)
        grad_means, grad_scales, grad_quaternions = cuda_rasterizer.project_points_backward(
            grad_points_img, grad_cov_inv_img, means, scales, quaternions, opacities,
            world_to_camera, intrinsic, ctx.width, ctx.height, cov_img, mask)
        return (grad_means, grad_scales, grad_quaternions) + (None,) * 10


class SphericalHarmonicsFunction(torch.autograd.Function):
    """wrapper.py:88-118."""

    @staticmethod
    def forward(ctx, camera_pos, means, sh_coeffs_dc, sh_coeffs_rest, mask, sh_sigmoid=False):
        colors = cuda_rasterizer.evaluate_spherical_harmonics(
            camera_pos, means, sh_coeffs_dc, sh_coeffs_rest, mask, sh_sigmoid)
        ctx.save_for_backward(camera_pos, means, sh_coeffs_dc, sh_coeffs_rest, colors, mask)
        ctx.sh_sigmoid = sh_sigmoid
        return colors

    @staticmethod
    def backward(ctx, grad_colors):
        camera_pos, means, sh_coeffs_dc, sh_coeffs_rest, colors, mask = ctx.saved_tensors
        grad_means, grad_dc, grad_rest = cuda_rasterizer.evaluate_spherical_harmonics_backward(
            grad_colors, camera_pos, means, sh_coeffs_dc, sh_coeffs_rest, colors, mask,
            ctx.sh_sigmoid)
        return None, grad_means, grad_dc, grad_rest, None, None


class RasterizeFunction(torch.autograd.Function):
    """wrapper.py:121-220."""

    @staticmethod
    def forward(ctx, indexing_offset, gaussian_ids_sorted, points_img, cov_inv_img, opacities,
                colors, width, height, tile_size, alpha_threshold, transmittance_threshold,
                chi_squared_threshold):
        image = cuda_rasterizer.rasterize(
            indexing_offset, gaussian_ids_sorted, points_img, cov_inv_img, opacities, colors,
            width, height, tile_size, alpha_threshold, transmittance_threshold,
            chi_squared_threshold)
        ctx.save_for_backward(indexing_offset, gaussian_ids_sorted, points_img, cov_inv_img,
                              opacities, colors)
        ctx.args = (width, height, tile_size, alpha_threshold, transmittance_threshold,
                    chi_squared_threshold)
        return image

    @staticmethod
    def backward(ctx, grad_rendered_image):
        indexing_offset, ids, points_img, cov_inv_img, opacities, colors = ctx.saved_tensors
        gp, gc, go, gcol = cuda_rasterizer.rasterize_backward(
            grad_rendered_image, indexing_offset, ids, points_img, cov_inv_img, opacities,
            colors, *ctx.args)
        return (None, None, gp, gc, go, gcol) + (None,) * 6


# ---------------------------------------------------------------------------
# fused path
# ---------------------------------------------------------------------------

def _require(name, t, dtype, dev, shape_tail=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device != dev:
        raise RuntimeError(f"{name} is on {t.device}, expected {dev}")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")
    if shape_tail is not None and tuple(t.shape[1:]) != tuple(shape_tail):
        raise RuntimeError(f"{name} has shape {tuple(t.shape)}, expected (N, *{shape_tail})")
    return t if t.is_contiguous() else t.contiguous()


class _Preprocess(torch.autograd.Function):
    """Fused projection + covariance + SH + tile counts; backward is the
    fused chain through projection, covariance and SH."""

    @staticmethod
    def forward(ctx, means, scales, quaternions, opacities, sh_dc, sh_rest, world_to_camera,
                intrinsic, camera_pos, opts):
        dev = means.device
        n = means.shape[0]
        f = dict(device=dev, dtype=torch.float32)
        points = torch.empty((n, 2), **f)
        depths = torch.empty((n,), **f)
        radii = torch.empty((n, 2), **f)
        mask = torch.empty((n,), device=dev, dtype=torch.bool)
        splat = torch.empty((n, 8), **f)
        counts = torch.empty((max(n, 1),), device=dev, dtype=torch.int32)
        total_dev = torch.empty((1,), device=dev, dtype=torch.int64)
        nat.call("gs_preprocess_forward", n, means.data_ptr(), scales.data_ptr(),
                 quaternions.data_ptr(), opacities.data_ptr(), sh_dc.data_ptr(),
                 sh_rest.data_ptr(), world_to_camera.data_ptr(), intrinsic.data_ptr(),
                 camera_pos.data_ptr(), opts["near_plane"], opts["far_plane"],
                 opts["min_opacity"], opts["min_radius"], opts["max_radius"], opts["width"],
                 opts["height"], int(opts["sh_sigmoid"]), 0, points.data_ptr(), depths.data_ptr(),
                 radii.data_ptr(), mask.view(torch.uint8).data_ptr(), splat.data_ptr(),
                 counts.data_ptr(), total_dev.data_ptr(), nat.stream_ptr(dev))
        ctx.save_for_backward(means, scales, quaternions, sh_dc, sh_rest, world_to_camera,
                              intrinsic, camera_pos, mask)
        ctx.opts = opts
        ctx.mark_non_differentiable(depths, radii, mask, counts, total_dev)
        return points, splat, depths, radii, mask, counts, total_dev

    @staticmethod
    def backward(ctx, g_points, g_splat, _gd, _gr, _gm, _go, _gt):
        means, scales, quats, sh_dc, sh_rest, w2c, K, campos, mask = ctx.saved_tensors
        o = ctx.opts
        dev = means.device
        n = means.shape[0]
        f = dict(device=dev, dtype=torch.float32)
        if g_points is None:
            g_points = torch.zeros((n, 2), **f)
        if g_splat is None:
            g_splat = torch.zeros((n, 8), **f)
        if g_points.stride(-1) != 1 or g_points.dtype != torch.float32:
            g_points = g_points.contiguous().float()
        if g_splat.stride(-1) != 1 or g_splat.dtype != torch.float32:
            g_splat = g_splat.contiguous().float()
        gm = torch.empty((n, 3), **f)
        gs = torch.empty((n, 3), **f)
        gq = torch.empty((n, 4), **f)
        go = torch.empty((n,), **f)
        gdc = torch.empty((n, 3), **f)
        grest = torch.empty((n, 15, 3), **f)
        nat.call("gs_preprocess_backward", n, means.data_ptr(), scales.data_ptr(),
                 quats.data_ptr(), None, sh_dc.data_ptr(), sh_rest.data_ptr(), w2c.data_ptr(),
                 K.data_ptr(), campos.data_ptr(), o["width"], o["height"], int(o["sh_sigmoid"]),
                 0, 0, mask.view(torch.uint8).data_ptr(), g_points.data_ptr(),
                 g_points.stride(0) if n > 0 else 2, g_splat.data_ptr(),
                 g_splat.stride(0) if n > 0 else 8, gm.data_ptr(), gs.data_ptr(), gq.data_ptr(),
                 go.data_ptr(), gdc.data_ptr(), grest.data_ptr(), nat.stream_ptr(dev))
        return gm, gs, gq, go, gdc, grest, None, None, None, None


class _Blend(torch.autograd.Function):
    """Blend forward/backward over the splat records of the fused path."""

    @staticmethod
    def forward(ctx, points, splat, indexing_offset, ids, opts):
        dev = points.device
        W, H = opts["width"], opts["height"]
        image = torch.empty((H, W, 3), device=dev, dtype=torch.float32)
        final_t = torch.empty((H * W,), device=dev, dtype=torch.float32)
        pixel_end = torch.empty((H * W,), device=dev, dtype=torch.int32)
        # each list entry's reach mask, written by the forward, read by the backward
        reach = torch.empty((max(ids.shape[0], 1),), device=dev, dtype=torch.uint8)
        # tiles blended longest list first (both passes)
        T = indexing_offset.shape[0]
        order = torch.empty((max(T, 1),), device=dev, dtype=torch.int32)
        st = nat.stream_ptr(dev)
        nat.call("gs_tile_order", T, indexing_offset.data_ptr(), ids.shape[0], order.data_ptr(),
                 st)
        nat.call("gs_blend_forward", T, indexing_offset.data_ptr(),
                 ids.shape[0], ids.data_ptr(), points.shape[0], points.data_ptr(),
                 splat.data_ptr(), W, H,
                 opts["alpha_threshold"], opts["transmittance_threshold"],
                 opts["chi_squared_threshold"], image.data_ptr(), final_t.data_ptr(),
                 pixel_end.data_ptr(), reach.data_ptr(), order.data_ptr(), st)
        ctx.save_for_backward(points, splat, indexing_offset, ids, final_t, pixel_end, reach,
                              order)
        ctx.opts = opts
        return image

    @staticmethod
    def backward(ctx, grad_image):
        points, splat, indexing_offset, ids, final_t, pixel_end, reach, order = ctx.saved_tensors
        o = ctx.opts
        dev = points.device
        n = points.shape[0]
        g = grad_image if grad_image.is_contiguous() else grad_image.contiguous()
        g_points = torch.zeros((n, 2), device=dev, dtype=torch.float32)
        g_splat = torch.zeros((n, 8), device=dev, dtype=torch.float32)
        nat.call("gs_blend_backward", indexing_offset.shape[0], indexing_offset.data_ptr(),
                 ids.shape[0], ids.data_ptr(), n, points.data_ptr(), splat.data_ptr(),
                 g.data_ptr(),
                 final_t.data_ptr(), pixel_end.data_ptr(), o["width"], o["height"],
                 o["alpha_threshold"], o["transmittance_threshold"],
                 o["chi_squared_threshold"], g_points.data_ptr(), g_splat.data_ptr(),
                 reach.data_ptr(), order.data_ptr(), nat.stream_ptr(dev))
        return g_points, g_splat, None, None, None


def render(world_to_camera, intrinsic, width, height, means, scales, quaternions, opacities,
           sh_coeffs_dc, sh_coeffs_rest, near_plane=0.01, far_plane=100.0, min_opacity=1 / 255,
           min_radius=0.5, max_radius=128.0, alpha_threshold=1e-4, transmittance_threshold=1e-4,
           chi_squared_threshold=9.21, sh_sigmoid=False):
    """Render one view; signature and result as src/cuda/wrapper.py:223-294.

    Inputs are already activated (exp scales, unit (x, y, z, w) quaternions,
    sigmoid opacities), fp32 CUDA tensors on one device. Returns
    (image (H, W, 3) clamped to [0, 1] and scaled by 255, points_img (N, 2),
    radii (N, 2)).
    """
    dev = means.device
    if dev.type != "cuda":
        raise RuntimeError("render() needs CUDA tensors; there is no CPU path")
    width, height = int(width), int(height)
    means = _require("means", means, torch.float32, dev, (3,))
    n = means.shape[0]
    scales = _require("scales", scales, torch.float32, dev, (3,))
    quaternions = _require("quaternions", quaternions, torch.float32, dev, (4,))
    opacities = _require("opacities", opacities, torch.float32, dev)
    sh_coeffs_dc = _require("sh_coeffs_dc", sh_coeffs_dc, torch.float32, dev, (3,))
    sh_coeffs_rest = _require("sh_coeffs_rest", sh_coeffs_rest, torch.float32, dev, (15, 3))
    world_to_camera = _require("world_to_camera", world_to_camera, torch.float32, dev)
    intrinsic = _require("intrinsic", intrinsic, torch.float32, dev)
    for nm, t in (("scales", scales), ("quaternions", quaternions), ("opacities", opacities),
                  ("sh_coeffs_dc", sh_coeffs_dc), ("sh_coeffs_rest", sh_coeffs_rest)):
        if t.shape[0] != n:
            raise RuntimeError(f"{nm} has {t.shape[0]} rows, means has {n}")
    opts = dict(width=width, height=height, near_plane=float(near_plane),
                far_plane=float(far_plane), min_opacity=float(min_opacity),
                min_radius=float(min_radius), max_radius=float(max_radius),
                alpha_threshold=float(alpha_threshold),
                transmittance_threshold=float(transmittance_threshold),
                chi_squared_threshold=float(chi_squared_threshold), sh_sigmoid=bool(sh_sigmoid))
    with torch.cuda.device(dev):
        # wrapper.py:260, computed the same way
        camera_pos = (-world_to_camera[:3, :3].t() @ world_to_camera[:3, 3]).contiguous()
        points, splat, depths, radii, mask, counts, total_dev = _Preprocess.apply(
            means, scales, quaternions, opacities, sh_coeffs_dc, sh_coeffs_rest,
            world_to_camera, intrinsic, camera_pos.detach(), opts)
        total = cuda_rasterizer._read_total(total_dev, dev)
        indexing_offset, ids = cuda_rasterizer.tile_layout_from_counts(
            points.detach(), radii, depths, counts, total, width, height)
        image = _Blend.apply(points, splat, indexing_offset, ids, opts)
    return image.clamp(0, 1) * 255, points, radii
