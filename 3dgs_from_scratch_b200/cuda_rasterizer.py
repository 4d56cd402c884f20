"""The reference's native module API, served by the B200 kernels.

ruguangyou/3dgs_from_scratch builds a pybind11 module `cuda_rasterizer`
(src/cuda/rasterizer.cpp:442-464) with seven functions. This module offers the
same seven functions, with the same argument order, output tuples, dtypes
and zero / one initialisation of outputs, on top of the C ABI of
lib3dgs_b200.so. Putting `3dgs_from_scratch_b200/dropin` on sys.path makes
`import cuda_rasterizer` resolve here, so the reference's own
src/cuda/wrapper.py and scripts/check_cuda_gradients.py run unchanged.

Tensors must be CUDA fp32 (bool mask, int32 layout tensors) on one device;
everything is launched on torch's current stream. Errors raise RuntimeError.
"""
from __future__ import annotations

import torch

from . import _native as nat

TILE = 16


def _check(name, t, dtype, device):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if t.device.type != "cuda":
        raise RuntimeError(f"{name} must be a CUDA tensor (got {t.device})")
    if device is not None and t.device != device:
        raise RuntimeError(f"{name} is on {t.device}, expected {device}")
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype} (got {t.dtype})")


def _c(t):
    return t if t.is_contiguous() else t.contiguous()


def _ptr(t):
    return t.data_ptr() if t is not None else None


def _mask_u8(mask):
    # a bool tensor is one byte per element; the kernels read it as uint8
    return mask.view(torch.uint8) if mask.dtype == torch.bool else mask


def project_points(points_world, scales, quaternions, opacities, world_to_camera, intrinsic,
                   near_plane, far_plane, min_opacity, min_radius, max_radius, width, height):
    """rasterizer.cpp:141-191. Returns (points_image, depths, cov_image,
    cov_inv_image, radii, mask)."""
    dev = points_world.device
    for nm, t in (("points_world", points_world), ("scales", scales),
                  ("quaternions", quaternions), ("opacities", opacities),
                  ("world_to_camera", world_to_camera), ("intrinsic", intrinsic)):
        _check(nm, t, torch.float32, dev)
    pw, sc, qt, op = map(_c, (points_world, scales, quaternions, opacities))
    w2c, K = _c(world_to_camera), _c(intrinsic)
    n = pw.shape[0]
    f = dict(device=dev, dtype=torch.float32)
    points = torch.zeros((n, 2), **f)
    depths = torch.zeros((n,), **f)
    cov = torch.zeros((n, 3), **f)
    conic = torch.zeros((n, 3), **f)
    radii = torch.zeros((n, 2), **f)
    mask = torch.ones((n,), device=dev, dtype=torch.bool)
    with torch.cuda.device(dev):
        nat.call("gs_project_points", n, pw.data_ptr(), sc.data_ptr(), qt.data_ptr(),
                 op.data_ptr(), w2c.data_ptr(), K.data_ptr(), float(near_plane),
                 float(far_plane), float(min_opacity), float(min_radius), float(max_radius),
                 int(width), int(height), points.data_ptr(), depths.data_ptr(), cov.data_ptr(),
                 conic.data_ptr(), radii.data_ptr(), _mask_u8(mask).data_ptr(),
                 nat.stream_ptr(dev))
    return points, depths, cov, conic, radii, mask


def project_points_backward(grad_points_image, grad_cov_inv_image, points_world, scales,
                            quaternions, opacities, world_to_camera, intrinsic, width, height,
                            cov_image, mask):
    """rasterizer.cpp:193-232. Returns (grad_points_world, grad_scales,
    grad_quaternions)."""
    dev = points_world.device
    gp, gc, pw, sc, qt = map(_c, (grad_points_image, grad_cov_inv_image, points_world, scales,
                                  quaternions))
    w2c, K, cov, m = _c(world_to_camera), _c(intrinsic), _c(cov_image), _c(mask)
    n = pw.shape[0]
    f = dict(device=dev, dtype=torch.float32)
    g_means = torch.zeros((n, 3), **f)
    g_scales = torch.zeros((n, 3), **f)
    g_quats = torch.zeros((n, 4), **f)
    with torch.cuda.device(dev):
        nat.call("gs_project_points_backward", n, gp.data_ptr(), gc.data_ptr(), pw.data_ptr(),
                 sc.data_ptr(), qt.data_ptr(), w2c.data_ptr(), K.data_ptr(), cov.data_ptr(),
                 _mask_u8(m).data_ptr(), int(width), int(height), g_means.data_ptr(),
                 g_scales.data_ptr(), g_quats.data_ptr(), nat.stream_ptr(dev))
    return g_means, g_scales, g_quats


def evaluate_spherical_harmonics(camera_pos, points_world, sh_coeffs_dc, sh_coeffs_rest, mask,
                                 sh_sigmoid=False):
    """rasterizer.cpp:234-257. Returns colors (N, 3)."""
    dev = points_world.device
    cp, pw, dc, rest, m = map(_c, (camera_pos, points_world, sh_coeffs_dc, sh_coeffs_rest, mask))
    n = pw.shape[0]
    colors = torch.zeros((n, 3), device=dev, dtype=torch.float32)
    with torch.cuda.device(dev):
        nat.call("gs_evaluate_sh", n, cp.data_ptr(), pw.data_ptr(), dc.data_ptr(),
                 rest.data_ptr(), _mask_u8(m).data_ptr(), int(bool(sh_sigmoid)),
                 colors.data_ptr(), nat.stream_ptr(dev))
    return colors


def evaluate_spherical_harmonics_backward(grad_colors, camera_pos, points_world, sh_coeffs_dc,
                                          sh_coeffs_rest, colors, mask, sh_sigmoid=False):
    """rasterizer.cpp:259-290. Returns (grad_points_world, grad_sh_coeffs_dc,
    grad_sh_coeffs_rest)."""
    dev = points_world.device
    gcol, cp, pw, rest, col, m = map(_c, (grad_colors, camera_pos, points_world, sh_coeffs_rest,
                                          colors, mask))
    n = pw.shape[0]
    f = dict(device=dev, dtype=torch.float32)
    g_means = torch.zeros((n, 3), **f)
    g_dc = torch.zeros((n, 3), **f)
    g_rest = torch.zeros((n, 15, 3), **f)
    with torch.cuda.device(dev):
        nat.call("gs_evaluate_sh_backward", n, gcol.data_ptr(), cp.data_ptr(), pw.data_ptr(),
                 rest.data_ptr(), col.data_ptr(), _mask_u8(m).data_ptr(),
                 int(bool(sh_sigmoid)), g_means.data_ptr(), g_dc.data_ptr(), g_rest.data_ptr(),
                 nat.stream_ptr(dev))
    return g_means, g_dc, g_rest


def _read_total(total_dev, dev):
    host = torch.zeros(1, dtype=torch.int64)
    nat.call("gs_read_total", total_dev.data_ptr(), host.data_ptr(), nat.stream_ptr(dev))
    return int(host.item())


# The binned layout (gs_tile_bins) is used while the pairs average at most
# this many per tile: its per-tile radix sorts are cheap for lists of up to
# 4096 entries; scenes whose lists run far longer (the clustered 4K scene of
# configuration 3 averages ~3000 pairs per tile, most of them in lists above
# 4096) go to the two stable sorts of gs_tile_layout. Both give the same
# lists and offsets bit for bit.
BIN_MAX_PAIRS_PER_TILE = 2560


def tile_layout_from_counts(points_image, radii, depths, counts, total, width, height,
                            return_keys=False, method="auto"):
    """Tile layout (pairs sorted by tile then depth bits, and per-tile start
    offsets) from the per-Gaussian tile counts and their total. method:
    "sort" (gs_tile_layout, the two stable sorts; also whenever the keys are
    returned), "bins" (gs_tile_bins) or "auto" (bins while the pairs average
    at most BIN_MAX_PAIRS_PER_TILE per tile)."""
    if method not in ("auto", "sort", "bins"):
        raise ValueError(f"unknown tile layout method {method!r}")
    dev = points_image.device
    tx, ty = (width + TILE - 1) // TILE, (height + TILE - 1) // TILE
    n = points_image.shape[0]
    bins = method == "bins" or (method == "auto" and total <= BIN_MAX_PAIRS_PER_TILE * tx * ty)
    if bins and not return_keys and total > 0:
        # capacity = the exact total, so the device-side count always fits
        offsets = torch.empty((tx * ty + 1,), device=dev, dtype=torch.int32)
        ids = torch.empty((total,), device=dev, dtype=torch.int32)
        total_dev = torch.empty((1,), device=dev, dtype=torch.int64)
        nbytes = int(nat.query("gs_tile_bins_scratch_bytes", n, int(total), int(width),
                               int(height)))
        scratch = torch.empty((max(nbytes, 8),), device=dev, dtype=torch.uint8)
        nat.call("gs_tile_bins", n, points_image.data_ptr(), radii.data_ptr(), depths.data_ptr(),
                 counts.data_ptr(), int(total), int(width), int(height), ids.data_ptr(),
                 offsets.data_ptr(), total_dev.data_ptr(), scratch.data_ptr(), nbytes, None,
                 nat.stream_ptr(dev))
        return offsets[:tx * ty], ids
    indexing_offset = torch.empty((tx * ty,), device=dev, dtype=torch.int32)
    ids = torch.empty((total,), device=dev, dtype=torch.int32)
    keys = torch.empty((total,), device=dev, dtype=torch.int64) if return_keys else None
    nbytes = int(nat.query("gs_tile_layout_scratch_bytes", n, total, int(width), int(height)))
    scratch = torch.empty((nbytes,), device=dev, dtype=torch.uint8)
    nat.call("gs_tile_layout", n, points_image.data_ptr(), radii.data_ptr(), depths.data_ptr(),
             counts.data_ptr(), int(total), int(width), int(height),
             keys.data_ptr() if keys is not None else None, ids.data_ptr(),
             indexing_offset.data_ptr(), scratch.data_ptr(), nbytes, nat.stream_ptr(dev))
    if return_keys:
        return indexing_offset, ids, keys
    return indexing_offset, ids


def compute_tile_intersection(points_image, radii, depths, mask, width, height, tile_size=16,
                              return_keys=False):
    """rasterizer.cpp:292-359. Returns (indexing_offset int32[tiles],
    gaussian_ids_sorted int32[K])."""
    if int(tile_size) != TILE:
        raise ValueError("only 16x16 tiles are supported (the reference hard-codes 16)")
    dev = points_image.device
    pts, rad, dep, m = map(_c, (points_image, radii, depths, mask))
    n = pts.shape[0]
    with torch.cuda.device(dev):
        st = nat.stream_ptr(dev)
        counts = torch.zeros((max(n, 1),), device=dev, dtype=torch.int32)
        offsets = torch.empty((max(n, 1),), device=dev, dtype=torch.int32)
        total_dev = torch.zeros((1,), device=dev, dtype=torch.int64)
        nat.call("gs_count_tiles", n, pts.data_ptr(), rad.data_ptr(), _mask_u8(m).data_ptr(),
                 int(width), int(height), counts.data_ptr(), st)
        sbytes = int(nat.query("gs_scan_scratch_bytes", n))
        scratch = torch.empty((max(sbytes, 8),), device=dev, dtype=torch.uint8)
        nat.call("gs_exclusive_scan", n, counts.data_ptr(), offsets.data_ptr(),
                 total_dev.data_ptr(), scratch.data_ptr(), sbytes, st)
        total = _read_total(total_dev, dev)
        return tile_layout_from_counts(pts, rad, dep, counts, total, int(width), int(height),
                                       return_keys=return_keys)


def rasterize(indexing_offset, gaussian_ids_sorted, points_image, cov_inv_image, opacities,
              colors, width, height, tile_size, alpha_threshold, transmittance_threshold,
              chi_squared_threshold):
    """rasterizer.cpp:361-395. Returns the image (H, W, 3)."""
    if int(tile_size) != TILE:
        raise ValueError("only 16x16 tiles are supported (the reference hard-codes 16)")
    dev = points_image.device
    off, ids, pts, conic, op, col = map(_c, (indexing_offset, gaussian_ids_sorted, points_image,
                                             cov_inv_image, opacities, colors))
    image = torch.zeros((int(height), int(width), 3), device=dev, dtype=torch.float32)
    work_t = torch.empty((int(height) * int(width),), device=dev, dtype=torch.float32)
    work_e = torch.empty((int(height) * int(width),), device=dev, dtype=torch.int32)
    with torch.cuda.device(dev):
        nat.call("gs_rasterize", off.shape[0], off.data_ptr(), ids.shape[0], ids.data_ptr(),
                 pts.shape[0], pts.data_ptr(), conic.data_ptr(), op.data_ptr(), col.data_ptr(), int(width),
                 int(height), float(alpha_threshold), float(transmittance_threshold),
                 float(chi_squared_threshold), image.data_ptr(), work_t.data_ptr(),
                 work_e.data_ptr(), nat.stream_ptr(dev))
    return image


def rasterize_backward(grad_rendered_image, indexing_offset, gaussian_ids_sorted, points_image,
                       cov_inv_image, opacities, colors, width, height, tile_size,
                       alpha_threshold, transmittance_threshold, chi_squared_threshold):
    """rasterizer.cpp:397-440. Returns (grad_points_image, grad_cov_inv_image,
    grad_opacities, grad_colors)."""
    if int(tile_size) != TILE:
        raise ValueError("only 16x16 tiles are supported (the reference hard-codes 16)")
    dev = points_image.device
    g, off, ids, pts, conic, op, col = map(_c, (grad_rendered_image, indexing_offset,
                                                gaussian_ids_sorted, points_image, cov_inv_image,
                                                opacities, colors))
    n = pts.shape[0]
    f = dict(device=dev, dtype=torch.float32)
    gp = torch.zeros((n, 2), **f)
    gc = torch.zeros((n, 3), **f)
    go = torch.zeros((n,), **f)
    gcol = torch.zeros((n, 3), **f)
    work_t = torch.empty((int(height) * int(width),), **f)
    work_e = torch.empty((int(height) * int(width),), device=dev, dtype=torch.int32)
    with torch.cuda.device(dev):
        nat.call("gs_rasterize_backward", off.shape[0], off.data_ptr(), ids.shape[0],
                 ids.data_ptr(), n, g.data_ptr(), pts.data_ptr(), conic.data_ptr(), op.data_ptr(),
                 col.data_ptr(), int(width), int(height), float(alpha_threshold),
                 float(transmittance_threshold), float(chi_squared_threshold), gp.data_ptr(),
                 gc.data_ptr(), go.data_ptr(), gcol.data_ptr(), work_t.data_ptr(),
                 work_e.data_ptr(), nat.stream_ptr(dev))
    return gp, gc, go, gcol
