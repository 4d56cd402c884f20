"""numpy front end of the CPU oracle (oracle/gs_oracle.c).

TEST INFRASTRUCTURE ONLY: the parity checker for the CUDA path and the timed
CPU baseline of bench.py. The shipped package never imports this module.

Each function mirrors one function of the reference's native module
`cuda_rasterizer` (src/cuda/rasterizer.cpp:141-440): same argument order and
meaning, same outputs, same zero / one initialisation of the outputs. Arrays
are numpy float32 / int32 / bool, C-contiguous. `render_forward` and
`render_backward` compose them the way src/cuda/wrapper.py:223-294 does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "gs_oracle.c")
LIB = os.path.join(HERE, "_build", "libgs_oracle.so")
TILE = 16

_lib = None


def build() -> str:
    """Compile gs_oracle.c into oracle/_build/libgs_oracle.so (skipped if fresh)."""
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    cmd = ["gcc", "-O2", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-Wall",
           "-o", LIB, SRC, "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _lib.or_num_threads.restype = ctypes.c_int
    return _lib


def set_num_threads(n: int) -> None:
    lib().or_set_num_threads(ctypes.c_int(int(n)))


def num_threads() -> int:
    return int(lib().or_num_threads())


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _f(x):
    return ctypes.c_float(float(x))


def _i(x):
    return ctypes.c_int(int(x))


def camera_position(world_to_camera):
    """-R^T t in float32 (src/cuda/wrapper.py:260)."""
    W = _f32(world_to_camera)
    R = W[:3, :3]
    t = W[:3, 3]
    out = np.zeros(3, np.float32)
    for j in range(3):
        acc = np.float32(0.0)
        for i in range(3):
            acc = np.float32(acc + R[i, j] * t[i])
        out[j] = -acc
    return out


def project_points(means, scales, quats, opacities, world_to_camera, intrinsic, near_plane,
                   far_plane, min_opacity, min_radius, max_radius, width, height):
    """Reference `project_points` (rasterizer.cpp:141-191, kernel.cu:411-500)."""
    means, scales, quats, opacities = map(_f32, (means, scales, quats, opacities))
    W, K = _f32(world_to_camera).reshape(16), _f32(intrinsic).reshape(9)
    n = means.shape[0]
    points = np.zeros((n, 2), np.float32)
    depths = np.zeros(n, np.float32)
    cov = np.zeros((n, 3), np.float32)
    conic = np.zeros((n, 3), np.float32)
    radii = np.zeros((n, 2), np.float32)
    mask = np.ones(n, np.uint8)
    lib().or_project_points(_i(n), _p(means), _p(scales), _p(quats), _p(opacities), _p(W), _p(K),
                            _f(near_plane), _f(far_plane), _f(min_opacity), _f(min_radius),
                            _f(max_radius), _i(width), _i(height), _p(points), _p(depths),
                            _p(cov), _p(conic), _p(radii), _p(mask))
    return points, depths, cov, conic, radii, mask.astype(bool)


def project_points_backward(g_points, g_conic, means, scales, quats, opacities,
                            world_to_camera, intrinsic, width, height, cov, mask):
    """Reference `project_points_backward` (rasterizer.cpp:193-232)."""
    g_points, g_conic, means, scales, quats, cov = map(
        _f32, (g_points, g_conic, means, scales, quats, cov))
    W, K = _f32(world_to_camera).reshape(16), _f32(intrinsic).reshape(9)
    m = np.ascontiguousarray(mask, dtype=np.uint8)
    n = means.shape[0]
    gm = np.zeros((n, 3), np.float32)
    gs = np.zeros((n, 3), np.float32)
    gq = np.zeros((n, 4), np.float32)
    lib().or_project_points_backward(_i(n), _p(g_points), _p(g_conic), _p(means), _p(scales),
                                     _p(quats), _p(W), _p(K), _p(cov), _p(m), _i(width),
                                     _i(height), _p(gm), _p(gs), _p(gq))
    return gm, gs, gq


def evaluate_spherical_harmonics(camera_pos, means, sh_dc, sh_rest, mask, sh_sigmoid=False):
    """Reference `evaluate_spherical_harmonics` (rasterizer.cpp:234-257)."""
    campos, means, sh_dc, sh_rest = map(_f32, (camera_pos, means, sh_dc, sh_rest))
    m = np.ascontiguousarray(mask, dtype=np.uint8)
    n = means.shape[0]
    colors = np.zeros((n, 3), np.float32)
    lib().or_sh_forward(_i(n), _p(campos), _p(means), _p(sh_dc), _p(sh_rest), _p(m),
                        _i(bool(sh_sigmoid)), _p(colors))
    return colors


def evaluate_spherical_harmonics_backward(g_colors, camera_pos, means, sh_dc, sh_rest, colors,
                                          mask, sh_sigmoid=False):
    """Reference `evaluate_spherical_harmonics_backward` (rasterizer.cpp:259-290)."""
    g_colors, campos, means, sh_rest, colors = map(
        _f32, (g_colors, camera_pos, means, sh_rest, colors))
    m = np.ascontiguousarray(mask, dtype=np.uint8)
    n = means.shape[0]
    gm = np.zeros((n, 3), np.float32)
    gdc = np.zeros((n, 3), np.float32)
    grest = np.zeros((n, 15, 3), np.float32)
    lib().or_sh_backward(_i(n), _p(g_colors), _p(campos), _p(means), _p(sh_rest), _p(colors),
                         _p(m), _i(bool(sh_sigmoid)), _p(gm), _p(gdc), _p(grest))
    return gm, gdc, grest


def count_tiles(points, radii, mask, width, height, tile_size=TILE):
    points, radii = _f32(points), _f32(radii)
    m = np.ascontiguousarray(mask, dtype=np.uint8)
    n = points.shape[0]
    counts = np.zeros(n, np.int32)
    lib().or_count_tiles(_i(n), _p(points), _p(radii), _p(m), _i(width), _i(height),
                         _i(tile_size), _p(counts))
    return counts


def compute_tile_intersection(points, radii, depths, mask, width, height, tile_size=TILE,
                              return_keys=False):
    """Reference `compute_tile_intersection` (rasterizer.cpp:292-359).

    Returns (indexing_offset int32[tiles], gaussian_ids_sorted int32[K]) and,
    with return_keys, the sorted int64 keys too.
    """
    points, radii, depths = _f32(points), _f32(radii), _f32(depths)
    m = np.ascontiguousarray(mask, dtype=np.uint8)
    n = points.shape[0]
    counts = count_tiles(points, radii, m, width, height, tile_size)
    total = int(counts.astype(np.int64).sum())
    tx = (width + tile_size - 1) // tile_size
    ty = (height + tile_size - 1) // tile_size
    offsets = np.zeros(tx * ty, np.int32)
    keys = np.zeros(total, np.int64)
    ids = np.zeros(total, np.int32)
    lib().or_tile_layout(_i(n), _p(points), _p(radii), _p(depths), _p(m), _p(counts),
                         _i(width), _i(height), _i(tile_size), ctypes.c_int64(total), _p(keys),
                         _p(ids), _p(offsets))
    if return_keys:
        return offsets, ids, keys
    return offsets, ids


def rasterize(indexing_offset, gaussian_ids_sorted, points, conic, opacities, colors, width,
              height, tile_size, alpha_threshold, transmittance_threshold, chi_squared_threshold):
    """Reference `rasterize` (rasterizer.cpp:361-395)."""
    off = np.ascontiguousarray(indexing_offset, dtype=np.int32)
    ids = np.ascontiguousarray(gaussian_ids_sorted, dtype=np.int32)
    points, conic, opacities, colors = map(_f32, (points, conic, opacities, colors))
    image = np.zeros((height, width, 3), np.float32)
    if off.shape[0] == 0 or ids.shape[0] == 0:
        return image
    lib().or_rasterize(_p(off), _i(off.shape[0]), _p(ids), ctypes.c_int64(ids.shape[0]),
                       _p(points), _p(conic), _p(opacities), _p(colors), _i(width), _i(height),
                       _i(tile_size), _f(alpha_threshold), _f(transmittance_threshold),
                       _f(chi_squared_threshold), _p(image))
    return image


def rasterize_backward(g_image, indexing_offset, gaussian_ids_sorted, points, conic, opacities,
                       colors, width, height, tile_size, alpha_threshold,
                       transmittance_threshold, chi_squared_threshold):
    """Reference `rasterize_backward` (rasterizer.cpp:397-440)."""
    off = np.ascontiguousarray(indexing_offset, dtype=np.int32)
    ids = np.ascontiguousarray(gaussian_ids_sorted, dtype=np.int32)
    g_image, points, conic, opacities, colors = map(
        _f32, (g_image, points, conic, opacities, colors))
    n = points.shape[0]
    gp = np.zeros((n, 2), np.float32)
    gc = np.zeros((n, 3), np.float32)
    go = np.zeros(n, np.float32)
    gcol = np.zeros((n, 3), np.float32)
    if off.shape[0] == 0 or ids.shape[0] == 0:
        return gp, gc, go, gcol
    lib().or_rasterize_backward(_p(g_image), _p(off), _i(off.shape[0]), _p(ids),
                                ctypes.c_int64(ids.shape[0]), _i(n), _p(points), _p(conic),
                                _p(opacities), _p(colors), _i(width), _i(height),
                                _i(tile_size), _f(alpha_threshold),
                                _f(transmittance_threshold), _f(chi_squared_threshold), _p(gp),
                                _p(gc), _p(go), _p(gcol))
    return gp, gc, go, gcol


DEFAULTS = dict(near_plane=0.01, far_plane=100.0, min_opacity=1 / 255, min_radius=0.5,
                max_radius=128.0, alpha_threshold=1e-4, transmittance_threshold=1e-4,
                chi_squared_threshold=9.21, sh_sigmoid=False)


def render_forward(world_to_camera, intrinsic, width, height, means, scales, quats, opacities,
                   sh_dc, sh_rest, **kw):
    """Forward of src/cuda/wrapper.py:223-294. Returns (image_0_255, state)."""
    o = dict(DEFAULTS)
    o.update(kw)
    pts, depths, cov, conic, radii, mask = project_points(
        means, scales, quats, opacities, world_to_camera, intrinsic, o["near_plane"],
        o["far_plane"], o["min_opacity"], o["min_radius"], o["max_radius"], width, height)
    campos = camera_position(world_to_camera)
    raw = evaluate_spherical_harmonics(campos, means, sh_dc, sh_rest, mask, o["sh_sigmoid"])
    colors = raw if o["sh_sigmoid"] else np.maximum(raw + np.float32(0.5), np.float32(0.0))
    off, ids = compute_tile_intersection(pts, radii, depths, mask, width, height, TILE)
    img = rasterize(off, ids, pts, conic, opacities, colors, width, height, TILE,
                    o["alpha_threshold"], o["transmittance_threshold"],
                    o["chi_squared_threshold"])
    out = np.clip(img, 0.0, 1.0) * np.float32(255.0)
    state = dict(points=pts, depths=depths, cov=cov, conic=conic, radii=radii, mask=mask,
                 campos=campos, raw_colors=raw, colors=colors, offsets=off, ids=ids, image=img,
                 opts=o)
    return out.astype(np.float32), state


def render_backward(g_out, state, world_to_camera, intrinsic, width, height, means, scales,
                    quats, opacities, sh_dc, sh_rest):
    """Backward of render(): gradients w.r.t. (means, scales, quats, opacities,
    sh_dc, sh_rest) and points_img, given d loss / d image_0_255."""
    o = state["opts"]
    img = state["image"]
    g_img = (np.float32(255.0) * _f32(g_out) * ((img >= 0) & (img <= 1))).astype(np.float32)
    gp, gc, go, gcol = rasterize_backward(
        g_img, state["offsets"], state["ids"], state["points"], state["conic"], opacities,
        state["colors"], width, height, TILE, o["alpha_threshold"],
        o["transmittance_threshold"], o["chi_squared_threshold"])
    if o["sh_sigmoid"]:
        graw = gcol
    else:
        graw = (gcol * (state["raw_colors"] + np.float32(0.5) >= 0)).astype(np.float32)
    gm_sh, gdc, grest = evaluate_spherical_harmonics_backward(
        graw, state["campos"], means, sh_dc, sh_rest, state["raw_colors"], state["mask"],
        o["sh_sigmoid"])
    gm_pr, gs, gq = project_points_backward(gp, gc, means, scales, quats, opacities,
                                            world_to_camera, intrinsic, width, height,
                                            state["cov"], state["mask"])
    return dict(means=gm_pr + gm_sh, scales=gs, quaternions=gq, opacities=go, sh_coeffs_dc=gdc,
                sh_coeffs_rest=grest, points_img=gp)
