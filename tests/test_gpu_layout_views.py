"""gs_tile_layout_views (every view's tile layout in one cooperative launch)
against one gs_tile_layout per view -- itself bit-exact against the
reference extension and the CPU oracle -- on the same preprocess outputs:
the sorted id lists and the per-tile offsets must be identical. Cases: small
ragged scenes with 1-3 views, a view that sees nothing, configuration 1 (4
views of 1M Gaussians), a clustered 4K view (~100M pairs, 15-bit tile ids)
and an image with more than 65536 tiles (32-bit tile keys, 3 passes)."""
import ctypes
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
nat = importlib.import_module("3dgs_from_scratch_b200._native")
cr = importlib.import_module("3dgs_from_scratch_b200.cuda_rasterizer")
GROUPS = ("means", "scales", "quaternions", "opacities", "sh_coeffs_dc", "sh_coeffs_rest")


def preprocess(gs, raw, w2c, K, W, H):
    V, n = w2c.shape[0], raw["means"].shape[0]
    Ks = K.expand(V, 3, 3).contiguous()
    campos = (-(w2c[:, :3, :3].transpose(1, 2) @ w2c[:, :3, 3:4])).squeeze(-1).contiguous()
    f = dict(device=DEV, dtype=torch.float32)
    b = dict(points=torch.empty((V, n, 2), **f), depths=torch.empty((V, n), **f),
             radii=torch.empty((V, n, 2), **f),
             mask=torch.empty((V, n), device=DEV, dtype=torch.uint8),
             splat=torch.empty((V, n, 8), **f),
             counts=torch.empty((V, max(n, 1)), device=DEV, dtype=torch.int32))
    totals = torch.empty(V, dtype=torch.int64, device=DEV)
    nat.call("gs_preprocess_forward_views", n, V, *[raw[k].data_ptr() for k in GROUPS],
             w2c.data_ptr(), Ks.data_ptr(), campos.data_ptr(), 0.01, 100.0, 1 / 255, 0.5, 128.0,
             W, H, 0, 1, b["points"].data_ptr(), b["depths"].data_ptr(), b["radii"].data_ptr(),
             b["mask"].data_ptr(), b["splat"].data_ptr(), b["counts"].data_ptr(),
             totals.data_ptr(), nat.stream_ptr())
    return b, [int(x) for x in totals.cpu()]


def layout_views(b, totals, n, W, H):
    V = len(totals)
    tot_c = (ctypes.c_int64 * V)(*totals)
    T = ((W + 15) // 16) * ((H + 15) // 16)
    ids = torch.full((max(sum(totals), 1),), -7, device=DEV, dtype=torch.int32)
    offs = torch.full((V, T), -7, device=DEV, dtype=torch.int32)
    nb = int(nat.query("gs_tile_layout_views_scratch_bytes", n, V,
                       ctypes.cast(tot_c, ctypes.c_void_p), W, H))
    scratch = torch.empty((max(nb, 1),), device=DEV, dtype=torch.uint8)
    nat.call("gs_tile_layout_views", n, V, b["points"].data_ptr(), b["radii"].data_ptr(),
             b["depths"].data_ptr(), b["counts"].data_ptr(), ctypes.cast(tot_c, ctypes.c_void_p),
             W, H, ids.data_ptr(), offs.data_ptr(), scratch.data_ptr(), nb, nat.stream_ptr())
    torch.cuda.synchronize()
    assert nat.query("gs_check_status", nat.stream_ptr()) == 0
    return ids, offs


def check(gs, cfg, n, W, H, w2c, seed=0):
    raw = {k: v.to(DEV) for k, v in gs.scenes.make_gaussians(cfg, seed=seed, n=n).items()}
    n = raw["means"].shape[0]
    K = gs.scenes.intrinsic_for(cfg, W, H).to(DEV)
    w2c = w2c.to(DEV).contiguous()
    b, totals = preprocess(gs, raw, w2c, K, W, H)
    ids, offs = layout_views(b, totals, n, W, H)
    start = 0
    for v, tot in enumerate(totals):
        r_off, r_ids = cr.tile_layout_from_counts(b["points"][v], b["radii"][v], b["depths"][v],
                                                  b["counts"][v], tot, W, H, method="sort")
        assert torch.equal(offs[v], r_off), f"view {v} offsets"
        assert torch.equal(ids[start:start + tot], r_ids), f"view {v} ids"
        start += tot
    return totals


@pytest.mark.parametrize("n,V", [(20_000, 1), (20_000 + 37, 3), (513, 2), (1, 1)])
def test_small_scenes(gs, n, V):
    cfg = gs.scenes.CONFIGS[0]
    totals = check(gs, cfg, n, 256, 256, gs.scenes.orbit_cameras(cfg, V))
    if n > 1000:
        assert min(totals) > 0


def test_a_view_that_sees_nothing(gs):
    cfg = gs.scenes.CONFIGS[0]
    cams = gs.scenes.orbit_cameras(cfg, 3)
    away = gs.scenes.look_at((0.0, 0.0, -4.0), (0.0, 0.0, -10.0))  # scene behind the camera
    totals = check(gs, cfg, 20_000, 200, 120, torch.stack([cams[0], away, cams[2]]))
    assert totals[1] == 0 and totals[0] > 0 and totals[2] > 0


def test_config1_four_views(gs):
    cfg = gs.scenes.CONFIGS[1]
    totals = check(gs, cfg, None, cfg.width, cfg.height, gs.scenes.orbit_cameras(cfg, 4))
    assert sum(totals) > 15_000_000


def test_config3_4k_view(gs):
    cfg = gs.scenes.CONFIGS[3]
    totals = check(gs, cfg, None, cfg.width, cfg.height, gs.scenes.primary_camera(cfg)[None])
    assert totals[0] > 50_000_000


def test_more_than_65536_tiles(gs):
    cfg = gs.scenes.CONFIGS[1]
    W, H = 5120, 3840  # 320 x 240 = 76800 tiles: 32-bit tile keys, 17 bits
    check(gs, cfg, 200_000, W, H, gs.scenes.orbit_cameras(cfg, 2))
