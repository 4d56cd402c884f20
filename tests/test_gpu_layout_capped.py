"""The tile layouts without a host-side pair count -- gs_tile_layout_capped
(two radix sorts) and gs_tile_bins (per-tile binning and bucket sorts) --
against gs_tile_layout, itself bit-exact against the reference extension and
the CPU oracle, on the same preprocess outputs: identical sorted id lists and
per-tile offsets, offsets[tiles] and *total_dev equal to the pair count,
nothing written past it. A count beyond the capacity leaves every list
empty, records GS_ERR_CAPACITY and writes no element of the buffers.
NativeTrainer's step with either (no host synchronisation) equals the
host-sized per-view layout step, and a step that overflows its capacity is
repeated with grown buffers to the same result."""
import importlib

import numpy as np

import pytest
import torch

from test_gpu_layout_views import DEV, GROUPS, cr, nat, preprocess

pytestmark = pytest.mark.gpu

ENTRIES = {"capped": ("gs_tile_layout_capped", "gs_tile_layout_scratch_bytes"),
           "bins": ("gs_tile_bins", "gs_tile_bins_scratch_bytes")}


def capped(b, v, n, cap, W, H, guard=4096, entry="capped"):
    fn, sfn = ENTRIES[entry]
    T = ((W + 15) // 16) * ((H + 15) // 16)
    ids = torch.full((cap + guard,), -7, device=DEV, dtype=torch.int32)
    offs = torch.full((T + 1 + guard,), -7, device=DEV, dtype=torch.int32)
    tot = torch.full((1,), -5, device=DEV, dtype=torch.int64)
    nb = int(nat.query(sfn, n, max(cap, 1), W, H))
    scratch = torch.empty((max(nb, 1),), device=DEV, dtype=torch.uint8)
    # the binned layout also writes the blend order of the tiles
    order = torch.full((T,), -1, device=DEV, dtype=torch.int32) if entry == "bins" else None
    extra = (order.data_ptr(),) if order is not None else ()
    nat.call(fn, n, b["points"][v].data_ptr(), b["radii"][v].data_ptr(),
             b["depths"][v].data_ptr(), b["counts"][v].data_ptr(), cap, W, H, ids.data_ptr(),
             offs.data_ptr(), tot.data_ptr(), scratch.data_ptr(), nb, *extra, nat.stream_ptr())
    torch.cuda.synchronize()
    if order is not None:
        check_blend_order(order, offs[:T + 1])
    return ids, offs, int(tot.item()), T


def check_blend_order(order, offsets):
    """order holds every tile once, longest length class first."""
    order = order.cpu().numpy()
    offs = offsets.cpu().numpy().astype(np.int64)
    T = offs.shape[0] - 1
    assert np.array_equal(np.sort(order), np.arange(T))
    lens = offs[1:] - offs[:-1]
    assert np.all(np.diff(_length_class(lens[order])) <= 0)


def setup(gs, cfg, n, W, H, cams, seed=0):
    raw = {k: v.to(DEV) for k, v in gs.scenes.make_gaussians(cfg, seed=seed, n=n).items()}
    n = raw["means"].shape[0]
    K = gs.scenes.intrinsic_for(cfg, W, H).to(DEV)
    b, totals = preprocess(gs, raw, cams.to(DEV).contiguous(), K, W, H)
    return b, totals, n


CASES = [(0, 20_000, 256, 256, 2), (0, 513, 200, 120, 1), (0, 40, 64, 48, 1),
         (1, None, 1920, 1080, 2), (1, 200_000, 5120, 3840, 1),
         (2, None, 1600, 1064, 1)]  # config 2: a quarter of the buckets above 2048 entries


@pytest.mark.parametrize("entry", ["capped", "bins"])
@pytest.mark.parametrize("cfg_i,n,W,H,V", CASES)
def test_capped_equals_host_sized_layout(gs, cfg_i, n, W, H, V, entry):
    cfg = gs.scenes.CONFIGS[cfg_i]
    b, totals, n = setup(gs, cfg, n, W, H, gs.scenes.orbit_cameras(cfg, V))
    for v, tot in enumerate(totals):
        r_off, r_ids = cr.tile_layout_from_counts(b["points"][v], b["radii"][v], b["depths"][v],
                                                  b["counts"][v], tot, W, H, method="sort")
        for cap in (tot, tot + 12_345):  # exact fit and headroom
            ids, offs, dtot, T = capped(b, v, n, cap, W, H, entry=entry)
            assert nat.query("gs_check_status", nat.stream_ptr()) == 0
            assert dtot == tot
            assert torch.equal(offs[:T], r_off), f"view {v} offsets"
            assert int(offs[T].item()) == tot
            assert torch.equal(ids[:tot], r_ids), f"view {v} ids"
            assert bool((ids[cap:] == -7).all()) and bool((offs[T + 1:] == -7).all())


@pytest.mark.parametrize("cfg_i,n,W,H,V", CASES)
def test_drop_in_layout_methods_agree(gs, cfg_i, n, W, H, V):
    """tile_layout_from_counts (the layout render() and compute_tile_intersection
    use): binned and two-sort forms give the same offsets (one per tile) and
    ids, and "auto" gives them too."""
    cfg = gs.scenes.CONFIGS[cfg_i]
    b, totals, n = setup(gs, cfg, n, W, H, gs.scenes.orbit_cameras(cfg, V))
    for v, tot in enumerate(totals):
        args = (b["points"][v], b["radii"][v], b["depths"][v], b["counts"][v], tot, W, H)
        s_off, s_ids = cr.tile_layout_from_counts(*args, method="sort")
        for method in ("bins", "auto"):
            off, ids = cr.tile_layout_from_counts(*args, method=method)
            assert off.shape == s_off.shape and ids.shape == s_ids.shape, method
            assert torch.equal(off, s_off) and torch.equal(ids, s_ids), (v, method)


def test_bins_config3_clustered_4k_bit_exact(gs):
    """~100M pairs of clustered Gaussians at 3840x2160: buckets far above
    the on-chip chunk, sorted as chunks merged through global scratch."""
    cfg = gs.scenes.CONFIGS[3]
    b, totals, n = setup(gs, cfg, None, cfg.width, cfg.height, gs.scenes.primary_camera(cfg)[None])
    tot = totals[0]
    assert tot > 50_000_000
    r_off, r_ids = cr.tile_layout_from_counts(b["points"][0], b["radii"][0], b["depths"][0],
                                              b["counts"][0], tot, cfg.width, cfg.height,
                                              method="sort")
    ids, offs, dtot, T = capped(b, 0, n, tot, cfg.width, cfg.height, guard=16, entry="bins")
    assert nat.query("gs_check_status", nat.stream_ptr()) == 0
    assert dtot == tot
    lens = torch.diff(torch.cat([r_off, torch.tensor([tot], device=DEV, dtype=torch.int32)]))
    assert int(lens.max()) > 2048  # the merge path ran
    assert torch.equal(offs[:T], r_off)
    assert torch.equal(ids[:tot], r_ids)


@pytest.mark.parametrize("entry", ["capped", "bins"])
def test_capped_overflow_empties_lists_and_reports(gs, entry):
    cfg = gs.scenes.CONFIGS[0]
    b, totals, n = setup(gs, cfg, 20_000, 256, 256, gs.scenes.orbit_cameras(cfg, 1))
    tot = totals[0]
    assert tot > 1000
    ids, offs, dtot, T = capped(b, 0, n, tot - 1, 256, 256, entry=entry)
    assert nat.query("gs_check_status", nat.stream_ptr()) == nat.GS_ERR_CAPACITY
    assert dtot == tot  # the count is reported for the caller to grow its buffers
    assert bool((offs[:T + 1] == 0).all())
    assert bool((ids == -7).all())  # nothing written
    assert nat.query("gs_check_status", nat.stream_ptr()) == 0  # the read cleared it


def _trainer(gs, cfg, layout, n=60_000, W=320, H=240):
    tr_mod = importlib.import_module("3dgs_from_scratch_b200.trainer")
    raw = {k: v.to(DEV) for k, v in gs.scenes.make_gaussians(cfg, seed=5, n=n).items()}
    return tr_mod.NativeTrainer(raw, W, H, layout=layout)


def _scene(gs, V, W=320, H=240, seed=3):
    cfg = gs.scenes.CONFIGS[1]
    K = gs.scenes.intrinsic_for(cfg, W, H).to(DEV)
    cams = gs.scenes.orbit_cameras(cfg, V).to(DEV)
    g = torch.Generator(device=DEV).manual_seed(seed)
    targets = [torch.rand((H, W, 3), device=DEV, generator=g) * 255 for _ in range(V)]
    return cfg, K, cams, targets


def _same_step(a, r):
    """Two trainers after one step from the same parameters: gradients equal
    up to the order of the blend's atomics (the reference's pass rule), so
    each parameter differs by at most the two Adam updates' difference."""
    from conftest import assert_close_metric

    for k in GROUPS:
        s0, n = a.fp.spans[k]
        assert_close_metric(k, a.fp.grad[s0:s0 + n].double().cpu().numpy(),
                            r.fp.grad[s0:s0 + n].double().cpu().numpy(), 0.99999, 1e-4)
        d = (a.params[k] - r.params[k]).abs().max().item()
        assert d <= 2.0 * a.fp.lrs[k] * 1.001, (k, d)


@pytest.mark.parametrize("layout", ["capped", "binned"])
def test_trainer_capped_step_equals_host_sized_step(gs, layout):
    cfg, K, cams, targets = _scene(gs, 3)
    a = _trainer(gs, cfg, layout)
    r = _trainer(gs, cfg, "per_view")
    for step in range(2):
        la = a.step(cams, K, targets, check_status=step == 1)
        lr = r.step(cams, K, targets)
        torch.cuda.synchronize()
        if step == 0:
            assert torch.allclose(la, lr, rtol=1e-9, atol=0)  # identical forward
            _same_step(a, r)
        else:  # the first step without a host read (the first one sized the buffers)
            assert a._cap is not None
            assert torch.allclose(la, lr, rtol=1e-5, atol=0)
    a.check_status()


@pytest.mark.parametrize("layout", ["capped", "binned"])
def test_trainer_repeats_a_step_that_overflows(gs, layout):
    cfg, K, cams, targets = _scene(gs, 2, seed=4)
    a = _trainer(gs, cfg, layout)
    r = _trainer(gs, cfg, "per_view")
    a.forward_views(cams, K)  # sizes the capacity form's buffers
    torch.cuda.synchronize()
    cap, key, bufs = a._cap
    a._cap = (1024, key, bufs)  # below every view's pair count
    la = a.step(cams, K, targets)  # overflows, skips its update, grows, repeats
    lr = r.step(cams, K, targets)
    torch.cuda.synchronize()
    assert a._cap[0] > 1024
    assert torch.allclose(la, lr, rtol=1e-9, atol=0)
    _same_step(a, r)


@pytest.mark.parametrize("cfg_i,n,W,H", [(0, 20_000, 256, 256), (1, None, 1920, 1080)])
def test_blend_backward_reading_kept_reach_masks(gs, cfg_i, n, W, H):
    """gs_blend_backward given the reach masks its forward kept gives the
    gradients it gives when it recomputes them: the same (pixel, entry)
    pairs contribute, so the two agree up to the order of the atomics."""
    tr_mod = importlib.import_module("3dgs_from_scratch_b200.trainer")
    cfg = gs.scenes.CONFIGS[cfg_i]
    raw = {k: v.to(DEV) for k, v in gs.scenes.make_gaussians(cfg, seed=4, n=n).items()}
    tr = tr_mod.NativeTrainer(raw, W, H, layout="binned")
    K = gs.scenes.intrinsic_for(cfg, W, H).to(DEV)
    cams = gs.scenes.orbit_cameras(cfg, 1).to(DEV)
    views = tr.render_views(cams, K)
    s, o, n = views[0], tr.opts, tr.n
    g = torch.Generator(device=DEV).manual_seed(11)
    grad_img = torch.randn((H, W, 3), device=DEV, generator=g)
    out = []
    for reach in (s["reach"], None):
        gp = torch.zeros((n, 2), device=DEV)
        gsp = torch.zeros((n, 8), device=DEV)
        nat.call("gs_blend_backward", tr.tx * tr.ty, s["offsets"].data_ptr(), s["total"],
                 s["ids"].data_ptr(), n, s["points"].data_ptr(), s["splat"].data_ptr(),
                 grad_img.data_ptr(), s["final_t"].data_ptr(), s["pixel_end"].data_ptr(), W, H,
                 o["alpha_threshold"], o["transmittance_threshold"],
                 o["chi_squared_threshold"], gp.data_ptr(), gsp.data_ptr(),
                 reach.data_ptr() if reach is not None else None, None, nat.stream_ptr())
        out.append((gp, gsp))
    torch.cuda.synchronize()
    assert nat.query("gs_check_status", nat.stream_ptr()) == 0
    for a, b in zip(out[0], out[1]):
        scale = b.abs().max().item()
        assert scale > 0
        assert (a - b).abs().max().item() <= 1e-5 * scale


def _length_class(n):
    """Host restatement of the tile-order length class (exact below 8, then
    8 classes per power of two)."""
    n = n.astype(np.int64)
    e = np.floor(np.log2(np.maximum(n, 1))).astype(np.int64)
    cls = (e << 3) | ((n >> np.maximum(e - 3, 0)) & 7)
    return np.where(n < 8, np.maximum(n, 0), cls)


@pytest.mark.parametrize("cfg_i,n,W,H", [(0, 20_000, 256, 256), (1, None, 1920, 1080)])
def test_tile_order_and_ordered_blend(gs, cfg_i, n, W, H):
    """gs_tile_order returns every tile once, longest length class first; the
    forward blend in that order writes the same image, final transmittance
    and end indices bit for bit, and the backward the same gradients up to
    the order of the atomics."""
    tr_mod = importlib.import_module("3dgs_from_scratch_b200.trainer")
    cfg = gs.scenes.CONFIGS[cfg_i]
    raw = {k: v.to(DEV) for k, v in gs.scenes.make_gaussians(cfg, seed=4, n=n).items()}
    tr = tr_mod.NativeTrainer(raw, W, H, layout="binned")
    K = gs.scenes.intrinsic_for(cfg, W, H).to(DEV)
    cams = gs.scenes.orbit_cameras(cfg, 1).to(DEV)
    s = tr.render_views(cams, K)[0]
    o, n, T = tr.opts, tr.n, tr.tx * tr.ty
    check_blend_order(s["order"], s["offsets"])  # written by the binned layout
    standalone = torch.full((T,), -1, device=DEV, dtype=torch.int32)
    nat.call("gs_tile_order", T, s["offsets"].data_ptr(), s["total"], standalone.data_ptr(),
             nat.stream_ptr())
    check_blend_order(standalone, s["offsets"])
    g = torch.Generator(device=DEV).manual_seed(12)
    grad_img = torch.randn((H, W, 3), device=DEV, generator=g)
    res = []
    for ordered in (True, False):
        img = torch.empty((H, W, 3), device=DEV)
        ft = torch.empty((H * W,), device=DEV)
        pe = torch.empty((H * W,), device=DEV, dtype=torch.int32)
        reach = torch.empty_like(s["reach"])
        ordp = s["order"].data_ptr() if ordered else None
        nat.call("gs_blend_forward", T, s["offsets"].data_ptr(), s["total"], s["ids"].data_ptr(),
                 n, s["points"].data_ptr(), s["splat"].data_ptr(), W, H, o["alpha_threshold"],
                 o["transmittance_threshold"], o["chi_squared_threshold"], img.data_ptr(),
                 ft.data_ptr(), pe.data_ptr(), reach.data_ptr(), ordp, nat.stream_ptr())
        gp = torch.zeros((n, 2), device=DEV)
        gsp = torch.zeros((n, 8), device=DEV)
        nat.call("gs_blend_backward", T, s["offsets"].data_ptr(), s["total"],
                 s["ids"].data_ptr(), n, s["points"].data_ptr(), s["splat"].data_ptr(),
                 grad_img.data_ptr(), ft.data_ptr(), pe.data_ptr(), W, H,
                 o["alpha_threshold"], o["transmittance_threshold"],
                 o["chi_squared_threshold"], gp.data_ptr(), gsp.data_ptr(), reach.data_ptr(),
                 ordp, nat.stream_ptr())
        res.append((img, ft, pe, gp, gsp))
    torch.cuda.synchronize()
    assert nat.query("gs_check_status", nat.stream_ptr()) == 0
    for a, b in zip(res[0][:3], res[1][:3]):
        assert torch.equal(a, b)
    for a, b in zip(res[0][3:], res[1][3:]):
        assert (a - b).abs().max().item() <= 1e-5 * b.abs().max().item()
