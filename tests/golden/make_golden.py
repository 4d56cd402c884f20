"""Generate the golden vectors in tests/golden/ from the reference's own code.

Run where the reference checkout is present (its path in $GS_REFERENCE_ROOT,
or a directory named "reference" beside the repository); the generated .npz
files are committed and the tests never read the reference at run time.

What it does:
* imports the reference's Python modules (src/torch_rasterizer.py,
  src/gaussian.py, scripts/check_cuda_gradients.py) with stub modules for
  the packages that are absent here (fused_ssim, pycolmap, imageio) and with
  `cuda_rasterizer` bound to the CPU oracle (oracle/oracle.py);
* runs the reference's gradient checks (check_project_points,
  check_rasterize, check_rasterize_multitile,
  check_rasterize_multitile_truncated, check_sh, check_end_to_end) on the
  CPU, so the reference's own thresholds assess the oracle, and records their
  verdicts in manifest.json;
* captures the reference-side tensors of every check (inputs, upstream
  gradients, the reference's layout from build_reference_tile_layout, its
  image from rasterize_reference, its Torch-autograd gradients) into .npz
  fixtures;
* renders seeded synthetic scenes with the reference Torch rasterizer
  (src/torch_rasterizer.render, device="cpu") and stores image and
  gradients.
"""
from __future__ import annotations

import importlib
import json
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
REF = os.environ.get("GS_REFERENCE_ROOT") or os.path.join(os.path.dirname(REPO), "reference")
sys.path.insert(0, REPO)

from oracle import oracle as orc  # noqa: E402

SCENES = importlib.import_module("3dgs_from_scratch_b200.scenes")


def t2n(t):
    return t.detach().cpu().numpy()


def make_stub_cuda_rasterizer(record):
    """`cuda_rasterizer` backed by the CPU oracle; records every call."""
    m = types.ModuleType("cuda_rasterizer")

    def project_points(*a):
        record.append(("project_points", [x.detach().clone() if torch.is_tensor(x) else x for x in a]))
        np_args = [t2n(x) if torch.is_tensor(x) else x for x in a]
        out = orc.project_points(*np_args)
        return tuple(torch.from_numpy(np.ascontiguousarray(o)) for o in out)

    def project_points_backward(*a):
        record.append(("project_points_backward",
                       [x.detach().clone() if torch.is_tensor(x) else x for x in a]))
        np_args = [t2n(x) if torch.is_tensor(x) else x for x in a]
        out = orc.project_points_backward(*np_args)
        return tuple(torch.from_numpy(o) for o in out)

    def evaluate_spherical_harmonics(camera_pos, means, dc, rest, mask, sh_sigmoid=False):
        record.append(("evaluate_spherical_harmonics",
                       [x.detach().clone() if torch.is_tensor(x) else x
                        for x in (camera_pos, means, dc, rest, mask, sh_sigmoid)]))
        return torch.from_numpy(orc.evaluate_spherical_harmonics(
            t2n(camera_pos), t2n(means), t2n(dc), t2n(rest), t2n(mask), sh_sigmoid))

    def evaluate_spherical_harmonics_backward(g, camera_pos, means, dc, rest, colors, mask,
                                              sh_sigmoid=False):
        out = orc.evaluate_spherical_harmonics_backward(
            t2n(g), t2n(camera_pos), t2n(means), t2n(dc), t2n(rest), t2n(colors), t2n(mask),
            sh_sigmoid)
        return tuple(torch.from_numpy(o) for o in out)

    def compute_tile_intersection(points, radii, depths, mask, width, height, tile_size=16):
        record.append(("compute_tile_intersection",
                       [x.detach().clone() if torch.is_tensor(x) else x
                        for x in (points, radii, depths, mask, width, height, tile_size)]))
        off, ids = orc.compute_tile_intersection(t2n(points), t2n(radii), t2n(depths), t2n(mask),
                                                 width, height, tile_size)
        return torch.from_numpy(off), torch.from_numpy(ids)

    def rasterize(*a):
        record.append(("rasterize", [x.detach().clone() if torch.is_tensor(x) else x for x in a]))
        np_args = [t2n(x) if torch.is_tensor(x) else x for x in a]
        return torch.from_numpy(orc.rasterize(*np_args))

    def rasterize_backward(*a):
        record.append(("rasterize_backward",
                       [x.detach().clone() if torch.is_tensor(x) else x for x in a]))
        np_args = [t2n(x) if torch.is_tensor(x) else x for x in a]
        return tuple(torch.from_numpy(o) for o in orc.rasterize_backward(*np_args))

    for f in (project_points, project_points_backward, evaluate_spherical_harmonics,
              evaluate_spherical_harmonics_backward, compute_tile_intersection, rasterize,
              rasterize_backward):
        setattr(m, f.__name__, f)
    return m


def install_stubs(record):
    sys.modules["cuda_rasterizer"] = make_stub_cuda_rasterizer(record)
    fs = types.ModuleType("fused_ssim")
    fs.fused_ssim = lambda *a, **k: (_ for _ in ()).throw(RuntimeError("fused_ssim absent"))
    sys.modules["fused_ssim"] = fs
    pc = types.ModuleType("pycolmap")
    pc.SceneManager = object
    sys.modules["pycolmap"] = pc
    im = types.ModuleType("imageio")
    im.v2 = types.ModuleType("imageio.v2")
    sys.modules["imageio"] = im
    sys.modules["imageio.v2"] = im.v2
    sys.path.insert(0, REF)
    sys.path.insert(0, os.path.join(REF, "src"))


class Capture:
    """Records torch.autograd.grad results and metric() arguments."""

    def __init__(self, ccg):
        self.ccg = ccg
        self.grads = []
        self.metrics = []

    def __enter__(self):
        self._grad = torch.autograd.grad
        self._metric = self.ccg.metric

        def grad(*a, **k):
            out = self._grad(*a, **k)
            self.grads.append([g.detach().clone() for g in out])
            return out

        def metric(name, a, b):
            self.metrics.append((name, a.detach().clone(), b.detach().clone()))
            return self._metric(name, a, b)

        torch.autograd.grad = grad
        self.ccg.metric = metric
        return self

    def __exit__(self, *exc):
        torch.autograd.grad = self._grad
        self.ccg.metric = self._metric
        return False


def last_call(record, name):
    for n, args in reversed(record):
        if n == name:
            return args
    raise KeyError(name)


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    record = []
    install_stubs(record)
    ccg = importlib.import_module("scripts.check_cuda_gradients")
    trz = importlib.import_module("src.torch_rasterizer")
    thr = ccg.Thresholds()
    manifest = {"reference_root": REF, "checks": {}, "fixtures": []}

    def save(name, **arrays):
        path = os.path.join(HERE, name)
        np.savez_compressed(path, **{k: (t2n(v) if torch.is_tensor(v) else np.asarray(v))
                                     for k, v in arrays.items()})
        manifest["fixtures"].append(name)

    # 1. projection backward vs Torch autograd (check_cuda_gradients.py:196-338)
    with Capture(ccg) as cap:
        ok = ccg.check_project_points(0, "cpu", thr)
    manifest["checks"]["project_points_seed0"] = bool(ok)
    fwd = last_call(record, "project_points")
    bwd = last_call(record, "project_points_backward")
    ref_gp, ref_gs, ref_gq = cap.grads[-1]
    save("project_points_seed0.npz", means=fwd[0], scales=fwd[1], quats=fwd[2], opac=fwd[3],
         w2c=fwd[4], K=fwd[5], near=fwd[6], far=fwd[7], min_opac=fwd[8], min_rad=fwd[9],
         max_rad=fwd[10], width=fwd[11], height=fwd[12], up_points=bwd[0], up_conic=bwd[1],
         ref_grad_means=ref_gp, ref_grad_scales=ref_gs, ref_grad_quats=ref_gq)

    # 2. single-tile rasterize vs rasterize_reference autograd (:341-427)
    with Capture(ccg) as cap:
        ok = ccg.check_rasterize(100, "cpu", thr)
    manifest["checks"]["rasterize_seed100"] = bool(ok)
    a = last_call(record, "rasterize")
    b = last_call(record, "rasterize_backward")
    ref_img = ccg.rasterize_reference(*a)
    gp, gc, go, gcol = cap.grads[-1]
    save("rasterize_seed100.npz", offsets=a[0], ids=a[1], points=a[2], conic=a[3], opac=a[4],
         colors=a[5], width=a[6], height=a[7], athr=a[9], tthr=a[10], chi=a[11],
         upstream=b[0], ref_image=ref_img, ref_grad_points=gp, ref_grad_conic=gc,
         ref_grad_opac=go, ref_grad_colors=gcol)

    # 3/4. multi-tile layouts and blends (:430-785)
    for fn, seed, tag in ((ccg.check_rasterize_multitile, 150, "multitile_seed150"),
                          (ccg.check_rasterize_multitile_truncated, 175, "truncated_seed175")):
        with Capture(ccg) as cap:
            ok = fn(seed, "cpu", thr)
        manifest["checks"][tag] = bool(ok)
        lay = last_call(record, "compute_tile_intersection")
        a = last_call(record, "rasterize")
        b = last_call(record, "rasterize_backward")
        off_ref, ids_ref = ccg.build_reference_tile_layout(*lay)
        ref_img = ccg.rasterize_reference(off_ref, ids_ref, *a[2:])
        gp, gc, go, gcol = cap.grads[-1]
        save(f"{tag}.npz", points=lay[0], radii=lay[1], depths=lay[2], mask=lay[3],
             width=lay[4], height=lay[5], ref_offsets=off_ref, ref_ids=ids_ref, conic=a[3],
             opac=a[4], colors=a[5], athr=a[9], tthr=a[10], chi=a[11], upstream=b[0],
             ref_image=ref_img, ref_grad_points=gp, ref_grad_conic=gc, ref_grad_opac=go,
             ref_grad_colors=gcol)

    # 5. SH vs src.gaussian.evaluate_spherical_harmonics (:788-820)
    with Capture(ccg) as cap:
        ok = ccg.check_sh(200, "cpu", thr)
    manifest["checks"]["sh_seed200"] = bool(ok)
    sh = last_call(record, "evaluate_spherical_harmonics")
    mets = {name: (x, y) for name, x, y in cap.metrics}
    save("sh_seed200.npz", camera_pos=sh[0], means=sh[1], dc=sh[2], rest=sh[3],
         ref_grad_means=mets["means"][1], ref_grad_dc=mets["sh_dc"][1],
         ref_grad_rest=mets["sh_rest"][1])

    # 6. end to end, reference wrapper.render over the oracle vs Torch render (:823-912)
    import functools

    ccg.torch_render = functools.partial(trz.render, device="cpu")  # its default is "cuda"
    with Capture(ccg) as cap:
        ok = ccg.check_end_to_end(300, "cpu", thr)
    manifest["checks"]["end_to_end_seed300"] = bool(ok)
    torch.manual_seed(300)
    count = 384
    means = (torch.rand(count, 3) - 0.5) * 2.0
    means[:, 2] = torch.rand(count) * 2.0 + 1.5
    scales_raw = torch.randn(count, 3) * 0.1
    quats_raw = torch.randn(count, 4)
    opac_raw = torch.randn(count) * 0.5
    dc_raw = torch.randn(count, 3) * 0.2
    rest_raw = torch.randn(count, 15, 3) * 0.05
    seen = [args for n, args in record if n == "project_points"][-1]
    assert torch.equal(seen[0], means), "regenerated end-to-end inputs differ"
    mets = {name: (x, y) for name, x, y in cap.metrics}
    save("end_to_end_seed300.npz", means=means, scales_raw=scales_raw, quats_raw=quats_raw,
         opac_raw=opac_raw, dc_raw=dc_raw, rest_raw=rest_raw, w2c=seen[4], K=seen[5],
         **{f"torch_grad_{k}": v[1] for k, v in mets.items()},
         **{f"oracle_grad_{k}": v[0] for k, v in mets.items()})

    # 7. Torch rasterizer on seeded synthetic scenes (config 0 and a small one)
    for tag, cfg, n, w, h, f, grads in (
            ("torch_render_cfg0", SCENES.CONFIGS[0], None, None, None, None, False),
            ("torch_render_small", SCENES.CONFIGS[0], 2000, 128, 96, 150.0, True)):
        w = cfg.width if w is None else w
        h = cfg.height if h is None else h
        f = cfg.focal if f is None else f
        raw = SCENES.make_gaussians(cfg, seed=1, n=n)
        params = {k: v.clone().requires_grad_(grads) for k, v in raw.items()}
        act = SCENES.activate(params)
        w2c = SCENES.primary_camera(cfg)
        K = torch.tensor([[f, 0, w / 2.0], [0, f, h / 2.0], [0, 0, 1]], dtype=torch.float32)
        img, _, _ = trz.render(w2c, K, w, h, act["means"], act["scales"], act["quaternions"],
                               act["opacities"], act["sh_coeffs_dc"], act["sh_coeffs_rest"],
                               device="cpu")
        out = dict(seed=1, n=raw["means"].shape[0], width=w, height=h, focal=f, w2c=w2c, K=K,
                   image=img)
        if grads:
            target = torch.rand(img.shape, generator=torch.Generator().manual_seed(5)) * 255.0
            loss = torch.nn.functional.l1_loss(img, target)
            loss.backward()
            out.update(target=target, **{f"grad_{k}": v.grad for k, v in params.items()})
        save(f"{tag}.npz", **out)

    with open(os.path.join(HERE, "manifest.json"), "w") as fh:
        json.dump(manifest, fh, indent=1, sort_keys=True)
    print(json.dumps(manifest["checks"], indent=1))


if __name__ == "__main__":
    main()
