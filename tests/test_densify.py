"""Device densification (DeviceStrategy, csrc/densify.cu) against the
reference's Strategy (src/strategy.py), pinned by golden vectors the
reference itself produced on the CPU (tests/golden/make_densify_golden.py):
the same views, the same refining step, the reference's split samples handed
to the kernels; parameters and Adam moments compared group by group."""
import importlib
import os
import socket

import numpy as np
import pytest
import torch

from conftest import golden

dp = importlib.import_module("3dgs_from_scratch_b200.dp")
dens = importlib.import_module("3dgs_from_scratch_b200.densify")
GROUPS = dp.GROUPS
DEV = "cuda"
CASES = ["densify_step600.npz", "densify_step3000.npz", "densify_step3100.npz"]


def _setup(g, device):
    fp = dp.FlatParams({k: torch.tensor(g["before_" + k], device=device) for k in GROUPS})
    fp.exp_avg = torch.zeros(fp.padded, device=device)
    fp.exp_avg_sq = torch.zeros(fp.padded, device=device)
    for k in GROUPS:
        a, n = fp.spans[k]
        fp.exp_avg[a:a + n] = torch.tensor(g["m_before_" + k].ravel(), device=device)
        fp.exp_avg_sq[a:a + n] = torch.tensor(g["v_before_" + k].ravel(), device=device)
    fp.step_count = 2
    return fp


def test_fixtures_are_consistent():
    for name in CASES:
        g = golden(name)
        n_after = g["after_means"].shape[0]
        assert g["probe"].shape[0] == 2 and g["probe"].shape[2] == 3
        for k in GROUPS:
            assert g["after_" + k].shape[0] == n_after
            assert g["m_after_" + k].shape == g["after_" + k].shape


@pytest.mark.gpu
@pytest.mark.parametrize("name", CASES)
def test_refine_matches_reference(name):
    g = golden(name)
    fp = _setup(g, DEV)
    ds = dens.DeviceStrategy()
    step = int(g["step"])
    W, H = int(g["width"]), int(g["height"])
    nv = g["view_grads"].shape[0]
    out = {}
    for v in range(nv):
        gp = torch.tensor(g["view_grads"][v], device=DEV)
        rd = torch.tensor(g["view_radii"][v], device=DEV)
        s = step - (nv - 1) + v
        noise = torch.tensor(g["probe"], device=DEV) if s == step else None
        out = ds.adjust(fp, s, gp, rd, W, H, noise=noise)
    torch.cuda.synchronize()
    assert fp.num_gaussians == g["after_means"].shape[0]
    assert out["split"] == g["probe"].shape[1]
    assert out.get("reset_opacities", False) == (step % 3000 == 0)
    for k in GROUPS:
        a, n = fp.spans[k]
        np.testing.assert_allclose(fp.data[a:a + n].cpu().numpy(), g["after_" + k].ravel(),
                                   rtol=2e-6, atol=2e-7, err_msg=k)
        np.testing.assert_array_equal(fp.exp_avg[a:a + n].cpu().numpy(),
                                      g["m_after_" + k].ravel(), err_msg="m " + k)
        np.testing.assert_array_equal(fp.exp_avg_sq[a:a + n].cpu().numpy(),
                                      g["v_after_" + k].ravel(), err_msg="v " + k)
    assert float(ds.grads.abs().sum()) == 0.0 and ds.grads.shape[0] == fp.num_gaussians


def _quat_to_rot(q):
    q = torch.nn.functional.normalize(q, dim=1)
    x, y, z, w = q.unbind(1)
    return torch.stack([
        torch.stack([1 - 2 * (y * y + z * z), 2 * (x * y - z * w), 2 * (x * z + y * w)], 1),
        torch.stack([2 * (x * y + z * w), 1 - 2 * (x * x + z * z), 2 * (y * z - x * w)], 1),
        torch.stack([2 * (x * z - y * w), 2 * (y * z + x * w), 1 - 2 * (x * x + y * y)], 1)], 1)


@pytest.mark.gpu
def test_generated_split_samples_are_standard_normal():
    """Without given samples the kernel draws its own (Philox): run the same
    refinement with zero samples (outputs = the parents' means) and with
    generated ones, and recover z = R^T (mean' - mean) / scale."""
    g = golden("densify_step600.npz")
    runs = []
    for noise in ("zero", None):
        fp = _setup(g, DEV)
        ds = dens.DeviceStrategy(seed=5)
        for v in range(g["view_grads"].shape[0]):
            ds.accumulate(torch.tensor(g["view_grads"][v], device=DEV),
                          torch.tensor(g["view_radii"][v], device=DEV), 160, 120)
        n_split = int(g["probe"].shape[1])
        z0 = torch.zeros(2, n_split, 3, device=DEV) if noise == "zero" else None
        out = ds.refine(fp, 600, noise=z0)
        runs.append((fp, out))
    (fz, oz), (fr, orr) = runs
    assert oz == orr
    ns, nc = oz["split"], oz["cloned"]
    lo = fz.num_gaussians - 2 * ns
    mean0 = fz.params["means"].detach()[lo:].view(2, ns, 3)
    mean1 = fr.params["means"].detach()[lo:].view(2, ns, 3)
    R = _quat_to_rot(fz.params["quaternions"].detach()[lo:lo + ns])
    sc = torch.exp(fz.params["scales"].detach()[lo:lo + ns]) * 1.6
    z = torch.einsum("sji,ksj->ksi", R, mean1 - mean0) / sc
    assert torch.equal(mean0[0], mean0[1])
    assert abs(float(z.mean())) < 0.15 and abs(float(z.std()) - 1.0) < 0.15
    assert not torch.equal(z[0], z[1])


@pytest.mark.gpu
def test_clone_budget_cap():
    g = golden("densify_step600.npz")
    fp = _setup(g, DEV)
    ref = _setup(g, DEV)
    ds, ds_ref = dens.DeviceStrategy(), dens.DeviceStrategy()
    for v in range(g["view_grads"].shape[0] - 1):
        for d in (ds, ds_ref):
            d.accumulate(torch.tensor(g["view_grads"][v], device=DEV),
                         torch.tensor(g["view_radii"][v], device=DEV), 160, 120)
    full = ds_ref.refine(ref, 600)
    survivors = int(g["n"]) - full["pruned"]
    ds.max_gaussians = survivors + full["cloned"] // 2
    capped = ds.refine(fp, 600)
    assert capped["cloned"] == full["cloned"] // 2
    assert capped["split"] == full["split"]
    assert fp.num_gaussians == survivors - full["split"] + capped["cloned"] + 2 * full["split"]
    # the survivors' section is unchanged
    nk = survivors - full["split"]
    for k in GROUPS:
        a, n = fp.spans[k]
        b, _ = ref.spans[k]
        per = n // fp.num_gaussians
        assert torch.equal(fp.data[a:a + nk * per], ref.data[b:b + nk * per])


@pytest.mark.gpu
def test_no_growth_at_the_cap():
    g = golden("densify_step600.npz")
    fp = _setup(g, DEV)
    ds = dens.DeviceStrategy()
    ds.max_gaussians = 10
    for v in range(g["view_grads"].shape[0]):
        ds.accumulate(torch.tensor(g["view_grads"][v], device=DEV),
                      torch.tensor(g["view_radii"][v], device=DEV), 160, 120)
    out = ds.refine(fp, 600)
    assert out["cloned"] == 0 and out["split"] == 0
    assert fp.num_gaussians == int(g["n"]) - out["pruned"]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _stats_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ds = dens.DeviceStrategy()
        ds.grads = torch.full((7,), float(rank + 1))
        ds.count = torch.full((7,), 2.0 * (rank + 1))
        ds._allreduce_stats()
        np.save(os.path.join(out_dir, f"s{rank}.npy"), torch.stack([ds.grads, ds.count]).numpy())
    finally:
        dist.destroy_process_group()


def test_statistics_are_summed_over_ranks(tmp_path):
    import torch.multiprocessing as mp

    mp.start_processes(_stats_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    for r in range(2):
        s = np.load(tmp_path / f"s{r}.npy")
        assert np.all(s[0] == 3.0) and np.all(s[1] == 6.0)


@pytest.mark.gpu
def test_native_trainer_with_strategy_runs_through_refinement():
    gs = importlib.import_module("3dgs_from_scratch_b200")
    tr_mod = importlib.import_module("3dgs_from_scratch_b200.trainer")
    cfg = gs.scenes.CONFIGS[0]
    raw = gs.scenes.make_gaussians(cfg, seed=4, n=4000)
    W, H, f = 160, 120, 170.0
    K = torch.tensor([[f, 0, W / 2], [0, f, H / 2], [0, 0, 1]], dtype=torch.float32)
    w2cs = gs.scenes.orbit_cameras(cfg, 2)
    gen = torch.Generator().manual_seed(3)
    targets = [(torch.rand((H, W, 3), generator=gen) * 255).round().to(torch.uint8).to(DEV)
               for _ in range(2)]
    ds = dens.DeviceStrategy()
    ds.refine_start_step, ds.refine_every_n_steps, ds.grow_grad = 0, 2, 1e-7
    tr = tr_mod.NativeTrainer({k: v.to(DEV) for k, v in raw.items()}, W, H, strategy=ds,
                              ssim_lambda=0.2)
    sizes = []
    for step in range(1, 6):
        losses = tr.step(w2cs, K, targets, step_index=step)
        assert torch.isfinite(losses).all()
        sizes.append(tr.n)
    assert sizes[0] == 4000 and sizes[1] != 4000  # refined at step 2
    assert all(torch.isfinite(p).all() for p in tr.params.values())
    assert ds.grads.shape[0] == tr.n
