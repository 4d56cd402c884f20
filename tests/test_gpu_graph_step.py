"""The training step replayed from CUDA graphs (NativeTrainer.step_graph)
against the eager step, and the table-driven Adam launch it uses against
gs_adam_step: the same update bit for bit, whatever step the uploaded table
describes."""
import importlib

import pytest
import torch

from test_gpu_layout_capped import GROUPS, _same_step, _scene, _trainer

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
nat = importlib.import_module("3dgs_from_scratch_b200._native")
dp = importlib.import_module("3dgs_from_scratch_b200.dp")


def test_table_adam_equals_adam_step_bit_for_bit(gs):
    cfg = gs.scenes.CONFIGS[0]
    raw = {k: v.to(DEV) for k, v in gs.scenes.make_gaussians(cfg, seed=2, n=3001).items()}
    a = dp.FlatParams(dict(raw))
    b = dp.FlatParams(dict(raw))
    b.prepare_table()
    g = torch.Generator(device=DEV).manual_seed(7)
    for step in range(1, 5):
        grad = torch.randn(a.grad.shape, device=DEV, generator=g)
        a.grad.copy_(grad)
        b.grad.copy_(grad)
        a.adam_step()
        b.upload_table(step)
        b.table_adam_step()
        b.step_count = step
        torch.cuda.synchronize()
        assert torch.equal(a.data, b.data), step
        assert torch.equal(a.exp_avg, b.exp_avg) and torch.equal(a.exp_avg_sq, b.exp_avg_sq)


@pytest.mark.parametrize("u8", [False, True])
def test_graph_steps_equal_eager_steps(gs, u8):
    cfg, K, cams, targets = _scene(gs, 3, seed=6)
    if u8:
        targets = [t.round().to(torch.uint8) for t in targets]
    a = _trainer(gs, cfg, "binned")
    r = _trainer(gs, cfg, "binned")
    assert a.graph_capable()
    la = a.step_graph(cams, K, targets, check_status=True)  # eager: sizes the buffers
    lr = r.step(cams, K, targets)
    torch.cuda.synchronize()
    _same_step(a, r)
    launches = []
    for step in range(3):
        n0 = nat.launch_count()
        la = a.step_graph(cams, K, targets, check_status=step == 2).clone()
        launches.append(nat.launch_count() - n0)
        lr = r.step(cams, K, targets)
        torch.cuda.synchronize()
        assert torch.allclose(la, lr, rtol=1e-4, atol=0), (step, la, lr)
    assert a._graph is not None and a.fp.step_count == r.fp.step_count == 4
    assert launches[1] == launches[2] == a._graph["kernels"] > 10
    for k in ("means", "opacities", "sh_coeffs_rest"):
        d = (a.params[k] - r.params[k]).abs().max().item()
        assert d <= 8.0 * a.fp.lrs[k], (k, d)


def test_graph_step_with_host_targets_and_new_cameras(gs):
    """Pinned host targets and cameras that change between replays: the
    replay renders the new views (its losses equal an eager step's from the
    same parameters)."""
    cfg, K, cams, targets = _scene(gs, 2, seed=8)
    host = [t.round().to(torch.uint8).cpu().pin_memory() for t in targets]
    a = _trainer(gs, cfg, "binned")
    for _ in range(2):
        a.step_graph(cams, K, host)
    torch.cuda.synchronize()
    cams2 = gs.scenes.orbit_cameras(cfg, 5)[3:5].to(DEV)
    r = _trainer(gs, cfg, "binned")
    with torch.no_grad():
        r.fp.data.copy_(a.fp.data)
    views = r.forward_views(cams2, K)
    lr = r.loss_and_backward(views, [h.to(DEV) for h in host])
    la = a.step_graph(cams2.cpu().pin_memory(), K.cpu(), host, check_status=True)
    torch.cuda.synchronize()
    assert torch.allclose(la, lr, rtol=1e-6, atol=0)


@pytest.mark.parametrize("graph", [False, True])
def test_adam_overlapped_with_the_backward_equals_one_launch(gs, graph):
    """adam_overlap: the preprocess backward in ranges of Gaussians, each
    range's Adam (gs_adam_step_ranges over its slices of the six groups) on
    a second stream -- the same update as one Adam launch after the whole
    backward (up to the blend's atomics), eagerly and replayed from graphs."""
    cfg, K, cams, targets = _scene(gs, 2, seed=9)
    a = _trainer(gs, cfg, "binned")
    a.adam_overlap = True
    r = _trainer(gs, cfg, "binned")
    assert a.overlap_adam() and not r.overlap_adam()
    run = a.step_graph if graph else a.step
    for step in range(3):
        la = run(cams, K, targets, check_status=True).clone()
        lr = r.step(cams, K, targets)
        torch.cuda.synchronize()
        if step == 0:
            _same_step(a, r)
        assert torch.allclose(la, lr, rtol=1e-4, atol=0)
    assert a.fp.step_count == r.fp.step_count == 3
    for k in GROUPS:
        d = (a.params[k] - r.params[k]).abs().max().item()
        assert d <= 6.0 * a.fp.lrs[k], (k, d)
