"""bench.py's host-side workload planning, on the CPU: which views a rank
renders per step, the loss, and the scaling mode each configuration
reports (config 2: a fixed 32-view batch sharded over the ranks with the
L1 + 0.2 (1 - SSIM) loss; the others: --views-per-rank views on every rank
with L1)."""
import importlib
import sys

import pytest

from conftest import REPO

sys.path.insert(0, REPO)
bench = importlib.import_module("bench")


def plan(argv, world, rank):
    old = sys.argv
    sys.argv = ["bench.py"] + argv
    try:
        args = bench.parse()
    finally:
        sys.argv = old
    out = bench.view_plan(args, world, rank)
    return args, out


def test_default_is_config1_weak_scaling():
    for world in (1, 2, 8):
        args, (total, mine, lam) = plan([], world, world - 1)
        assert (total, mine, lam) == (4 * world, 4, 0.0)
        assert args.strong is False
        cfg = bench.workload_config(args, bench.scenes.CONFIGS[1], mine)
        assert cfg["global_batch"] == 4 * world and "L1 vs" in cfg["workload"]


def test_config2_shards_a_fixed_batch():
    for world in (1, 2, 4, 8):
        views = [plan(["--config", "2"], world, r)[1][1] for r in range(world)]
        assert sum(views) == 32 and max(views) - min(views) <= 1
        args, (total, _, lam) = plan(["--config", "2"], world, 0)
        assert total == 32 and lam == 0.2 and args.strong is True


def test_explicit_views_and_lambda():
    args, (total, mine, lam) = plan(["--config", "2", "--views-per-rank", "3",
                                     "--ssim-lambda", "0.5"], 2, 1)
    assert (total, mine, lam) == (6, 3, 0.5) and args.strong is False
    args, (total, mine, _) = plan(["--global-views", "7"], 2, 1)
    assert (total, mine) == (7, 3) and args.strong is True
    with pytest.raises(SystemExit):
        plan(["--global-views", "1"], 2, 0)


def test_state_snapshot_round_trip():
    """snapshot_state / restore_state put parameters, Adam moments and the
    step count back in the same buffers (the e2e region replays the
    device-timed steps from that state)."""
    import types

    import torch

    dp = importlib.import_module("3dgs_from_scratch_b200.dp")
    raw = bench.scenes.make_gaussians(bench.scenes.CONFIGS[0], seed=1, n=257)
    fp = dp.FlatParams(raw)
    fp.exp_avg = torch.randn_like(fp.data)
    fp.exp_avg_sq = torch.rand_like(fp.data)
    fp.step_count = 7
    tr = types.SimpleNamespace(fp=fp)
    ptrs = (fp.data.data_ptr(), fp.exp_avg.data_ptr(), fp.exp_avg_sq.data_ptr())
    before = (fp.data.clone(), fp.exp_avg.clone(), fp.exp_avg_sq.clone())
    state = bench.snapshot_state(tr)
    with torch.no_grad():
        fp.data.add_(1.0)
        fp.exp_avg.mul_(3.0)
        fp.exp_avg_sq.zero_()
    fp.step_count = 12
    bench.restore_state(tr, state)
    assert (fp.data.data_ptr(), fp.exp_avg.data_ptr(), fp.exp_avg_sq.data_ptr()) == ptrs
    for a, b in zip((fp.data, fp.exp_avg, fp.exp_avg_sq), before):
        assert torch.equal(a, b)
    assert fp.step_count == 7
