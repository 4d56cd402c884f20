"""Data-parallel host logic on CPU ranks (gloo, world size 2): view sharding,
the flat gradient buffer that autograd accumulates into, and the all-reduce
that makes every rank's gradients equal to the sum over ranks."""
import importlib
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

dp = importlib.import_module("3dgs_from_scratch_b200.dp")


def test_shard_views_partitions():
    for n in (0, 1, 7, 32, 33):
        for w in (1, 2, 3, 8):
            shards = [dp.shard_views(n, r, w) for r in range(w)]
            flat = [v for s in shards for v in s]
            assert flat == list(range(n))
            assert max(len(s) for s in shards) - min(len(s) for s in shards) <= 1


def _tensors(n, seed):
    g = torch.Generator().manual_seed(seed)
    return {"means": torch.randn(n, 3, generator=g), "scales": torch.randn(n, 3, generator=g),
            "quaternions": torch.randn(n, 4, generator=g), "opacities": torch.randn(n, generator=g),
            "sh_coeffs_dc": torch.randn(n, 3, generator=g),
            "sh_coeffs_rest": torch.randn(n, 15, 3, generator=g)}


def test_flat_params_views_and_in_place_accumulation():
    fp = dp.FlatParams(_tensors(5, 0))
    assert fp.numel % 4 == 0
    for k in dp.GROUPS:
        p = fp[k]
        assert p.is_leaf and p.requires_grad
        assert p.data_ptr() >= fp.data.data_ptr()
    loss = sum((fp[k] * (i + 1)).sum() for i, k in enumerate(dp.GROUPS))
    loss.backward()
    loss2 = sum((fp[k] * 2).sum() for k in dp.GROUPS)
    loss2.backward()
    for i, k in enumerate(dp.GROUPS):
        a, n = fp.spans[k]
        assert torch.allclose(fp.grad[a:a + n], torch.full((n,), float(i + 1 + 2)))
        assert fp[k].grad.data_ptr() == fp.grad[a:].data_ptr()  # still a view of the flat buffer
    fp.zero_grad()
    assert float(fp.grad.abs().sum()) == 0.0


def _worker(rank, world, port, n, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        fp = dp.FlatParams(_tensors(n, 0))  # identical replicas
        views = dp.shard_views(8, rank, world)
        # each rank's "render" of its views: a loss that depends on the view index
        loss = sum(((fp["means"] * (v + 1)).sum() + (fp["sh_coeffs_rest"] ** 2).sum() * v)
                   for v in views)
        loss.backward()
        fp.allreduce_grads()
        out[rank] = fp.grad.clone()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_allreduce_over_two_gloo_ranks():
    n = 6
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, n, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    # single-process expectation: the gradient of the loss over all 8 views
    fp = dp.FlatParams(_tensors(n, 0))
    loss = sum(((fp["means"] * (v + 1)).sum() + (fp["sh_coeffs_rest"] ** 2).sum() * v)
               for v in range(8))
    loss.backward()
    for r in range(world):
        assert torch.allclose(out[r], fp.grad, rtol=1e-6, atol=1e-6)
    assert torch.equal(out[0], out[1])


def _dying_worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    import time

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=10))
    fp = dp.FlatParams(_tensors(4, 0))
    if rank == 1:
        os._exit(3)  # a rank that dies between steps, before the gradient exchange
    t0 = time.time()
    try:
        fp.allreduce_grads()
        out[rank] = "no error"
    except Exception as exc:  # the survivor must see an error, not hang
        out[rank] = f"error after {time.time() - t0:.1f}s: {type(exc).__name__}"
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_dead_rank_surfaces_as_error_not_hang():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(90)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    assert str(out.get(0, "")).startswith("error"), out.get(0)


def test_flat_params_rebuild_relayouts_every_group():
    """FlatParams.rebuild re-lays the six groups out for a new Gaussian count
    and hands the fill function both layouts (host-side logic; the device
    fill is gs_densify_apply)."""
    n, n_new = 5, 8
    fp = dp.FlatParams(_tensors(n, 1))
    fp.exp_avg = torch.arange(fp.padded, dtype=torch.float32)
    fp.exp_avg_sq = torch.arange(fp.padded, dtype=torch.float32) * 2
    old = {k: fp[k].detach().clone() for k in dp.GROUPS}
    seen = {}

    def fill(old_data, old_off, new_data, new_off, old_m, old_v, new_m, new_v):
        seen["offsets"] = (list(old_off), list(new_off))
        for i, k in enumerate(dp.GROUPS):
            per = old[k][0].numel()
            a, b = old_off[i], new_off[i]
            # keep the first n Gaussians, then repeat the first n_new - n
            new_data[b:b + n * per] = old_data[a:a + n * per]
            new_data[b + n * per:b + n_new * per] = old_data[a:a + (n_new - n) * per]
            new_m[b:b + n * per] = old_m[a:a + n * per]
            new_v[b:b + n * per] = old_v[a:a + n * per]

    fp.rebuild(n_new, fill)
    assert fp.num_gaussians == n_new
    for k in dp.GROUPS:
        p = fp[k]
        assert p.shape == (n_new,) + old[k].shape[1:]
        assert torch.equal(p[:n].detach(), old[k])
        assert torch.equal(p[n:].detach(), old[k][:n_new - n])
        assert p.grad is not None and float(p.grad.abs().sum()) == 0.0
        assert p.data_ptr() >= fp.data.data_ptr()
    old_off, new_off = seen["offsets"]
    assert old_off[0] == new_off[0] == 0 and new_off[-1] > old_off[-1]
    assert all(o % 4 == 0 for o in new_off)
    assert fp.exp_avg.shape[0] == fp.padded
    a, _ = fp.spans["means"]
    assert torch.equal(fp.exp_avg[a:a + 3 * n], torch.arange(3 * n, dtype=torch.float32))
