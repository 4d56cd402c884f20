"""The fused data-parallel optimizer step (gs_dp_adam_step): reduce-scatter
of the flat gradient, Adam on the rank's shard, all-gather of the
parameters, in one kernel over peer memory / NVSwitch multicast.

* CPU: the shard padding.
* one GPU: world = 1 (the kernel's barrier with itself, its Adam against the
  one-launch Adam) and the bounded-wait path (a second rank that never
  arrives; all buffers local, the kernel gives up after 4 s and reports
  GS_ERR_DEVICE_TIMEOUT).
* two or more GPUs (skipped otherwise): 2 ranks over NCCL, fused step
  (multicast and peer-store variants) against all_reduce + Adam.
"""
import ctypes
import importlib
import os
import socket

import numpy as np
import pytest
import torch

dp = importlib.import_module("3dgs_from_scratch_b200.dp")
nat = importlib.import_module("3dgs_from_scratch_b200._native")


def test_padded_numel():
    for n in (1, 4, 59, 1000, 59_000_004):
        for w in (1, 2, 3, 8):
            p = dp.padded_numel(n, w)
            assert p >= n and p % (4 * w) == 0 and p - n < 4 * w


def _flat_inputs(n, seed, device):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(n, generator=g).to(device)


def _group_table(n):
    ends = [n // 8, n // 4, n // 2, n - 8, n - 4, n]
    ends = [e // 4 * 4 for e in ends]
    lrs = [1e-3, 5e-3, 1e-2, 5e-2, 2.5e-3, 1.25e-4]
    return ((ctypes.c_int64 * 6)(*ends), (ctypes.c_float * 6)(*lrs),
            (ctypes.c_float * 6)(*([1e-15] * 6)))


def _vp(*ptrs):
    return (ctypes.c_void_p * len(ptrs))(*ptrs)


@pytest.mark.gpu
def test_world1_matches_adam():
    n = 4096 * 3 + 8
    dev = torch.device("cuda", 0)
    params = _flat_inputs(n, 1, dev)
    grad = _flat_inputs(n, 2, dev)
    ref = params.clone()
    m_ref, v_ref = torch.zeros_like(ref), torch.zeros_like(ref)
    m, v = torch.zeros_like(ref), torch.zeros_like(ref)
    words = nat.query("gs_dp_flag_words", 4)
    flags = torch.zeros(words, dtype=torch.int32, device=dev)
    out = torch.empty_like(grad)
    ends, lrs, eps = _group_table(n)
    st = nat.stream_ptr(dev)
    for step in (1, 2, 3):
        nat.call("gs_adam_step", n, ref.data_ptr(), grad.data_ptr(), m_ref.data_ptr(),
                 v_ref.data_ptr(), 6, ctypes.cast(ends, ctypes.c_void_p),
                 ctypes.cast(lrs, ctypes.c_void_p), ctypes.cast(eps, ctypes.c_void_p), 0.9, 0.999,
                 step, st)
        nat.call("gs_dp_adam_step", 1, 0, _vp(grad.data_ptr()), _vp(params.data_ptr()),
                 _vp(flags.data_ptr()), None, None, n, m.data_ptr(), v.data_ptr(), 6,
                 ctypes.cast(ends, ctypes.c_void_p), ctypes.cast(lrs, ctypes.c_void_p),
                 ctypes.cast(eps, ctypes.c_void_p), 0.9, 0.999, step, step, 4, out.data_ptr(), st)
    assert nat.query("gs_check_status", st) == 0
    assert torch.equal(params, ref)
    assert torch.equal(m, m_ref) and torch.equal(v, v_ref)
    assert torch.equal(out, grad)


@pytest.mark.gpu
def test_missing_rank_times_out_and_context_survives():
    """world = 2 with rank 1 absent: every buffer is on this GPU (the
    "peer" buffers are local allocations), nothing ever sets rank 1's flag,
    so each block's entry wait ends after its bound and records a timeout."""
    n = 1024
    dev = torch.device("cuda", 0)
    params = [_flat_inputs(n, 1, dev), _flat_inputs(n, 1, dev)]
    grads = [_flat_inputs(n, 2, dev), _flat_inputs(n, 3, dev)]
    before = params[0].clone()
    words = nat.query("gs_dp_flag_words", 2)
    flags = [torch.zeros(words, dtype=torch.int32, device=dev) for _ in range(2)]
    m = torch.zeros(n // 2, device=dev)
    v = torch.zeros(n // 2, device=dev)
    ends, lrs, eps = _group_table(n)
    st = nat.stream_ptr(dev)
    nat.call("gs_dp_adam_step", 2, 0, _vp(*[g.data_ptr() for g in grads]),
             _vp(*[p.data_ptr() for p in params]), _vp(*[f.data_ptr() for f in flags]), None, None,
             n, m.data_ptr(), v.data_ptr(), 6, ctypes.cast(ends, ctypes.c_void_p),
             ctypes.cast(lrs, ctypes.c_void_p), ctypes.cast(eps, ctypes.c_void_p), 0.9, 0.999, 1, 1,
             2, None, st)
    assert nat.query("gs_check_status", st) == nat.GS_ERR_DEVICE_TIMEOUT
    assert torch.equal(params[0], before)  # nothing was updated
    assert int(flags[1][:2 * 8].view(2, 8)[:, 0].max()) == 1  # rank 0 did signal rank 1
    assert torch.arange(10, device=dev).sum().item() == 45


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, result_dir):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        tens = {k: v.to(dev) for k, v in _tensors(1001, 0).items()}
        fused = dp.FlatParams(tens, fused_dp=mode)
        plain = dp.FlatParams(tens, fused_dp=False)
        for step in range(3):
            g = torch.Generator(device=dev).manual_seed(100 * step + rank)
            gr = torch.randn(fused.numel, generator=g, device=dev)
            fused.grad[:fused.numel].copy_(gr)
            plain.grad.copy_(gr)
            fused.step()
            plain.step()
        torch.cuda.synchronize()
        assert nat.query("gs_check_status", nat.stream_ptr(dev)) == 0
        mine = fused.data[:fused.numel].clone()
        allp = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allp, mine)
        np.savez(os.path.join(result_dir, f"r{rank}.npz"), fused=mine.cpu().numpy(),
                 plain=plain.data.cpu().numpy(), all=torch.stack(allp).cpu().numpy(),
                 multicast=np.array(bool(fused.multicast)))
        dist.barrier()
    finally:
        del fused
        dist.destroy_process_group()


def _tensors(n, seed):
    g = torch.Generator().manual_seed(seed)
    return {"means": torch.randn(n, 3, generator=g), "scales": torch.randn(n, 3, generator=g),
            "quaternions": torch.randn(n, 4, generator=g), "opacities": torch.randn(n, generator=g),
            "sh_coeffs_dc": torch.randn(n, 3, generator=g),
            "sh_coeffs_rest": torch.randn(n, 15, 3, generator=g)}


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["p2p", "multicast", "auto"])
def test_two_ranks_fused_step_matches_allreduce_adam(tmp_path, mode):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    mp.start_processes(_worker, args=(2, _free_port(), mode, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    r = [np.load(tmp_path / f"r{i}.npz") for i in range(2)]
    # every rank holds the same parameters after the step ...
    assert np.array_equal(r[0]["all"][0], r[0]["all"][1])
    # ... equal to all-reduce + Adam up to the order of the gradient sum
    np.testing.assert_allclose(r[0]["fused"], r[0]["plain"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(r[1]["fused"], r[1]["plain"], rtol=1e-5, atol=1e-6)
