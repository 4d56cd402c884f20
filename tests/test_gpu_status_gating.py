"""A step whose kernels recorded an error must not update the parameters.

The optimizer kernels (gs_adam_step, gs_dp_adam_step) read the device
status word first and skip their update while it holds an error (a bounded
wait that gave up earlier in the step, so the gradient may be incomplete).
The error is planted with gs_selftest_set_timeout: a one-thread kernel that
polls a flag nothing sets until its spin limit and records
GS_ERR_DEVICE_TIMEOUT, as any of the library's bounded waits would -- no
fault, and the context stays usable."""
import ctypes
import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
nat = importlib.import_module("3dgs_from_scratch_b200._native")
DEV = torch.device("cuda", 0)


def plant_timeout():
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    nat.call("gs_selftest_set_timeout", flag.data_ptr(), nat.stream_ptr(DEV))
    torch.cuda.synchronize()
    return flag


def small_trainer(gs):
    cfg = gs.scenes.CONFIGS[0]
    raw = gs.scenes.make_gaussians(cfg, seed=5, n=3000)
    trainer = importlib.import_module("3dgs_from_scratch_b200.trainer")
    tr = trainer.NativeTrainer({k: v.to(DEV) for k, v in raw.items()}, 96, 64)
    w2c = torch.stack([gs.scenes.primary_camera(cfg), gs.scenes.orbit_cameras(cfg, 2)[1]])
    K = torch.tensor([[120.0, 0, 48], [0, 120.0, 32], [0, 0, 1]])
    tg = torch.rand((2, 64, 96, 3), generator=torch.Generator().manual_seed(1)) * 255
    return tr, w2c.to(DEV), K.to(DEV), [t.to(DEV) for t in tg]


def test_adam_skips_update_while_status_holds_an_error(gs):
    tr, w2c, K, tg = small_trainer(gs)
    tr.step(w2c, K, tg)  # moments exist; a clean step
    views = tr.forward_views(w2c, K)
    tr.loss_and_backward(views, tg)
    before = tr.fp.data.clone()
    m_before = tr.fp.exp_avg.clone()
    plant_timeout()
    tr.fp.step()
    assert nat.query("gs_check_status", nat.stream_ptr(DEV)) == nat.GS_ERR_DEVICE_TIMEOUT
    assert torch.equal(tr.fp.data, before)
    assert torch.equal(tr.fp.exp_avg, m_before)
    # with the word cleared the same gradient is applied
    tr.fp.step()
    assert nat.query("gs_check_status", nat.stream_ptr(DEV)) == 0
    assert not torch.equal(tr.fp.data, before)


@pytest.mark.parametrize("overlap", [True, False])
def test_step_raises_in_the_same_step_with_parameters_unchanged(gs, overlap):
    """Whether Adam runs range by range behind the backward (the one-GPU
    default) or as one launch after it."""
    tr, w2c, K, tg = small_trainer(gs)
    tr.adam_overlap = overlap
    assert tr.overlap_adam() == overlap
    tr.step(w2c, K, tg)
    before = tr.fp.data.clone()
    m_before = tr.fp.exp_avg.clone()
    steps_before = tr.fp.step_count
    clean = tr.loss_and_backward

    def backward_after_a_failed_wait(*args, **kwargs):
        plant_timeout()  # as if a bounded wait of this step's layout had given up
        return clean(*args, **kwargs)

    tr.loss_and_backward = backward_after_a_failed_wait
    with pytest.raises(nat.NativeError) as e:
        tr.step(w2c, K, tg)
    assert e.value.code == nat.GS_ERR_DEVICE_TIMEOUT
    assert torch.equal(tr.fp.data, before)
    assert torch.equal(tr.fp.exp_avg, m_before)
    tr.loss_and_backward = clean
    tr.fp.step_count = steps_before  # the failed step's update did not happen
    tr.step(w2c, K, tg)  # the next step runs normally
    assert not torch.equal(tr.fp.data, before)


def test_dp_kernel_skips_update_while_status_holds_an_error():
    n = 4096
    params = torch.randn(n, device=DEV)
    grad = torch.randn(n, device=DEV)
    m, v = torch.zeros_like(params), torch.zeros_like(params)
    flags = torch.zeros(int(nat.query("gs_dp_flag_words", 2)), dtype=torch.int32, device=DEV)
    ends = (ctypes.c_int64 * 1)(n)
    lrs = (ctypes.c_float * 1)(1e-2)
    eps = (ctypes.c_float * 1)(1e-15)
    vp = ctypes.c_void_p * 1
    before = params.clone()
    st = nat.stream_ptr(DEV)

    def dp_step(epoch):
        nat.call("gs_dp_adam_step", 1, 0, vp(grad.data_ptr()), vp(params.data_ptr()),
                 vp(flags.data_ptr()), None, None, n, m.data_ptr(), v.data_ptr(), 1,
                 ctypes.cast(ends, ctypes.c_void_p), ctypes.cast(lrs, ctypes.c_void_p),
                 ctypes.cast(eps, ctypes.c_void_p), 0.9, 0.999, 1, epoch, 2, None, st)

    plant_timeout()
    dp_step(1)
    assert nat.query("gs_check_status", st) == nat.GS_ERR_DEVICE_TIMEOUT
    assert torch.equal(params, before) and not bool(m.any())
    dp_step(2)
    assert nat.query("gs_check_status", st) == 0
    assert not torch.equal(params, before)
