"""Benchmark: data-parallel training step of the Gaussian-splatting rasterizer.

Workload: N = 1,000,000 SH-degree-3 Gaussians with
the config's seeded synthetic distributions, 1920x1080 views, fx = fy = 1100,
cameras on a radius-8 orbit around the scene (view 0 is the config's camera
at (0, 0, -8)), L1 loss against a uniform-random target image. One step per
rank = activations, `views_per_rank` rendered views fwd+bwd through the
package's public render(), gradient all-reduce over NCCL when world > 1,
and one Adam step over the six parameter groups. Weak scaling: every rank
renders its own views of a replicated scene.

value = views/s over all ranks, device-timed with CUDA events, max over
ranks. e2e = the same step through render() with each step's target images
(uint8) and cameras copied from pinned host memory and the loss read back,
wall-clock timed. The roofline of each stage is its algorithmic bytes (or
FLOPs) per launch, listed below, over the launch's CUDA-event time.

--trainer native (default) runs the step with trainer.NativeTrainer: the same
math with the activations fused into the preprocess kernels, one host
synchronisation per step, the L1 loss and its gradient in one kernel, and
gradients accumulated straight into the flat buffer. --trainer autograd runs
it through the public render() with Torch activations, loss and autograd.
"""
from __future__ import annotations

import argparse
import importlib
import json
import math
import os
import platform
import statistics
import subprocess
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
gs = importlib.import_module("3dgs_from_scratch_b200")
nat = importlib.import_module("3dgs_from_scratch_b200._native")
dp = importlib.import_module("3dgs_from_scratch_b200.dp")
trainer_mod = importlib.import_module("3dgs_from_scratch_b200.trainer")
gs_ssim = importlib.import_module("3dgs_from_scratch_b200.ssim")
scenes = gs.scenes

METRIC = "fwd+bwd ms/view (1M SH3 Gauss, 1080p); train views/s at 1/2/4/8 B200"
PEAKS_PATH = os.path.join(HERE, "MEASURED_PEAKS.json")
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

# algorithmic bytes / flops per unit (Gaussian, pair or evaluated pixel-Gaussian pair)
PRE_FWD_BYTES_PER_G = 281
PRE_BWD_BYTES_PER_G = 504
LAYOUT_BYTES_PER_PAIR = 12 + 144 + 8
PARAM_BYTES_PER_G = 236     # the 59 fp32 parameters of one Gaussian
PRE_OUT_BYTES_PER_G = 45    # per view: points 8, depth 4, conic 12, radii 8, rgb 12, mask 1
PRE_UP_BYTES_PER_G = 40     # per view: upstream gradients of points (8) and splat (32)
BLEND_FWD_FLOP_PER_PAIR = 22
BLEND_BWD_FLOP_PER_PAIR = 60

# DRAM bytes (read + write) per launch at config 1 (4 views per step):
# dram__bytes_read.sum + dram__bytes_write.sum from one-kernel ncu captures of
# the same kernels on the same workload (preprocess_fwd is the one multi-view
# launch).
NCU_TRAFFIC_BYTES = {"preprocess_fwd": 415.7e6, "preprocess_bwd": 599.3e6, "blend_fwd": 54.0e6,
                     "blend_bwd": 111.0e6, "loss": 50.8e6}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--views-per-rank", type=int, default=None,
                   help="views each rank renders per step (weak scaling; default 4)")
    p.add_argument("--global-views", type=int, default=None,
                   help="views per step over all ranks, sharded (strong scaling); "
                        "config 2 defaults to its batch of 32")
    p.add_argument("--no-graph", action="store_true",
                   help="run the native step eagerly instead of replaying it from CUDA graphs "
                        "(graphs are used on one GPU)")
    p.add_argument("--streams", type=int, default=2,
                   help="CUDA streams the native trainer spreads a step's views over")
    p.add_argument("--layout", choices=["auto", "binned", "capped", "batched", "per_view"],
                   default="auto",
                   help="tile layout: one per view into fixed-capacity buffers with the pair "
                        "counts kept on the device (no host synchronisation in a step), by "
                        "per-tile binning or by two radix sorts (auto: binning up to 2560 pairs "
                        "per tile on average); every view in one cooperative launch; or one per "
                        "view sized by a host read of the pair counts")
    p.add_argument("--dp", choices=["nccl", "fused", "fused-p2p", "fused-mc"], default="fused",
                   help="multi-GPU optimizer step: NCCL all-reduce + Adam, or the fused "
                        "reduce-scatter / sharded Adam / all-gather kernel (fused: peer loads "
                        "and stores at 2 GPUs, NVSwitch multicast above when available; "
                        "fused-p2p / fused-mc force one of the two)")
    p.add_argument("--ssim-lambda", type=float, default=None,
                   help="loss = (1 - l) L1 + l (1 - SSIM); default 0.2 for config 2, else 0")
    p.add_argument("--config", type=int, default=1)
    p.add_argument("--n", type=int, default=None, help="override Gaussian count (tests/profiling)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--cpu-sample-views", type=int, default=2)
    p.add_argument("--mode", choices=["train", "render"], default="train",
                   help="render: forward-only novel-view rendering (config 4), frames/s")
    p.add_argument("--no-subrecords", action="store_true",
                   help="skip the config-2 / config-4 / render() / GPU-reference / Torch-CPU "
                        "sub-records and the multi-GPU parity check")
    p.add_argument("--trainer", choices=["native", "autograd"], default="native",
                   help="native: NativeTrainer (fused activations/loss, flat-buffer gradients); "
                        "autograd: render() + Torch activations/loss + autograd")
    return p.parse_args()


def peaks():
    try:
        with open(PEAKS_PATH) as fh:
            d = json.load(fh)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """SM clock and throttle-reason sampling (NVML, every 10 ms) during the
    timed region, in a background thread."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
               "sw_power_cap": 0x4}

    def __init__(self, index):
        self.index = index
        self.samples = []
        self._stop = None

    def __enter__(self):
        import threading

        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._stop = None
            return self
        self._stop = threading.Event()

        def run():
            while not self._stop.is_set():
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                    rs = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    self.samples.append((mhz, rs))
                except Exception:
                    pass
                self._stop.wait(0.01)

        self._thread = threading.Thread(target=run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        if self._stop is not None:
            self._stop.set()
            self._thread.join(2)
        return False

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        reasons = sorted({name for _, rs in self.samples for name, bit in self.REASONS.items()
                          if rs & bit})
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(self.samples)}


class StageTimer:
    """CUDA events around each C-ABI call of interest, on the launching stream."""

    WATCH = ("gs_preprocess_forward", "gs_tile_layout", "gs_tile_layout_capped",
             "gs_tile_bins", "gs_tile_layout_views", "gs_tile_order",
             "gs_blend_forward", "gs_blend_backward",
             "gs_preprocess_backward", "gs_l1_loss_grad", "gs_l1_ssim_loss_grad", "gs_adam_step",
             "gs_dp_adam_step", "gs_preprocess_forward_views", "gs_preprocess_backward_views")

    def __init__(self):
        self.events = {k: [] for k in self.WATCH}
        self._orig = None

    def __enter__(self):
        self._orig = nat.call
        timer = self

        def call(name, *args):
            if name not in timer.events:
                return timer._orig(name, *args)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            rc = timer._orig(name, *args)
            b.record()
            timer.events[name].append((a, b))
            return rc

        nat.call = call
        return self

    def __exit__(self, *exc):
        nat.call = self._orig
        return False

    def mean_ms(self):
        torch.cuda.synchronize()
        return {k: (sum(a.elapsed_time(b) for a, b in v) / len(v) if v else None)
                for k, v in self.events.items()}


def setup_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU leg: the oracle port (the reference's algorithm restated in C)
# ---------------------------------------------------------------------------

def cpu_fwd_bwd_views(cfg, raw_np, views, targets, ssim_lambda=0.0):
    from oracle import oracle as orc
    from oracle import ssim_oracle

    ssim_oracle.set_separable(True)
    a = raw_np
    K = scenes.intrinsic_for(cfg).numpy()
    t0 = time.perf_counter()
    for w2c, tgt in zip(views, targets):
        img, st = orc.render_forward(w2c, K, cfg.width, cfg.height, a["means"], a["scales"],
                                     a["quaternions"], a["opacities"], a["sh_coeffs_dc"],
                                     a["sh_coeffs_rest"])
        if ssim_lambda > 0:  # image is clamp(raw) * 255: the loss's clamp is then the identity
            _, g = ssim_oracle.l1_ssim_loss(img / 255.0, tgt, ssim_lambda)
            g = (g / 255.0).astype(np.float32)
        else:
            g = (np.sign(img - tgt) / img.size).astype(np.float32)
        orc.render_backward(g, st, w2c, K, cfg.width, cfg.height, a["means"], a["scales"],
                            a["quaternions"], a["opacities"], a["sh_coeffs_dc"],
                            a["sh_coeffs_rest"])
    return time.perf_counter() - t0


def cpu_setup(cfg, n, views):
    from oracle import oracle as orc

    orc.set_num_threads(os.cpu_count() or 1)
    raw = scenes.make_gaussians(cfg, seed=0, n=n)
    act = {k: v.numpy() for k, v in scenes.activate(raw).items()}
    cams = bench_cameras(cfg, views).numpy()
    rng = np.random.default_rng(0)
    tg = [rng.uniform(0, 255, (cfg.height, cfg.width, 3)).astype(np.float32) for _ in range(views)]
    return act, cams, tg, orc.num_threads()


def cpu_model():
    try:
        with open("/proc/cpuinfo") as fh:
            for line in fh:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return platform.processor()


def run_reference(args, world, rank):
    if rank != 0:
        return
    cfg = scenes.CONFIGS[args.config]
    _, _, lam = view_plan(args, 1, 0)
    act, cams, tg, threads = cpu_setup(cfg, args.n, 1)
    for _ in range(args.warmup):
        cpu_fwd_bwd_views(cfg, act, cams[:1], tg[:1], lam)
    times = [cpu_fwd_bwd_views(cfg, act, cams[:1], tg[:1], lam) for _ in range(args.steps)]
    sec = statistics.median(times)
    value = 1.0 / sec
    sample = (f"1 full view per step (N={act['means'].shape[0]}, {cfg.width}x{cfg.height}), "
              f"fwd+bwd, median of {args.steps}")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "views/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": sec * 1000.0, "ms_per_view": sec * 1000.0, "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, cfg, 1),
        "cpu_baseline": {"value": value, "unit": "views/s", "cores": threads, "kind": "port",
                         "sample": sample, "cpu": cpu_model()},
        "e2e": {"value": value, "unit": "views/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_cameras(cfg, count):
    """The configuration's views: a seeded-uniform sphere of cameras for
    configuration 2 ("cameras on a radius-10 sphere"), an orbit in the
    horizontal plane otherwise (view 0 at (0, 0, -distance))."""
    return scenes.orbit_cameras(cfg, count, sphere=cfg.name == "cfg2")


def view_plan(args, world, rank):
    """(views per step over all ranks, this rank's views, SSIM lambda).
    Config 2 is a fixed batch of 32 views sharded over the ranks (strong
    scaling) with the L1 + 0.2 (1 - SSIM) loss; the others render
    --views-per-rank views on every rank (weak scaling) with L1."""
    gv = args.global_views
    if gv is None and args.config == 2 and args.views_per_rank is None:
        gv = 32
    if gv is not None:
        total = int(gv)
        if total < world:
            raise SystemExit("--global-views must be at least the number of ranks")
    else:
        total = (args.views_per_rank or 4) * world
    args.global_views_resolved = total
    args.strong = gv is not None
    lam = args.ssim_lambda
    if lam is None:
        lam = 0.2 if args.config == 2 else 0.0
    args.ssim_lambda_resolved = float(lam)
    return total, len(dp.shard_views(total, rank, world)), float(lam)


def workload_config(args, cfg, views_per_rank):
    lam = getattr(args, "ssim_lambda_resolved", 0.0)
    loss = f"{1 - lam:g} L1 + {lam:g} (1 - SSIM valid)" if lam > 0 else "L1"
    what = ("forward-only rendering to uint8 frames, replicas (no communication)"
            if getattr(args, "mode", "train") == "render"
            else f"{loss} vs uniform target, Adam step")
    total = getattr(args, "global_views_resolved", views_per_rank * max(args.gpus, 1))
    return {"workload": f"config {args.config}: {cfg.n if args.n is None else args.n} SH3 "
                        f"Gaussians, {cfg.width}x{cfg.height}, {views_per_rank} view(s)/rank per "
                        f"step, orbit r={cfg.camera_distance}, {what}",
            "global_batch": total, "views_per_rank": views_per_rank,
            "parallelism": f"dp{max(args.gpus, 1)} (views sharded; " + (
                "NCCL all-reduce of grads + Adam)" if getattr(args, "dp", "nccl") == "nccl" else
                "fused reduce-scatter / sharded Adam / all-gather kernel, "
                + ("NVSwitch multicast when available)" if args.dp == "fused" else
                   "peer loads and stores)")),
            "l2": "inputs larger than L2 (236 MB params + 472 MB Adam state per rank)",
            "optimizer": "Adam, six groups in one flat buffer, one native launch",
            "trainer": args.trainer, "streams": getattr(args, "streams", 1),
            "layout": getattr(args, "layout", "batched")}


# ---------------------------------------------------------------------------
# GPU leg
# ---------------------------------------------------------------------------

class Trainer:
    def __init__(self, cfg, n, total_views, world, rank, device, ssim_lambda=0.0):
        self.cfg = cfg
        self.world = world
        self.device = device
        self.ssim_lambda = float(ssim_lambda)
        raw = scenes.make_gaussians(cfg, seed=0, n=n, device=device)
        self.fp = dp.FlatParams(raw)  # replicas: identical on every rank
        self.params = self.fp.params
        cams = bench_cameras(cfg, total_views)
        mine = dp.shard_views(total_views, rank, world)
        views = len(mine)
        self.cams = cams[mine].to(device)
        self.K = scenes.intrinsic_for(cfg).to(device)
        g = torch.Generator(device=device).manual_seed(1234 + rank)
        self.targets = [torch.rand((cfg.height, cfg.width, 3), device=device, generator=g) * 255.0
                        for _ in range(views)]
        # e2e inputs: uint8 targets and cameras in pinned host memory
        self.host_targets = [(t.cpu().round().clamp(0, 255).to(torch.uint8)).pin_memory()
                             for t in self.targets]
        self.host_cams = self.cams.cpu().pin_memory()
        self.host_K = self.K.cpu().pin_memory()
        self.host_loss = torch.zeros(len(self.targets), dtype=torch.float32).pin_memory()

    def step(self, e2e=False):
        act = scenes.activate(self.params)
        losses = []
        for v in range(len(self.targets)):
            if e2e:
                w2c = self.host_cams[v].to(self.device, non_blocking=True)
                K = self.host_K.to(self.device, non_blocking=True)
                tgt = self.host_targets[v].to(self.device, non_blocking=True).float()
            else:
                w2c, K, tgt = self.cams[v], self.K, self.targets[v]
            img, pts, radii = gs.render(w2c, K, self.cfg.width, self.cfg.height, act["means"],
                                        act["scales"], act["quaternions"], act["opacities"],
                                        act["sh_coeffs_dc"], act["sh_coeffs_rest"])
            rn, tn = img / 255.0, tgt / 255.0
            loss = torch.nn.functional.l1_loss(rn, tn)
            if self.ssim_lambda > 0:  # scripts/train.py:193-203
                ss = gs_ssim.fused_ssim(rn.permute(2, 0, 1).unsqueeze(0),
                                        tn.permute(2, 0, 1).unsqueeze(0), padding="valid")
                loss = (1 - self.ssim_lambda) * loss + self.ssim_lambda * (1 - ss)
            losses.append(loss)
        # one backward per step: the views' gradients meet at the activated
        # parameters, so the activation backward runs once
        torch.stack(losses).sum().backward()
        self.fp.allreduce_grads()
        self.fp.adam_step()
        self.fp.zero_grad()
        total = torch.stack([x.detach() for x in losses])
        if e2e:
            self.host_loss.copy_(total, non_blocking=True)
        return total


class NativeBenchTrainer:
    """The same step as Trainer, run by trainer.NativeTrainer."""

    def __init__(self, cfg, n, total_views, world, rank, device, ssim_lambda=0.0, dp_mode="nccl",
                 streams=2, layout="auto", graph=True):
        self.cfg = cfg
        self.world = world
        self.device = device
        self.graph = graph
        raw = scenes.make_gaussians(cfg, seed=0, n=n, device=device)
        fused = {"nccl": False, "fused": "auto", "fused-p2p": "p2p",
                 "fused-mc": "multicast"}[dp_mode]
        self.nt = trainer_mod.NativeTrainer(raw, cfg.width, cfg.height, ssim_lambda=ssim_lambda,
                                            fused_dp=fused, streams=streams, layout=layout)
        self.fp = self.nt.fp
        self.params = self.fp.params
        cams = bench_cameras(cfg, total_views)
        mine = dp.shard_views(total_views, rank, world)
        views = len(mine)
        self.cams = cams[mine].to(device)
        self.K = scenes.intrinsic_for(cfg).to(device)
        g = torch.Generator(device=device).manual_seed(1234 + rank)
        self.targets = [torch.rand((cfg.height, cfg.width, 3), device=device, generator=g) * 255.0
                        for _ in range(views)]
        self.host_targets = [(t.cpu().round().clamp(0, 255).to(torch.uint8)).pin_memory()
                             for t in self.targets]
        # the device-resident targets are the same uint8 images (what a data
        # loader hands over), so both timings run the same loss
        self.targets = [t.to(device) for t in self.host_targets]
        self.host_cams = self.cams.cpu().pin_memory()
        self.host_K = self.K.cpu().pin_memory()
        # two pinned loss buffers: step k's losses are read on the host while
        # step k + 1 runs (see e2e_pending)
        self.host_loss = [torch.zeros(len(self.targets), dtype=torch.float64).pin_memory()
                          for _ in range(2)]
        self._loss_slot = 0
        self.e2e_pending = None

    def step(self, e2e=False, check=False):
        if e2e:
            # the pinned host cameras and targets go to the trainer, which
            # copies them (the targets on a copy stream while the views are
            # rendered); the eager step takes device cameras
            if self.graph:
                cams, K = self.host_cams, self.host_K
            else:
                cams = self.host_cams.to(self.device, non_blocking=True)
                K = self.host_K.to(self.device, non_blocking=True)
            tg = self.host_targets
        else:
            cams, K, tg = self.cams, self.K, self.targets
        # Steps are queued with no host synchronisation (the warm-up steps
        # read the status word, which sizes the layout buffers); the timed
        # and e2e regions read it once at their end. With graph (one GPU)
        # the step is replayed from CUDA graphs.
        run = self.nt.step_graph if self.graph else self.nt.step
        losses = run(cams, K, tg, check_status=check)
        if e2e:
            # the losses go to a pinned host buffer; e2e_pending = (event,
            # buffer) lets the caller read them once the copy has landed,
            # after it has queued the next step
            buf = self.host_loss[self._loss_slot]
            self._loss_slot ^= 1
            buf.copy_(losses, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record()
            self.e2e_pending = (ev, buf)
        return losses

    def render_step(self, e2e=False):
        """Forward-only rendering of this rank's views into uint8 frames
        (configuration 4); with e2e the frames are copied to pinned host
        memory."""
        if e2e:
            cams = self.host_cams.to(self.device, non_blocking=True)
            K = self.host_K.to(self.device, non_blocking=True)
        else:
            cams, K = self.cams, self.K
        views = self.nt.render_views(cams, K)
        frames = [(v["image"].clamp(0, 1) * 255).round().to(torch.uint8) for v in views]
        if e2e:
            if not hasattr(self, "host_frames"):
                self.host_frames = [torch.empty_like(f, device="cpu").pin_memory() for f in frames]
            for h, f in zip(self.host_frames, frames):
                h.copy_(f, non_blocking=True)
        return frames


def count_pairs(tr, view=0):
    """Evaluated (pixel, Gaussian) pairs of one view, in the reference's
    counting: list entries visited before the transmittance break."""
    cr = gs.cuda_rasterizer
    cfg = tr.cfg
    with torch.no_grad():
        act = scenes.activate(tr.params)
        w2c = tr.cams[view]
        pts, depths, cov, conic, radii, mask = cr.project_points(
            act["means"], act["scales"], act["quaternions"], act["opacities"], w2c, tr.K, 0.01,
            100.0, 1 / 255, 0.5, 128.0, cfg.width, cfg.height)
        off, ids = cr.compute_tile_intersection(pts, radii, depths, mask, cfg.width, cfg.height)
        W, H = cfg.width, cfg.height
        colors = torch.full((pts.shape[0], 3), 0.5, device=pts.device)
        work_t = torch.empty(H * W, device=pts.device)
        work_e = torch.empty(H * W, device=pts.device, dtype=torch.int32)
        image = torch.zeros((H, W, 3), device=pts.device)
        nat.call("gs_rasterize", off.shape[0], off.data_ptr(), ids.shape[0], ids.data_ptr(),
                 pts.shape[0], pts.data_ptr(), conic.data_ptr(), act["opacities"].data_ptr(), colors.data_ptr(),
                 W, H, 1e-4, 1e-4, 9.21, image.data_ptr(), work_t.data_ptr(), work_e.data_ptr(),
                 nat.stream_ptr())
        tx = (W + 15) // 16
        vv, uu = torch.meshgrid(torch.arange(H, device=pts.device),
                                torch.arange(W, device=pts.device), indexing="ij")
        tile = ((vv // 16) * tx + (uu // 16)).reshape(-1)
        offl = torch.cat([off.long(), torch.tensor([ids.shape[0]], device=off.device)])
        s = offl[tile]
        e = offl[tile + 1]
        broke = work_t < 1e-4
        visited = torch.where(broke, work_e.long() - s, e - s)
        return int(visited.sum().item()), int(ids.shape[0]), int(mask.sum().item())


# ---------------------------------------------------------------------------
# Sub-records: the other configurations and paths, measured in the same run
# ---------------------------------------------------------------------------

def sub_record(fn, *args):
    """A sub-record's result, or its failure written into the record (the
    headline line is printed either way; a failed sub-record says why)."""
    try:
        return fn(*args)
    except Exception as exc:  # recorded, not hidden: the line carries the error
        import traceback

        traceback.print_exc()
        torch.cuda.empty_cache()
        return {"error": f"{type(exc).__name__}: {exc}"}


def snapshot_state(tr):
    """The training state (parameters, Adam moments, step count) of a bench
    trainer, so that two timed regions can run the same steps from the same
    state: training moves the Gaussians, and with them each step's pair
    counts and cost."""
    fp = tr.fp
    moments = None if fp.exp_avg is None else (fp.exp_avg.clone(), fp.exp_avg_sq.clone())
    return fp.data.clone(), moments, fp.step_count


def restore_state(tr, state):
    """Puts a snapshot_state() back in place (the same buffers, so captured
    graphs and peer mappings stay valid)."""
    fp = tr.fp
    data, moments, step_count = state
    with torch.no_grad():
        fp.data.copy_(data)
        if moments is not None:
            fp.exp_avg.copy_(moments[0])
            fp.exp_avg_sq.copy_(moments[1])
    fp.step_count = step_count
    if fp.data.is_cuda:
        torch.cuda.synchronize(fp.data.device)


def timed_steps(fn, steps, warmup, world):
    """warmup untimed calls, then `steps` calls between barriers and device
    synchronisations, timed with CUDA events on the current stream; returns
    the total in ms, max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    barrier(world)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize()
    barrier(world)
    return max_over_ranks(a.elapsed_time(b), world)


def sub_config2(args, world, rank, device, steps=3, warmup=2):
    """Configuration 2: 3M Gaussians, a fixed batch of 32 views of 1600x1064
    on a radius-10 sphere sharded over the ranks (strong scaling),
    0.8 L1 + 0.2 (1 - SSIM), the optimizer step of the main run's --dp mode."""
    cfg = scenes.CONFIGS[2]
    total = 32
    tr = NativeBenchTrainer(cfg, None, total, world, rank, device, ssim_lambda=0.2,
                            dp_mode=args.dp, streams=args.streams, layout=args.layout,
                            graph=not args.no_graph)
    V = len(tr.targets)
    ms = timed_steps(tr.step, steps, warmup, world)
    tr.graph = False  # the stage timer sees eager launches only (a replay is one graph launch)
    with StageTimer() as st:
        tr.step()
        torch.cuda.synchronize()
    sm = st.mean_ms()
    opt = sm.get("gs_dp_adam_step") or sm.get("gs_adam_step")
    opt = max_over_ranks(opt or 0.0, world)
    rec = {"workload": f"config 2: {cfg.n} SH3 Gaussians, {cfg.width}x{cfg.height}, batch of "
                       f"{total} views on a radius-{cfg.camera_distance} sphere sharded over "
                       f"{world} rank(s), 0.8 L1 + 0.2 (1 - SSIM valid), Adam",
           "value": total * steps / (ms / 1000.0), "unit": "views/s", "scaling": "strong",
           "global_batch": total, "views_per_rank": V, "steps": steps, "warmup": warmup,
           "ms_per_step": ms / steps, "optimizer_ms": opt,
           "optimizer_share": opt / (ms / steps) if ms > 0 else None,
           "optimizer": "fused DP kernel" if tr.fp.fused else (
               "NCCL all-reduce + Adam" if world > 1 else "Adam")}
    del tr
    torch.cuda.empty_cache()
    return rec


def render_frames(nt, cams, K, chunk):
    """Forward-only rendering of `cams` into uint8 frames, `chunk` views per
    multi-view preprocess launch."""
    frames = []
    for c in range(0, cams.shape[0], chunk):
        views = nt.render_views(cams[c:c + chunk], K)
        frames += [(v["image"].clamp(0, 1) * 255).round().to(torch.uint8) for v in views]
        del views
    return frames


def sub_config4(args, world, rank, device, steps=2, warmup=1, chunk=8):
    """Configuration 4: inference of 6M Gaussians, 256 views of 1920x1080 on a
    radius-12 orbit sharded over the ranks with no communication."""
    cfg = scenes.CONFIGS[4]
    total = 256
    raw = scenes.make_gaussians(cfg, seed=0, device=device)
    nt = trainer_mod.NativeTrainer(raw, cfg.width, cfg.height, streams=args.streams,
                                   layout=args.layout)
    del raw
    mine = dp.shard_views(total, rank, world)
    cams = scenes.orbit_cameras(cfg, total)[mine].to(device)
    K = scenes.intrinsic_for(cfg).to(device)
    ms = timed_steps(lambda: render_frames(nt, cams, K, chunk), steps, warmup, world)
    rec = {"workload": f"config 4: {cfg.n} SH3 Gaussians, {total} views of {cfg.width}x"
                       f"{cfg.height} on a radius-{cfg.camera_distance} orbit sharded over "
                       f"{world} rank(s), forward only to uint8 frames, no communication",
           "value": total * steps / (ms / 1000.0), "unit": "frames/s", "scaling": "strong",
           "views_per_rank": len(mine), "views_per_launch": chunk, "steps": steps,
           "warmup": warmup, "ms_per_step": ms / steps}
    del nt
    torch.cuda.empty_cache()
    return rec


def sub_render_api(args, world, rank, device, steps=10, warmup=3):
    """The drop-in path scripts/train.py drives unchanged: render() with Torch
    activations, L1 loss and autograd, one view per rank per step (the
    reference's script steps once per view), gradient all-reduce over NCCL
    (world > 1) and the one-launch Adam; configuration 1."""
    cfg = scenes.CONFIGS[1]
    tr = Trainer(cfg, None, world, world, rank, device)
    ms = timed_steps(tr.step, steps, warmup, world)
    rec = {"workload": f"config 1 through render() + autograd, 1 view per rank per step, "
                       f"{world} rank(s)",
           "value": world * steps / (ms / 1000.0), "unit": "views/s", "scaling": "weak",
           "steps": steps, "warmup": warmup, "ms_per_step": ms / steps}
    del tr
    torch.cuda.empty_cache()
    return rec


def sub_gpu_reference(device, ours_ms, reps=3):
    """The reference's own CUDA extension (its rasterizer.cpp + kernel.cu
    built for sm_100a into oracle/_ref) on configuration 1's first view, per
    stage with CUDA events (median of `reps` after one warm-up), beside this
    library's per-view stage times from the same run."""
    from oracle import build_ref

    ref = build_ref.load_module()
    if ref is None:
        return {"unavailable": "reference extension not built (oracle/_ref)"}
    cfg = scenes.CONFIGS[1]
    W, H = cfg.width, cfg.height
    a = scenes.activate(scenes.make_gaussians(cfg, seed=0, device=device))
    w2c = scenes.primary_camera(cfg).to(device)
    K = scenes.intrinsic_for(cfg).to(device)
    campos = (-w2c[:3, :3].t() @ w2c[:3, 3]).contiguous()
    tgt = torch.rand((H, W, 3), device=device, generator=torch.Generator(device).manual_seed(5))
    args = (0.01, 100.0, 1 / 255, 0.5, 128.0)
    st = {}

    def ev(name, fn):
        x = torch.cuda.Event(enable_timing=True)
        y = torch.cuda.Event(enable_timing=True)
        x.record()
        out = fn()
        y.record()
        st.setdefault(name, []).append((x, y))
        return out

    for _ in range(reps + 1):
        pp = ev("project_points", lambda: ref.project_points(
            a["means"], a["scales"], a["quaternions"], a["opacities"], w2c, K, *args, W, H))
        pts, depths, cov, conic, radii, mask = pp
        raw_col = ev("spherical_harmonics", lambda: ref.evaluate_spherical_harmonics(
            campos, a["means"], a["sh_coeffs_dc"], a["sh_coeffs_rest"], mask, False))
        colors = torch.clamp_min(raw_col + 0.5, 0.0)
        off, ids = ev("compute_tile_intersection", lambda: ref.compute_tile_intersection(
            pts, radii, depths, mask, W, H, 16))
        rargs = (off, ids, pts, conic, a["opacities"], colors, W, H, 16, 1e-4, 1e-4, 9.21)
        img = ev("rasterize", lambda: ref.rasterize(*rargs))
        up = (torch.sign(img.clamp(0, 1) - tgt) / img.numel()).contiguous()
        gp, gc, go, gcol = ev("rasterize_backward", lambda: ref.rasterize_backward(up, *rargs))
        ev("spherical_harmonics_backward", lambda: ref.evaluate_spherical_harmonics_backward(
            gcol.contiguous(), campos, a["means"], a["sh_coeffs_dc"], a["sh_coeffs_rest"],
            raw_col, mask, False))
        ev("project_points_backward", lambda: ref.project_points_backward(
            gp.contiguous(), gc.contiguous(), a["means"], a["scales"], a["quaternions"],
            a["opacities"], w2c, K, W, H, cov, mask))
    torch.cuda.synchronize()
    ref_ms = {k: statistics.median(x.elapsed_time(y) for x, y in v[1:]) for k, v in st.items()}
    groups = {
        "preprocess_fwd": ["project_points", "spherical_harmonics"],
        "tile_layout": ["compute_tile_intersection"],
        "blend_fwd": ["rasterize"],
        "blend_bwd": ["rasterize_backward"],
        "preprocess_bwd": ["spherical_harmonics_backward", "project_points_backward"],
    }
    per_stage = {}
    for g, names in groups.items():
        r = sum(ref_ms[n] for n in names)
        o = ours_ms.get(g)
        per_stage[g] = {"reference_ms": r, "ours_ms": o,
                        "speedup": (r / o) if o else None}
    ref_total = sum(ref_ms.values())
    ours_total = sum(v for v in ours_ms.values() if v is not None)
    del a, pp, pts, depths, cov, conic, radii, mask, off, ids, img, up, gp, gc, go, gcol
    torch.cuda.empty_cache()
    return {"what": "reference src/cuda extension (rasterizer.cpp + kernel.cu) built for "
                    "sm_100a, config 1 view 0 (1M SH3 Gaussians, 1920x1080), L1 gradient; "
                    "CUDA events per stage, median of 3",
            "reference_stage_ms": ref_ms, "per_stage": per_stage,
            "reference_ms_per_view": ref_total, "ours_ms_per_view": ours_total,
            "speedup_per_view": ref_total / ours_total if ours_total else None,
            "ours_basis": "per-view stage times of this run (multi-view launches divided by "
                          "their views)"}


def cpu_torch_reference_cfg0(iters=3):
    """The reference's own CPU path: src/torch_rasterizer.render(device="cpu"),
    forward + backward of configuration 0 (20k Gaussians, 256x256, L1 against a
    uniform target) with torch.set_num_threads(os.cpu_count()); one warm-up,
    median of `iters`. The module is the reference's, byte-compiled by
    oracle/build_ref.py into oracle/_ref/py."""
    from oracle import build_ref

    build_ref.stage_python()
    if not build_ref.install_staged_importer():
        return {"unavailable": "reference Python modules not staged (oracle/_ref/py)"}
    tr_mod = importlib.import_module("src.torch_rasterizer")
    prev = torch.get_num_threads()
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    try:
        cfg = scenes.CONFIGS[0]
        raw = scenes.make_gaussians(cfg, seed=0)
        w2c = scenes.primary_camera(cfg)
        K = scenes.intrinsic_for(cfg)
        tgt = torch.rand((cfg.height, cfg.width, 3), generator=torch.Generator().manual_seed(0))
        times = []
        for it in range(iters + 1):
            p = {k: v.clone().requires_grad_(True) for k, v in raw.items()}
            act = scenes.activate(p)
            t0 = time.perf_counter()
            img, _, _ = tr_mod.render(w2c, K, cfg.width, cfg.height, act["means"], act["scales"],
                                      act["quaternions"], act["opacities"], act["sh_coeffs_dc"],
                                      act["sh_coeffs_rest"], device="cpu")
            torch.nn.functional.l1_loss(img / 255.0, tgt).backward()
            if it > 0:
                times.append(time.perf_counter() - t0)
        sec = statistics.median(times)
    finally:
        torch.set_num_threads(prev)
    return {"value": 1.0 / sec, "unit": "views/s", "cores": cores, "kind": "reference",
            "ms_per_view": sec * 1000.0,
            "sample": f"config 0 (N={cfg.n}, {cfg.width}x{cfg.height}), fwd+bwd through "
                      f"src/torch_rasterizer.render(device='cpu'), median of {iters}",
            "cpu": cpu_model()}


def nccl_allreduce_bus_gbs(numel, world, device, iters=5):
    """NCCL all-reduce bus bandwidth over this run's ranks for a flat fp32
    buffer of `numel` elements: 2 (w - 1) / w * bytes / time, max over ranks."""
    import torch.distributed as dist

    x = torch.ones(numel, device=device, dtype=torch.float32)
    for _ in range(2):
        dist.all_reduce(x)
    torch.cuda.synchronize()
    barrier(world)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        dist.all_reduce(x)
    b.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(a.elapsed_time(b) / iters, world)
    del x
    return 2 * (world - 1) / world * 4 * numel / (ms * 1e-3) / 1e9, ms


def dp_parity(tr, world, rank):
    """Multi-GPU correctness in the bench itself: (a) every rank's flat
    parameters are bitwise identical to rank 0's after the timed steps;
    (b) from one state and one set of per-rank gradients, the fused data-
    parallel step equals an NCCL all-reduce of the gradients followed by the
    one-GPU Adam kernel (parameters within 1e-5)."""
    import torch.distributed as dist

    fp = tr.fp
    dev = fp.device
    torch.cuda.synchronize()
    r0 = fp.data.clone()
    dist.broadcast(r0, 0)
    same = torch.tensor([1 if torch.equal(r0, fp.data) else 0], device=dev, dtype=torch.int32)
    dist.all_reduce(same, op=dist.ReduceOp.MIN)
    del r0
    out = {"ranks_bitwise_identical": bool(same.item()), "world": world}
    nt = getattr(tr, "nt", None)
    if not fp.fused or nt is None:
        out["fused_vs_nccl"] = None
        out["pass"] = out["ranks_bitwise_identical"]
        return out
    views = nt.forward_views(tr.cams, tr.K)
    nt.loss_and_backward(views, tr.targets)
    del views
    torch.cuda.synchronize()
    g = fp.grad.clone()
    p0 = fp.data.clone()
    m0, v0 = fp.full_moments()
    step0 = fp.step_count
    fp.fused_step()
    torch.cuda.synchronize()
    p_fused = fp.data.clone()
    dist.all_reduce(g)
    p_ref, m, v = p0.clone(), m0.clone(), v0.clone()
    ends_c, lrs_c, eps_c = fp._group_table()
    import ctypes

    nat.call("gs_adam_step", fp.padded, p_ref.data_ptr(), g.data_ptr(), m.data_ptr(),
             v.data_ptr(), len(dp.GROUPS), ctypes.cast(ends_c, ctypes.c_void_p),
             ctypes.cast(lrs_c, ctypes.c_void_p), ctypes.cast(eps_c, ctypes.c_void_p),
             fp.betas[0], fp.betas[1], step0 + 1, nat.stream_ptr(dev))
    torch.cuda.synchronize()
    d = (p_fused - p_ref).abs()
    du = ((p_fused - p0) - (p_ref - p0)).norm() / (p_ref - p0).norm().clamp_min(1e-30)
    mx = max_over_ranks(float(d.max()), world)
    out["fused_vs_nccl"] = {"max_abs_param_diff": mx, "update_rel_l2": float(du),
                            "elements_over_1e-5": int((d > 1e-5).sum()),
                            "multicast": bool(getattr(fp, "multicast", False))}
    out["pass"] = out["ranks_bitwise_identical"] and mx <= 1e-5
    del g, p0, m0, v0, p_fused, p_ref, m, v, d
    torch.cuda.empty_cache()
    return out


def main():
    args = parse()
    world, rank, local = setup_dist(args)
    if args.impl == "reference":
        run_reference(args, world, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    device = torch.device("cuda", local)
    cfg = scenes.CONFIGS[args.config]
    total_views, V, lam = view_plan(args, world, rank)
    if args.trainer == "native":
        tr = NativeBenchTrainer(cfg, args.n, total_views, world, rank, device, ssim_lambda=lam,
                                dp_mode=args.dp, streams=args.streams, layout=args.layout,
                                graph=not args.no_graph)
    else:
        if args.dp != "nccl":
            raise SystemExit("--dp fused needs --trainer native")
        tr = Trainer(cfg, args.n, total_views, world, rank, device, ssim_lambda=lam)
    n = tr.params["means"].shape[0]
    render_mode = args.mode == "render"
    if render_mode and args.trainer != "native":
        raise SystemExit("--mode render uses the native path")
    run_step = tr.render_step if render_mode else tr.step

    for _ in range(args.warmup):
        # warm-up steps read the status word: a pair count beyond the layout
        # capacity grows the buffers there (and repeats the step), so the
        # timed steps queue without any host synchronisation
        if isinstance(tr, NativeBenchTrainer) and not render_mode:
            run_step(check=True)
        else:
            run_step()
    torch.cuda.synchronize()
    barrier(world)

    # the e2e region below replays the timed steps from this same state
    state0 = snapshot_state(tr) if not render_mode else None
    launches0 = nat.launch_count()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        start.record()
        for _ in range(args.steps):
            run_step()
        end.record()
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
    launches = nat.launch_count() - launches0
    rc = nat.query("gs_check_status", nat.stream_ptr())
    if rc:
        raise nat.NativeError("timed steps", rc, nat.lib().gs_last_cuda_error())
    ms_total = max_over_ranks(start.elapsed_time(end), world)
    ms_step = ms_total / args.steps
    value = total_views * args.steps / (ms_total / 1000.0)
    unit = "frames/s" if render_mode else "views/s"

    # e2e right after the device-timed steps (same thermal state), then the
    # per-stage breakdown
    e2e = None
    if not args.no_e2e:
        for _ in range(2):
            run_step(e2e=True)
        torch.cuda.synchronize()
        if state0 is not None:
            restore_state(tr, state0)  # the same steps as the device-timed region
        barrier(world)
        pipelined = isinstance(tr, NativeBenchTrainer) and not render_mode
        loss_sum = 0.0
        with ClockSampler(local) as clk_e2e:
            t0 = time.perf_counter()
            pending = None
            for _ in range(args.steps):
                run_step(e2e=True)
                if not pipelined:
                    torch.cuda.current_stream().synchronize()  # the step's result is on the host
                    continue
                # a training loop's order: queue step k + 1, then read step
                # k's losses on the host (their copy is in the stream behind
                # step k), so the GPU does not wait for the host between steps
                if pending is not None:
                    pending[0].synchronize()
                    loss_sum += float(pending[1].sum())
                pending = tr.e2e_pending
            if pending is not None:
                pending[0].synchronize()
                loss_sum += float(pending[1].sum())
            torch.cuda.current_stream().synchronize()
            barrier(world)
            sec = max_over_ranks(time.perf_counter() - t0, world)
        rc = nat.query("gs_check_status", nat.stream_ptr())
        if rc:
            raise nat.NativeError("e2e steps", rc, nat.lib().gs_last_cuda_error())
        if pipelined and not math.isfinite(loss_sum):
            raise RuntimeError(f"e2e steps: non-finite losses read back ({loss_sum})")
        if render_mode:
            h2d = V * (16 + 9) * 4
            d2h = V * cfg.width * cfg.height * 3
        else:
            h2d = sum(t.numel() for t in tr.host_targets) + V * (16 + 9) * 4
            d2h = V * 8
        e2e = {"value": total_views * args.steps / sec, "unit": unit,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "timing": ("wall clock, max over ranks, the device-timed steps replayed from "
                          "the same training state"
                          + ("; the host reads step k's losses after queuing step k + 1"
                             if pipelined else "; the host waits for each step's result")),
               "clocks": clk_e2e.summary()}

    # Per-stage times come from separate steps after the timed region, with
    # every view on one stream (in the timed steps views overlap on two
    # streams, which would fold one view's kernels into another's interval).
    nt = getattr(tr, "nt", None)
    saved_streams = nt.num_streams if nt is not None else None
    saved_graph = getattr(tr, "graph", False)
    if nt is not None:
        nt.num_streams = 1
        tr.graph = False  # stage events need the launches one by one
    with StageTimer() as stages:
        for _ in range(min(args.steps, 3)):
            run_step()
        torch.cuda.synchronize()
    if nt is not None:
        nt.num_streams = saved_streams
        tr.graph = saved_graph
    barrier(world)
    stage_ms = stages.mean_ms()

    # roofline of the dominant stage
    hbm, bf16, src = peaks()
    E, K, visible = count_pairs(tr)
    T = ((cfg.width + 15) // 16) * ((cfg.height + 15) // 16)
    clocks = clk.summary()
    sm_mhz = clocks.get("sm_max_mhz") or 1965.0
    fp32_peak = 148 * 128 * 2 * sm_mhz * 1e6 / 1e12  # TFLOP/s, nominal at max SM clock
    roof = {}
    if stage_ms.get("gs_preprocess_forward"):
        gbs = PRE_FWD_BYTES_PER_G * n / (stage_ms["gs_preprocess_forward"] * 1e-3) / 1e9
        roof["preprocess_fwd"] = {"bound": "hbm", "ms": stage_ms["gs_preprocess_forward"],
                                  "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}
    if stage_ms.get("gs_preprocess_backward"):
        gbs = PRE_BWD_BYTES_PER_G * n / (stage_ms["gs_preprocess_backward"] * 1e-3) / 1e9
        roof["preprocess_bwd"] = {"bound": "hbm", "ms": stage_ms["gs_preprocess_backward"],
                                  "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}
    # multi-view launches (NativeTrainer): one launch covers this rank's V views; the
    # algorithmic bytes are those of the fused operation -- parameters read once, every
    # view's outputs written (forward); parameters and every view's upstream gradients
    # read, the summed gradient written once (backward)
    if stage_ms.get("gs_preprocess_forward_views"):
        ms = stage_ms["gs_preprocess_forward_views"]
        gbs = (PARAM_BYTES_PER_G + PRE_OUT_BYTES_PER_G * V) * n / (ms * 1e-3) / 1e9
        roof["preprocess_fwd"] = {"bound": "hbm", "ms": ms / V, "ms_per_launch": ms,
                                  "views_per_launch": V, "achieved": gbs, "peak": hbm,
                                  "unit": "GB/s", "frac": gbs / hbm}
    if stage_ms.get("gs_preprocess_backward_views"):
        ms = stage_ms["gs_preprocess_backward_views"]
        gbs = (2 * PARAM_BYTES_PER_G + PRE_UP_BYTES_PER_G * V) * n / (ms * 1e-3) / 1e9
        roof["preprocess_bwd"] = {"bound": "hbm", "ms": ms / V, "ms_per_launch": ms,
                                  "views_per_launch": V, "achieved": gbs, "peak": hbm,
                                  "unit": "GB/s", "frac": gbs / hbm}
    lay_ms = (stage_ms.get("gs_tile_layout") or stage_ms.get("gs_tile_layout_capped")
              or stage_ms.get("gs_tile_bins"))
    if lay_ms:
        lay_ms += stage_ms.get("gs_tile_order") or 0.0  # the blend order is part of the layout
        gbs = (LAYOUT_BYTES_PER_PAIR * K + 4 * T) / (lay_ms * 1e-3) / 1e9
        roof["tile_layout"] = {"bound": "hbm", "ms": lay_ms, "achieved": gbs,
                               "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}
    if stage_ms.get("gs_tile_layout_views"):
        # one launch lays out every view of the step: the reference's bytes for
        # each view's pairs (its 6-pass 64-bit sort basis) and tile offsets
        ms = stage_ms["gs_tile_layout_views"]
        ktot = sum(getattr(getattr(tr, "nt", None), "last_totals", None) or [K] * V)
        gbs = (LAYOUT_BYTES_PER_PAIR * ktot + 4 * T * V) / (ms * 1e-3) / 1e9
        roof["tile_layout"] = {"bound": "hbm", "ms": ms / V, "ms_per_launch": ms,
                               "views_per_launch": V, "pairs_per_launch": int(ktot),
                               "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm,
                               "basis": "reference's bytes: (12 + 144 + 8) B per pair + "
                                        "4 B per tile"}
    for key, nm, fl in (("blend_fwd", "gs_blend_forward", BLEND_FWD_FLOP_PER_PAIR),
                        ("blend_bwd", "gs_blend_backward", BLEND_BWD_FLOP_PER_PAIR)):
        if stage_ms.get(nm):
            tf = fl * E / (stage_ms[nm] * 1e-3) / 1e12
            roof[key] = {"bound": "fp32", "ms": stage_ms[nm], "achieved": tf, "peak": fp32_peak,
                         "unit": "TFLOP/s", "frac": tf / fp32_peak}
    npx = cfg.width * cfg.height * 3
    tgt_bytes = 4  # float targets in the device-timed loop
    if stage_ms.get("gs_l1_loss_grad"):  # raw + target read, gradient written
        gbs = npx * (4 + tgt_bytes + 4) / (stage_ms["gs_l1_loss_grad"] * 1e-3) / 1e9
        roof["loss"] = {"bound": "hbm", "ms": stage_ms["gs_l1_loss_grad"], "achieved": gbs,
                        "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}
    if stage_ms.get("gs_l1_ssim_loss_grad"):
        # two kernels: raw + target read, three fp32 maps written; maps + raw + target read,
        # gradient written
        b = npx * ((4 + tgt_bytes + 12) + (12 + 4 + tgt_bytes + 4))
        gbs = b / (stage_ms["gs_l1_ssim_loss_grad"] * 1e-3) / 1e9
        roof["loss"] = {"bound": "hbm", "ms": stage_ms["gs_l1_ssim_loss_grad"], "achieved": gbs,
                        "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}
    numel = tr.fp.padded
    nccl = None
    if world > 1 and not render_mode:
        bus_gbs, ar_ms = nccl_allreduce_bus_gbs(numel, world, device)
        nccl = {"bus_gbs": bus_gbs, "ms": ar_ms, "bytes": 4 * numel,
                "what": "NCCL all-reduce of the flat gradient's size in this run, "
                        "2 (w - 1) / w * bytes / time, max over ranks"}
    if stage_ms.get("gs_adam_step"):  # param, grad, m, v read; param, m, v written
        gbs = 28 * numel / (stage_ms["gs_adam_step"] * 1e-3) / 1e9
        roof["optimizer"] = {"bound": "hbm", "ms": stage_ms["gs_adam_step"], "achieved": gbs,
                             "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}
    if stage_ms.get("gs_dp_adam_step"):
        # all-reduce-equivalent bus bytes per rank, 2 (w - 1) / w * 4 B * numel, against the
        # NCCL all-reduce bus bandwidth measured in this run at the same size
        bus = 2 * (world - 1) / world * 4 * numel
        gbs = bus / (stage_ms["gs_dp_adam_step"] * 1e-3) / 1e9
        peak_bus = nccl["bus_gbs"]
        roof["optimizer"] = {"bound": "nvlink", "ms": stage_ms["gs_dp_adam_step"],
                             "achieved": gbs, "peak": peak_bus, "unit": "GB/s",
                             "frac": gbs / peak_bus,
                             "peak_source": "NCCL all-reduce bus bandwidth of this run",
                             "multicast": bool(getattr(tr.fp, "multicast", False))}
    dom = max(roof, key=lambda k: roof[k]["ms"]) if roof else None
    roofline = None
    if dom:
        r = roof[dom]
        roofline = {"kernel": dom, "bound": r["bound"], "achieved": r["achieved"],
                    "peak": r["peak"], "unit": r["unit"], "frac": r["frac"],
                    "traffic": NCU_TRAFFIC_BYTES.get(dom) if args.config == 1 and args.n is None
                    else None,
                    "traffic_unit": "bytes/launch (ncu capture of this kernel, config 1)",
                    "peak_source": (f"{src} MEASURED_PEAKS.json hbm_gbs" if r["bound"] == "hbm"
                                    else "nominal FP32: 148 SMs x 128 lanes x 2 FLOP x max SM clock"
                                         " (MEASURED_PEAKS.json has no FP32 figure)"),
                    "work_per_launch": (f"{E} evaluated pairs" if r["bound"] == "fp32"
                                        else "algorithmic bytes per launch over its time")}

    parity = None
    if world > 1 and not render_mode and not args.no_subrecords:
        parity = dp_parity(tr, world, rank)
    subs = {}
    headline = args.config == 1 and args.n is None and not render_mode
    if headline and not args.no_subrecords:
        ours_view_ms = {k: (roof[k]["ms"] if k in roof else None)
                        for k in ("preprocess_fwd", "tile_layout", "blend_fwd", "blend_bwd",
                                  "preprocess_bwd")}
        del tr
        torch.cuda.empty_cache()
        subs["config2"] = sub_record(sub_config2, args, world, rank, device)
        subs["config4"] = sub_record(sub_config4, args, world, rank, device)
        subs["render_api"] = sub_record(sub_render_api, args, world, rank, device)
        if world == 1:
            subs["gpu_reference"] = sub_record(sub_gpu_reference, device, ours_view_ms)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not render_mode:
        act, cams, tg, threads = cpu_setup(cfg, args.n, args.cpu_sample_views)
        sec = cpu_fwd_bwd_views(cfg, act, cams, tg, lam)
        cpu = {"value": args.cpu_sample_views / sec, "unit": "views/s", "cores": threads,
               "kind": "port",
               "sample": f"{args.cpu_sample_views} full views fwd+bwd of the same scene "
                         f"(oracle/gs_oracle.c, OpenMP)", "cpu": cpu_model()}

    if rank == 0:
        line = {
            "metric": METRIC if not render_mode else "inference frames/s (config 4)",
            "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "ms_per_view": ms_step / V, "higher_is_better": True,
            "scaling": "strong" if args.strong else "weak",
            "mode": args.mode,
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(args, cfg, V), "e2e": e2e, "gpu_launches": int(launches),
            "clocks": clocks, "roofline": roofline, "stages": roof,
            "stages_timing": "CUDA events around each stage in separate steps after the timed "
                             "region, all views on one stream",
            "pairs": {"K": K, "evaluated_fwd": E, "visible": visible, "tiles": T},
            "cpu_baseline": cpu,
        }
        if headline and not args.no_cpu_baseline and world == 1:
            line["cpu_reference_cfg0"] = sub_record(cpu_torch_reference_cfg0)
        if nccl is not None:
            line["nccl_allreduce"] = nccl
        if parity is not None:
            line["dp_parity"] = parity
        line.update(subs)
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        torch.cuda.synchronize()
        barrier(world)
        tr = None  # symmetric-memory buffers go before the process group
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
