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
# 8-rank NCCL all-reduce bus bandwidth at 1 GiB measured on this pool's B200s (GB/s): the
# reference figure for the fused data-parallel optimizer step
NVLINK_ALLREDUCE_BUS_GBS = 725.0
BLEND_FWD_FLOP_PER_PAIR = 22
BLEND_BWD_FLOP_PER_PAIR = 60

# DRAM bytes (read + write) per launch at config 1 (4 views per step), from the
# ncu --set full captures summarised in profiles/kernels_cfg1_full.md and
# profiles/blend_kernels_cfg1.md (dram__bytes_read.sum + dram__bytes_write.sum;
# preprocess_fwd is the one multi-view launch).
NCU_TRAFFIC_BYTES = {"preprocess_fwd": 416.7e6, "blend_fwd": 57.2e6, "blend_bwd": 110.0e6,
                     "loss": 50.8e6}


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
    p.add_argument("--streams", type=int, default=2,
                   help="CUDA streams the native trainer spreads a step's views over")
    p.add_argument("--dp", choices=["nccl", "fused", "fused-p2p"], default="fused",
                   help="multi-GPU optimizer step: NCCL all-reduce + Adam, or the fused "
                        "reduce-scatter / sharded Adam / all-gather kernel (multicast when "
                        "available, or peer stores only)")
    p.add_argument("--ssim-lambda", type=float, default=None,
                   help="loss = (1 - l) L1 + l (1 - SSIM); default 0.2 for config 2, else 0")
    p.add_argument("--config", type=int, default=1)
    p.add_argument("--n", type=int, default=None, help="override Gaussian count (tests/profiling)")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--cpu-sample-views", type=int, default=2)
    p.add_argument("--mode", choices=["train", "render"], default="train",
                   help="render: forward-only novel-view rendering (config 4), frames/s")
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

    WATCH = ("gs_preprocess_forward", "gs_tile_layout", "gs_blend_forward", "gs_blend_backward",
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
    cams = scenes.orbit_cameras(cfg, views).numpy()
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
            "trainer": args.trainer, "streams": getattr(args, "streams", 1)}


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
        cams = scenes.orbit_cameras(cfg, total_views)
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
                 streams=2):
        self.cfg = cfg
        self.world = world
        self.device = device
        raw = scenes.make_gaussians(cfg, seed=0, n=n, device=device)
        fused = {"nccl": False, "fused": "auto", "fused-p2p": "p2p"}[dp_mode]
        self.nt = trainer_mod.NativeTrainer(raw, cfg.width, cfg.height, ssim_lambda=ssim_lambda,
                                            fused_dp=fused, streams=streams)
        self.fp = self.nt.fp
        self.params = self.fp.params
        cams = scenes.orbit_cameras(cfg, total_views)
        mine = dp.shard_views(total_views, rank, world)
        views = len(mine)
        self.cams = cams[mine].to(device)
        self.K = scenes.intrinsic_for(cfg).to(device)
        g = torch.Generator(device=device).manual_seed(1234 + rank)
        self.targets = [torch.rand((cfg.height, cfg.width, 3), device=device, generator=g) * 255.0
                        for _ in range(views)]
        self.host_targets = [(t.cpu().round().clamp(0, 255).to(torch.uint8)).pin_memory()
                             for t in self.targets]
        self.host_cams = self.cams.cpu().pin_memory()
        self.host_K = self.K.cpu().pin_memory()
        self.host_loss = torch.zeros(len(self.targets), dtype=torch.float64).pin_memory()

    def step(self, e2e=False):
        if e2e:
            # cameras copied here; the pinned host targets go to the trainer, which
            # copies them on a copy stream while the views are rendered
            cams = self.host_cams.to(self.device, non_blocking=True)
            K = self.host_K.to(self.device, non_blocking=True)
            tg = self.host_targets
        else:
            cams, K, tg = self.cams, self.K, self.targets
        losses = self.nt.step(cams, K, tg)
        if e2e:
            self.host_loss.copy_(losses, non_blocking=True)
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
        views = self.nt.forward_views(cams, K)
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
                                dp_mode=args.dp, streams=args.streams)
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
        run_step()
    torch.cuda.synchronize()
    barrier(world)

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
    ms_total = max_over_ranks(start.elapsed_time(end), world)
    ms_step = ms_total / args.steps
    value = total_views * args.steps / (ms_total / 1000.0)
    unit = "frames/s" if render_mode else "views/s"

    # Per-stage times come from separate steps after the timed region, with
    # every view on one stream (in the timed steps views overlap on two
    # streams, which would fold one view's kernels into another's interval).
    nt = getattr(tr, "nt", None)
    saved_streams = nt.num_streams if nt is not None else None
    if nt is not None:
        nt.num_streams = 1
    with StageTimer() as stages:
        for _ in range(min(args.steps, 3)):
            run_step()
        torch.cuda.synchronize()
    if nt is not None:
        nt.num_streams = saved_streams
    barrier(world)
    stage_ms = stages.mean_ms()

    e2e = None
    if not args.no_e2e:
        for _ in range(2):
            run_step(e2e=True)
        torch.cuda.synchronize()
        barrier(world)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            run_step(e2e=True)
            torch.cuda.current_stream().synchronize()  # the step's result is on the host
        barrier(world)
        sec = max_over_ranks(time.perf_counter() - t0, world)
        if render_mode:
            h2d = V * (16 + 9) * 4
            d2h = V * cfg.width * cfg.height * 3
        else:
            h2d = sum(t.numel() for t in tr.host_targets) + V * (16 + 9) * 4
            d2h = V * 8
        e2e = {"value": total_views * args.steps / sec, "unit": unit,
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "timing": "wall clock, max over ranks"}

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
    if stage_ms.get("gs_tile_layout"):
        gbs = (LAYOUT_BYTES_PER_PAIR * K + 4 * T) / (stage_ms["gs_tile_layout"] * 1e-3) / 1e9
        roof["tile_layout"] = {"bound": "hbm", "ms": stage_ms["gs_tile_layout"], "achieved": gbs,
                               "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}
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
    if stage_ms.get("gs_adam_step"):  # param, grad, m, v read; param, m, v written
        gbs = 28 * numel / (stage_ms["gs_adam_step"] * 1e-3) / 1e9
        roof["optimizer"] = {"bound": "hbm", "ms": stage_ms["gs_adam_step"], "achieved": gbs,
                             "peak": hbm, "unit": "GB/s", "frac": gbs / hbm}
    if stage_ms.get("gs_dp_adam_step"):
        # all-reduce-equivalent bus bytes per rank, 2 (w - 1) / w * 4 B * numel, against the
        # measured 8-rank NCCL all-reduce bus bandwidth of this pool
        bus = 2 * (world - 1) / world * 4 * numel
        gbs = bus / (stage_ms["gs_dp_adam_step"] * 1e-3) / 1e9
        roof["optimizer"] = {"bound": "nvlink", "ms": stage_ms["gs_dp_adam_step"],
                             "achieved": gbs, "peak": NVLINK_ALLREDUCE_BUS_GBS, "unit": "GB/s",
                             "frac": gbs / NVLINK_ALLREDUCE_BUS_GBS,
                             "multicast": bool(getattr(tr.fp, "multicast", False))}
    dom = max(roof, key=lambda k: roof[k]["ms"]) if roof else None
    roofline = None
    if dom:
        r = roof[dom]
        roofline = {"kernel": dom, "bound": r["bound"], "achieved": r["achieved"],
                    "peak": r["peak"], "unit": r["unit"], "frac": r["frac"],
                    "traffic": NCU_TRAFFIC_BYTES.get(dom) if args.config == 1 and args.n is None
                    else None,
                    "traffic_unit": "bytes/launch (ncu, profiles/)",
                    "peak_source": (f"{src} MEASURED_PEAKS.json hbm_gbs" if r["bound"] == "hbm"
                                    else "nominal FP32: 148 SMs x 128 lanes x 2 FLOP x max SM clock"
                                         " (MEASURED_PEAKS.json has no FP32 figure)"),
                    "work_per_launch": (f"{E} evaluated pairs" if r["bound"] == "fp32"
                                        else "algorithmic bytes per launch over its time")}

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
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        torch.cuda.synchronize()
        barrier(world)
        del tr  # symmetric-memory buffers go before the process group
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
