"""Adaptive density control on the device (the reference's Strategy).

The reference's Strategy (src/strategy.py:5-250) accumulates, per Gaussian,
the norm of the screen-space means gradient (scaled to NDC) and a
visibility count every step, and every `refine_every_n_steps` steps between
`refine_start_step` and `refine_stop_step` prunes, clones and splits
Gaussians, rebuilding every parameter and Adam-state tensor with host-driven
index_select / torch.cat; every `reset_every_n_steps` steps it clamps the
opacities. DeviceStrategy keeps the same schedule, thresholds and output
order, but works on the flat buffers of dp.FlatParams with this library's
kernels: the statistics are accumulated by gs_densify_accumulate, the
decisions and output slots come from gs_densify_plan and three exclusive
scans, and one gs_densify_apply launch writes the new parameter and Adam
buffers (one host synchronisation per refinement, for the three counts).
Under torch.distributed the statistics are summed over the ranks before the
decisions, and the split samples come from a counter-based generator keyed
by (seed, step, split slot), so every rank makes the same changes.
"""
from __future__ import annotations

import math

import torch

from . import _native as nat
from .dp import FlatParams


class DeviceStrategy:
    # src/strategy.py:6-14
    refine_start_step = 500
    refine_stop_step = 15000
    refine_every_n_steps = 100
    reset_every_n_steps = 3000
    prune_opacity = 0.005
    prune_scale = 0.1
    grow_grad = 0.0002
    split_scale = 0.01
    max_gaussians = 1000000

    def __init__(self, seed: int = 0, group=None):
        self.seed = int(seed)
        self.group = group
        self.grads = None
        self.count = None

    # ---- statistics (strategy.py:48-72) ---------------------------------------

    def _ensure_state(self, n, device):
        if self.grads is None or self.grads.shape[0] != n:
            self.grads = torch.zeros(n, device=device, dtype=torch.float32)
            self.count = torch.zeros(n, device=device, dtype=torch.float32)

    def accumulate(self, grad_points: torch.Tensor, radii: torch.Tensor, width: int,
                   height: int):
        """One view's contribution: grad_points is d loss / d points_img (N, 2),
        radii (N, 2) as render() returns them."""
        n = grad_points.shape[0]
        dev = grad_points.device
        self._ensure_state(n, dev)
        g = grad_points.detach().to(torch.float32).contiguous()
        r = radii.detach().to(torch.float32).contiguous()
        nat.call("gs_densify_accumulate", n, g.data_ptr(), r.data_ptr(), int(width), int(height),
                 self.grads.data_ptr(), self.count.data_ptr(), nat.stream_ptr(dev))

    # ---- the schedule (strategy.py:20-46) -------------------------------------

    def adjust(self, fp: FlatParams, step: int, grad_points=None, radii=None, width=None,
               height=None, noise=None):
        """strategy.adjust for the Gaussians of `fp` after the optimizer step
        of `step`. With grad_points / radii (one view), they are accumulated
        first, as the reference does; a caller with several views per step
        calls accumulate() per view instead. `noise` (2 x n_split x 3, as the
        reference's torch.randn draw) replaces the generated split samples.
        Returns a dict of what changed (empty when nothing was refined)."""
        if step > self.refine_stop_step:
            return {}
        if grad_points is not None:
            self.accumulate(grad_points, radii, width, height)
        out = {}
        if step > self.refine_start_step and step % self.refine_every_n_steps == 0:
            out = self.refine(fp, step, noise)
        if step > 0 and step % self.reset_every_n_steps == 0:
            self.reset_opacities(fp)
            out["reset_opacities"] = True
        return out

    # ---- prune + grow (strategy.py:74-233) --------------------------------------

    def refine(self, fp: FlatParams, step: int, noise: torch.Tensor | None = None):
        dev = fp.device
        n = fp.num_gaussians
        self._ensure_state(n, dev)
        self._allreduce_stats()
        st = nat.stream_ptr(dev)
        codes = torch.empty(n, dtype=torch.uint8, device=dev)
        flags = torch.empty((3, max(n, 1)), dtype=torch.int32, device=dev)
        pos = torch.empty((3, max(n, 1)), dtype=torch.int32, device=dev)
        totals = torch.zeros(3, dtype=torch.int64, device=dev)
        prune_by_scale = int(step > self.reset_every_n_steps)

        def plan(grow_grad):
            nat.call("gs_densify_plan", n, fp.data.data_ptr(), fp.group_offsets(),
                     self.grads.data_ptr(), self.count.data_ptr(), self.prune_opacity,
                     prune_by_scale, self.prune_scale, grow_grad, self.split_scale,
                     codes.data_ptr(), flags[0].data_ptr(), flags[1].data_ptr(),
                     flags[2].data_ptr(), st)

        def scan(k):
            scratch = torch.empty(nat.query("gs_scan_scratch_bytes", n), dtype=torch.uint8,
                                  device=dev)
            nat.call("gs_exclusive_scan", n, flags[k].data_ptr(), pos[k].data_ptr(),
                     totals[k:].data_ptr(), scratch.data_ptr(), scratch.numel(), st)

        plan(self.grow_grad)
        for k in range(3):
            scan(k)
        n_keep, n_clone, n_split = (int(x) for x in totals.cpu())
        survivors = n_keep + n_split
        if survivors >= self.max_gaussians:
            # strategy.py:118-123: at the cap, no growth at all
            plan(math.inf)
            for k in range(3):
                scan(k)
            n_keep, n_clone, n_split = (int(x) for x in totals.cpu())
        elif n_clone > self.max_gaussians - survivors:
            # strategy.py:131-138: a random subset of the clones fills the budget
            budget = self.max_gaussians - survivors
            cand = torch.nonzero(flags[1][:n]).squeeze(1)
            gen = torch.Generator(device=dev).manual_seed(self.seed * 1000003 + step)
            pick = cand[torch.randperm(n_clone, generator=gen, device=dev)[:budget]]
            flags[1].zero_()
            flags[1][pick] = 1
            codes[cand] = 1
            codes[pick] = 2
            scan(1)
            n_clone = budget
        n_new = n_keep + n_clone + 2 * n_split
        if noise is not None:
            noise = noise.to(device=dev, dtype=torch.float32).contiguous()
            if noise.numel() != 2 * n_split * 3:
                raise ValueError("noise must hold 2 x n_split x 3 values")
        seed = (self.seed * 0x9E3779B97F4A7C15 + step) & 0xFFFFFFFFFFFFFFFF

        def fill(old_data, old_off, new_data, new_off, old_m, old_v, new_m, new_v):
            nat.call("gs_densify_apply", n, codes.data_ptr(), pos[0].data_ptr(),
                     pos[1].data_ptr(), pos[2].data_ptr(), n_keep, n_clone, n_split,
                     old_data.data_ptr(), old_off, new_data.data_ptr(), new_off,
                     0 if old_m is None else old_m.data_ptr(),
                     0 if old_v is None else old_v.data_ptr(),
                     0 if new_m is None else new_m.data_ptr(),
                     0 if new_v is None else new_v.data_ptr(),
                     0 if noise is None else noise.data_ptr(), seed, 1.6, st)

        fp.rebuild(n_new, fill)
        # strategy.py:38-40: the statistics restart
        self.grads = torch.zeros(n_new, device=dev, dtype=torch.float32)
        self.count = torch.zeros(n_new, device=dev, dtype=torch.float32)
        return {"pruned": n - n_keep - n_split, "cloned": n_clone, "split": n_split,
                "num_gaussians": n_new}

    def _allreduce_stats(self):
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            both = torch.stack([self.grads, self.count])
            dist.all_reduce(both, op=dist.ReduceOp.SUM, group=self.group)
            self.grads.copy_(both[0])
            self.count.copy_(both[1])

    # ---- opacity reset (strategy.py:235-250) -----------------------------------

    def reset_opacities(self, fp: FlatParams):
        dev = fp.device
        n = fp.num_gaussians
        # torch.logit of prune_opacity * 2 in fp32, as strategy.py:238
        thr = float(torch.logit(torch.tensor(self.prune_opacity * 2.0, dtype=torch.float32)))
        a, _ = fp.spans["opacities"]
        logits = fp.data[a:a + n]
        m_ptr = v_ptr = 0
        if fp.exp_avg is not None:
            if fp.fused:
                self._zero_sharded_opacity_moments(fp, a, n)
            else:
                m_ptr = fp.exp_avg[a:a + n].data_ptr()
                v_ptr = fp.exp_avg_sq[a:a + n].data_ptr()
        nat.call("gs_reset_opacities", n, logits.data_ptr(), m_ptr, v_ptr, thr,
                 nat.stream_ptr(dev))

    @staticmethod
    def _zero_sharded_opacity_moments(fp: FlatParams, a: int, n: int):
        shard = fp.padded // fp.world
        lo, hi = max(a, fp.rank * shard), min(a + n, (fp.rank + 1) * shard)
        if lo < hi:
            fp.exp_avg[lo - fp.rank * shard:hi - fp.rank * shard].zero_()
            fp.exp_avg_sq[lo - fp.rank * shard:hi - fp.rank * shard].zero_()
