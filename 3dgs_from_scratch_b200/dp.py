"""Data-parallel training over camera views.

Each rank holds a full replica of the Gaussians, renders its own share of
the step's views, and accumulates the parameter gradients into one flat fp32
buffer; one all_reduce(SUM) of that buffer per step (NCCL over NVLink on
GPUs, gloo on CPU) makes the gradients identical on every rank, and every
rank then applies the same optimizer step. The reference trains on one GPU
with one view per step (scripts/train.py:160-166); this module is the
multi-GPU extension of that loop.

The six parameter groups of the reference (means, scales, quaternions,
opacities, sh_coeffs_dc, sh_coeffs_rest; scripts/train.py:17-44) live back to
back in one flat buffer (each group padded to a multiple of 4 elements), so
the all-reduce and the optimizer are one call each.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native as nat

GROUPS = ("means", "scales", "quaternions", "opacities", "sh_coeffs_dc", "sh_coeffs_rest")

# scripts/train.py:17-44 (batch_size = 1)
DEFAULT_LRS = {"means": 1.6e-4, "scales": 5e-3, "quaternions": 1e-3, "opacities": 5e-2,
               "sh_coeffs_dc": 2.5e-3, "sh_coeffs_rest": 2.5e-3 / 20}


def shard_views(num_views: int, rank: int, world: int) -> list[int]:
    """Contiguous, balanced split of view indices over ranks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(num_views, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


class FlatParams:
    """Gaussian parameters as views into one flat buffer, with a matching flat
    gradient buffer (each parameter's .grad is a view of it, so autograd
    accumulates in place) and flat Adam state."""

    def __init__(self, tensors: dict, lrs: dict | None = None, eps: float = 1e-15,
                 betas=(0.9, 0.999)):
        first = tensors[GROUPS[0]]
        self.device = first.device
        self.shapes = {k: tuple(tensors[k].shape) for k in GROUPS}
        self.spans = {}
        off = 0
        for k in GROUPS:
            n = tensors[k].numel()
            self.spans[k] = (off, n)
            off += (n + 3) // 4 * 4
        self.numel = off
        f = dict(device=self.device, dtype=torch.float32)
        self.data = torch.zeros(off, **f)
        self.grad = torch.zeros(off, **f)
        self.params = {}
        for k in GROUPS:
            a, n = self.spans[k]
            self.data[a:a + n].copy_(tensors[k].reshape(-1))
            p = torch.nn.Parameter(self.data[a:a + n].view(self.shapes[k]))
            p.grad = self.grad[a:a + n].view(self.shapes[k])
            self.params[k] = p
        self.lrs = dict(DEFAULT_LRS if lrs is None else lrs)
        self.eps = float(eps)
        self.betas = (float(betas[0]), float(betas[1]))
        self.exp_avg = None
        self.exp_avg_sq = None
        self.step_count = 0

    def __getitem__(self, k):
        return self.params[k]

    def zero_grad(self):
        self.grad.zero_()

    def allreduce_grads(self, group=None):
        """Sum the flat gradient over the ranks of `group` (no-op at world 1)."""
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.grad, op=dist.ReduceOp.SUM, group=group)

    def adam_step(self):
        """One Adam step over every group with the native one-launch kernel."""
        if self.device.type != "cuda":
            raise RuntimeError("adam_step runs on the GPU kernel only")
        if self.exp_avg is None:
            self.exp_avg = torch.zeros_like(self.data)
            self.exp_avg_sq = torch.zeros_like(self.data)
        self.step_count += 1
        ends = []
        lrs = []
        for i, k in enumerate(GROUPS):
            a, n = self.spans[k]
            nxt = self.spans[GROUPS[i + 1]][0] if i + 1 < len(GROUPS) else self.numel
            ends.append(nxt)
            lrs.append(self.lrs[k])
        ends_c = (ctypes.c_int64 * len(GROUPS))(*ends)
        lrs_c = (ctypes.c_float * len(GROUPS))(*lrs)
        eps_c = (ctypes.c_float * len(GROUPS))(*([self.eps] * len(GROUPS)))
        nat.call("gs_adam_step", self.numel, self.data.data_ptr(), self.grad.data_ptr(),
                 self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), len(GROUPS),
                 ctypes.cast(ends_c, ctypes.c_void_p), ctypes.cast(lrs_c, ctypes.c_void_p),
                 ctypes.cast(eps_c, ctypes.c_void_p), self.betas[0], self.betas[1],
                 self.step_count, nat.stream_ptr(self.device))
