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
    accumulates in place) and flat Adam state.

    With `fused_dp` set and a process group of world > 1 on CUDA, the two
    flat buffers live in symmetric memory (every rank can address every
    other rank's buffers, and the NVSwitch multicast mapping is used when
    the system has one) and `step()` runs the fused data-parallel optimizer
    step (gs_dp_adam_step: reduce-scatter of the gradient, Adam on this
    rank's 1/world shard, all-gather of the parameters, in one kernel);
    each rank then keeps only its shard of the Adam moments. fused_dp is
    "auto", "multicast" (the NVSwitch multicast mapping when the system has
    one, else peer loads and stores), "p2p" (always peer loads and stores)
    or False (NCCL all-reduce + full Adam). "auto" (also True) takes peer
    loads and stores at world 2 and multicast above: a multicast reduce
    fetches every rank's copy through the switch, the rank's own included,
    so per step each GPU's links carry about (1 + 1/world) times the
    gradient bytes each way, against 2 (world - 1) / world times for peer
    loads and stores -- 1.5 against 1 at world 2 (measured on two B200s at
    config 1: 0.70 against 0.56 ms per optimizer step), 1.125 against 1.75
    at world 8."""

    def __init__(self, tensors: dict, lrs: dict | None = None, eps: float = 1e-15,
                 betas=(0.9, 0.999), group=None, fused_dp=False):
        first = tensors[GROUPS[0]]
        self.device = first.device
        self.group = group
        self.world, self.rank = _world_rank(group)
        self.fused = bool(fused_dp) and self.world > 1 and self.device.type == "cuda"
        if fused_dp and fused_dp not in (True, "auto", "multicast", "p2p"):
            raise ValueError("fused_dp must be False, True, 'auto', 'multicast' or 'p2p'")
        self._force_p2p = fused_dp == "p2p" or (fused_dp in (True, "auto") and self.world <= 2)
        self._set_layout({k: tuple(tensors[k].shape) for k in GROUPS})
        self._alloc_buffers()
        for k in GROUPS:
            a, n = self.spans[k]
            self.data[a:a + n].copy_(tensors[k].reshape(-1))
        self._make_params()
        self.lrs = dict(DEFAULT_LRS if lrs is None else lrs)
        self.eps = float(eps)
        self.betas = (float(betas[0]), float(betas[1]))
        self.exp_avg = None
        self.exp_avg_sq = None
        self.step_count = 0
        self._epoch = 0

    def _set_layout(self, shapes):
        self.shapes = dict(shapes)
        self.spans = {}
        off = 0
        for k in GROUPS:
            n = 1
            for d in self.shapes[k]:
                n *= d
            self.spans[k] = (off, n)
            off += (n + 3) // 4 * 4
        self.numel = off
        self.padded = padded_numel(off, self.world) if self.fused else off

    def _alloc_buffers(self):
        if self.fused:
            self._setup_symmetric()
        else:
            f = dict(device=self.device, dtype=torch.float32)
            self.data = torch.zeros(self.padded, **f)
            self.grad = torch.zeros(self.padded, **f)

    def _make_params(self):
        self.params = {}
        for k in GROUPS:
            a, n = self.spans[k]
            p = torch.nn.Parameter(self.data[a:a + n].view(self.shapes[k]))
            p.grad = self.grad[a:a + n].view(self.shapes[k])
            self.params[k] = p

    @property
    def num_gaussians(self) -> int:
        return self.shapes[GROUPS[0]][0]

    def group_offsets(self):
        """Element offset of each group in the flat buffers (host int64 array)."""
        return (ctypes.c_int64 * len(GROUPS))(*[self.spans[k][0] for k in GROUPS])

    def full_moments(self):
        """The Adam moments over the whole flat buffer (gathered from the
        ranks' shards with the fused step), or (None, None) before the first
        step."""
        if self.exp_avg is None:
            return None, None
        if not self.fused:
            return self.exp_avg, self.exp_avg_sq
        import torch.distributed as dist

        full = []
        for t in (self.exp_avg, self.exp_avg_sq):
            out = torch.empty(self.padded, device=self.device, dtype=torch.float32)
            dist.all_gather_into_tensor(out, t, group=self.group)
            full.append(out)
        return full[0], full[1]

    def rebuild(self, num_gaussians: int, fill):
        """Re-lay the buffers out for `num_gaussians` Gaussians. fill(old_data,
        old_offsets, new_data, new_offsets, old_m, old_v, new_m, new_v) writes
        the new parameters (and, when the moments exist, the new moments) from
        the old; the gradient buffer comes back zeroed. With the fused step
        this is a collective (new symmetric buffers, re-sharded moments)."""
        old_data, old_offsets = self.data, self.group_offsets()
        old_m, old_v = self.full_moments()
        self._set_layout({k: (int(num_gaussians),) + tuple(self.shapes[k][1:]) for k in GROUPS})
        self._alloc_buffers()
        new_m = new_v = None
        if old_m is not None:
            new_m = torch.zeros(self.padded, device=self.device, dtype=torch.float32)
            new_v = torch.zeros(self.padded, device=self.device, dtype=torch.float32)
        fill(old_data, old_offsets, self.data, self.group_offsets(), old_m, old_v, new_m, new_v)
        if new_m is not None:
            if self.fused:
                shard = self.padded // self.world
                sl = slice(self.rank * shard, (self.rank + 1) * shard)
                new_m, new_v = new_m[sl].clone(), new_v[sl].clone()
            self.exp_avg, self.exp_avg_sq = new_m, new_v
        self._make_params()

    # ---- symmetric-memory set-up (fused data-parallel step) -----------------

    def _setup_symmetric(self):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        gname = (self.group if self.group is not None else dist.group.WORLD).group_name
        self.data = symm.empty(self.padded, dtype=torch.float32, device=self.device)
        self.grad = symm.empty(self.padded, dtype=torch.float32, device=self.device)
        self.data.zero_()
        self.grad.zero_()
        self.num_blocks = max(1, min(int(nat.query("gs_dp_max_blocks")),
                                     -(-self.padded // (self.world * 4 * 512))))
        words = int(nat.query("gs_dp_flag_words", self.num_blocks))
        self.flags = symm.empty(words, dtype=torch.int32, device=self.device)
        self.flags.zero_()
        torch.cuda.synchronize(self.device)
        self._h_data = symm.rendezvous(self.data, gname)
        self._h_grad = symm.rendezvous(self.grad, gname)
        self._h_flags = symm.rendezvous(self.flags, gname)
        vp = ctypes.c_void_p * self.world
        g_ptrs, mc_g = self._peer_ptrs(self.grad, self._h_grad)
        p_ptrs, mc_p = self._peer_ptrs(self.data, self._h_data)
        f_ptrs, _ = self._peer_ptrs(self.flags, self._h_flags)
        self._grad_ptrs, self._param_ptrs, self._flag_ptrs = vp(*g_ptrs), vp(*p_ptrs), vp(*f_ptrs)
        self.multicast = (not self._force_p2p) and mc_g != 0 and mc_p != 0
        self._mc = (mc_g, mc_p) if self.multicast else (None, None)
        dist.barrier(group=self.group)

    def _peer_ptrs(self, t, h):
        """Every rank's address of tensor t and its multicast address (0 if
        none), from the rendezvous handle of t. The handle must address t
        itself on this rank (anything else is refused rather than guessed)."""
        ptrs = [int(x) for x in h.buffer_ptrs]
        if len(ptrs) != self.world or ptrs[self.rank] != t.data_ptr():
            raise RuntimeError("symmetric-memory handle does not address the tensor")
        if any(x % 16 for x in ptrs):
            raise RuntimeError("symmetric buffers must be 16-byte aligned")
        mc = int(getattr(h, "multicast_ptr", 0) or 0)
        if mc % 16:
            mc = 0
        return ptrs, mc

    def __getitem__(self, k):
        return self.params[k]

    def zero_grad(self):
        self.grad.zero_()

    def allreduce_grads(self, group=None):
        """Sum the flat gradient over the ranks of `group` (no-op at world 1)."""
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            dist.all_reduce(self.grad, op=dist.ReduceOp.SUM, group=group)

    def _group_table(self):
        ends, lrs = [], []
        for i, k in enumerate(GROUPS):
            nxt = self.spans[GROUPS[i + 1]][0] if i + 1 < len(GROUPS) else self.padded
            ends.append(nxt)
            lrs.append(self.lrs[k])
        ends_c = (ctypes.c_int64 * len(GROUPS))(*ends)
        lrs_c = (ctypes.c_float * len(GROUPS))(*lrs)
        eps_c = (ctypes.c_float * len(GROUPS))(*([self.eps] * len(GROUPS)))
        return ends_c, lrs_c, eps_c

    def adam_step(self):
        """One Adam step over every group with the native one-launch kernel
        (on this rank's full buffer; the gradient must already be summed)."""
        if self.device.type != "cuda":
            raise RuntimeError("adam_step runs on the GPU kernel only")
        if self.fused:
            raise RuntimeError("with fused_dp the optimizer runs in step()")
        if self.exp_avg is None:
            self.exp_avg = torch.zeros_like(self.data)
            self.exp_avg_sq = torch.zeros_like(self.data)
        self.step_count += 1
        ends_c, lrs_c, eps_c = self._group_table()
        nat.call("gs_adam_step", self.padded, self.data.data_ptr(), self.grad.data_ptr(),
                 self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), len(GROUPS),
                 ctypes.cast(ends_c, ctypes.c_void_p), ctypes.cast(lrs_c, ctypes.c_void_p),
                 ctypes.cast(eps_c, ctypes.c_void_p), self.betas[0], self.betas[1],
                 self.step_count, nat.stream_ptr(self.device))

    # ---- the optimizer step inside a CUDA graph (world 1) -------------------
    #
    # A captured launch keeps the arguments it was captured with, so the step
    # count (through Adam's bias corrections) cannot be an argument: the
    # graph's Adam launch reads its group table from a device buffer, and
    # upload_table() copies the table of the coming step there (from a ring
    # of pinned host buffers, each reused only after its copy completed)
    # before every replay.
    _RING = 8

    def table_adam_step(self):
        """The Adam launch of a graph: reads the table last uploaded."""
        if self.exp_avg is None or self.fused:
            raise RuntimeError("table_adam_step needs the Adam state of a one-GPU FlatParams")
        nat.call("gs_adam_step_table", self.padded, self.data.data_ptr(), self.grad.data_ptr(),
                 self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(),
                 self._table_dev.data_ptr(), self.betas[0], self.betas[1],
                 nat.stream_ptr(self.device))

    def prepare_table(self):
        """Adam state and the device table buffer, allocated before a capture."""
        if self.exp_avg is None:
            self.exp_avg = torch.zeros_like(self.data)
            self.exp_avg_sq = torch.zeros_like(self.data)
        if getattr(self, "_table_dev", None) is None:
            nb = int(nat.query("gs_adam_table_bytes"))
            self._table_dev = torch.zeros(-(-nb // 8), dtype=torch.int64, device=self.device)
            self._table_host = [torch.zeros(-(-nb // 8), dtype=torch.int64).pin_memory()
                                for _ in range(self._RING)]
            self._table_done = [None] * self._RING
            self._table_slot = 0

    def upload_table(self, step):
        """Copies the group table of Adam step `step` to the device buffer,
        on the current stream (ahead of the replay that reads it)."""
        k = self._table_slot
        self._table_slot = (k + 1) % self._RING
        if self._table_done[k] is not None:
            self._table_done[k].synchronize()  # the slot's previous copy has read it
        host = self._table_host[k]
        ends_c, lrs_c, eps_c = self._group_table()
        nat.call("gs_adam_table", self.padded, len(GROUPS), ctypes.cast(ends_c, ctypes.c_void_p),
                 ctypes.cast(lrs_c, ctypes.c_void_p), ctypes.cast(eps_c, ctypes.c_void_p),
                 self.betas[0], self.betas[1], int(step), host.data_ptr(),
                 host.numel() * 8)
        self._table_dev.copy_(host, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record()
        self._table_done[k] = ev

    def gaussian_ranges(self, lo, hi):
        """Element ranges (host int64 arrays: starts, counts) of the flat
        buffer that hold Gaussians lo .. hi - 1 in each of the six groups (a
        group holds its Gaussians contiguously); the range that ends the
        group also takes its padding. lo and hi multiples of 4 (or hi = N)."""
        n = self.num_gaussians
        starts, counts = [], []
        for k in GROUPS:
            off, numel = self.spans[k]
            w = numel // n if n else 0
            a = off + w * lo
            b = off + ((numel + 3) // 4 * 4 if hi >= n else w * hi)
            starts.append(a)
            counts.append(b - a)
        return ((ctypes.c_int64 * len(GROUPS))(*starts),
                (ctypes.c_int64 * len(GROUPS))(*counts))

    def range_adam_step(self, ranges):
        """Adam on the element ranges of gaussian_ranges(), reading the group
        table last uploaded (upload_table) -- in a CUDA graph or not."""
        starts_c, counts_c = ranges
        nat.call("gs_adam_step_ranges", self.data.data_ptr(), self.grad.data_ptr(),
                 self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), len(GROUPS),
                 ctypes.cast(starts_c, ctypes.c_void_p), ctypes.cast(counts_c, ctypes.c_void_p),
                 self._table_dev.data_ptr(), self.betas[0], self.betas[1],
                 nat.stream_ptr(self.device))

    def fused_step(self, grad_shard_out=None):
        """The fused data-parallel optimizer step (see the class docstring).
        grad_shard_out, if given, receives this rank's shard of the summed
        gradient (padded // world floats)."""
        if not self.fused:
            raise RuntimeError("fused_step needs fused_dp and world > 1")
        shard = self.padded // self.world
        if self.exp_avg is None:
            self.exp_avg = torch.zeros(shard, device=self.device, dtype=torch.float32)
            self.exp_avg_sq = torch.zeros(shard, device=self.device, dtype=torch.float32)
        self.step_count += 1
        self._epoch = (self._epoch + 1) & 0x7FFFFFFF
        ends_c, lrs_c, eps_c = self._group_table()
        out = 0 if grad_shard_out is None else grad_shard_out.data_ptr()
        nat.call("gs_dp_adam_step", self.world, self.rank, self._grad_ptrs, self._param_ptrs,
                 self._flag_ptrs, self._mc[0], self._mc[1], self.padded,
                 self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), len(GROUPS),
                 ctypes.cast(ends_c, ctypes.c_void_p), ctypes.cast(lrs_c, ctypes.c_void_p),
                 ctypes.cast(eps_c, ctypes.c_void_p), self.betas[0], self.betas[1],
                 self.step_count, self._epoch, self.num_blocks, out,
                 nat.stream_ptr(self.device))

    def merge_status(self):
        """Every rank's device status word, max-reduced over the group and
        merged into the local word (gs_status_export / gs_status_merge), so
        that the status-gated Adam kernel skips or applies the update on all
        ranks alike. No-op at world 1."""
        import torch.distributed as dist

        if self.device.type != "cuda" or not (dist.is_available() and dist.is_initialized()):
            return
        if dist.get_world_size(self.group) <= 1:
            return
        st = torch.zeros(1, dtype=torch.int32, device=self.device)
        nat.call("gs_status_export", st.data_ptr(), nat.stream_ptr(self.device))
        dist.all_reduce(st, op=dist.ReduceOp.MAX, group=self.group)
        nat.call("gs_status_merge", st.data_ptr(), nat.stream_ptr(self.device))

    def step(self):
        """The step's gradient sum over the ranks and the Adam update: the
        fused kernel with fused_dp, else NCCL all-reduce + one-launch Adam.
        Both skip the update on every rank when any rank's device status
        word holds an error from earlier in the step."""
        if self.fused:
            self.fused_step()
        else:
            self.allreduce_grads(self.group)
            self.merge_status()
            self.adam_step()


def padded_numel(numel: int, world: int) -> int:
    """Flat length rounded up so that each of `world` shards is a whole
    number of float4s (the fused step's unit of work)."""
    q = 4 * max(int(world), 1)
    return -(-int(numel) // q) * q


def _world_rank(group):
    import torch.distributed as dist

    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size(group), dist.get_rank(group)
    return 1, 0
