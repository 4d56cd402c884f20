"""Native data-parallel training step.

The reference's training step (scripts/train.py:133-222) is, per view:
activations in Torch (exp scales, normalised quaternions, sigmoid
opacities), render(), L1 loss against the target image, backward through
the rasterizer and the activations, Adam on the six parameter groups. This
module runs the same step entirely in this library's kernels, for a batch of
views sharded across ranks:

* activations fused into the preprocess kernels (their Jacobians in the
  preprocess backward), so gradients come out w.r.t. the raw parameters;
* no host synchronisation inside a step: the tile layouts take the pair
  counts from the device (the reference reads each view's count with a
  blocking .item(), rasterizer.cpp:322) and write into buffers of a fixed
  capacity, sized at the first step and grown when a step overflows them
  (the overflowing step is skipped on device and repeated);
* the clamp*255 of render() and the loss with its gradient in one kernel
  (L1, or with ssim_lambda > 0 the reference's (1 - lambda) L1 +
  lambda (1 - SSIM) of scripts/train.py:186-203, in two kernels);
* every view's preprocess in one launch that reads each Gaussian's
  parameters once (gs_preprocess_forward_views), and every view's
  raw-parameter gradients summed on chip by one multi-view preprocess
  backward written straight into the flat gradient buffer
  (gs_preprocess_backward_views), so neither autograd nor a per-view
  gradient pass over the parameters is involved;
* the optimizer step of dp.FlatParams: one NCCL all-reduce of the flat
  gradient (world > 1) and the one-launch Adam, or with fused_dp one kernel
  that reduce-scatters the gradient over NVLink / NVSwitch, applies Adam to
  the rank's shard and all-gathers the parameters.

The renders are the same as render()'s (same kernels); tests compare one step
of this trainer with the autograd path (render() + Torch activations +
torch.nn.functional.l1_loss).
"""
from __future__ import annotations

import torch

from . import _native as nat
from . import cuda_rasterizer
from .dp import GROUPS, FlatParams

RENDER_DEFAULTS = dict(near_plane=0.01, far_plane=100.0, min_opacity=1 / 255, min_radius=0.5,
                       max_radius=128.0, alpha_threshold=1e-4, transmittance_threshold=1e-4,
                       chi_squared_threshold=9.21)


class NativeTrainer:
    """Gaussians as raw parameters (means, log-scales, raw quaternions,
    opacity logits, SH dc, SH rest) in one flat buffer on one CUDA device."""

    AUTO_BIN_PAIRS_PER_TILE = 2560  # as cuda_rasterizer.BIN_MAX_PAIRS_PER_TILE

    def __init__(self, raw: dict, width: int, height: int, lrs: dict | None = None,
                 ssim_lambda: float = 0.0, group=None, fused_dp=False, strategy=None,
                 streams: int = 2, layout: str = "auto", adam_overlap: bool = False,
                 **render_opts):
        self.fp = FlatParams({k: raw[k] for k in GROUPS}, lrs=lrs, group=group, fused_dp=fused_dp)
        if not 0.0 <= float(ssim_lambda) <= 1.0:
            raise ValueError("ssim_lambda must lie in [0, 1]")
        self.ssim_lambda = float(ssim_lambda)
        self.device = self.fp.device
        if self.device.type != "cuda":
            raise RuntimeError("NativeTrainer needs the parameters on a CUDA device")
        self.width, self.height = int(width), int(height)
        self.opts = dict(RENDER_DEFAULTS)
        self.opts.update(render_opts)
        self.strategy = strategy  # a densify.DeviceStrategy, or None
        self.adam_overlap = bool(adam_overlap)
        # Views are independent between the batched preprocess and the batched
        # preprocess backward: view v's layout, blend and loss run on stream
        # v % streams, so one view's latency-bound layout kernels overlap
        # another's throughput-bound blend.
        if streams < 1:
            raise ValueError("streams must be at least 1")
        self.num_streams = int(streams)
        self._side = [torch.cuda.Stream(device=self.device) for _ in range(self.num_streams - 1)]
        self._ssim_scratch = [None] * self.num_streams
        # "batched": every view's tile layout in one cooperative launch
        # (gs_tile_layout_views); "per_view": one gs_tile_layout per view on
        # the view's stream (both sized by a host read of the pair counts);
        # "binned": per-view layouts by per-tile binning (gs_tile_bins);
        # "capped": per-view layouts by the two radix sorts
        # (gs_tile_layout_capped). Both write into buffers of a fixed
        # capacity and keep the pair counts on the device (no host
        # synchronisation in a step; a count beyond the capacity fails the
        # step, which step() repeats with grown buffers).
        # "auto" picks one of the two at every sizing of the buffers: binning
        # while the views average at most AUTO_BIN_PAIRS_PER_TILE pairs per
        # tile (its per-tile radix sorts are cheap for lists of up to 4096
        # entries: configurations 1, 2 and 4), the two sorts above for longer
        # lists (the clustered 4K scene of configuration 3).
        if layout not in ("auto", "binned", "capped", "batched", "per_view"):
            raise ValueError("layout must be 'auto', 'binned', 'capped', 'batched' or 'per_view'")
        self.layout = layout
        self._capacity_form = layout in ("auto", "binned", "capped")
        self._capacity_entry = "gs_tile_layout_capped" if layout == "capped" else "gs_tile_bins"
        self._cap = None  # (capacity, (views, n), buffers) of the capacity form
        self.tx = (self.width + 15) // 16
        self.ty = (self.height + 15) // 16

    def _view_stream(self, v):
        k = v % self.num_streams
        return torch.cuda.current_stream(self.device) if k == 0 else self._side[k - 1]

    def _fork(self):
        """Side streams start after the work queued so far on the current stream."""
        ev = torch.cuda.current_stream(self.device).record_event()
        for s in self._side:
            s.wait_event(ev)

    def _join(self):
        """The current stream continues after the side streams' work."""
        cur = torch.cuda.current_stream(self.device)
        for s in self._side:
            cur.wait_event(s.record_event())

    @property
    def params(self):
        return self.fp.params

    @property
    def n(self) -> int:
        return self.fp.num_gaussians

    def _ptr(self, name):
        return self.fp.params[name].data_ptr()

    def _gptr(self, name):
        a, _ = self.fp.spans[name]
        return self.fp.grad.data_ptr() + 4 * a

    def forward_views(self, world_to_cameras, intrinsics):
        """Render the views (forward only). Returns the per-view state list;
        state["image"] is the raw blended image (H, W, 3) before clamp * 255."""
        o = self.opts
        dev = self.device
        st = nat.stream_ptr(dev)
        n, W, H = self.n, self.width, self.height
        w2c = world_to_cameras.to(dev, torch.float32).contiguous()
        Ks = intrinsics.to(dev, torch.float32)
        if Ks.dim() == 2:
            Ks = Ks.unsqueeze(0).expand(w2c.shape[0], 3, 3)
        Ks = Ks.contiguous()
        V = w2c.shape[0]
        campos = (-(w2c[:, :3, :3].transpose(1, 2) @ w2c[:, :3, 3:4])).squeeze(-1).contiguous()
        totals = torch.empty(V, dtype=torch.int64, device=dev)
        f = dict(device=dev, dtype=torch.float32)
        # every view's preprocess outputs in (V, n, ...) arrays, filled by one
        # launch that reads each Gaussian's parameters once for all views
        batch = dict(points=torch.empty((V, n, 2), **f), depths=torch.empty((V, n), **f),
                     radii=torch.empty((V, n, 2), **f),
                     mask=torch.empty((V, n), device=dev, dtype=torch.uint8),
                     splat=torch.empty((V, n, 8), **f),
                     counts=torch.empty((V, max(n, 1)), device=dev, dtype=torch.int32))
        nat.call("gs_preprocess_forward_views", n, V, self._ptr("means"), self._ptr("scales"),
                 self._ptr("quaternions"), self._ptr("opacities"), self._ptr("sh_coeffs_dc"),
                 self._ptr("sh_coeffs_rest"), w2c.data_ptr(), Ks.data_ptr(), campos.data_ptr(),
                 o["near_plane"], o["far_plane"], o["min_opacity"], o["min_radius"],
                 o["max_radius"], W, H, 0, 1, batch["points"].data_ptr(),
                 batch["depths"].data_ptr(), batch["radii"].data_ptr(), batch["mask"].data_ptr(),
                 batch["splat"].data_ptr(), batch["counts"].data_ptr(), totals.data_ptr(), st)
        views = []
        for v in range(V):
            s = {k: t[v] for k, t in batch.items()}
            s.update(w2c=w2c[v], K=Ks[v], campos=campos[v])
            views.append(s)
        self._batch = dict(batch, w2c=w2c, K=Ks, campos=campos, totals=totals)
        T = self.tx * self.ty
        capped = self._capacity_form and self._cap is not None and self._cap[1] == (V, n)
        if not capped:
            # one host synchronisation for every view's pair count
            host_totals = totals.cpu()
            rc = nat.query("gs_check_status", st)
            if rc:
                raise nat.NativeError("gs_check_status", rc, nat.lib().gs_last_cuda_error())
            self.last_totals = [int(x) for x in host_totals]
            if self._capacity_form:
                self._grow_capacity(V, self.last_totals)
                capped = True
            elif self.layout == "batched":
                self._layout_views(views, self.last_totals)
        self._fork()
        for v, s in enumerate(views):
            s["stream"] = self._view_stream(v)
            with torch.cuda.stream(s["stream"]):
                vst = nat.stream_ptr(dev)
                if capped:
                    # capacity form: the pair count stays on the device (no
                    # host synchronisation); the lists' end is offsets[T]
                    k = v % self.num_streams
                    cap, _, bufs = self._cap
                    s["ids"], s["offsets"] = bufs["ids"][v], bufs["offsets"][v]
                    s["reach"], s["order"] = bufs["reach"][v], bufs["order"][v]
                    s["total_dev"] = bufs["totals"][v:v + 1]
                    scratch = bufs["scratch"][k]
                    # the binned layout writes the blend order in the same launch
                    # as its offsets; after the two-sort layout gs_tile_order does
                    fused_order = self._capacity_entry == "gs_tile_bins"
                    extra = (s["order"].data_ptr(),) if fused_order else ()
                    nat.call(self._capacity_entry, n, s["points"].data_ptr(),
                             s["radii"].data_ptr(), s["depths"].data_ptr(),
                             s["counts"].data_ptr(), cap, W, H, s["ids"].data_ptr(),
                             s["offsets"].data_ptr(), s["total_dev"].data_ptr(),
                             scratch.data_ptr(), scratch.numel(), *extra, vst)
                    s["total"] = -1
                else:
                    total = self.last_totals[v]
                    s["total"] = total
                    if self.layout != "batched":
                        s["offsets"], s["ids"] = cuda_rasterizer.tile_layout_from_counts(
                            s["points"], s["radii"], s["depths"], s["counts"], total, W, H)
                    s["reach"] = torch.empty((max(total, 1),), device=dev, dtype=torch.uint8)
                    s["order"] = torch.empty((T,), device=dev, dtype=torch.int32)
                    fused_order = False
                if not fused_order:
                    # the tiles in blend order, longest lists first (both passes)
                    nat.call("gs_tile_order", T, s["offsets"].data_ptr(), s["total"],
                             s["order"].data_ptr(), vst)
                s["image"] = torch.empty((H, W, 3), **f)
                s["final_t"] = torch.empty((H * W,), **f)
                s["pixel_end"] = torch.empty((H * W,), device=dev, dtype=torch.int32)
                nat.call("gs_blend_forward", T, s["offsets"].data_ptr(), s["total"],
                         s["ids"].data_ptr(), n, s["points"].data_ptr(), s["splat"].data_ptr(),
                         W, H, o["alpha_threshold"], o["transmittance_threshold"],
                         o["chi_squared_threshold"], s["image"].data_ptr(),
                         s["final_t"].data_ptr(), s["pixel_end"].data_ptr(),
                         s["reach"].data_ptr(), s["order"].data_ptr(), vst)
        self._join()
        return views

    def render_views(self, world_to_cameras, intrinsics):
        """Forward-only rendering (inference): forward_views followed by one
        read of the status word; a view whose pair count exceeded the layout
        capacity is rendered again with grown buffers, any other error is
        raised. Returns the per-view state list (state["image"] is the raw
        blended image)."""
        for _ in range(3):
            views = self.forward_views(world_to_cameras, intrinsics)
            rc = nat.query("gs_check_status", nat.stream_ptr(self.device))
            if rc == nat.GS_OK:
                return views
            if rc != nat.GS_ERR_CAPACITY or not self._capacity_form:
                raise nat.NativeError("gs_check_status", rc, nat.lib().gs_last_cuda_error())
            self.last_totals = [int(x) for x in self._batch["totals"].cpu()]
            self._grow_capacity(len(views), self.last_totals)
        raise nat.NativeError("gs_check_status", nat.GS_ERR_CAPACITY)

    def _grow_capacity(self, V, totals):
        """Pair buffers of the capacity form for V views of the current n:
        every view's list capacity is the largest pair count seen, plus
        headroom for the counts to drift between steps (25% + 64 Ki pairs,
        rounded up to 64 Ki). Buffers are kept across steps and rebuilt only
        when V, n or the needed capacity change."""
        dev = self.device
        n, T = self.n, self.tx * self.ty
        need = max(list(totals) + [0])
        cap = (int(need * 1.25) + 2 * 65536) // 65536 * 65536
        old = self._cap
        if old is not None and old[1] == (V, n) and old[0] >= need:
            return
        if self.layout == "auto":
            binned = need <= self.AUTO_BIN_PAIRS_PER_TILE * T
            self._capacity_entry = "gs_tile_bins" if binned else "gs_tile_layout_capped"
        query = ("gs_tile_bins_scratch_bytes" if self._capacity_entry == "gs_tile_bins"
                 else "gs_tile_layout_scratch_bytes")
        nbytes = int(nat.query(query, n, cap, self.width, self.height))
        bufs = dict(
            ids=[torch.empty((cap,), device=dev, dtype=torch.int32) for _ in range(V)],
            # per list entry: the reach mask the forward blend keeps for the backward
            reach=[torch.empty((cap,), device=dev, dtype=torch.uint8) for _ in range(V)],
            order=[torch.empty((T,), device=dev, dtype=torch.int32) for _ in range(V)],
            offsets=[torch.empty((T + 1,), device=dev, dtype=torch.int32) for _ in range(V)],
            totals=torch.zeros((V,), device=dev, dtype=torch.int64),
            scratch=[torch.empty((max(nbytes, 1),), device=dev, dtype=torch.uint8)
                     for _ in range(self.num_streams)])
        self._cap = (cap, (V, n), bufs)

    def _layout_views(self, views, totals):
        """Every view's tile layout in one launch on the current stream: the
        views' sorted id lists concatenated in one buffer, their per-tile
        offsets (view-local) in one (views, tiles) array."""
        import ctypes

        dev = self.device
        b = self._batch
        V, n = len(views), self.n
        tot_c = (ctypes.c_int64 * V)(*totals)
        ktot = sum(totals)
        ids = torch.empty((max(ktot, 1),), device=dev, dtype=torch.int32)
        offsets = torch.empty((V, self.tx * self.ty), device=dev, dtype=torch.int32)
        nbytes = int(nat.query("gs_tile_layout_views_scratch_bytes", n, V,
                               ctypes.cast(tot_c, ctypes.c_void_p), self.width, self.height))
        if nbytes == 0 and ktot > 0:
            raise nat.NativeError("gs_tile_layout_views_scratch_bytes", nat.GS_ERR_CAPACITY)
        scratch = torch.empty((max(nbytes, 1),), device=dev, dtype=torch.uint8)
        nat.call("gs_tile_layout_views", n, V, b["points"].data_ptr(), b["radii"].data_ptr(),
                 b["depths"].data_ptr(), b["counts"].data_ptr(),
                 ctypes.cast(tot_c, ctypes.c_void_p), self.width, self.height, ids.data_ptr(),
                 offsets.data_ptr(), scratch.data_ptr(), nbytes, nat.stream_ptr(dev))
        start = 0
        for v, s in enumerate(views):
            s["offsets"] = offsets[v]
            s["ids"] = ids[start:start + totals[v]]
            start += totals[v]

    def _stage_targets(self, targets):
        """Targets held in host memory (pinned, for the copy to be
        asynchronous) are copied to the device on a copy stream, so the copy
        overlaps the forward pass; returns the device targets and the event
        the copies complete on (None when they were already on the device)."""
        if all(t.device == self.device for t in targets):
            return list(targets), None
        if not hasattr(self, "_copy_stream"):
            self._copy_stream = torch.cuda.Stream(device=self.device)
        with torch.cuda.stream(self._copy_stream):
            dev = [t.to(self.device, non_blocking=True) for t in targets]
        return dev, self._copy_stream.record_event()

    # Gaussians per range of the backward overlapped with Adam (a multiple
    # of the preprocess kernels' 128-Gaussian chunk)
    ADAM_OVERLAP_RANGES = 4

    def overlap_adam(self):
        """Adam runs range by range behind the preprocess backward: opted in
        with adam_overlap (measured 1% slower than one Adam launch after the
        backward at config 1 -- the split backward launches are smaller and
        Adam takes SMs from them), one GPU (the one-launch Adam, not the
        data-parallel step) and enough Gaussians to split."""
        return (self.adam_overlap and self.fp.world == 1 and not self.fp.fused
                and self.fp.device.type == "cuda"
                and self.n >= 4 * 128 * self.ADAM_OVERLAP_RANGES)

    def _backward_with_adam(self, n, V, pargs, adam):
        """The multi-view preprocess backward in ADAM_OVERLAP_RANGES ranges of
        Gaussians on the current stream, each range's Adam update (its slices
        of the six groups, gs_adam_step_ranges) on a second stream as soon
        as its gradient is complete -- so Adam (HBM-bound) overlaps the
        backward of the next range (latency-bound). adam = "eager" uploads
        the group table of the coming step first and counts the step;
        "graph" leaves both to the caller of the graph replay."""
        dev = self.device
        fp = self.fp
        if adam == "eager":
            fp.prepare_table()
            fp.upload_table(fp.step_count + 1)
            fp.step_count += 1
        if not hasattr(self, "_adam_stream"):
            self._adam_stream = torch.cuda.Stream(device=dev)
        cur = torch.cuda.current_stream(dev)
        R = self.ADAM_OVERLAP_RANGES
        per = -(-n // R)
        per = -(-per // 128) * 128
        bounds = [min(n, i * per) for i in range(R + 1)]
        for i in range(R):
            lo, hi = bounds[i], bounds[i + 1]
            if hi <= lo:
                continue
            nat.call("gs_preprocess_backward_views_range", n, lo, hi - lo, V, *pargs,
                     nat.stream_ptr(dev))
            self._adam_stream.wait_event(cur.record_event())
            with torch.cuda.stream(self._adam_stream):
                fp.range_adam_step(fp.gaussian_ranges(lo, hi))
        cur.wait_event(self._adam_stream.record_event())

    def loss_and_backward(self, views, targets, accumulate=False, targets_ready=None,
                          adam=None):
        """Loss of every view against its target (H, W, 3; float in [0, 255]
        or uint8) -- L1, or (1 - ssim_lambda) L1 + ssim_lambda (1 - SSIM)
        when ssim_lambda > 0 -- and the backward into the flat gradient buffer.
        The views' gradients are summed by one multi-view preprocess backward
        and overwrite the buffer (every element is written, zeros for
        Gaussians every view culled) unless `accumulate`, which adds them.
        With adam ("eager" or "graph", see _backward_with_adam) the Adam
        step runs range by range behind the backward. Returns the per-view
        losses (device tensor)."""
        o = self.opts
        dev = self.device
        st = nat.stream_ptr(dev)
        n, W, H = self.n, self.width, self.height
        npx = H * W * 3
        V = len(views)
        lam = self.ssim_lambda
        loss_sums = torch.zeros((V, 2), dtype=torch.float64, device=dev)
        grad_imgs = [torch.empty((H, W, 3), device=dev, dtype=torch.float32)
                     for _ in range(min(V, self.num_streams))]
        if lam > 0:
            for k in range(len(grad_imgs)):
                if self._ssim_scratch[k] is None:
                    self._ssim_scratch[k] = torch.empty(
                        nat.query("gs_ssim_scratch_bytes", 3, H, W) // 4, device=dev,
                        dtype=torch.float32)
        # every view's blend gradients, consumed by one multi-view preprocess backward
        g_points_all = torch.zeros((V, n, 2), device=dev, dtype=torch.float32)
        g_splat_all = torch.zeros((V, n, 8), device=dev, dtype=torch.float32)
        self._fork()
        for v, s in enumerate(views):
            k = v % self.num_streams
            vs = self._view_stream(v)
            if targets_ready is not None:  # targets copied on another stream
                vs.wait_event(targets_ready)
                targets[v].record_stream(vs)
            with torch.cuda.stream(vs):
                self._view_backward(s, targets[v], grad_imgs[k], self._ssim_scratch[k],
                                    loss_sums[v], g_points_all[v], g_splat_all[v])
        self._join()
        st = nat.stream_ptr(dev)
        if self.strategy is not None:  # strategy.py:48-72, per view
            for v, s in enumerate(views):
                self.strategy.accumulate(g_points_all[v], s["radii"], W, H)
        b = self._batch
        if V != b["mask"].shape[0]:
            raise ValueError("loss_and_backward takes the views of the last forward_views call")
        pargs = (self._ptr("means"), self._ptr("scales"), self._ptr("quaternions"),
                 self._ptr("opacities"), self._ptr("sh_coeffs_dc"), self._ptr("sh_coeffs_rest"),
                 b["w2c"].data_ptr(), b["K"].data_ptr(), b["campos"].data_ptr(), W, H, 0, 1,
                 int(accumulate), b["mask"].data_ptr(), g_points_all.data_ptr(), 2,
                 g_splat_all.data_ptr(), 8, self._gptr("means"), self._gptr("scales"),
                 self._gptr("quaternions"), self._gptr("opacities"), self._gptr("sh_coeffs_dc"),
                 self._gptr("sh_coeffs_rest"))
        if adam is None:
            nat.call("gs_preprocess_backward_views", n, V, *pargs, st)
        else:
            self._backward_with_adam(n, V, pargs, adam)
        l1 = loss_sums[:, 0] / npx
        if lam == 0:
            return l1
        ssim = loss_sums[:, 1] / (3 * (H - 10) * (W - 10))
        return (1 - lam) * l1 + lam * (1 - ssim)

    def _view_backward(self, s, tgt, grad_img, ssim_scratch, loss_slot, g_points, g_splat):
        """One view's loss, its gradient w.r.t. the raw image and the blend
        backward into g_points / g_splat, on the current stream."""
        o = self.opts
        dev = self.device
        st = nat.stream_ptr(dev)
        n, W, H = self.n, self.width, self.height
        if tgt.device != dev or not tgt.is_contiguous():
            tgt = tgt.to(dev).contiguous()
        if tgt.dtype not in (torch.uint8, torch.float32):
            tgt = tgt.float()
        if self.ssim_lambda > 0:
            nat.call("gs_l1_ssim_loss_grad", H, W, s["image"].data_ptr(), tgt.data_ptr(),
                     int(tgt.dtype == torch.uint8), self.ssim_lambda, grad_img.data_ptr(),
                     loss_slot.data_ptr(), ssim_scratch.data_ptr(), ssim_scratch.numel() * 4,
                     st)
        else:
            nat.call("gs_l1_loss_grad", H * W * 3, s["image"].data_ptr(), tgt.data_ptr(),
                     int(tgt.dtype == torch.uint8), grad_img.data_ptr(), loss_slot.data_ptr(),
                     st)
        nat.call("gs_blend_backward", self.tx * self.ty, s["offsets"].data_ptr(),
                 s["total"], s["ids"].data_ptr(), n, s["points"].data_ptr(),
                 s["splat"].data_ptr(), grad_img.data_ptr(), s["final_t"].data_ptr(),
                 s["pixel_end"].data_ptr(), W, H, o["alpha_threshold"],
                 o["transmittance_threshold"], o["chi_squared_threshold"], g_points.data_ptr(),
                 g_splat.data_ptr(), s["reach"].data_ptr(), s["order"].data_ptr(), st)

    def check_status(self):
        """Synchronise the device and raise NativeError if a kernel of this
        library recorded an error since the last check (the status word is
        then cleared)."""
        rc = nat.query("gs_check_status", nat.stream_ptr(self.device))
        if rc:
            raise nat.NativeError("gs_check_status", rc, nat.lib().gs_last_cuda_error())

    def step(self, world_to_cameras, intrinsics, targets, optimizer_step=True, step_index=None,
             check_status=True):
        """One training step over this rank's views: render, loss, backward
        (the first view overwrites the flat gradient, so no zeroing is needed
        between steps), then the gradient sum over the ranks and Adam
        (FlatParams.step: NCCL all-reduce + one-launch Adam, or with
        fused_dp the one-kernel reduce-scatter / sharded Adam / all-gather).
        The optimizer kernels skip their update when the device status word
        holds an error from this step (a bounded wait that gave up, or a pair
        count beyond the layout's capacity, on any rank), so a failed step
        leaves the parameters unchanged. With check_status the word is read
        once after the optimizer (one synchronisation): a capacity error
        grows the pair buffers and repeats the step (on every rank), any
        other error is raised in the same step. Without check_status the step
        queues with no synchronisation at all and an error surfaces at the
        next check (check_status(), or a later step's), the updates of the
        steps in between skipped. With a strategy and step_index, the
        densification schedule of scripts/train.py:224-227 runs after the
        optimizer step (it may change the number of Gaussians). Targets in
        host memory are copied while the views are rendered. Returns the
        losses."""
        targets, ready = self._stage_targets(targets)
        overlap = optimizer_step and self.overlap_adam()
        for attempt in range(3):
            views = self.forward_views(world_to_cameras, intrinsics)
            losses = self.loss_and_backward(views, targets, targets_ready=ready,
                                            adam="eager" if overlap else None)
            if optimizer_step and not overlap:
                self.fp.step()
            if not check_status:
                break
            rc = nat.query("gs_check_status", nat.stream_ptr(self.device))
            if not self._repeat_for_capacity(rc, len(views)):
                break
            if optimizer_step:  # the skipped update does not count as an Adam step
                self.fp.step_count -= 1
        if optimizer_step and self.strategy is not None and step_index is not None:
            self.strategy.adjust(self.fp, int(step_index))
        return losses

    # ---- the step replayed from CUDA graphs ----------------------------------

    def graph_capable(self):
        """Steps can be replayed from CUDA graphs: one GPU (world 1, the
        one-launch Adam), a capacity-form layout, no densification."""
        return self.fp.world == 1 and self._capacity_form and self.strategy is None

    def step_graph(self, world_to_cameras, intrinsics, targets, check_status=False):
        """One training step (the same as step()) replayed from two CUDA
        graphs captured on first use: the forward of every view, then the
        loss, the backward and Adam. Per call the host only copies the
        inputs into the graphs' static buffers -- cameras on the current
        stream, targets on a copy stream that overlaps the forward replay --
        uploads Adam's group table for the coming step, and launches the two
        graphs, so the GPU is not left waiting on Python between steps. The
        first call on a new shape runs an ordinary step(), which sizes the
        layout buffers and Adam's state; a pair count beyond the capacity
        (seen with check_status) grows the buffers, re-captures and repeats
        the step. Falls back to step() when graph_capable() is False.
        Inputs may be device tensors or host tensors; host inputs in pinned
        memory keep the call asynchronous (a pageable one is copied through
        a staging buffer, which can block the host until the copy stream's
        earlier work is done). Returns the per-view losses (a static device
        tensor, overwritten by the next call)."""
        if not self.graph_capable():
            return self.step(world_to_cameras, intrinsics, targets, check_status=check_status)
        w2c = world_to_cameras.to(torch.float32)
        V = w2c.shape[0]
        K1 = intrinsics.to(torch.float32)
        Ks = K1.unsqueeze(0).expand(V, 3, 3) if K1.dim() == 2 else K1
        key = (V, self.n, tuple(t.dtype for t in targets), tuple(targets[0].shape))
        g = getattr(self, "_graph", None)
        if g is None or g["key"] != key or g["cap"] != (self._cap[0] if self._cap else None):
            self._graph = None
            if self._cap is None or self._cap[1] != (V, self.n) or self.fp.exp_avg is None:
                return self.step(world_to_cameras, intrinsics, targets, check_status=True)
            self._capture(w2c, Ks, targets, key)
            g = self._graph
        if not hasattr(self, "_copy_stream"):
            self._copy_stream = torch.cuda.Stream(device=self.device)
        cs = self._copy_stream
        cur = torch.cuda.current_stream(self.device)
        # Inputs on the copy stream, once the previous replay has read them:
        # the cameras first -- the forward waits for them alone -- then the
        # targets and Adam's table for the coming step, overlapping the
        # forward. (Queued behind the large target copy on the same copy
        # engine, a small camera copy on the compute stream would hold the
        # forward back for the whole transfer.)
        if g.get("bwd_done") is not None:
            cs.wait_event(g["bwd_done"])
        with torch.cuda.stream(cs):
            g["w2c"].copy_(w2c, non_blocking=True)
            if K1.dim() == 2 and not K1.is_cuda:
                # one intrinsic for every view: the 3x3 goes to the device and
                # is broadcast there (a broadcast host tensor would be copied
                # through pageable memory, which blocks the host until the
                # copy stream's earlier work -- the previous step -- is done)
                g["K"].copy_(K1.to(self.device, non_blocking=True).expand(V, 3, 3))
            else:
                g["K"].copy_(Ks, non_blocking=True)
            cams_ready = cs.record_event()
        cur.wait_event(cams_ready)
        g["fwd"].replay()  # queued before the rest of the host work of the step
        with torch.cuda.stream(cs):
            for src, dst in zip(targets, g["targets"]):
                dst.copy_(src, non_blocking=True)
            self.fp.upload_table(self.fp.step_count + 1)
            inputs_ready = cs.record_event()
        cur.wait_event(inputs_ready)
        g["bwd"].replay()
        g["bwd_done"] = cur.record_event()
        nat.lib().gs_note_launches(g["kernels"])
        self.fp.step_count += 1
        if check_status:
            rc = nat.query("gs_check_status", nat.stream_ptr(self.device))
            if self._repeat_for_capacity(rc, V):
                # the step overflowed the layout buffers and skipped its
                # update: the grown buffers redo it in one ordinary step, the
                # next call captures again
                self.fp.step_count -= 1
                self._graph = None
                return self.step(world_to_cameras, intrinsics, targets, check_status=True)
        return g["losses"]

    def _capture(self, w2c, Ks, targets, key):
        """Captures the forward graph and the loss / backward / Adam graph
        over static input buffers (sharing one memory pool, so the views the
        forward leaves behind stay valid for the backward)."""
        dev = self.device
        self.fp.prepare_table()
        g = {"key": key, "cap": self._cap[0],
             "w2c": torch.empty(w2c.shape, device=dev, dtype=torch.float32),
             "K": torch.empty(Ks.shape, device=dev, dtype=torch.float32),
             "targets": [torch.empty(t.shape, device=dev, dtype=t.dtype) for t in targets]}
        g["w2c"].copy_(w2c)
        g["K"].copy_(Ks)
        for src, dst in zip(targets, g["targets"]):
            dst.copy_(src)
        self.fp.upload_table(self.fp.step_count + 1)
        torch.cuda.synchronize(dev)
        fwd, bwd = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        n0 = nat.launch_count()
        with torch.cuda.graph(fwd):
            views = self.forward_views(g["w2c"], g["K"])
        with torch.cuda.graph(bwd, pool=fwd.pool()):
            if self.overlap_adam():
                g["losses"] = self.loss_and_backward(views, g["targets"], adam="graph")
            else:
                g["losses"] = self.loss_and_backward(views, g["targets"])
                self.fp.table_adam_step()
        # launches recorded into the graphs, counted again at every replay
        g["kernels"] = nat.launch_count() - n0
        nat.lib().gs_note_launches(-g["kernels"])
        g["views"], g["fwd"], g["bwd"] = views, fwd, bwd
        torch.cuda.synchronize(dev)
        self._graph = g

    def _repeat_for_capacity(self, rc, V):
        """After a step's status read: True when the step must be repeated
        because a view's pair count exceeded the layout capacity on this or
        (world > 1) any rank -- the buffers are then grown to the counts of
        the failed step; raises for any other error; False when the step
        succeeded everywhere."""
        cap_err = rc == nat.GS_ERR_CAPACITY
        other = rc not in (nat.GS_OK, nat.GS_ERR_CAPACITY, nat.GS_ERR_PEER)
        if self.fp.world > 1:
            import torch.distributed as dist

            flags = torch.tensor([int(cap_err), int(other), int(rc != nat.GS_OK)],
                                 dtype=torch.int32, device=self.device)
            dist.all_reduce(flags, op=dist.ReduceOp.MAX, group=self.fp.group)
            any_cap, any_other, any_err = (int(x) for x in flags.cpu())
        else:
            any_cap, any_other, any_err = int(cap_err), int(other), int(rc != nat.GS_OK)
        if not any_err:
            return False
        if any_other or not any_cap:
            raise nat.NativeError("gs_check_status", rc or nat.GS_ERR_PEER,
                                  nat.lib().gs_last_cuda_error())
        if self._capacity_form:
            self.last_totals = [int(x) for x in self._batch["totals"].cpu()]
            self._grow_capacity(V, self.last_totals)
        return True
