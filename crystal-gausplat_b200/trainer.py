"""View-sharded data-parallel training step (Trainer#train_step,
src/gaussian_splatting/trainer.cr:178-215, batched over views).

One process per GPU. Every rank holds a full replica of the Gaussians and
renders + backpropagates its own slice of the view batch, accumulating fp32
gradients in one flat arena; one all-reduce (NCCL over NVLink) sums the
arena, and the fused Adam kernel applies the view mean (grad_scale = 1/views).
The order is grads -> all-reduce -> Adam -> zero (the reference zeroes the
gradients BEFORE its optimiser step, trainer.cr:202-203, so it never updates).
"""
import ctypes as C

import torch

from . import _abi
from ._abi import check, lib
from .gaussian import FIELDS
from .loss import combined_with_grad
from .optim import Adam
from .rasterizer import Rasterizer, RasterizerContext, RasterizerGradients, context


def shard(n_items, rank, world):
    """Contiguous slice of [0, n_items) owned by `rank`."""
    lo = (n_items * rank) // world
    hi = (n_items * (rank + 1)) // world
    return lo, hi


def _symmetric_copy(t, group):
    """t copied into torch symmetric memory (peer-addressable over NVLink)."""
    import torch.distributed._symmetric_memory as symm_mem
    s = symm_mem.empty(t.numel(), dtype=t.dtype, device=t.device)
    s.copy_(t)
    hdl = symm_mem.rendezvous(s, group.group_name)
    return s, hdl


def _peer_ptrs(t, hdl):
    base = hdl.buffer_ptrs[hdl.rank]
    off = t.data_ptr() - base
    return [p + off for p in hdl.buffer_ptrs]


# smallest world size at which multicast="auto" uses the NVSwitch multicast form
MULTICAST_MIN_RANKS = 4


def _multicast_ptr(t, hdl):
    """NVLink multicast address of tensor t inside a symmetric-memory
    buffer, or 0 when the buffer has no multicast object."""
    try:
        mc = int(hdl.multicast_ptr)
    except (AttributeError, RuntimeError, TypeError):
        return 0
    if not mc:
        return 0
    return mc + (t.data_ptr() - hdl.buffer_ptrs[hdl.rank])


class DataParallelTrainer:
    """exchange="nccl": all-reduce of the gradient arena, then Adam on every
    replica. exchange="fused": gsc_dp_adam_step -- each rank sums its shard of
    the peers' gradients over NVLink, applies Adam once and stores the new
    parameters into every replica (arenas in torch symmetric memory);
    multicast=True does the sum and the stores through the NVSwitch's
    multicast object where the box has one (exchange_path "multimem", else
    "peer"). Per NVLink direction the multicast form moves (1 + 1/P) arenas
    and the peer form 2 (P - 1)/P: multicast="auto" takes the multicast form
    from P = MULTICAST_MIN_RANKS ranks on (at P = 2 it measured 1.85 against
    1.05 ms per 3M-Gaussian exchange).

    loss="l1": the L1 gradient fused into the backward compositing (the
    benchmark configurations). loss="combined": Trainer#train_step's
    (1 - lambda_ssim) L1 + lambda_ssim (1 - SSIM) (trainer.cr:190), computed on
    the rendered image by gsc_combined_loss_grad and fed back as dL/dimage."""

    def __init__(self, gaussians, cameras, config, lrs=None, process_group=None, exchange="nccl",
                 loss="l1", lambda_ssim=0.2, batch_views=_abi.GSC_MAX_BATCH_VIEWS,
                 barrier_timeout_s=60.0, multicast="auto", tile_hints=True):
        self.g = gaussians
        self.cameras = cameras
        self.cfg = config
        self.pg = process_group
        self.world = torch.distributed.get_world_size(process_group) if process_group is not None else 1
        self.rank = torch.distributed.get_rank(process_group) if process_group is not None else 0
        self.lo, self.hi = shard(len(cameras), self.rank, self.world)
        self.exchange = exchange if self.world > 1 else "nccl"
        grad_arena = None
        if self.exchange == "fused":
            arena, self.hdl_params = _symmetric_copy(gaussians.arena, process_group)
            gaussians.rebind_arena(arena)
            grad_arena, self.hdl_grads = _symmetric_copy(torch.zeros_like(arena), process_group)
        self.grads = RasterizerGradients(gaussians, arena=grad_arena, screen=False)
        self.opt = Adam.for_gaussians(gaussians, self.grads, lrs)
        self.barrier_timeout_s = barrier_timeout_s
        self.multicast = multicast
        self.exchange_path = None
        if self.exchange == "fused":
            self._setup_fused()
        # batch_views > 1: compositing backward per view, then one preprocess
        # backward per batch_views views (gsc_rasterize_backward_batch)
        self.batch = max(1, min(int(batch_views), _abi.GSC_MAX_BATCH_VIEWS))
        self.ctxs = [RasterizerContext(gaussians.arena.device) for _ in range(self.batch)]
        self.ctx = self.last_ctx = self.ctxs[0]
        self._pending = []
        self._slot = {}  # view -> context of the current forward batch
        if self.batch > 1:
            H, W = cameras[0].height, cameras[0].width
            self.images = [torch.empty(H, W, 3, device=gaussians.arena.device) for _ in range(self.batch)]
        self.loss = torch.zeros(1, device=gaussians.arena.device)
        self.cam_structs = [c.to_struct() for c in cameras]
        # occluded binning: one per-tile depth cut per view of this rank, made
        # by the view's forward and read by its next one (gsc_frame_set_tile_hint)
        self.tile_hints = {}
        if tile_hints and self.batch > 1 and config.binning == _abi.GSC_BIN_OCCLUDED:
            for v in self.my_views:
                c = cameras[v]
                T = ((c.width + 15) // 16) * ((c.height + 15) // 16)
                self.tile_hints[v] = [torch.empty(T, dtype=torch.float32, device=gaussians.arena.device), False]
        if loss not in ("l1", "combined"):
            raise ValueError(f"unknown loss {loss!r}")
        self.loss_kind, self.lambda_ssim = loss, lambda_ssim
        if loss == "combined":
            dev = gaussians.arena.device
            H, W = cameras[0].height, cameras[0].width
            self.image = torch.empty(H, W, 3, device=dev)
            self.dimage = torch.empty(H, W, 3, device=dev)
            self.loss_terms = torch.zeros(3, device=dev)

    @property
    def my_views(self):
        return range(self.lo, self.hi)

    def zero(self):
        ctx = context(self.g.arena.device)
        check(lib().gsc_memset(ctx, C.c_void_p(self.grads.arena.data_ptr()), 0,
                               self.grads.arena.numel() * 4), "gsc_memset")
        check(lib().gsc_memset(ctx, C.c_void_p(self.loss.data_ptr()), 0, 4), "gsc_memset")

    def view_fwd_bwd(self, v, target, ready=None):
        """Forward + backward of view v against a device target [H,W,3]; with
        `ready` (a CUDA event), the target is only waited for right before the
        backward that reads it (the forward does not need it)."""
        cam = self.cameras[v]
        defer = self.batch > 1
        if defer:
            # forward of the next views of this rank as one batch, then one
            # deferred backward per view, then one preprocess backward
            if v not in self._slot:
                self.flush()
                views = list(range(v, min(v + self.batch, max(self.hi, v + 1))))
                self._slot = {u: k for k, u in enumerate(views)}
                for k, u in enumerate(views):
                    if u in self.tile_hints:
                        self.ctxs[k].set_tile_hint(*self.tile_hints[u])
                        self.tile_hints[u][1] = True  # this forward writes it
                    elif self.tile_hints:
                        self.ctxs[k].set_tile_hint(None, False)
                Rasterizer.forward_batch(self.g, [self.cameras[u] for u in views], self.ctxs,
                                         config=self.cfg, images=self.images[:len(views)])
            k = self._slot[v]
            ctx = self.last_ctx = self.ctxs[k]
            image = self.images[k]
        else:
            ctx = self.last_ctx = self.ctxs[0]
            image = self.image if self.loss_kind == "combined" else None
            Rasterizer.forward(self.g, cam, context=ctx, config=self.cfg, out=image)
        if ready is not None:
            torch.cuda.current_stream(self.g.arena.device).wait_event(ready)
        if self.loss_kind == "combined":
            combined_with_grad(image, target, self.lambda_ssim, out=self.loss_terms, grad=self.dimage)
            self.loss += self.loss_terms[0]
            Rasterizer.backward(self.dimage, self.g, cam, ctx, grads=self.grads, config=self.cfg,
                                defer=defer)
        else:
            Rasterizer.backward(None, self.g, cam, ctx, grads=self.grads, target=target,
                                l1_scale=1.0 / target.numel(), loss_sum=self.loss, config=self.cfg,
                                defer=defer)
        if defer:
            self._pending.append(v)
            if len(self._pending) == len(self._slot):
                self.flush()

    def flush(self):
        """Preprocess backward of the views whose compositing backward is done."""
        if not self._pending:
            self._slot = {}
            return
        Rasterizer.backward_batch([self.ctxs[self._slot[v]] for v in self._pending], self.g,
                                  [self.cameras[v] for v in self._pending], self.grads, config=self.cfg)
        self._pending = []
        self._slot = {}

    def _setup_fused(self):
        g = self.g
        self.m = torch.zeros_like(g.arena)
        self.v = torch.zeros_like(g.arena)
        a = _abi.DpAdamArgs()
        a.nranks, a.rank = self.world, self.rank
        for p, (pg, pp) in enumerate(zip(_peer_ptrs(self.grads.arena, self.hdl_grads),
                                         _peer_ptrs(g.arena, self.hdl_params))):
            a.peer_grads[p] = pg
            a.peer_params[p] = pp
        a.m, a.v = self.m.data_ptr(), self.v.data_ptr()
        a.ngroups = len(FIELDS)
        for i, (name, w) in enumerate(FIELDS):
            a.offset[i] = g.offsets[name]
            a.numel[i] = g.count * w
            a.lr[i] = self.opt.groups[i]["lr"]
            a.weight_decay[i] = self.opt.groups[i]["weight_decay"]
        a.beta1, a.beta2, a.eps = self.opt.beta1, self.opt.beta2, self.opt.eps
        a.grad_scale = 1.0 / len(self.cameras)
        # NVSwitch multicast (multimem loads with in-switch sums, multimem
        # stores into every replica) where the arenas are bound to a multicast
        # object; otherwise plain peer loads and stores
        use_mc = self.world >= MULTICAST_MIN_RANKS if self.multicast == "auto" else bool(self.multicast)
        mc_g = _multicast_ptr(self.grads.arena, self.hdl_grads) if use_mc else 0
        mc_p = _multicast_ptr(g.arena, self.hdl_params) if use_mc else 0
        if mc_g and mc_p:
            a.mc_grads, a.mc_params = mc_g, mc_p
            self.exchange_path = "multimem"
        else:
            self.exchange_path = "peer"
        self.dp_args = a
        # bounded cross-rank barrier (gsc_dp_barrier) over one flag word per
        # rank in symmetric memory; every barrier call uses the next epoch
        self.flags, self.hdl_flags = _symmetric_copy(
            torch.zeros(self.world, dtype=torch.int32, device=g.arena.device), self.pg)
        b = _abi.DpBarrierArgs()
        b.nranks, b.rank = self.world, self.rank
        for p, fp in enumerate(_peer_ptrs(self.flags, self.hdl_flags)):
            b.peer_flags[p] = fp
        b.timeout_us = int(self.barrier_timeout_s * 1e6)
        self.barrier_args = b
        self.epoch = 0
        self.hdl_flags.barrier(channel=0)  # every rank's zeroed flags exist before the first signal

    def _barrier(self):
        self.epoch += 1
        self.barrier_args.epoch = self.epoch
        check(lib().gsc_dp_barrier(context(self.g.arena.device), C.byref(self.barrier_args)),
              "gsc_dp_barrier")

    def check(self):
        """Wait for the queued work and raise GscError if a cross-rank wait
        gave up (a peer that never arrived) or a device check failed."""
        check(lib().gsc_sync(context(self.g.arena.device)), "gsc_sync")

    def reduce_and_step(self):
        self.flush()
        if self.exchange == "fused":
            torch.distributed.all_reduce(self.loss, group=self.pg)
            self.opt.step_count += 1
            self.dp_args.step = self.opt.step_count
            self._barrier()  # every rank's gradients are complete
            check(lib().gsc_dp_adam_step(context(self.g.arena.device), C.byref(self.dp_args)),
                  "gsc_dp_adam_step")
            self._barrier()  # every shard's parameters have landed
            return
        if self.world > 1:
            torch.distributed.all_reduce(self.grads.arena, group=self.pg)
            torch.distributed.all_reduce(self.loss, group=self.pg)
        self.opt.step(grad_scale=1.0 / len(self.cameras))

    def step_from_host(self, feeder):
        """One training step with targets streamed from pinned host memory
        (feeder: HostTargetFeeder over this rank's views, indexed from 0)."""
        self.zero()
        feeder.run(range(self.hi - self.lo), lambda k, t, ready: self.view_fwd_bwd(self.lo + k, t, ready))
        self.reduce_and_step()
        return self.loss

    def step(self, targets):
        """One training step over all views; `targets(v)` gives view v's device target."""
        self.zero()
        for v in self.my_views:
            self.view_fwd_bwd(v, targets(v))
        self.reduce_and_step()
        return self.loss


class HostTargetFeeder:
    """Streams per-view targets from pinned host memory to the device on a
    side stream, `depth` views ahead (default: one forward batch), so that the
    copies run under the batched forward and the earlier backwards. `host` is
    a pinned [V, H, W, 3] tensor."""

    def __init__(self, host, device, depth=_abi.GSC_MAX_BATCH_VIEWS):
        self.host = host
        self.copy_stream = torch.cuda.Stream(device=device)
        depth = max(1, min(int(depth), host.shape[0]))
        self.bufs = [torch.empty_like(host[0], device=device) for _ in range(depth)]
        self.ready = [torch.cuda.Event() for _ in range(depth)]
        self.free = [torch.cuda.Event() for _ in range(depth)]
        for e in self.free:
            e.record(torch.cuda.current_stream(device))

    def _issue(self, slot, v):
        with torch.cuda.stream(self.copy_stream):
            self.copy_stream.wait_event(self.free[slot])
            self.bufs[slot].copy_(self.host[v], non_blocking=True)
            self.ready[slot].record(self.copy_stream)

    def run(self, views, fn):
        """Calls fn(v, device_target, ready_event) for each view; fn makes the
        current stream wait for ready_event before it reads the target."""
        views = list(views)
        if not views:
            return
        cur = torch.cuda.current_stream(self.bufs[0].device)
        D = len(self.bufs)
        for k in range(min(D, len(views))):
            self._issue(k, views[k])
        for k, v in enumerate(views):
            slot = k % D
            fn(v, self.bufs[slot], self.ready[slot])
            self.free[slot].record(cur)
            if k + D < len(views):
                self._issue(slot, views[k + D])


# ---- the reference's single-view training loop ------------------------------

class TrainerConfig:
    """TrainerConfig (src/gaussian_splatting/trainer.cr:15-57), same fields and defaults."""

    def __init__(self, iterations=30000, lr_position=0.00016, lr_scale=0.005, lr_rotation=0.001,
                 lr_opacity=0.05, lr_sh=0.0025, lambda_ssim=0.2, densify_from=500, densify_until=15000,
                 densify_interval=100, densify_grad_threshold=0.0002, densify_size_threshold=0.01,
                 prune_interval=100, opacity_threshold=0.005, max_screen_size=20.0,
                 opacity_reset_interval=3000):
        self.iterations = iterations
        self.lr_position, self.lr_scale, self.lr_rotation = lr_position, lr_scale, lr_rotation
        self.lr_opacity, self.lr_sh, self.lambda_ssim = lr_opacity, lr_sh, lambda_ssim
        self.densify_from, self.densify_until = densify_from, densify_until
        self.densify_interval = densify_interval
        self.densify_grad_threshold = densify_grad_threshold
        self.densify_size_threshold = densify_size_threshold
        self.prune_interval, self.opacity_threshold = prune_interval, opacity_threshold
        self.max_screen_size = max_screen_size
        self.opacity_reset_interval = opacity_reset_interval

    def lrs(self):
        return {"position": self.lr_position, "log_scale": self.lr_scale, "rotation": self.lr_rotation,
                "logit_opacity": self.lr_opacity, "sh_coeffs": self.lr_sh}


class TrainStats:
    """TrainStats (trainer.cr:61-74)."""

    def __init__(self, iteration=0, loss=0.0, psnr=0.0, num_gaussians=0, lr=0.0):
        self.iteration, self.loss, self.psnr = iteration, loss, psnr
        self.num_gaussians, self.lr = num_gaussians, lr

    def __str__(self):
        return (f"Iter {self.iteration}: loss={self.loss:.4f}, PSNR={self.psnr:.2f}dB, "
                f"gaussians={self.num_gaussians}")


class Trainer:
    """Trainer (trainer.cr:125-420): one sampled view per step, combined
    L1 + SSIM loss, screen-space gradient accumulation, densification and
    pruning every densify_interval steps in [densify_from, densify_until),
    opacity reset every opacity_reset_interval steps. Every camera carries its
    device target as `camera.image` ([H, W, 3] fp32).

    The order inside a step is gradients -> Adam -> zero (the reference zeroes
    before its optimiser step, trainer.cr:202-203, so it never updates); after
    densification the optimiser state is recreated, as recreate_optimizers!
    (trainer.cr:412-419) does. Camera sampling uses a seeded generator."""

    def __init__(self, gaussians, cameras, config=None, seed=0, raster_config=None):
        import numpy as np

        from .densify import GradientAccumulator
        self.gaussians = gaussians
        self.cameras = cameras
        self.config = config or TrainerConfig()
        self.rcfg = raster_config or _abi.default_config()
        self.rng = np.random.default_rng(seed)
        self.iteration = 0
        self.context = RasterizerContext(gaussians.arena.device)
        self.grad_accum = GradientAccumulator(gaussians.count, device=gaussians.arena.device)
        self._recreate()

    def _recreate(self):
        """recreate_optimizers! (trainer.cr:412-419) and fresh gradient buffers."""
        self.grads = RasterizerGradients(self.gaussians, screen=True)
        self.optimizer = Adam.for_gaussians(self.gaussians, self.grads, self.config.lrs())

    def train(self, callback=None):
        """Trainer#train (trainer.cr:157-180)."""
        c = self.config
        for i in range(c.iterations):
            self.iteration = i
            stats = self.train_step()
            if callback is not None:
                callback(stats)
            if c.densify_from <= i < c.densify_until and i % c.densify_interval == 0:
                self.densify_and_prune()
            if i > 0 and i % c.opacity_reset_interval == 0:
                self.reset_opacity()

    def train_step(self):
        """Trainer#train_step (trainer.cr:183-215)."""
        from .loss import psnr
        cam = self.cameras.sample(self.rng) if hasattr(self.cameras, "sample") else \
            self.cameras[int(self.rng.integers(len(self.cameras)))]
        target = getattr(cam, "image", None)
        if target is None:
            raise ValueError("Camera has no target image")
        rendered, ctx = Rasterizer.forward(self.gaussians, cam, context=self.context, config=self.rcfg)
        loss, grad_image = combined_with_grad(rendered, target, self.config.lambda_ssim)
        self.grads.zero_()
        Rasterizer.backward(grad_image, self.gaussians, cam, ctx, grads=self.grads, config=self.rcfg)
        self.grad_accum.accumulate(self.grads)
        self.optimizer.step()
        return TrainStats(iteration=self.iteration, loss=float(loss), psnr=psnr(rendered, target),
                          num_gaussians=self.gaussians.count, lr=self.config.lr_position)

    def densify_and_prune(self):
        """Trainer#densify_and_prune! (trainer.cr:293-330) on the device."""
        from .densify import densify_and_prune
        c = self.config
        self.gaussians = densify_and_prune(self.gaussians, self.grad_accum, c.densify_grad_threshold,
                                           c.densify_size_threshold, c.opacity_threshold,
                                           seed=self.iteration)
        self._recreate()

    def reset_opacity(self):
        """Trainer#reset_opacity! (trainer.cr:407-410): logit opacity -1."""
        from .densify import reset_opacity
        reset_opacity(self.gaussians, -1.0)
