"""Rasterizer, RasterizerContext and RasterizerGradients over libgsplat_cuda.so,
with the reference's API (src/gaussian_splatting/rasterizer.cr:48-104,
rasterizer_context.cr:10-162), plus GPURadixSort (src/metal/gpu_radix_sort.cr).

Every call goes through the C ABI; work is enqueued on torch's current CUDA
stream of the tensors' device.
"""
import ctypes as C

import torch

from . import _abi
from ._abi import check, lib

_contexts = {}


def context(device=None):
    """The library context of a CUDA device, bound to torch's current stream."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       torch.device(device).index or 0)
    ctx = _contexts.get(dev.index)
    if ctx is None:
        h = C.c_void_p()
        with torch.cuda.device(dev):
            check(lib().gsc_init(dev.index, C.byref(h)), "gsc_init")
        ctx = h
        _contexts[dev.index] = ctx
    stream = torch.cuda.current_stream(dev).cuda_stream
    check(lib().gsc_set_stream(ctx, C.c_void_p(stream)), "gsc_set_stream")
    return ctx


def ptr(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def gaussians_struct(g):
    s = _abi.Gaussians()
    s.position = g.position.data_ptr()
    s.log_scale = g.log_scale.data_ptr()
    s.rotation = g.rotation.data_ptr()
    s.logit_opacity = g.logit_opacity.data_ptr()
    s.sh = g.sh_coeffs.data_ptr()
    s.count = g.count
    return s


class RasterizerGradients:
    """RasterizerGradients (rasterizer_context.cr:133-162) plus the gradients of
    the stored parameters (log_scale, rotation, logit_opacity) that the
    trainer's chain rule produces (trainer.cr:218-255)."""

    def __init__(self, gaussians, arena=None, screen=True):
        n = gaussians.count
        dev = gaussians.arena.device
        self.arena = arena if arena is not None else torch.zeros_like(gaussians.arena)
        v = gaussians.views_of(self.arena)
        self.dL_dposition = v["position"]
        self.dL_dlog_scale = v["log_scale"]
        self.dL_drotation = v["rotation"]
        self.dL_dlogit_opacity = v["logit_opacity"]
        self.dL_dsh = v["sh_coeffs"]
        if screen:
            self.dL_dmean2d = torch.zeros(n, 2, device=dev)
            self.dL_dcov2d = torch.zeros(n, 3, device=dev)
            self.dL_dopacity = torch.zeros(n, device=dev)
            self.dL_dcolors = torch.zeros(n, 3, device=dev)
        else:
            self.dL_dmean2d = self.dL_dcov2d = self.dL_dopacity = self.dL_dcolors = None

    def struct(self):
        s = _abi.GaussianGrads()
        s.position = self.dL_dposition.data_ptr()
        s.log_scale = self.dL_dlog_scale.data_ptr()
        s.rotation = self.dL_drotation.data_ptr()
        s.logit_opacity = self.dL_dlogit_opacity.data_ptr()
        s.sh = self.dL_dsh.data_ptr()
        return s

    def screen_struct(self):
        if self.dL_dmean2d is None:
            return None
        s = _abi.Grads2D()
        s.mean2d = self.dL_dmean2d.data_ptr()
        s.cov2d = self.dL_dcov2d.data_ptr()
        s.opacity = self.dL_dopacity.data_ptr()
        s.colors = self.dL_dcolors.data_ptr()
        return s

    def zero_(self):
        self.arena.zero_()
        for t in (self.dL_dmean2d, self.dL_dcov2d, self.dL_dopacity, self.dL_dcolors):
            if t is not None:
                t.zero_()


class RasterizerContext:
    """Per-view state kept between forward and backward (a gsc_frame)."""

    def __init__(self, device=None):
        self.ctx = context(device)
        h = C.c_void_p()
        check(lib().gsc_frame_create(self.ctx, C.byref(h)), "gsc_frame_create")
        self.frame = h
        self.num_rendered = 0
        self.width = self.height = 0
        self.rendered_image = None
        self.background = (0.0, 0.0, 0.0)

    def __del__(self):
        try:
            if self.frame:
                lib().gsc_frame_destroy(self.frame)
                self.frame = None
        except Exception:
            pass

    def get(self, which, dtype):
        """Host copy (numpy) of a frame-owned device buffer (GSC_FRAME_*)."""
        import numpy as np
        p = C.c_void_p()
        n = C.c_int64()
        check(lib().gsc_frame_get(self.frame, which, C.byref(p), C.byref(n)), "gsc_frame_get")
        out = np.empty(n.value, dtype=dtype)
        if p.value and n.value:
            check(lib().gsc_memcpy_d2h(self.ctx, out.ctypes.data_as(C.c_void_p), p, out.nbytes),
                  "gsc_memcpy_d2h")
        return out

    def set_tile_hint(self, cut, valid):
        """Bind a view's per-tile depth cut (a float32 device tensor of
        tiles_x * tiles_y entries, or None) for the next occluded forwards on
        this context (gsc_frame_set_tile_hint): valid=True reads it, and every
        such forward rewrites it for the view's next one. Results do not
        depend on its contents."""
        if cut is not None:
            assert cut.dtype == torch.float32 and cut.is_cuda and cut.is_contiguous()
        check(lib().gsc_frame_set_tile_hint(self.frame, ptr(cut), cut.numel() if cut is not None else 0,
                                            1 if (cut is not None and valid) else 0), "gsc_frame_set_tile_hint")

    @property
    def tiles_x(self):
        return (self.width + 15) // 16

    @property
    def tiles_y(self):
        return (self.height + 15) // 16


class Rasterizer:
    """Rasterizer.forward / .backward (rasterizer.cr:48-104)."""

    @staticmethod
    def forward(gaussians, camera, context=None, background=(0.0, 0.0, 0.0), config=None,
                out=None, n_contrib=None, final_T=None):
        ctx = context or RasterizerContext(gaussians.arena.device)
        cfg = config or _abi.default_config(background=background)
        if config is not None and background != (0.0, 0.0, 0.0):
            for i in range(3):
                cfg.background[i] = background[i]
        H, W = camera.height, camera.width
        image = out if out is not None else torch.empty(H, W, 3, device=gaussians.arena.device)
        nr = C.c_int64()
        g = gaussians_struct(gaussians)
        cam = camera.to_struct()
        check(lib().gsc_rasterize_forward(ctx.ctx, ctx.frame, C.byref(g), C.byref(cam), C.byref(cfg),
                                          ptr(image), ptr(n_contrib), ptr(final_T), C.byref(nr)),
              "gsc_rasterize_forward")
        ctx.num_rendered = nr.value
        ctx.width, ctx.height = W, H
        ctx.rendered_image = image
        ctx.background = tuple(cfg.background)
        ctx.config = cfg
        return image, ctx

    @staticmethod
    def forward_batch(gaussians, cameras, contexts, config=None, images=None):
        """Rasterizer.forward of up to GSC_MAX_BATCH_VIEWS views of one size, one
        context each, sharing one preprocess pass. Returns the images."""
        k = len(cameras)
        assert len(contexts) >= k
        cfg = config or _abi.default_config()
        H, W = cameras[0].height, cameras[0].width
        dev = gaussians.arena.device
        if images is None:
            images = [torch.empty(H, W, 3, device=dev) for _ in range(k)]
        frames = (C.c_void_p * k)(*[c.frame.value for c in contexts[:k]])
        cams = (_abi.Camera * k)(*[c.to_struct() for c in cameras])
        imgs = (C.c_void_p * k)(*[im.data_ptr() for im in images])
        nr = (C.c_int64 * k)()
        g = gaussians_struct(gaussians)
        check(lib().gsc_rasterize_forward_batch(contexts[0].ctx, frames, cams, k, C.byref(g), C.byref(cfg),
                                                imgs, nr), "gsc_rasterize_forward_batch")
        for c, im, m in zip(contexts, images, nr):
            c.num_rendered = m
            c.width, c.height = W, H
            c.rendered_image = im
            c.background = tuple(cfg.background)
            c.config = cfg
        return images

    @staticmethod
    def backward(dL_dimage, gaussians, camera, context, grads=None, target=None, l1_scale=None,
                 loss_sum=None, config=None, defer=False):
        """Gradients for the last forward on `context`. With `target`, the pixel
        gradient is the fused L1 gradient sign(image - target) * l1_scale
        (default 1/numel, Loss.l1_with_grad) and dL_dimage must be None.
        defer=True stops after the compositing backward (screen-space
        gradients stay in the context) for a later Rasterizer.backward_batch."""
        cfg = config or context.config
        if target is not None and l1_scale is None:
            l1_scale = 1.0 / target.numel()
        g = gaussians_struct(gaussians)
        cam = camera.to_struct()
        if defer:
            check(lib().gsc_rasterize_backward(
                context.ctx, context.frame, C.byref(g), C.byref(cam), C.byref(cfg), ptr(dL_dimage),
                ptr(target), C.c_float(l1_scale or 0.0), ptr(loss_sum), None, None),
                "gsc_rasterize_backward")
            return None
        grads = grads if grads is not None else RasterizerGradients(gaussians)
        gs = grads.struct()
        g2d = grads.screen_struct()
        check(lib().gsc_rasterize_backward(
            context.ctx, context.frame, C.byref(g), C.byref(cam), C.byref(cfg), ptr(dL_dimage),
            ptr(target), C.c_float(l1_scale or 0.0), ptr(loss_sum), C.byref(gs),
            C.byref(g2d) if g2d is not None else None), "gsc_rasterize_backward")
        return grads

    @staticmethod
    def backward_batch(contexts, gaussians, cameras, grads, config=None):
        """Parameter gradients of up to GSC_MAX_BATCH_VIEWS deferred backwards
        (one context and camera per view), summed into `grads` in one pass."""
        k = len(contexts)
        cfg = config or contexts[0].config
        frames = (C.c_void_p * k)(*[c.frame.value for c in contexts])
        cams = (_abi.Camera * k)(*[c.to_struct() for c in cameras])
        g = gaussians_struct(gaussians)
        gs = grads.struct()
        check(lib().gsc_rasterize_backward_batch(contexts[0].ctx, frames, cams, k, C.byref(g),
                                                 C.byref(cfg), C.byref(gs)),
              "gsc_rasterize_backward_batch")
        return grads


class GPURadixSort:
    """GPURadixSort (src/metal/gpu_radix_sort.cr:46-233) on the library's onesweep sort."""

    @staticmethod
    def sort(keys, values, n=None, begin_bit=0, end_bit=64):
        """In-place stable sort of (u64 key, u32 value) pairs (sort!)."""
        n = keys.numel() if n is None else n
        check(lib().gsc_sort_pairs_u64(context(keys.device), ptr(keys), ptr(values), n, begin_bit,
                                       end_bit), "gsc_sort_pairs_u64")

    @staticmethod
    def compute_tile_ranges(sorted_keys, ranges, n, num_tiles):
        check(lib().gsc_tile_ranges(context(sorted_keys.device), ptr(sorted_keys), n, num_tiles,
                                    ptr(ranges)), "gsc_tile_ranges")


def sync(device=None):
    check(lib().gsc_sync(context(device)), "gsc_sync")
