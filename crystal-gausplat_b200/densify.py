"""Densification and pruning on the device: GradientAccumulator
(src/gaussian_splatting/trainer.cr:77-123), Trainer#densify_and_prune! with
split_gaussians! and add_position_noise! (trainer.cr:293-392), and
Gaussian3D#reset_opacity! (gaussian.cr:269-271).

The decisions and the new set are computed by libgsplat_cuda.so; only the
three group sizes come back to the host (to size the new arena). Random
position offsets come from a seeded counter-based hash, so a densification
is reproducible; the reference draws them from an unseeded host RNG.
"""
import ctypes as C
import math

import torch

from . import _abi
from ._abi import check, lib
from .gaussian import Gaussian3D
from .rasterizer import context, gaussians_struct, ptr


class GradientAccumulator:
    """Per-Gaussian sum of |dL/dmean2d| and the number of views accumulated."""

    def __init__(self, count, device="cuda"):
        self.position_grad_accum = torch.zeros(count, dtype=torch.float32, device=device)
        self.position_grad_count = torch.zeros(count, dtype=torch.int32, device=device)

    @property
    def count(self):
        return self.position_grad_accum.numel()

    def accumulate(self, grads):
        """grads: RasterizerGradients (its dL_dmean2d [N,2]) or an [N,2] / [N,k>=2] tensor."""
        d = grads.dL_dmean2d if hasattr(grads, "dL_dmean2d") else grads
        n = self.count
        assert d.dtype == torch.float32 and d.is_contiguous() and d.shape[0] == n
        stride = d.numel() // max(n, 1)
        check(lib().gsc_grad_accumulate(context(d.device), ptr(d), stride, n,
                                        ptr(self.position_grad_accum),
                                        ptr(self.position_grad_count)), "gsc_grad_accumulate")

    def get_average(self, index=None):
        avg = torch.where(self.position_grad_count == 0, torch.zeros_like(self.position_grad_accum),
                          self.position_grad_accum / self.position_grad_count.clamp(min=1).float())
        return avg if index is None else float(avg[index])

    def reset(self):
        self.position_grad_accum.zero_()
        self.position_grad_count.zero_()

    def resize(self, new_count):
        dev = self.position_grad_accum.device
        keep = min(new_count, self.count)
        a = torch.zeros(new_count, dtype=torch.float32, device=dev)
        c = torch.zeros(new_count, dtype=torch.int32, device=dev)
        a[:keep] = self.position_grad_accum[:keep]
        c[:keep] = self.position_grad_count[:keep]
        self.position_grad_accum, self.position_grad_count = a, c


def densify_plan(gaussians, accum, grad_threshold=0.0002, size_threshold=0.01,
                 opacity_threshold=0.005):
    """flags (uint8 [N], GSC_DENSIFY_* bits) and (kept, clones, splits).
    Defaults are TrainerConfig's (trainer.cr:41-44)."""
    n = gaussians.count
    dev = gaussians.arena.device
    flags = torch.zeros(max(n, 1), dtype=torch.uint8, device=dev)
    counts = (C.c_int64 * 3)()
    s = gaussians_struct(gaussians)
    check(lib().gsc_densify_plan(context(dev), C.byref(s), ptr(accum.position_grad_accum),
                                 ptr(accum.position_grad_count), grad_threshold, size_threshold,
                                 opacity_threshold, ptr(flags), counts), "gsc_densify_plan")
    return flags[:n], tuple(counts)


def densify_apply(gaussians, flags, counts, clone_noise=0.001, scale_factor=1.6, seed=0):
    """The densified set as a new Gaussian3D: [kept][clones][split halves 1][split halves 2]."""
    kept, clones, splits = counts
    dev = gaussians.arena.device
    out = Gaussian3D.empty(kept + clones + 2 * splits, device=dev)
    o = _abi.GaussiansOut()
    o.position = out.position.data_ptr()
    o.log_scale = out.log_scale.data_ptr()
    o.rotation = out.rotation.data_ptr()
    o.logit_opacity = out.logit_opacity.data_ptr()
    o.sh = out.sh_coeffs.data_ptr()
    s = gaussians_struct(gaussians)
    check(lib().gsc_densify_apply(context(dev), C.byref(s), ptr(flags), C.byref(o), clone_noise,
                                  math.log(scale_factor), seed), "gsc_densify_apply")
    return out


def densify_and_prune(gaussians, accum, grad_threshold=0.0002, size_threshold=0.01,
                      opacity_threshold=0.005, clone_noise=0.001, scale_factor=1.6, seed=0):
    """Trainer#densify_and_prune!: returns the new Gaussian3D and resets `accum`
    to its size. Optimizer state must be recreated for the new set, as the
    reference's recreate_optimizers! does."""
    flags, counts = densify_plan(gaussians, accum, grad_threshold, size_threshold,
                                 opacity_threshold)
    out = densify_apply(gaussians, flags, counts, clone_noise, scale_factor, seed)
    accum.resize(out.count)
    accum.reset()
    return out


def reset_opacity(gaussians, value=-1.0):
    """Gaussian3D#reset_opacity!: every logit opacity set to `value` (the reference's -1)."""
    t = gaussians.logit_opacity
    check(lib().gsc_reset_opacity(context(t.device), ptr(t), gaussians.count, value),
          "gsc_reset_opacity")
