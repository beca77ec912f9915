"""The reference's Loss module (src/ops/loss.cr) over libgsplat_cuda.so:
l1, l1_with_grad, mse, mse_with_grad, ssim, ssim_loss, ssim_loss_with_grad,
combined, combined_with_grad and psnr. Images are [H, W, C] fp32 CUDA
tensors. Values come back as 0-d device tensors (no host sync) unless a
Python float is asked for with float(...).

mode: GSC_MODE_FULL (default) evaluates SSIM with the separable window and
the exact gradient of 1 - SSIM; GSC_MODE_REF reproduces the reference
(2D window, two-pass variance, and its surrogate gradient 2 (pred - target) / n).
"""
import ctypes as C
import math

import torch

from ._abi import GSC_MODE_FULL, check, lib
from .optim import l1_with_grad as _l1_with_grad
from .rasterizer import context, ptr

SSIM_C1 = 0.01 ** 2
SSIM_C2 = 0.03 ** 2


def _hwc(pred, target):
    if pred.shape != target.shape:
        raise ValueError("Shape mismatch")
    if pred.dim() != 3:
        raise ValueError("Expected 3D tensor [H, W, C]")
    assert pred.dtype == torch.float32 and pred.is_contiguous() and target.is_contiguous()
    return pred.shape


def _out(pred):
    return torch.zeros(3, dtype=torch.float32, device=pred.device)


def ssim_loss_with_grad(pred, target, window_size=11, mode=GSC_MODE_FULL, ssim_map=None,
                        want_grad=True):
    """(1 - SSIM, d(1 - SSIM)/dpred)."""
    H, W, Cn = _hwc(pred, target)
    out = _out(pred)
    grad = torch.empty_like(pred) if want_grad else None
    check(lib().gsc_ssim_loss_grad(context(pred.device), ptr(pred), ptr(target), H, W, Cn,
                                   window_size, mode, ptr(grad), ptr(ssim_map), ptr(out)),
          "gsc_ssim_loss_grad")
    return out[0], grad


def ssim(pred, target, window_size=11, mode=GSC_MODE_FULL):
    """Mean local SSIM over the valid region and channels (Loss.ssim)."""
    H, W, Cn = _hwc(pred, target)
    out = _out(pred)
    check(lib().gsc_ssim_loss_grad(context(pred.device), ptr(pred), ptr(target), H, W, Cn,
                                   window_size, mode, None, None, ptr(out)), "gsc_ssim_loss_grad")
    return out[2]


def ssim_loss(pred, target, window_size=11, mode=GSC_MODE_FULL):
    return 1.0 - ssim(pred, target, window_size, mode)


def combined_with_grad(pred, target, lambda_ssim=0.2, mode=GSC_MODE_FULL, out=None, grad=None):
    """((1 - lambda) L1 + lambda (1 - SSIM), its gradient) — Loss.combined_with_grad.
    `out` (3 floats: loss, L1, SSIM) and `grad` may be preallocated."""
    H, W, Cn = _hwc(pred, target)
    out = _out(pred) if out is None else out
    grad = torch.empty_like(pred) if grad is None else grad
    check(lib().gsc_combined_loss_grad(context(pred.device), ptr(pred), ptr(target), H, W, Cn,
                                       C.c_float(lambda_ssim), mode, ptr(grad), ptr(out)),
          "gsc_combined_loss_grad")
    return out[0], grad


def combined(pred, target, lambda_ssim=0.2, mode=GSC_MODE_FULL):
    H, W, Cn = _hwc(pred, target)
    out = _out(pred)
    check(lib().gsc_combined_loss_grad(context(pred.device), ptr(pred), ptr(target), H, W, Cn,
                                       C.c_float(lambda_ssim), mode, None, ptr(out)),
          "gsc_combined_loss_grad")
    return out[0]


def mse_with_grad(pred, target):
    if pred.shape != target.shape:
        raise ValueError("Shape mismatch")
    out = _out(pred)
    grad = torch.empty_like(pred)
    check(lib().gsc_mse_loss_grad(context(pred.device), ptr(pred), ptr(target), pred.numel(),
                                  ptr(grad), ptr(out)), "gsc_mse_loss_grad")
    return out[0], grad


def mse(pred, target):
    if pred.shape != target.shape:
        raise ValueError("Shape mismatch")
    out = _out(pred)
    check(lib().gsc_mse_loss_grad(context(pred.device), ptr(pred), ptr(target), pred.numel(),
                                  None, ptr(out)), "gsc_mse_loss_grad")
    return out[0]


def l1_with_grad(pred, target):
    loss, grad = _l1_with_grad(pred, target)
    return loss[0], grad


def l1(pred, target):
    return l1_with_grad(pred, target)[0]


def psnr(pred, target, max_val=1.0):
    """Loss.psnr (loss.cr:291-296): inf below an MSE of 1e-10."""
    m = float(mse(pred, target))
    if m < 1e-10:
        return math.inf
    return 10.0 * math.log10(max_val * max_val / m)
