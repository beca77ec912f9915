"""Adam (src/optim/adam.cr:35-176) as one fused launch over all parameter
groups, and the L1 loss (src/ops/loss.cr:33-57)."""
import ctypes as C

import torch

from . import _abi
from ._abi import check, lib
from .rasterizer import context, ptr

# Trainer learning rates (src/gaussian_splatting/trainer.cr:41-45).
DEFAULT_LRS = {"position": 1.6e-4, "log_scale": 5e-3, "rotation": 1e-3, "logit_opacity": 5e-2,
               "sh_coeffs": 2.5e-3}


class Adam:
    """Adam with parameter groups; state m, v and the step count per optimiser
    (AdamState, adam.cr:20-33). `groups` is a list of (param, grad, lr)
    tensors of equal shape; m and v are allocated here."""

    def __init__(self, groups, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=0.0):
        if not 0 < len(groups) <= 8:
            raise ValueError("1..8 parameter groups")
        self.beta1, self.beta2, self.eps = beta1, beta2, eps
        self.step_count = 0
        self.groups = []
        for g in groups:
            param, grad, lr = g[0], g[1], g[2]
            wd = g[3] if len(g) > 3 else weight_decay
            self.groups.append({"param": param, "grad": grad, "lr": float(lr), "weight_decay": float(wd),
                                "m": torch.zeros_like(param), "v": torch.zeros_like(param)})

    @classmethod
    def for_gaussians(cls, gaussians, grads, lrs=None, **kw):
        lrs = dict(DEFAULT_LRS, **(lrs or {}))
        gv = gaussians.views_of(grads.arena if hasattr(grads, "arena") else grads)
        params = dict(zip(("position", "log_scale", "rotation", "logit_opacity", "sh_coeffs"),
                          gaussians.parameters()))
        return cls([(params[k], gv[k], lrs[k]) for k in params], **kw)

    def step(self, grad_scale=1.0):
        """Adam#step (adam.cr:86-110); gradients are multiplied by grad_scale."""
        self.step_count += 1
        arr = (_abi.AdamGroup * len(self.groups))()
        for i, g in enumerate(self.groups):
            arr[i].param = g["param"].data_ptr()
            arr[i].grad = g["grad"].data_ptr()
            arr[i].m = g["m"].data_ptr()
            arr[i].v = g["v"].data_ptr()
            arr[i].numel = g["param"].numel()
            arr[i].lr = g["lr"]
            arr[i].weight_decay = g["weight_decay"]
        check(lib().gsc_adam_step(context(self.groups[0]["param"].device), arr, len(self.groups),
                                  self.beta1, self.beta2, self.eps, self.step_count, grad_scale),
              "gsc_adam_step")

    def state_dict(self):
        return {"step": self.step_count,
                "m": [g["m"].clone() for g in self.groups], "v": [g["v"].clone() for g in self.groups]}

    def load_state_dict(self, sd):
        self.step_count = int(sd["step"])
        for g, m, v in zip(self.groups, sd["m"], sd["v"]):
            g["m"].copy_(m)
            g["v"].copy_(v)


def l1_with_grad(pred, target, scale=None):
    """Loss.l1_with_grad: (mean |pred - target|, sign(pred - target)/numel)."""
    scale = 1.0 / pred.numel() if scale is None else scale
    grad = torch.empty_like(pred)
    loss = torch.zeros(1, device=pred.device)
    check(lib().gsc_l1_loss_grad(context(pred.device), ptr(pred), ptr(target), pred.numel(),
                                 C.c_float(scale), ptr(grad), ptr(loss)), "gsc_l1_loss_grad")
    return loss, grad
