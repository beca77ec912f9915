"""Shared helpers for the parity tests (CUDA path via the C ABI vs the CPU oracle)."""
import ctypes as C
import importlib

import numpy as np

gs = importlib.import_module("crystal-gausplat_b200")
_abi = importlib.import_module("crystal-gausplat_b200._abi")
R = importlib.import_module("crystal-gausplat_b200.rasterizer")


def to_dev(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t):
    return t.detach().cpu().numpy()


def u64_dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.uint64).view(np.int64)).cuda()


def u64_host(t):
    return t.cpu().numpy().view(np.uint64)


def u32_dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.uint32).view(np.int32)).cuda()


def u32_host(t):
    return t.cpu().numpy().view(np.uint32)


def scene(n, seed, extent=1.0):
    return gs.synthetic_arrays(n, seed, extent)


def gpu_preprocess(g, cam, cfg):
    """gsc_preprocess with every reference-visible output."""
    import torch
    n = g.count
    out = {"splats": torch.zeros(n, 12, device="cuda"), "mean2d": torch.zeros(n, 2, device="cuda"),
           "cov2d": torch.zeros(n, 3, device="cuda"), "conic": torch.zeros(n, 3, device="cuda"),
           "depth": torch.zeros(n, device="cuda"), "radius": torch.zeros(n, device="cuda"),
           "colors": torch.zeros(n, 3, device="cuda"), "opacity": torch.zeros(n, device="cuda"),
           "tiles_touched": torch.zeros(n, dtype=torch.int32, device="cuda"),
           "cov3d": torch.zeros(n, 6, device="cuda")}
    p = _abi.Projected()
    for k, v in out.items():
        setattr(p, k, v.data_ptr())
    gsx = R.gaussians_struct(g)
    _abi.check(_abi.lib().gsc_preprocess(R.context(), C.byref(gsx), C.byref(cam), C.byref(cfg),
                                         C.byref(p)), "gsc_preprocess")
    return out


def rel_err(a, b, floor):
    """max |a-b| / max(|b|, floor)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b) / np.maximum(np.abs(b), floor))) if a.size else 0.0
