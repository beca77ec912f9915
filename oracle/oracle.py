"""numpy front end of the CPU oracle (oracle/_build/libgs_oracle.so).

TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
bench.py CPU-baseline / reference arm as the checker. The product path never
imports it. Parity is unpinned by the reference (no golden vectors exist for
this path upstream); the oracle is pinned by known-answer tests and float64
finite differences in tests/.
"""
import ctypes as C
import importlib
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB_PATH = os.path.join(HERE, "_build", "libgs_oracle.so")

if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
_abi = importlib.import_module("crystal-gausplat_b200._abi")  # struct layouts of include/gsplat_cuda.h

P = C.c_void_p
_lib = None


def build():
    subprocess.check_call(["make", "-s", "-C", HERE])
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(
                os.path.getmtime(os.path.join(HERE, f)) for f in ("gs_oracle.cpp", "gs_oracle.h")):
            build()
        L = C.CDLL(LIB_PATH)
        L.gso_expf.restype = C.c_float
        L.gso_expf.argtypes = [C.c_float]
        L.gso_powi_f32.restype = C.c_float
        L.gso_powi_f32.argtypes = [C.c_float, C.c_int32]
        L.gso_emit_keys.restype = C.c_int64
        L.gso_render_view.restype = C.c_int64
        _lib = L
    return _lib


def default_config(mode=_abi.GSC_MODE_FULL, sh_degree=3, background=(0.0, 0.0, 0.0), t_stop=None,
                   binning=None):
    """The reference's rasterizer constants from the oracle library (no CUDA
    library is loaded), with the overrides of the product's default_config."""
    cfg = _abi.RasterConfig()
    lib().gso_raster_config_default(C.byref(cfg))
    if binning is not None:
        cfg.binning = binning
    cfg.mode = mode
    cfg.sh_degree = sh_degree
    for i in range(3):
        cfg.background[i] = background[i]
    if t_stop is not None:
        cfg.t_stop = t_stop
    return cfg


def powi_f32(a, b):
    return np.float32(lib().gso_powi_f32(C.c_float(a), int(b)))


def set_threads(n):
    lib().gso_set_threads(int(n))


def set_exact_sums(on):
    """Composite-backward sums in double (default) or in fp32 as they come."""
    lib().gso_set_exact_sums(1 if on else 0)


def _p(a):
    return None if a is None else a.ctypes.data_as(P)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def expf(x):
    x = _f32(x).reshape(-1)
    return np.array([lib().gso_expf(C.c_float(v)) for v in x], dtype=np.float32)


class Scene:
    """Host Gaussian arrays (dict from gaussian.synthetic_arrays) as a C struct."""

    def __init__(self, arrays):
        self.pos = _f32(arrays["position"]).reshape(-1, 3)
        self.log_scale = _f32(arrays["log_scale"]).reshape(-1, 3)
        self.rot = _f32(arrays["rotation"]).reshape(-1, 4)
        self.logit = _f32(arrays["logit_opacity"]).reshape(-1)
        self.sh = _f32(arrays["sh_coeffs"]).reshape(-1, 48)
        self.n = self.pos.shape[0]
        s = _abi.Gaussians()
        s.position = self.pos.ctypes.data
        s.log_scale = self.log_scale.ctypes.data
        s.rotation = self.rot.ctypes.data
        s.logit_opacity = self.logit.ctypes.data
        s.sh = self.sh.ctypes.data
        s.count = self.n
        self.struct = s

    def zero_grads(self):
        g = {"position": np.zeros((self.n, 3), np.float32), "log_scale": np.zeros((self.n, 3), np.float32),
             "rotation": np.zeros((self.n, 4), np.float32), "logit_opacity": np.zeros(self.n, np.float32),
             "sh_coeffs": np.zeros((self.n, 48), np.float32)}
        s = _abi.GaussianGrads()
        s.position = g["position"].ctypes.data
        s.log_scale = g["log_scale"].ctypes.data
        s.rotation = g["rotation"].ctypes.data
        s.logit_opacity = g["logit_opacity"].ctypes.data
        s.sh = g["sh_coeffs"].ctypes.data
        return g, s


def preprocess(scene, cam, cfg):
    n = scene.n
    out = {"mean2d": np.zeros((n, 2), np.float32), "cov2d": np.zeros((n, 3), np.float32),
           "conic": np.zeros((n, 3), np.float32), "depth": np.zeros(n, np.float32),
           "radius": np.zeros(n, np.float32), "colors": np.zeros((n, 3), np.float32),
           "opacity": np.zeros(n, np.float32), "tiles_touched": np.zeros(n, np.uint32),
           "cov3d": np.zeros((n, 6), np.float32)}
    lib().gso_preprocess(C.byref(scene.struct), C.byref(cam), C.byref(cfg), *(_p(out[k]) for k in (
        "mean2d", "cov2d", "conic", "depth", "radius", "colors", "opacity", "tiles_touched", "cov3d")))
    return out


def emit_keys(pre, tiles_x, tiles_y):
    n = pre["depth"].shape[0]
    m = lib().gso_emit_keys(C.c_int64(n), _p(pre["mean2d"]), _p(pre["depth"]), _p(pre["radius"]),
                            tiles_x, tiles_y, None, None, C.c_int64(0))
    keys = np.zeros(m, np.uint64)
    vals = np.zeros(m, np.uint32)
    lib().gso_emit_keys(C.c_int64(n), _p(pre["mean2d"]), _p(pre["depth"]), _p(pre["radius"]),
                        tiles_x, tiles_y, _p(keys), _p(vals), C.c_int64(m))
    return keys, vals


def sort_pairs(keys, vals, begin_bit=0, end_bit=64):
    keys = np.ascontiguousarray(keys, np.uint64).copy()
    vals = np.ascontiguousarray(vals, np.uint32).copy()
    lib().gso_sort_pairs(C.c_int64(keys.size), _p(keys), _p(vals), begin_bit, end_bit)
    return keys, vals


def tile_ranges(keys, num_tiles):
    ranges = np.zeros(num_tiles * 2, np.uint32)
    lib().gso_tile_ranges(C.c_int64(keys.size), _p(keys), num_tiles, _p(ranges))
    return ranges


def composite_forward(W, H, ranges, vals, pre, cfg):
    img = np.zeros((H, W, 3), np.float32)
    nc = np.zeros((H, W), np.uint32)
    fT = np.zeros((H, W), np.float32)
    last = np.zeros((H, W), np.uint32)
    lib().gso_composite_forward(W, H, _p(ranges), _p(vals), _p(pre["mean2d"]), _p(pre["cov2d"]),
                                _p(pre["opacity"]), _p(pre["colors"]), C.byref(cfg), _p(img),
                                _p(nc), _p(fT), _p(last))
    return img, nc, fT, last


def composite_forward_literal(W, H, ranges, vals, pre, cfg):
    """rasterize_tile with the reference's unfused expression forms."""
    img = np.zeros((H, W, 3), np.float32)
    nc = np.zeros((H, W), np.uint32)
    fT = np.zeros((H, W), np.float32)
    lib().gso_composite_forward_literal(W, H, _p(ranges), _p(vals), _p(pre["mean2d"]), _p(pre["cov2d"]),
                                        _p(pre["opacity"]), _p(pre["colors"]), C.byref(cfg), _p(img),
                                        _p(nc), _p(fT))
    return img, nc, fT


def composite_backward(W, H, ranges, vals, pre, cfg, final_T, last, dL_dimage=None, image=None,
                       target=None, l1_scale=0.0):
    n = pre["depth"].shape[0]
    g2d = np.zeros((n, 9), np.float32)
    loss = C.c_double(0.0)
    lib().gso_composite_backward(W, H, _p(ranges), _p(vals), _p(pre["mean2d"]), _p(pre["cov2d"]),
                                 _p(pre["opacity"]), _p(pre["colors"]), C.byref(cfg),
                                 _p(None if dL_dimage is None else _f32(dL_dimage)),
                                 _p(None if image is None else _f32(image)),
                                 _p(None if target is None else _f32(target)), C.c_float(l1_scale),
                                 _p(final_T), _p(last), _p(g2d), C.byref(loss))
    return g2d, loss.value


def preprocess_backward(scene, cam, cfg, grad2d):
    g, gs = scene.zero_grads()
    n = scene.n
    views = {"mean2d": np.zeros((n, 2), np.float32), "cov2d": np.zeros((n, 3), np.float32),
             "opacity": np.zeros(n, np.float32), "colors": np.zeros((n, 3), np.float32)}
    lib().gso_preprocess_backward(C.byref(scene.struct), C.byref(cam), C.byref(cfg),
                                  _p(_f32(grad2d)), C.byref(gs), _p(views["mean2d"]),
                                  _p(views["cov2d"]), _p(views["opacity"]), _p(views["colors"]))
    return g, views


def l1_loss_grad(pred, target, scale):
    pred, target = _f32(pred), _f32(target)
    grad = np.zeros_like(pred)
    loss = C.c_double(0.0)
    lib().gso_l1_loss_grad(C.c_int64(pred.size), _p(pred), _p(target), C.c_float(scale), _p(grad),
                           C.byref(loss))
    return loss.value, grad


def adam_step(groups, beta1, beta2, eps, step, grad_scale=1.0):
    """groups: list of dicts with numpy param/grad/m/v (updated in place), lr, weight_decay."""
    arr = (_abi.AdamGroup * len(groups))()
    for i, g in enumerate(groups):
        arr[i].param = g["param"].ctypes.data
        arr[i].grad = g["grad"].ctypes.data
        arr[i].m = g["m"].ctypes.data
        arr[i].v = g["v"].ctypes.data
        arr[i].numel = g["param"].size
        arr[i].lr = g["lr"]
        arr[i].weight_decay = g.get("weight_decay", 0.0)
    lib().gso_adam_step(arr, len(groups), C.c_float(beta1), C.c_float(beta2), C.c_float(eps), step,
                        C.c_float(grad_scale))


def loss_grad(pred, target, window_size=11, mode=0, w_l1=0.0, w_ssim=1.0, want_grad=True,
              want_map=False):
    """gso_loss_grad on [H, W, C] arrays: (out[3], grad or None, ssim map or None)."""
    pred, target = _f32(pred), _f32(target)
    H, W, Cn = pred.shape
    out = np.zeros(3, np.float32)
    grad = np.zeros_like(pred) if want_grad else None
    smap = np.zeros_like(pred) if want_map else None
    lib().gso_loss_grad(_p(pred), _p(target), H, W, Cn, window_size, mode, C.c_float(w_l1),
                        C.c_float(w_ssim), _p(grad), _p(smap), _p(out))
    return out, grad, smap


def mse_loss_grad(pred, target):
    pred, target = _f32(pred), _f32(target)
    out = np.zeros(3, np.float32)
    grad = np.zeros_like(pred)
    lib().gso_mse_loss_grad(_p(pred), _p(target), C.c_int64(pred.size), _p(grad), _p(out))
    return out, grad


def image_to_target(img, width, height, channels):
    """gso_image_to_target on an [h, w, c] uint8 array."""
    img = np.ascontiguousarray(img, np.uint8)
    sh, sw, sc = img.shape
    out = np.zeros((height, width, channels), np.float32)
    lib().gso_image_to_target(_p(img), sw, sh, sc, _p(out), width, height, channels)
    return out


def grad_accumulate(dmean2d, accum, count):
    """accum/count (numpy float32 / int32) updated in place from an [N, stride] gradient."""
    d = _f32(dmean2d)
    n = accum.size
    lib().gso_grad_accumulate(_p(d), C.c_int32(d.size // max(n, 1)), C.c_int64(n), _p(accum),
                              _p(count))


def densify_plan(scene, accum, count, grad_threshold, size_threshold, opacity_threshold):
    flags = np.zeros(scene.n, np.uint8)
    counts = (C.c_int64 * 3)()
    lib().gso_densify_plan(C.byref(scene.struct), _p(_f32(accum)),
                           _p(np.ascontiguousarray(count, np.int32)), C.c_float(grad_threshold),
                           C.c_float(size_threshold), C.c_float(opacity_threshold), _p(flags), counts)
    return flags, tuple(counts)


def densify_apply(scene, flags, clone_noise, ln_split, seed):
    """New host arrays (position, log_scale, rotation, logit_opacity, sh_coeffs)."""
    f = np.ascontiguousarray(flags, np.uint8)
    split = (f & _abi.GSC_DENSIFY_SPLIT) != 0
    keep = ~split & ((f & _abi.GSC_DENSIFY_PRUNE) == 0)
    m = int(keep.sum() + ((f & _abi.GSC_DENSIFY_CLONE) != 0).sum() + 2 * split.sum())
    out = {"position": np.zeros((m, 3), np.float32), "log_scale": np.zeros((m, 3), np.float32),
           "rotation": np.zeros((m, 4), np.float32), "logit_opacity": np.zeros(m, np.float32),
           "sh_coeffs": np.zeros((m, 48), np.float32)}
    o = _abi.GaussiansOut()
    o.position = out["position"].ctypes.data
    o.log_scale = out["log_scale"].ctypes.data
    o.rotation = out["rotation"].ctypes.data
    o.logit_opacity = out["logit_opacity"].ctypes.data
    o.sh = out["sh_coeffs"].ctypes.data
    lib().gso_densify_apply(C.byref(scene.struct), _p(f), C.byref(o), C.c_float(clone_noise),
                            C.c_float(ln_split), C.c_uint64(seed))
    return out


def contributing_lists(W, H, skeys, svals, pre, alpha_min):
    """gso_contributing_lists: the sorted lists without provably non-contributing pairs."""
    m = skeys.size
    ok = np.zeros(m, np.uint64)
    ov = np.zeros(m, np.uint32)
    L = lib()
    L.gso_contributing_lists.restype = C.c_int64
    k = L.gso_contributing_lists(W, H, C.c_int64(m), _p(skeys), _p(svals), _p(pre["mean2d"]),
                                 _p(pre["conic"]), _p(pre["opacity"]), _p(pre["tiles_touched"]),
                                 C.c_float(alpha_min), _p(ok), _p(ov))
    return ok[:k].copy(), ov[:k].copy()


def occluded_lists(W, H, skeys, svals, ranges, last):
    """GSC_BIN_OCCLUDED's final lists: per tile, the first max(last) entries of
    its (contributing) list -- every entry that a pixel of the tile composited
    up to its stop, i.e. all that the backward reads."""
    tx, ty = (W + 15) // 16, (H + 15) // 16
    r = ranges.reshape(-1, 2).astype(np.int64)
    lp = np.zeros((ty * 16, tx * 16), np.int64)
    lp[:H, :W] = last
    keep = lp.reshape(ty, 16, tx, 16).max(axis=(1, 3)).reshape(-1)
    keep = np.minimum(keep, r[:, 1] - r[:, 0])
    sel = np.concatenate([np.arange(a, a + k) for a, k in zip(r[:, 0], keep)]) if keep.sum() else \
        np.zeros(0, np.int64)
    out_r = np.zeros_like(r)
    out_r[:, 1] = np.cumsum(keep)
    out_r[:, 0] = out_r[:, 1] - keep
    out_r[keep == 0] = 0  # the reference's empty range {0, 0}
    return skeys[sel].copy(), svals[sel].copy(), out_r.astype(np.uint32).reshape(-1)


def forward_pipeline(scene, cam, cfg):
    """All forward intermediates of one view (preprocess .. composite)."""
    W, H = cam.width, cam.height
    tx, ty = (W + 15) // 16, (H + 15) // 16
    pre = preprocess(scene, cam, cfg)
    keys, vals = emit_keys(pre, tx, ty)
    end_bit = 32 + max(0, int(np.ceil(np.log2(tx * ty))) if tx * ty > 1 else 0)
    skeys, svals = sort_pairs(keys, vals, 0, end_bit)
    binning = getattr(cfg, "binning", _abi.GSC_BIN_REFERENCE)
    if binning in (_abi.GSC_BIN_CONTRIBUTING, _abi.GSC_BIN_OCCLUDED):
        skeys, svals = contributing_lists(W, H, skeys, svals, pre, cfg.alpha_min)
    ranges = tile_ranges(skeys, tx * ty)
    img, nc, fT, last = composite_forward(W, H, ranges, svals, pre, cfg)
    if binning == _abi.GSC_BIN_OCCLUDED:
        skeys, svals, ranges = occluded_lists(W, H, skeys, svals, ranges, last)
    return {"pre": pre, "keys": keys, "vals": vals, "sorted_keys": skeys, "sorted_vals": svals,
            "ranges": ranges, "image": img, "n_contrib": nc, "final_T": fT, "last": last}


def render_view(scene, cam, cfg, target=None, l1_scale=0.0):
    """Whole view through the oracle (forward; + fused L1 backward with a target)."""
    img = np.zeros((cam.height, cam.width, 3), np.float32)
    grads, gs = scene.zero_grads()
    loss = C.c_double(0.0)
    m = lib().gso_render_view(C.byref(scene.struct), C.byref(cam), C.byref(cfg), _p(img),
                              _p(None if target is None else _f32(target)), C.c_float(l1_scale),
                              C.byref(gs) if target is not None else None, C.byref(loss))
    return img, (grads if target is not None else None), loss.value, m
