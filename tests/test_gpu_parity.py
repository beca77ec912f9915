"""Parity of the CUDA path (through the C ABI) with the CPU oracle.

Bars: bit-exact for keys, values, tile ranges and the
per-tile lists; images within 1e-5 relative (the shared fp32 operation
order makes them bit-exact in practice, which is asserted where it holds);
gradients within 1e-4 relative. Float atomics reorder the per-Gaussian
screen-space sums (grad2d), so the whole-pipeline gradient gate is, per
tensor,
    ||gpu - oracle||_2 <= 1e-4 * ||oracle||_2   and
    |gpu - oracle| <= 1e-4 * (|oracle| + 1e-2 * max|oracle|) per element,
while the chain from a given grad2d to the 59 parameters
(gsc_preprocess_backward) runs the same fp32 operations as the oracle and is
checked bit for bit.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import (R, _abi, gpu_preprocess, gs, host, rel_err, scene, to_dev, u32_dev,
                     u32_host, u64_dev, u64_host)

pytestmark = pytest.mark.gpu

GRAD_RTOL = 1e-4
IMG_RTOL = 1e-5


def grad_close(a, b, rtol=GRAD_RTOL):
    """max of the norm-wise and the floored element-wise relative error."""
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    if not b.size:
        return 0.0
    nb = float(np.linalg.norm(b))
    if nb == 0.0:
        return float(np.abs(a).max())
    norm_err = float(np.linalg.norm(a - b)) / nb
    elem_err = float(np.max(np.abs(a - b) / (np.abs(b) + 1e-2 * float(np.abs(b).max()))))
    return max(norm_err, elem_err)


def make(n, W, H, seed=7, extent=1.0, eye=(0.0, 0.0, 4.0)):
    arrays = scene(n, seed, extent)
    g = gs.Gaussian3D(arrays)
    cam = gs.make_camera(W, H, eye)
    return arrays, g, cam


CASES = [  # (n, W, H, eye)
    (2000, 64, 48, (0.0, 0.0, 4.0)),
    (5000, 100, 75, (1.5, -2.0, 3.0)),   # ragged tile grid, off-axis camera
    (20000, 256, 256, (0.0, 0.0, 4.0)),
]


@pytest.mark.parametrize("mode", [gs.GSC_MODE_FULL, gs.GSC_MODE_REF])
@pytest.mark.parametrize("case", CASES)
def test_preprocess_bit_exact(cuda, oracle, case, mode):
    n, W, H, eye = case
    arrays, g, cam = make(n, W, H, eye=eye)
    cs = cam.to_struct()
    cfg = gs.default_config(mode=mode)
    got = gpu_preprocess(g, cs, cfg)
    ref = oracle.preprocess(oracle.Scene(arrays), cs, cfg)
    for k in ("mean2d", "cov2d", "conic", "depth", "radius", "colors", "opacity", "cov3d"):
        np.testing.assert_array_equal(host(got[k]).reshape(ref[k].shape), ref[k], err_msg=k)
    np.testing.assert_array_equal(u32_host(got["tiles_touched"]), ref["tiles_touched"])


@pytest.mark.parametrize("case", CASES)
def test_binning_sort_ranges_bit_exact(cuda, oracle, case):
    n, W, H, eye = case
    arrays, g, cam = make(n, W, H, eye=eye)
    cs = cam.to_struct()
    cfg = gs.default_config(binning=_abi.GSC_BIN_REFERENCE)  # the stage entry points build reference lists
    got = gpu_preprocess(g, cs, cfg)
    ref = oracle.forward_pipeline(oracle.Scene(arrays), cs, cfg)
    tx, ty = (W + 15) // 16, (H + 15) // 16
    m = ref["keys"].size
    keys = cuda.zeros(m + 1, dtype=cuda.int64, device="cuda")
    vals = cuda.zeros(m + 1, dtype=cuda.int32, device="cuda")
    nk = C.c_int64()
    lib = _abi.lib()
    _abi.check(lib.gsc_bin(R.context(), n, R.ptr(got["splats"]), tx, ty, R.ptr(keys), R.ptr(vals),
                           m + 1, C.byref(nk)))
    assert nk.value == m
    np.testing.assert_array_equal(u64_host(keys)[:m], ref["keys"])
    np.testing.assert_array_equal(u32_host(vals)[:m], ref["vals"])
    # capacity error, nothing written
    rc = lib.gsc_bin(R.context(), n, R.ptr(got["splats"]), tx, ty, R.ptr(keys), R.ptr(vals), m - 1,
                     C.byref(nk))
    assert rc == _abi.GSC_ERR_CAPACITY
    end_bit = 32 + int(np.ceil(np.log2(tx * ty)))
    _abi.check(lib.gsc_sort_pairs_u64(R.context(), R.ptr(keys), R.ptr(vals), m, 0, end_bit))
    np.testing.assert_array_equal(u64_host(keys)[:m], ref["sorted_keys"])
    np.testing.assert_array_equal(u32_host(vals)[:m], ref["sorted_vals"])
    ranges = cuda.zeros(tx * ty * 2, dtype=cuda.int32, device="cuda")
    _abi.check(lib.gsc_tile_ranges(R.context(), R.ptr(keys), m, tx * ty, R.ptr(ranges)))
    np.testing.assert_array_equal(u32_host(ranges), ref["ranges"])
    R.sync()


@pytest.mark.parametrize("n,begin,end", [(0, 0, 64), (1, 0, 64), (2, 0, 64), (511, 0, 64),
                                          (4096, 0, 64), (4097, 0, 45), (100003, 0, 45),
                                          (300000, 8, 40), (1 << 20, 0, 64)])
def test_sort_pairs_bit_exact(cuda, oracle, n, begin, end):
    rng = np.random.default_rng(n + begin)
    tiles = rng.integers(0, 8160, n, dtype=np.uint64)
    depth = rng.uniform(0.5, 10.0, n).astype(np.float32).view(np.uint32).astype(np.uint64)
    keys = (tiles << np.uint64(32)) | depth
    if n > 10:  # duplicate keys exercise stability
        keys[: n // 10] = keys[n // 10: 2 * (n // 10)]
    if end == 64 and n > 3:
        keys[::3] = rng.integers(0, 2**63, keys[::3].size, dtype=np.uint64) * np.uint64(2) + np.uint64(1)
    vals = np.arange(n, dtype=np.uint32)
    rk, rv = oracle.sort_pairs(keys, vals, begin, end)
    dk = u64_dev(keys) if n else cuda.zeros(1, dtype=cuda.int64, device="cuda")
    dv = u32_dev(vals) if n else cuda.zeros(1, dtype=cuda.int32, device="cuda")
    gs.GPURadixSort.sort(dk, dv, n, begin, end)
    R.sync()
    np.testing.assert_array_equal(u64_host(dk)[:n], rk)
    np.testing.assert_array_equal(u32_host(dv)[:n], rv)


def test_sort_c1_distribution_sorted(cuda, oracle):
    """Config-1 key distribution at 4M pairs: sortedness, permutation, stability."""
    n = 4_000_000
    rng = np.random.default_rng(1)
    tiles = rng.integers(0, 8160, n, dtype=np.uint64)
    depth = rng.uniform(0.5, 10.0, n).astype(np.float32).view(np.uint32).astype(np.uint64)
    keys = (tiles << np.uint64(32)) | depth
    vals = np.arange(n, dtype=np.uint32)
    dk, dv = u64_dev(keys), u32_dev(vals)
    gs.GPURadixSort.sort(dk, dv, n, 0, 45)
    R.sync()
    k, v = u64_host(dk), u32_host(dv)
    order = np.argsort(keys, kind="stable")
    np.testing.assert_array_equal(k, keys[order])
    np.testing.assert_array_equal(v, vals[order])


BINNINGS = [_abi.GSC_BIN_REFERENCE, _abi.GSC_BIN_CONTRIBUTING, _abi.GSC_BIN_OCCLUDED]
BIN_IDS = ["reference_lists", "contributing_lists", "occluded_lists"]


def expected_rendered(oracle, arrays, cam, cfg, ref):
    """num_rendered: the list length, or for OCCLUDED the contributing pairs before occlusion."""
    if cfg.binning != _abi.GSC_BIN_OCCLUDED:
        return ref["sorted_keys"].size
    c = gs.default_config(mode=cfg.mode, binning=_abi.GSC_BIN_CONTRIBUTING)
    c.t_stop, c.near_z, c.far_z = cfg.t_stop, cfg.near_z, cfg.far_z
    return oracle.forward_pipeline(oracle.Scene(arrays), cam.to_struct(), c)["sorted_keys"].size


@pytest.mark.parametrize("binning", BINNINGS, ids=BIN_IDS)
@pytest.mark.parametrize("mode", [gs.GSC_MODE_FULL, gs.GSC_MODE_REF])
@pytest.mark.parametrize("case", CASES)
def test_rasterize_forward_matches_oracle(cuda, oracle, case, mode, binning):
    n, W, H, eye = case
    arrays, g, cam = make(n, W, H, eye=eye)
    cfg = gs.default_config(mode=mode, background=(0.1, 0.2, 0.3), binning=binning)
    img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
    nc = ctx.get(_abi.GSC_FRAME_N_CONTRIB, np.uint32)
    fT = ctx.get(_abi.GSC_FRAME_FINAL_T, np.float32)
    last = ctx.get(_abi.GSC_FRAME_LAST, np.uint32)
    ref = oracle.forward_pipeline(oracle.Scene(arrays), cam.to_struct(), cfg)
    assert ctx.num_rendered == expected_rendered(oracle, arrays, cam, cfg, ref)
    if binning == _abi.GSC_BIN_REFERENCE:
        assert ctx.num_rendered == ref["keys"].size
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_KEYS, np.uint64), ref["sorted_keys"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_VALUES, np.uint32), ref["sorted_vals"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_RANGES, np.uint32), ref["ranges"])
    im = host(img)
    assert rel_err(im, ref["image"], 1e-6) <= IMG_RTOL
    np.testing.assert_array_equal(im, ref["image"])  # shared operation order: exact
    np.testing.assert_array_equal(nc.reshape(H, W), ref["n_contrib"])
    np.testing.assert_array_equal(fT.reshape(H, W), ref["final_T"])
    np.testing.assert_array_equal(last.reshape(H, W), ref["last"])


@pytest.mark.parametrize("mode", [gs.GSC_MODE_FULL, gs.GSC_MODE_REF])
@pytest.mark.parametrize("case", CASES)
def test_rasterize_backward_matches_oracle(cuda, oracle, case, mode):
    n, W, H, eye = case
    arrays, g, cam = make(n, W, H, eye=eye)
    cfg = gs.default_config(mode=mode)
    img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
    target = np.random.default_rng(3).uniform(0, 1, (H, W, 3)).astype(np.float32)
    scale = 1.0 / target.size
    loss = cuda.zeros(1, device="cuda")
    grads = gs.Rasterizer.backward(None, g, cam, ctx, target=to_dev(target), l1_scale=scale,
                                   loss_sum=loss)
    R.sync()
    sc = oracle.Scene(arrays)
    ref = oracle.forward_pipeline(sc, cam.to_struct(), cfg)
    g2d, rloss = oracle.composite_backward(W, H, ref["ranges"], ref["sorted_vals"], ref["pre"], cfg,
                                           ref["final_T"], ref["last"], image=ref["image"],
                                           target=target, l1_scale=scale)
    rg, views = oracle.preprocess_backward(sc, cam.to_struct(), cfg, g2d)
    assert abs(float(loss.item()) - rloss) <= 1e-5 * abs(rloss)
    pairs = [(grads.dL_dmean2d, views["mean2d"]), (grads.dL_dopacity, views["opacity"]),
             (grads.dL_dcolors, views["colors"]), (grads.dL_dcov2d, views["cov2d"]),
             (grads.dL_dposition, rg["position"]), (grads.dL_dlog_scale, rg["log_scale"]),
             (grads.dL_drotation, rg["rotation"]), (grads.dL_dlogit_opacity, rg["logit_opacity"]),
             (grads.dL_dsh, rg["sh_coeffs"])]
    names = ["mean2d", "opacity", "colors", "cov2d", "position", "log_scale", "rotation", "logit", "sh"]
    for name, (a, b) in zip(names, pairs):
        e = grad_close(host(a), b)
        assert e <= GRAD_RTOL, f"{name}: {e}"


@pytest.mark.parametrize("case", CASES)
def test_contributing_lists_change_nothing_but_the_lists(cuda, oracle, case):
    """CONTRIBUTING vs REFERENCE binning on the GPU: same image, n_contrib and
    final_T bit for bit, gradients within the atomics' reordering, and the
    contributing lists are an order-preserving subset of the reference ones."""
    n, W, H, eye = case
    arrays, g, cam = make(n, W, H, eye=eye)
    target = to_dev(np.random.default_rng(4).uniform(0, 1, (H, W, 3)).astype(np.float32))
    out = {}
    for b in BINNINGS:
        cfg = gs.default_config(binning=b)
        img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
        grads = gs.Rasterizer.backward(None, g, cam, ctx, target=target)
        R.sync()
        out[b] = (host(img), ctx.get(_abi.GSC_FRAME_N_CONTRIB, np.uint32),
                  ctx.get(_abi.GSC_FRAME_FINAL_T, np.float32), ctx.get(_abi.GSC_FRAME_KEYS, np.uint64),
                  ctx.get(_abi.GSC_FRAME_VALUES, np.uint32), host(grads.arena).copy())
    r, c = out[_abi.GSC_BIN_REFERENCE], out[_abi.GSC_BIN_CONTRIBUTING]
    for k in range(3):
        np.testing.assert_array_equal(c[k], r[k])
    assert c[3].size < r[3].size
    pairs_r = r[3] >> np.uint64(32) << np.uint64(32) | r[4].astype(np.uint64)
    pairs_c = c[3] >> np.uint64(32) << np.uint64(32) | c[4].astype(np.uint64)
    o = np.argsort(pairs_r, kind="stable")  # (tile, id) pairs are unique
    pos = o[np.searchsorted(pairs_r[o], pairs_c)]
    np.testing.assert_array_equal(pairs_r[pos], pairs_c)
    assert np.all(np.diff(pos) > 0)  # order preserved
    np.testing.assert_array_equal(r[3][pos], c[3])
    assert grad_close(c[5], r[5]) <= GRAD_RTOL
    o = out[_abi.GSC_BIN_OCCLUDED]  # depth-sliced: same results, shorter lists
    for k in range(3):
        np.testing.assert_array_equal(o[k], r[k])
    assert o[3].size <= c[3].size
    assert grad_close(o[5], r[5]) <= GRAD_RTOL


def test_backward_with_explicit_dl_dimage(cuda, oracle):
    n, W, H = 3000, 80, 64
    arrays, g, cam = make(n, W, H)
    cfg = gs.default_config()
    img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
    dl = np.random.default_rng(5).standard_normal((H, W, 3)).astype(np.float32) * 1e-3
    grads = gs.Rasterizer.backward(to_dev(dl), g, cam, ctx)
    R.sync()
    sc = oracle.Scene(arrays)
    ref = oracle.forward_pipeline(sc, cam.to_struct(), cfg)
    g2d, _ = oracle.composite_backward(W, H, ref["ranges"], ref["sorted_vals"], ref["pre"], cfg,
                                       ref["final_T"], ref["last"], dL_dimage=dl)
    rg, _ = oracle.preprocess_backward(sc, cam.to_struct(), cfg, g2d)
    assert grad_close(host(grads.dL_dposition), rg["position"]) <= GRAD_RTOL
    assert grad_close(host(grads.dL_dsh), rg["sh_coeffs"]) <= GRAD_RTOL
    assert grad_close(host(grads.dL_drotation), rg["rotation"]) <= GRAD_RTOL


def test_empty_and_culled(cuda, oracle):
    # all Gaussians behind the camera -> background everywhere, no keys
    arrays = scene(500, 11)
    arrays["position"][:, 2] = 10.0  # camera at z=4 looking to -z: all behind
    g = gs.Gaussian3D(arrays)
    cam = gs.make_camera(40, 40, (0.0, 0.0, 4.0))
    cfg = gs.default_config(background=(0.25, 0.5, 0.75))
    img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
    assert ctx.num_rendered == 0
    np.testing.assert_array_equal(host(img), np.broadcast_to(np.float32([0.25, 0.5, 0.75]), (40, 40, 3)))
    grads = gs.Rasterizer.backward(None, g, cam, ctx, target=to_dev(np.zeros((40, 40, 3), np.float32)))
    R.sync()
    assert float(grads.arena.abs().max()) == 0.0
    # zero Gaussians
    g0 = gs.Gaussian3D(scene(0, 1))
    img0, ctx0 = gs.Rasterizer.forward(g0, cam, config=cfg)
    assert ctx0.num_rendered == 0


def test_adam_bit_exact(cuda, oracle):
    rng = np.random.default_rng(9)
    sizes = [30001, 7, 4096, 3]
    host_groups, dev_groups = [], []
    for i, s in enumerate(sizes):
        p = rng.standard_normal(s).astype(np.float32)
        gr = rng.standard_normal(s).astype(np.float32)
        m = rng.standard_normal(s).astype(np.float32) * 0.1
        v = np.abs(rng.standard_normal(s).astype(np.float32)) * 0.01
        lr = [1.6e-4, 5e-3, 5e-2, 1e-3][i]
        wd = 0.01 if i == 2 else 0.0
        host_groups.append({"param": p.copy(), "grad": gr, "m": m.copy(), "v": v.copy(), "lr": lr,
                            "weight_decay": wd})
        dev_groups.append((to_dev(p), to_dev(gr), to_dev(m), to_dev(v), lr, wd))
    for step in (1, 2, 7):
        arr = (_abi.AdamGroup * len(sizes))()
        for i, (p, gr, m, v, lr, wd) in enumerate(dev_groups):
            arr[i].param, arr[i].grad, arr[i].m, arr[i].v = (p.data_ptr(), gr.data_ptr(), m.data_ptr(),
                                                             v.data_ptr())
            arr[i].numel, arr[i].lr, arr[i].weight_decay = p.numel(), lr, wd
        _abi.check(_abi.lib().gsc_adam_step(R.context(), arr, len(sizes), 0.9, 0.999, 1e-8, step, 0.5))
        oracle.adam_step(host_groups, 0.9, 0.999, 1e-8, step, 0.5)
    R.sync()
    for hg, dg in zip(host_groups, dev_groups):
        np.testing.assert_array_equal(host(dg[0]), hg["param"])
        np.testing.assert_array_equal(host(dg[2]), hg["m"])
        np.testing.assert_array_equal(host(dg[3]), hg["v"])


def test_l1_loss_grad(cuda, oracle):
    rng = np.random.default_rng(2)
    a = rng.uniform(0, 1, (37, 51, 3)).astype(np.float32)
    b = rng.uniform(0, 1, (37, 51, 3)).astype(np.float32)
    b[0, 0] = a[0, 0]
    loss, grad = gs.l1_with_grad(to_dev(a), to_dev(b))
    R.sync()
    rl, rg = oracle.l1_loss_grad(a, b, 1.0 / a.size)
    np.testing.assert_array_equal(host(grad), rg)
    assert abs(float(loss.item()) - rl) <= 1e-5 * rl


def test_training_step_decreases_loss(cuda):
    """Forward, fused L1 backward and Adam for a few steps on one view."""
    n, W, H = 5000, 96, 96
    arrays, g, cam = make(n, W, H)
    target = to_dev(np.random.default_rng(4).uniform(0, 1, (H, W, 3)).astype(np.float32))
    grads = gs.RasterizerGradients(g, screen=False)
    opt = gs.Adam.for_gaussians(g, grads)
    ctx = gs.RasterizerContext()
    losses = []
    for _ in range(20):
        grads.zero_()
        loss = cuda.zeros(1, device="cuda")
        gs.Rasterizer.forward(g, cam, context=ctx)
        gs.Rasterizer.backward(None, g, cam, ctx, grads=grads, target=target, loss_sum=loss)
        opt.step()
        losses.append(float(loss.item()))
    R.sync()
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("mode", [gs.GSC_MODE_FULL, gs.GSC_MODE_REF])
def test_composite_backward_grad2d_and_chain(cuda, oracle, mode):
    """Stage API: composite backward (grad2d) within tolerance; the
    preprocess backward fed the SAME grad2d is bit-exact."""
    n, W, H, eye = CASES[1]
    arrays, g, cam = make(n, W, H, eye=eye)
    cs = cam.to_struct()
    cfg = gs.default_config(mode=mode)
    img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
    target = np.random.default_rng(8).uniform(0, 1, (H, W, 3)).astype(np.float32)
    grads = gs.Rasterizer.backward(None, g, cam, ctx, target=to_dev(target), l1_scale=1.0 / target.size)
    R.sync()
    g2d_gpu = ctx.get(_abi.GSC_FRAME_GRAD2D, np.float32).reshape(n, 9)
    sc = oracle.Scene(arrays)
    ref = oracle.forward_pipeline(sc, cs, cfg)
    g2d_ref, _ = oracle.composite_backward(W, H, ref["ranges"], ref["sorted_vals"], ref["pre"], cfg,
                                           ref["final_T"], ref["last"], image=ref["image"],
                                           target=target, l1_scale=1.0 / target.size)
    for k in range(9):
        e = grad_close(g2d_gpu[:, k], g2d_ref[:, k])
        assert e <= GRAD_RTOL, (k, e)
    # chain: oracle on the GPU's grad2d == GPU
    rg, views = oracle.preprocess_backward(sc, cs, cfg, g2d_gpu)
    np.testing.assert_array_equal(host(grads.dL_dposition), rg["position"])
    np.testing.assert_array_equal(host(grads.dL_dlog_scale), rg["log_scale"])
    np.testing.assert_array_equal(host(grads.dL_drotation), rg["rotation"])
    np.testing.assert_array_equal(host(grads.dL_dlogit_opacity).reshape(-1), rg["logit_opacity"])
    np.testing.assert_array_equal(host(grads.dL_dsh).reshape(n, 48), rg["sh_coeffs"])
    np.testing.assert_array_equal(host(grads.dL_dcov2d), views["cov2d"])


@pytest.mark.parametrize("mode", [gs.GSC_MODE_FULL, gs.GSC_MODE_REF])
@pytest.mark.parametrize("k", [1, 3, 8])
def test_backward_batch_equals_per_view_backwards(cuda, mode, k):
    """gsc_rasterize_backward_batch over k deferred views == k single-view
    backwards (up to the order of the fp32 sums)."""
    n, W, H = 20000, 96, 80
    arrays, g, _ = make(n, W, H)
    cams = [gs.make_camera(W, H, tuple(e)) for e in gs.sphere_poses(k, 4.0, seed=k)]
    cfg = gs.default_config(mode=mode)
    rng = np.random.default_rng(k)
    targets = [to_dev(rng.uniform(0, 1, (H, W, 3)).astype(np.float32)) for _ in cams]
    single = gs.RasterizerGradients(g, screen=False)
    ctx = gs.RasterizerContext()
    for cam, t in zip(cams, targets):
        gs.Rasterizer.forward(g, cam, context=ctx, config=cfg)
        gs.Rasterizer.backward(None, g, cam, ctx, grads=single, target=t, config=cfg)
    batched = gs.RasterizerGradients(g, screen=False)
    ctxs = [gs.RasterizerContext() for _ in cams]
    for c, cam, t in zip(ctxs, cams, targets):
        gs.Rasterizer.forward(g, cam, context=c, config=cfg)
        assert gs.Rasterizer.backward(None, g, cam, c, target=t, config=cfg, defer=True) is None
    gs.Rasterizer.backward_batch(ctxs, g, cams, batched, config=cfg)
    R.sync()
    a, b = host(batched.arena), host(single.arena)
    assert np.abs(b).max() > 0
    assert grad_close(a, b) <= GRAD_RTOL


@pytest.mark.parametrize("binning", BINNINGS, ids=BIN_IDS)
def test_forward_batch_equals_single_view_forwards(cuda, binning):
    """gsc_rasterize_forward_batch == gsc_rasterize_forward per view, bit for bit."""
    n, W, H = 30000, 112, 72
    arrays, g, _ = make(n, W, H)
    cams = [gs.make_camera(W, H, tuple(e)) for e in gs.sphere_poses(5, 4.0, seed=3)]
    cfg = gs.default_config(binning=binning)
    ctxs = [gs.RasterizerContext() for _ in cams]
    imgs = gs.Rasterizer.forward_batch(g, cams, ctxs, config=cfg)
    one = gs.RasterizerContext()
    for cam, c, im in zip(cams, ctxs, imgs):
        ref, _ = gs.Rasterizer.forward(g, cam, context=one, config=cfg)
        assert c.num_rendered == one.num_rendered
        np.testing.assert_array_equal(host(im), host(ref))
        for which, dt in ((_abi.GSC_FRAME_VALUES, np.uint32), (_abi.GSC_FRAME_RANGES, np.uint32),
                          (_abi.GSC_FRAME_KEYS, np.uint64),
                          (_abi.GSC_FRAME_FINAL_T, np.float32), (_abi.GSC_FRAME_LAST, np.uint32)):
            np.testing.assert_array_equal(c.get(which, dt), one.get(which, dt))


@pytest.mark.parametrize("near_far", [(0.01, 1000.0), (0.5, 6.0), (-1.0, 1000.0), (0.01, float("inf"))],
                         ids=["default", "narrow", "negative_near", "infinite_far"])
@pytest.mark.parametrize("binning", [_abi.GSC_BIN_CONTRIBUTING, _abi.GSC_BIN_OCCLUDED],
                         ids=["contributing_lists", "occluded_lists"])
def test_forward_batch_depth_words(cuda, oracle, near_far, binning):
    """The batched depth sort (compact view/depth words where the near..far
    span allows, 36-bit words otherwise) gives the oracle's lists per view."""
    n, W, H = 6000, 80, 64
    arrays, g, _ = make(n, W, H, seed=12)
    cams = [gs.make_camera(W, H, tuple(e)) for e in gs.sphere_poses(3, 4.0, seed=5)]
    cfg = gs.default_config(binning=binning)
    cfg.near_z, cfg.far_z = near_far
    ctxs = [gs.RasterizerContext() for _ in cams]
    imgs = gs.Rasterizer.forward_batch(g, cams, ctxs, config=cfg)
    for cam, c, im in zip(cams, ctxs, imgs):
        ref = oracle.forward_pipeline(oracle.Scene(arrays), cam.to_struct(), cfg)
        assert c.num_rendered == expected_rendered(oracle, arrays, cam, cfg, ref)
        np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_KEYS, np.uint64), ref["sorted_keys"])
        np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_VALUES, np.uint32), ref["sorted_vals"])
        np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_RANGES, np.uint32), ref["ranges"])
        np.testing.assert_array_equal(host(im), ref["image"])


@pytest.mark.parametrize("n,W,H", [(300, 16, 16), (300, 13, 9), (1, 48, 48), (2, 48, 48)],
                         ids=["one_tile", "one_ragged_tile", "one_gaussian", "two_gaussians"])
@pytest.mark.parametrize("binning", [_abi.GSC_BIN_CONTRIBUTING, _abi.GSC_BIN_OCCLUDED],
                         ids=["contributing_lists", "occluded_lists"])
def test_forward_tiny_lists(cuda, oracle, n, W, H, binning):
    """One tile (no tile bits to sort) and lists of one or two pairs."""
    arrays = scene(n, 4)
    if n <= 2:
        arrays["position"][:] = 0.0
        arrays["log_scale"][:] = -5.0
    g = gs.Gaussian3D(arrays)
    cam = gs.make_camera(W, H, (0.0, 0.0, 4.0))
    cfg = gs.default_config(binning=binning)
    for views in (1, 2):
        cams = [cam] * views
        ctxs = [gs.RasterizerContext() for _ in cams]
        imgs = gs.Rasterizer.forward_batch(g, cams, ctxs, config=cfg)
        ref = oracle.forward_pipeline(oracle.Scene(arrays), cam.to_struct(), cfg)
        for c, im in zip(ctxs, imgs):
            assert c.num_rendered == expected_rendered(oracle, arrays, cam, cfg, ref)
            np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_KEYS, np.uint64), ref["sorted_keys"])
            np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_VALUES, np.uint32), ref["sorted_vals"])
            np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_RANGES, np.uint32), ref["ranges"])
            np.testing.assert_array_equal(host(im), ref["image"])
