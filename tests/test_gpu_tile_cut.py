"""Occluded binning with a per-tile depth cut (gsc_frame_set_tile_hint).

The cut only decides which depth slice a (tile, Gaussian) pair is binned in:
the first slice takes, per tile, the pairs in front of the tile's cut, the
second the rest of the tiles whose pixels did not all stop. Every tile's list
is still its depth order up to its saturation point, so the frame's lists,
ranges, per-pixel outputs and images must equal those of the forward without
a cut bit for bit, whatever the cut holds (the unhinted occluded forward
itself is checked against the oracle in test_gpu_north_star.py and
test_gpu_parity.py). The scenes include Gaussians whose rectangles exceed 64
tiles, which the cut's counting and emission walk warp-cooperatively.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import R, _abi, gs, host, to_dev

pytestmark = pytest.mark.gpu

W = H = 256
T = (W // 16) * (H // 16)
OUTS = {"keys": (_abi.GSC_FRAME_KEYS, np.uint64), "vals": (_abi.GSC_FRAME_VALUES, np.uint32),
        "ranges": (_abi.GSC_FRAME_RANGES, np.uint32), "final_T": (_abi.GSC_FRAME_FINAL_T, np.float32),
        "last": (_abi.GSC_FRAME_LAST, np.uint32), "n_contrib": (_abi.GSC_FRAME_N_CONTRIB, np.uint32)}


def big_scene(n, seed, big=300):
    a = gs.synthetic_arrays(n, seed)
    # scale ~0.5 at depth ~4: radius ~80 px, rectangles of ~100 tiles
    a["log_scale"][:big] = -0.7
    return a


def outputs(ctx, img):
    out = {k: ctx.get(w, dt) for k, (w, dt) in OUTS.items()}
    out["image"] = host(img).copy()
    out["rendered"] = int(ctx.num_rendered)
    return out


def assert_same(a, b, what):
    for k in a:
        np.testing.assert_array_equal(a[k], b[k], err_msg=f"{what}: {k}")


def binned_pairs(fn):
    """Pairs binned (emitted and sorted) by fn(), from the tracing counters."""
    lib, ctx = _abi.lib(), R.context()
    out = (C.c_uint64 * 2)()
    _abi.check(lib.gsc_profile_pairs(ctx, out, 1))
    _abi.check(lib.gsc_profile_enable(ctx, 1))
    try:
        fn()
        R.sync()
    finally:
        _abi.check(lib.gsc_profile_enable(ctx, 0))
    _abi.check(lib.gsc_profile_pairs(ctx, out, 1))
    return int(out[0]), int(out[1])


@pytest.mark.parametrize("t_stop", [1e-3, 1e-4], ids=["T1e-3", "T1e-4"])
@pytest.mark.parametrize("mode", [gs.GSC_MODE_FULL, gs.GSC_MODE_REF], ids=["full", "ref"])
def test_single_view_any_cut_gives_the_same_frame(cuda, mode, t_stop):
    g = gs.Gaussian3D(big_scene(100_000, 0x7C0100))
    cam = gs.make_camera(W, H, (0.0, 0.0, 4.0))
    cfg = gs.default_config(mode=mode, binning=_abi.GSC_BIN_OCCLUDED, t_stop=t_stop)
    ctx = R.RasterizerContext()

    def run(cut=None, valid=False):
        ctx.set_tile_hint(cut, valid)
        img, _ = gs.Rasterizer.forward(g, cam, context=ctx, config=cfg)
        R.sync()
        return outputs(ctx, img)

    base = run()
    b_plain, kept = binned_pairs(lambda: run())
    cut = cuda.empty(T, dtype=cuda.float32, device="cuda")
    assert_same(run(cut, False), base, "unread cut")  # writes the view's cut
    c = host(cut)
    finite = np.isfinite(c)
    assert finite.any() and (c[finite] > 0).all() and np.isposinf(c[~finite]).all()
    first = c.copy()
    b_cut, kept_cut = binned_pairs(lambda: run(cut, True))
    assert kept_cut == kept
    assert b_cut < b_plain, (b_cut, b_plain)  # the cut bins fewer pairs
    np.testing.assert_array_equal(host(cut), first)  # same scene, same cut
    assert_same(run(cut, True), base, "own cut")
    rng = np.random.default_rng(5)
    lo, hi = float(c[finite].min()) * 0.8, float(c[finite].max()) * 1.2
    for trial in range(4):
        r = rng.uniform(lo, hi, T).astype(np.float32)
        r[rng.random(T) < 0.1] = np.inf
        r[rng.random(T) < 0.1] = 0.0
        r[rng.random(T) < 0.05] = np.nan
        cut.copy_(to_dev(r))
        assert_same(run(cut, True), base, f"random cut {trial}")
    for v in (0.0, np.inf, np.nan):
        cut.fill_(float(v))
        assert_same(run(cut, True), base, f"cut {v}")


def test_batched_views_with_per_view_cuts_and_backward(cuda):
    arrays = big_scene(60_000, 0x7C0200)
    g = gs.Gaussian3D(arrays)
    eyes = gs.sphere_poses(4, 4.0, 0x7C0201)
    cams = [gs.make_camera(W, H, tuple(e)) for e in eyes]
    cfg = gs.default_config(binning=_abi.GSC_BIN_OCCLUDED)
    ctxs = [R.RasterizerContext() for _ in cams]
    cuts = [cuda.empty(T, dtype=cuda.float32, device="cuda") for _ in cams]
    targets = [to_dev(np.random.default_rng(40 + v).random((H, W, 3), dtype=np.float32)) for v in range(len(cams))]

    def step(bind):
        for k, c in enumerate(ctxs):
            bind(k, c)
        imgs = gs.Rasterizer.forward_batch(g, cams, ctxs, config=cfg)
        R.sync()
        outs = [outputs(c, im) for c, im in zip(ctxs, imgs)]
        grads = gs.RasterizerGradients(g, screen=False)
        loss = cuda.zeros(1, device="cuda")
        for k, (cam, c) in enumerate(zip(cams, ctxs)):
            gs.Rasterizer.backward(None, g, cam, c, grads=grads, target=targets[k], loss_sum=loss, defer=True)
        gs.Rasterizer.backward_batch(ctxs, g, cams, grads, config=cfg)
        R.sync()
        return outs, host(grads.arena).copy(), float(loss.item())

    base, g0, l0 = step(lambda k, c: c.set_tile_hint(None, False))
    step(lambda k, c: c.set_tile_hint(cuts[k], False))  # every view writes its cut
    # view 0 unbound, view 1 its cut unread, views 2 and 3 read their cuts
    outs, g1, l1 = step(lambda k, c: c.set_tile_hint(None if k == 0 else cuts[k], k >= 2))
    for k in range(len(cams)):
        assert_same(outs[k], base[k], f"view {k}")
    # same lists, so the gradients differ only by the order of the atomic adds
    assert abs(l1 - l0) <= 1e-6 * abs(l0)
    assert np.linalg.norm(g1 - g0) <= 1e-5 * np.linalg.norm(g0)


def test_short_cut_array_is_refused(cuda):
    g = gs.Gaussian3D(gs.synthetic_arrays(2_000, 0x7C0300))
    cam = gs.make_camera(W, H, (0.0, 0.0, 4.0))
    cfg = gs.default_config(binning=_abi.GSC_BIN_OCCLUDED)
    ctx = R.RasterizerContext()
    ctx.set_tile_hint(cuda.full((T - 1,), float("inf"), device="cuda"), True)
    with pytest.raises(_abi.GscError, match="shorter than the view's tiles"):
        gs.Rasterizer.forward(g, cam, context=ctx, config=cfg)
    ctx.set_tile_hint(None, False)
    img, _ = gs.Rasterizer.forward(g, cam, context=ctx, config=cfg)  # the frame still works
    R.sync()
    assert np.isfinite(host(img)).all()
