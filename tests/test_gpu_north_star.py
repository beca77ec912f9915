"""Parity at the benchmark's own configurations (2 and the
config-3 training path), CUDA path through the C ABI against the CPU oracle.

Bars: bit-exact for sorted keys, values, tile ranges and per-tile lists;
images within 1e-5 relative (bit-exact in practice: the kernels and the
oracle share the fp32 operation order, asserted); gradients against the
oracle with exact (double) per-Gaussian sums: norm-wise relative error
<= 1e-4 per tensor, element-wise within 1e-4 except for ill-conditioned
elements no more numerous than fp32 summation itself produces (see `gate`).

- config 0: 100k Gaussians, one 256x256 camera at (0,0,4): both tile-list
  kinds, both arithmetic modes, both transmittance stops (the reference's
  1e-3, gaussian.metal:400, and the north star's 1e-4).
- config 2: 1M Gaussians, one 1920x1080 camera on the radius-4 sphere, L1
  against a seeded target: the reference's sorted lists and ranges, the image
  and all 59 parameter gradients, at both stops.
- config 3 path: 3M Gaussians at 1920x1080, three views through the
  benchmark's own training path (DataParallelTrainer: one batched forward with
  depth-sliced occluded lists and batched depth words, deferred compositing
  backwards, one batched preprocess backward). Per view the lists equal the
  oracle's contributing lists cut after each tile's largest `last`, the
  contributing lists are an order-preserving subset of the reference's sorted
  lists, and images, contributor counts, final transmittance and `last` equal
  the oracle's (images also over the reference lists); the summed gradients
  of the three views pass the gradient gate. A second pass, whose forwards
  read each view's per-tile depth cut from the first, gives the same frames.
"""
import importlib
import os

import numpy as np
import pytest

from helpers import R, _abi, gs, host, rel_err, to_dev

pytestmark = pytest.mark.gpu

GRAD_RTOL = 1e-4
IMG_RTOL = 1e-5
C0_SEED = 0x6A5D0000
C2_SEED = 0x6A5D0002
C3_SEED = 0x6A5D0003


@pytest.fixture
def par_oracle(oracle):
    """The oracle on every host thread for the large cases."""
    oracle.set_threads(os.cpu_count() or 1)
    yield oracle
    oracle.set_threads(1)


def sphere_camera(seed, W, H, k=0, views=1):
    eyes = gs.sphere_poses(views, 4.0, seed + 101)
    return gs.make_camera(W, H, tuple(eyes[k]))


def target_of(seed, v, H, W):
    return np.random.default_rng(seed * 1000 + v).random((H, W, 3), dtype=np.float32)


def check_forward(ctx, img, ref, W, H, rendered=None):
    assert ctx.num_rendered == (ref["sorted_keys"].size if rendered is None else rendered)
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_KEYS, np.uint64), ref["sorted_keys"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_VALUES, np.uint32), ref["sorted_vals"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_RANGES, np.uint32), ref["ranges"])
    im = host(img)
    assert rel_err(im, ref["image"], 1e-6) <= IMG_RTOL
    np.testing.assert_array_equal(im, ref["image"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_N_CONTRIB, np.uint32).reshape(H, W), ref["n_contrib"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_FINAL_T, np.float32).reshape(H, W), ref["final_T"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_LAST, np.uint32).reshape(H, W), ref["last"])


def oracle_backward(o, sc, cs, cfg, ref, target, W, H, exact=True):
    """The oracle's screen-space and parameter gradients of one view; exact:
    per-Gaussian sums in double (default), else fp32 in thread order."""
    o.set_exact_sums(exact)
    try:
        g2d, rloss = o.composite_backward(W, H, ref["ranges"], ref["sorted_vals"], ref["pre"], cfg,
                                          ref["final_T"], ref["last"], image=ref["image"], target=target,
                                          l1_scale=1.0 / target.size)
    finally:
        o.set_exact_sums(True)
    rg, views = o.preprocess_backward(sc, cs, cfg, g2d)
    out = {k: v for k, v in rg.items()}
    out.update({"v_" + k: v for k, v in views.items()})
    return out, rloss


def elem_rel(a, b):
    """Per-element error floored at 1e-2 of the largest reference magnitude."""
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    if not b.size:
        return np.zeros(0)
    floor = 1e-2 * float(np.abs(b).max())
    if floor == 0.0:
        return np.abs(a - b)
    return np.abs(a - b) / (np.abs(b) + floor)


def norm_err(a, b):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    nb = float(np.linalg.norm(b))
    return float(np.linalg.norm(a - b)) / nb if nb else float(np.abs(a).max() if a.size else 0.0)


def gate(name, got, exact, fp32):
    """Gradient gate against the exact-sum oracle.

    - norm-wise relative error <= 1e-4 per tensor (the north star's bar);
    - element-wise (error floored at 1e-2 of the largest magnitude): every
      element within 1e-4, except as many as the oracle's own fp32 sums miss
      that bar by (at most 3x that count, or 10). Those are ill-conditioned
      elements -- the rotation and scale gradients of nearly isotropic
      Gaussians, whose terms cancel -- where any fp32 summation order moves
      the result by more than 1e-4; the reference adds with fp32 atomics in an
      unspecified order, so its own results carry that spread from run to run.
      Their worst error must stay within 10x the fp32 spread's worst."""
    ne = norm_err(got, exact)
    assert ne <= GRAD_RTOL, f"{name}: norm-wise {ne:.3e}"
    eg, ef = elem_rel(got, exact), elem_rel(fp32, exact)
    if not eg.size:
        return
    over_g, over_f = int((eg > GRAD_RTOL).sum()), int((ef > GRAD_RTOL).sum())
    assert over_g <= max(10, 3 * over_f), \
        f"{name}: {over_g} of {eg.size} elements beyond 1e-4 (fp32 sums: {over_f})"
    assert eg.max() <= max(GRAD_RTOL, 10.0 * ef.max()), \
        f"{name}: element-wise {eg.max():.3e}, fp32 spread {ef.max():.3e}"


def check_backward(o, sc, cs, cfg, ref, grads, loss, target, W, H):
    exact, rloss = oracle_backward(o, sc, cs, cfg, ref, target, W, H, exact=True)
    fp32, _ = oracle_backward(o, sc, cs, cfg, ref, target, W, H, exact=False)
    assert abs(float(loss.item()) - rloss) <= 1e-5 * abs(rloss)
    got = {"v_mean2d": grads.dL_dmean2d, "v_opacity": grads.dL_dopacity, "v_colors": grads.dL_dcolors,
           "v_cov2d": grads.dL_dcov2d, "position": grads.dL_dposition, "log_scale": grads.dL_dlog_scale,
           "rotation": grads.dL_drotation, "logit_opacity": grads.dL_dlogit_opacity, "sh_coeffs": grads.dL_dsh}
    for name, t in got.items():
        if cfg.mode == _abi.GSC_MODE_REF and name == "v_cov2d":
            continue  # the reference never writes it (zero on both sides)
        gate(name, host(t), exact[name], fp32[name])


# ---- config 0 ------------------------------------------------------------------

@pytest.mark.parametrize("t_stop", [1e-3, 1e-4], ids=["T1e-3", "T1e-4"])
@pytest.mark.parametrize("binning", [_abi.GSC_BIN_REFERENCE, _abi.GSC_BIN_CONTRIBUTING, _abi.GSC_BIN_OCCLUDED],
                         ids=["reference_lists", "contributing_lists", "occluded_lists"])
@pytest.mark.parametrize("mode", [gs.GSC_MODE_FULL, gs.GSC_MODE_REF], ids=["full", "ref"])
def test_c0_forward_backward(cuda, par_oracle, mode, binning, t_stop):
    W = H = 256
    arrays = gs.synthetic_arrays(100_000, C0_SEED)
    g = gs.Gaussian3D(arrays)
    cam = gs.make_camera(W, H, (0.0, 0.0, 4.0))
    cfg = gs.default_config(mode=mode, binning=binning, t_stop=t_stop)
    img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
    target = target_of(C0_SEED, 0, H, W)
    loss = cuda.zeros(1, device="cuda")
    grads = gs.Rasterizer.backward(None, g, cam, ctx, target=to_dev(target), loss_sum=loss)
    R.sync()
    sc = par_oracle.Scene(arrays)
    cs = cam.to_struct()
    ref = par_oracle.forward_pipeline(sc, cs, cfg)
    rendered = None
    if binning == _abi.GSC_BIN_OCCLUDED:  # num_rendered: the contributing pairs before occlusion
        c = gs.default_config(mode=mode, binning=_abi.GSC_BIN_CONTRIBUTING, t_stop=t_stop)
        rendered = par_oracle.forward_pipeline(sc, cs, c)["sorted_keys"].size
        assert ref["sorted_keys"].size < rendered
    else:
        assert ref["sorted_keys"].size > 100_000
    check_forward(ctx, img, ref, W, H, rendered)
    check_backward(par_oracle, sc, cs, cfg, ref, grads, loss, target, W, H)


# ---- config 2 ------------------------------------------------------------------

@pytest.mark.parametrize("t_stop", [1e-3, 1e-4], ids=["T1e-3", "T1e-4"])
def test_c2_single_view_forward_backward(cuda, par_oracle, t_stop):
    W, H = 1920, 1080
    arrays = gs.synthetic_arrays(1_000_000, C2_SEED)
    g = gs.Gaussian3D(arrays)
    cam = sphere_camera(C2_SEED, W, H)
    cfg = gs.default_config(binning=_abi.GSC_BIN_REFERENCE, t_stop=t_stop)
    img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
    target = target_of(C2_SEED, 0, H, W)
    loss = cuda.zeros(1, device="cuda")
    grads = gs.Rasterizer.backward(None, g, cam, ctx, target=to_dev(target), loss_sum=loss)
    R.sync()
    sc = par_oracle.Scene(arrays)
    cs = cam.to_struct()
    ref = par_oracle.forward_pipeline(sc, cs, cfg)
    assert ref["sorted_keys"].size > 5_000_000
    check_forward(ctx, img, ref, W, H)
    check_backward(par_oracle, sc, cs, cfg, ref, grads, loss, target, W, H)


# ---- config 3 training path ------------------------------------------------------

def test_c3_training_path_three_views(cuda, par_oracle):
    O = par_oracle
    trainer_mod = importlib.import_module("crystal-gausplat_b200.trainer")
    W, H, views = 1920, 1080, 3
    arrays = gs.synthetic_arrays(3_000_000, C3_SEED)
    g = gs.Gaussian3D(arrays)
    eyes = gs.sphere_poses(64, 4.0, C3_SEED + 101)[:views]  # the benchmark's first three poses
    cams = [gs.make_camera(W, H, tuple(e)) for e in eyes]
    cfg = gs.default_config(binning=_abi.GSC_BIN_OCCLUDED)  # the benchmark's lists
    tr = trainer_mod.DataParallelTrainer(g, cams, cfg)
    targets = [target_of(C3_SEED, v, H, W) for v in range(views)]
    dev_t = [to_dev(t) for t in targets]
    tr.zero()
    for v in range(views):
        tr.view_fwd_bwd(v, dev_t[v])
    tr.flush()
    R.sync()
    got = {v: {"keys": tr.ctxs[v].get(_abi.GSC_FRAME_KEYS, np.uint64),
               "vals": tr.ctxs[v].get(_abi.GSC_FRAME_VALUES, np.uint32),
               "ranges": tr.ctxs[v].get(_abi.GSC_FRAME_RANGES, np.uint32),
               "n_contrib": tr.ctxs[v].get(_abi.GSC_FRAME_N_CONTRIB, np.uint32).reshape(H, W),
               "last": tr.ctxs[v].get(_abi.GSC_FRAME_LAST, np.uint32).reshape(H, W),
               "rendered": tr.ctxs[v].num_rendered,
               "final_T": tr.ctxs[v].get(_abi.GSC_FRAME_FINAL_T, np.float32).reshape(H, W),
               "image": host(tr.images[v])} for v in range(views)}
    gpu_grads = host(tr.grads.arena).copy()
    gpu_loss = float(tr.loss.item())
    # the same pass again: now each view's forward reads the per-tile depth
    # cut its first forward wrote; lists, per-pixel outputs and images are
    # the same bit for bit, gradients up to the order of the atomic adds
    assert tr.tile_hints and all(h[1] for h in tr.tile_hints.values())
    tr.zero()
    for v in range(views):
        tr.view_fwd_bwd(v, dev_t[v])
    tr.flush()
    R.sync()
    for v in range(views):
        c = tr.ctxs[v]
        np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_KEYS, np.uint64), got[v]["keys"])
        np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_VALUES, np.uint32), got[v]["vals"])
        np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_RANGES, np.uint32), got[v]["ranges"])
        np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_LAST, np.uint32).reshape(H, W), got[v]["last"])
        np.testing.assert_array_equal(c.get(_abi.GSC_FRAME_FINAL_T, np.float32).reshape(H, W), got[v]["final_T"])
        np.testing.assert_array_equal(host(tr.images[v]), got[v]["image"])
        assert c.num_rendered == got[v]["rendered"]
    g2 = host(tr.grads.arena)
    assert np.linalg.norm(g2 - gpu_grads) <= 1e-5 * np.linalg.norm(gpu_grads)
    del tr

    sc = O.Scene(arrays)
    ref_cfg = O.default_config(binning=_abi.GSC_BIN_REFERENCE)
    tx, ty = (W + 15) // 16, (H + 15) // 16
    end_bit = 32 + int(np.ceil(np.log2(tx * ty)))
    FIELDS = importlib.import_module("crystal-gausplat_b200.gaussian").FIELDS
    ref_grads = f32_grads = None
    ref_loss = 0.0
    for v in range(views):
        cs = cams[v].to_struct()
        pre = O.preprocess(sc, cs, ref_cfg)
        keys, vals = O.emit_keys(pre, tx, ty)
        sk, sv = O.sort_pairs(keys, vals, 0, end_bit)
        del keys, vals
        ck, cv = O.contributing_lists(W, H, sk, sv, pre, ref_cfg.alpha_min)
        assert got[v]["rendered"] == ck.size  # contributing pairs before occlusion
        # compositing over the contributing lists gives every pixel's last
        # contributor; the GPU's final lists are those lists cut after each
        # tile's largest `last`, bit for bit
        cr = O.tile_ranges(ck, tx * ty)
        img_c, nc_c, fT_c, last_c = O.composite_forward(W, H, cr, cv, pre, ref_cfg)
        np.testing.assert_array_equal(got[v]["last"], last_c)
        ok, ov, orr = O.occluded_lists(W, H, ck, cv, cr, last_c)
        np.testing.assert_array_equal(got[v]["keys"], ok)
        np.testing.assert_array_equal(got[v]["vals"], ov)
        np.testing.assert_array_equal(got[v]["ranges"], orr)
        assert ok.size < ck.size
        # ... which are an order-preserving subset of the reference's sorted lists
        assert ck.size < sk.size
        # (tile, id) pairs are unique: locate each contributing pair in the
        # reference list; the positions must rise (order preserved)
        pr = (sk >> np.uint64(32) << np.uint64(32)) | sv.astype(np.uint64)
        pc = (ck >> np.uint64(32) << np.uint64(32)) | cv.astype(np.uint64)
        o = np.argsort(pr, kind="stable")
        pos = o[np.searchsorted(pr[o], pc)]
        np.testing.assert_array_equal(pr[pos], pc)
        assert np.all(np.diff(pos) > 0)
        np.testing.assert_array_equal(sk[pos], ck)
        del pr, pc, o, pos
        # the image over the reference lists equals the GPU's over the contributing lists
        ranges = O.tile_ranges(sk, tx * ty)
        img, nc, fT, last = O.composite_forward(W, H, ranges, sv, pre, ref_cfg)
        np.testing.assert_array_equal(img_c, img)
        np.testing.assert_array_equal(got[v]["image"], img)
        np.testing.assert_array_equal(got[v]["n_contrib"], nc)
        np.testing.assert_array_equal(got[v]["final_T"], fT)
        view_ref = {"ranges": ranges, "sorted_vals": sv, "pre": pre, "final_T": fT, "last": last, "image": img}
        ex, lv = oracle_backward(O, sc, cs, ref_cfg, view_ref, targets[v], W, H, exact=True)
        f32, _ = oracle_backward(O, sc, cs, ref_cfg, view_ref, targets[v], W, H, exact=False)
        ref_loss += lv
        flat = [np.concatenate([d[k].reshape(-1).astype(np.float64) for k, _ in FIELDS]) for d in (ex, f32)]
        ref_grads = flat[0] if ref_grads is None else ref_grads + flat[0]
        f32_grads = flat[1] if f32_grads is None else f32_grads + flat[1]
        del sk, sv, ck, cv, ex, f32, flat
    assert abs(gpu_loss - ref_loss) <= 1e-5 * abs(ref_loss)
    # the arena holds the five gradient fields in the same order, each block
    # padded to a 16-byte boundary
    n = 3_000_000
    parts = []
    gsmod = importlib.import_module("crystal-gausplat_b200.gaussian")
    offs, _ = gsmod.field_offsets(n)
    for name, w in gsmod.FIELDS:
        parts.append(gpu_grads[offs[name]: offs[name] + n * w].astype(np.float64))
    got_flat = np.concatenate(parts)
    start = 0
    for name, w in gsmod.FIELDS:
        sl = slice(start, start + n * w)
        gate(name, got_flat[sl], ref_grads[sl], f32_grads[sl])
        start += n * w
