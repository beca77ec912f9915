"""Known-answer tests pinning the CPU oracle (the reference ships no golden
vectors for this path, so these are derived from the mathematics)."""
import math

import numpy as np
import pytest

from helpers import _abi, gs


def test_expf_within_one_ulp(oracle):
    x = np.concatenate([np.linspace(-103.9, 88.7, 200001, dtype=np.float32),
                        np.float32([0.0, -0.0, 1.0, -1.0, 1e-30, -5.55, 88.72, -87.3])])
    got = oracle.expf(x).astype(np.float64)
    ref = np.exp(x.astype(np.float64))
    normal = ref > np.finfo(np.float32).tiny
    ulp = np.spacing(ref[normal].astype(np.float32)).astype(np.float64)
    assert np.max(np.abs(got[normal] - ref[normal]) / ulp) <= 1.0
    sub = ~normal
    assert np.all(np.abs(got[sub] - ref[sub]) <= 2 * 1.4e-45)
    s = oracle.expf(np.float32([np.inf, -np.inf, np.nan, 100.0, -200.0]))
    assert s[0] == np.inf and s[1] == 0.0 and np.isnan(s[2]) and s[3] == np.inf and s[4] == 0.0


def one_gaussian(gs, n=1, **over):
    a = gs.synthetic_arrays(n, 1)
    a["position"][:] = 0.0
    a["log_scale"][:] = np.float32(math.log(0.05))
    a["rotation"][:] = np.float32([1, 0, 0, 0])
    a["logit_opacity"][:] = 0.0
    a["sh_coeffs"][:] = 0.0
    for k, v in over.items():
        a[k][:] = v
    return a


def test_single_isotropic_gaussian(gs, oracle):
    W = H = 64
    a = one_gaussian(gs)
    a["sh_coeffs"][0, 0, :] = np.float32([1.0, 0.0, -1.0])  # DC: colour = 0.5 + C0 * dc
    cam = gs.make_camera(W, H, (0.0, 0.0, 4.0)).to_struct()
    cfg = gs.default_config(background=(0.1, 0.2, 0.3))
    r = oracle.forward_pipeline(oracle.Scene(a), cam, cfg)
    pre = r["pre"]
    fx = cam.fx
    assert pre["mean2d"][0] == pytest.approx([32.0, 32.0], abs=1e-5)
    assert pre["depth"][0] == pytest.approx(4.0, rel=1e-6)
    var = (fx * 0.05 / 4.0) ** 2
    assert pre["cov2d"][0] == pytest.approx([var + 0.3, 0.0, var + 0.3], rel=1e-5, abs=1e-6)
    assert pre["radius"][0] == math.ceil(3 * math.sqrt(var + 0.3))
    c0 = 0.28209479177387814
    col = np.array([0.5 + c0, 0.5, max(0.0, 0.5 - c0)])
    assert pre["colors"][0] == pytest.approx(col, rel=1e-6)
    assert pre["opacity"][0] == pytest.approx(0.5)
    # pixel (31, 31) has centre (31.5, 31.5): d = (-0.5, -0.5)
    A = 1.0 / (var + 0.3)
    alpha = 0.5 * math.exp(-0.5 * (0.25 * A + 0.25 * A))
    want = alpha * col + (1 - alpha) * np.array([0.1, 0.2, 0.3])
    assert r["image"][31, 31] == pytest.approx(want, rel=1e-5)
    assert r["n_contrib"][31, 31] == 1
    assert r["final_T"][31, 31] == pytest.approx(1 - alpha, rel=1e-6)
    # far corner: outside the support -> background, no contributor
    assert r["image"][0, 0] == pytest.approx([0.1, 0.2, 0.3])
    assert r["n_contrib"][0, 0] == 0


def test_two_gaussians_front_to_back(gs, oracle):
    W = H = 32
    a = one_gaussian(gs, n=2)
    a["position"][0] = [0.0, 0.0, -0.5]   # farther from the camera at z = +4
    a["position"][1] = [0.0, 0.0, 0.5]    # nearer
    a["sh_coeffs"][0, 0, :] = [1.5, 0.0, 0.0]
    a["sh_coeffs"][1, 0, :] = [0.0, 0.0, 1.5]
    a["logit_opacity"][:] = 1.0
    cam = gs.make_camera(W, H, (0.0, 0.0, 4.0)).to_struct()
    cfg = gs.default_config()
    r = oracle.forward_pipeline(oracle.Scene(a), cam, cfg)
    ranges = r["ranges"].reshape(-1, 2)
    t = 0  # tile (0,0) holds both, nearer first
    lst = r["sorted_vals"][ranges[t, 0]:ranges[t, 1]]
    assert list(lst) == [1, 0]
    pre = r["pre"]
    px = 15
    a_near = r["image"][px, px]
    def alpha(g):
        mx, my = pre["mean2d"][g]
        ca, cb, cc = pre["cov2d"][g].astype(np.float64)
        det = ca * cc - cb * cb
        dx, dy = px + 0.5 - mx, px + 0.5 - my
        p = -0.5 * (dx * dx * cc / det - 2 * dx * dy * cb / det + dy * dy * ca / det)
        return min(0.99, pre["opacity"][g] * math.exp(p))
    a1, a0 = alpha(1), alpha(0)
    want = a1 * pre["colors"][1] + (1 - a1) * a0 * pre["colors"][0]
    assert a_near == pytest.approx(want, rel=1e-5)


def test_all_culled_gives_background(gs, oracle):
    a = gs.synthetic_arrays(50, 2)
    a["position"][:, 2] = 9.0  # behind a camera at z=4 looking toward -z
    cam = gs.make_camera(40, 24, (0.0, 0.0, 4.0)).to_struct()
    cfg = gs.default_config(background=(0.25, 0.5, 0.75))
    r = oracle.forward_pipeline(oracle.Scene(a), cam, cfg)
    assert r["keys"].size == 0
    assert not r["ranges"].any()
    assert np.all(r["image"] == np.float32([0.25, 0.5, 0.75]))
    assert np.all(r["pre"]["mean2d"] == -1000.0) and np.all(r["pre"]["radius"] == 0.0)


def test_sort_is_stable_and_ranges_mark_empty_tiles(oracle):
    keys = np.array([(3 << 32) | 7, (1 << 32) | 9, (3 << 32) | 7, (1 << 32) | 2, (3 << 32) | 1],
                    dtype=np.uint64)
    vals = np.arange(5, dtype=np.uint32)
    k, v = oracle.sort_pairs(keys, vals)
    assert list(v) == [3, 1, 4, 0, 2]
    r = oracle.tile_ranges(k, 5).reshape(-1, 2)
    assert r.tolist() == [[0, 0], [0, 2], [0, 0], [2, 5], [0, 0]]
    # partial bit range: only bits [32, 64) -> ties broken by input order
    k2, v2 = oracle.sort_pairs(keys, vals, 32, 64)
    assert list(v2) == [1, 3, 0, 2, 4]


def test_key_emission_canonical_order(gs, oracle):
    a = one_gaussian(gs, n=2)
    a["log_scale"][:] = np.float32(math.log(0.2))  # spans several tiles
    cam = gs.make_camera(64, 64, (0.0, 0.0, 4.0)).to_struct()
    cfg = gs.default_config()
    pre = oracle.preprocess(oracle.Scene(a), cam, cfg)
    keys, vals = oracle.emit_keys(pre, 4, 4)
    assert keys.size == int(pre["tiles_touched"].sum())
    assert list(vals) == [0] * (keys.size // 2) + [1] * (keys.size // 2)
    tiles = (keys >> np.uint64(32)).astype(np.int64)[: keys.size // 2]
    assert np.all(np.diff(tiles) > 0)  # ty outer, tx inner, ascending
    assert np.all((keys & np.uint64(0xFFFFFFFF)) == np.float32(pre["depth"][0]).view(np.uint32))


def test_adam_closed_form_and_float32_order(oracle):
    rng = np.random.default_rng(0)
    n = 1000
    p0 = rng.standard_normal(n).astype(np.float32)
    g = rng.standard_normal(n).astype(np.float32)
    grp = {"param": p0.copy(), "grad": g, "m": np.zeros(n, np.float32), "v": np.zeros(n, np.float32),
           "lr": 1e-2, "weight_decay": 0.0}
    oracle.adam_step([grp], 0.9, 0.999, 1e-8, 1)
    # step 1: m_hat = g, v_hat = g^2  ->  p - lr * g / (|g| + eps)
    np.testing.assert_allclose(grp["param"], p0 - 1e-2 * g / (np.abs(g) + 1e-8), rtol=0, atol=2e-7)
    # the documented fp32 order, restated in numpy
    for step in (2, 3):
        p, m, v = grp["param"].copy(), grp["m"].copy(), grp["v"].copy()
        oracle.adam_step([grp], 0.9, 0.999, 1e-8, step, 0.5)
        f = np.float32
        gr = g * f(0.5)
        m = f(0.9) * m + (f(1) - f(0.9)) * gr
        v = f(0.999) * v + (f(1) - f(0.999)) * gr * gr
        bc1 = f(1) - powi_f32(f(0.9), step)  # beta^t as Float32#**(Int32)
        bc2 = f(1) - powi_f32(f(0.999), step)
        p = p - f(1e-2) * (m / bc1) / (np.sqrt(v / bc2) + f(1e-8))
        np.testing.assert_array_equal(grp["param"], p)
        np.testing.assert_array_equal(grp["m"], m)


def powi_f32(a, b):
    """Binary exponentiation in float32, lowest exponent bit first: what
    Float32#**(Int32) runs in the reference's Adam (adam.cr:129-130)."""
    a, r = np.float32(a), np.float32(1)
    while True:
        if b & 1:
            r = np.float32(r * a)
        b //= 2
        if b == 0:
            return r
        a = np.float32(a * a)


def test_powi_f32_is_the_references_fp32_power(oracle):
    f = np.float32
    for beta in (f(0.9), f(0.999)):
        assert oracle.powi_f32(beta, 1) == beta
        assert oracle.powi_f32(beta, 2) == f(beta * beta)
        assert oracle.powi_f32(beta, 3) == f(f(beta) * f(beta * beta))  # r = a, then a^2 * r
        for t in list(range(1, 200)) + [1000, 4095, 4096, 30000]:
            got = oracle.powi_f32(beta, t)
            assert got == powi_f32(beta, t), (beta, t)
            # each squaring doubles the relative error it inherits, so the
            # relative error of the fp32 power stays below t * 2^-23
            exact = np.float64(beta) ** t
            if exact > 1e-30:
                assert abs(float(got) / exact - 1.0) <= t * 2.0 ** -23, (beta, t)


def test_l1_loss_grad(oracle):
    a = np.float32([0.5, 0.2, 0.3, 0.9])
    b = np.float32([0.1, 0.2, 0.7, 0.0])
    loss, g = oracle.l1_loss_grad(a, b, 0.25)
    assert loss == pytest.approx((0.4 + 0.0 + 0.4 + 0.9) / 4, rel=1e-6)
    assert g.tolist() == [0.25, 0.0, -0.25, 0.25]


def test_ref_mode_sh_truncation(gs, oracle):
    """REF mode evaluates degree 2 for the red channel only and no degree 3
    (gaussian.metal:290-302); FULL evaluates every coefficient."""
    a = one_gaussian(gs)
    a["sh_coeffs"][0, 4:, :] = 0.3
    cam = gs.make_camera(32, 32, (1.0, 2.0, 3.0)).to_struct()
    full = oracle.preprocess(oracle.Scene(a), cam, gs.default_config())["colors"][0]
    ref = oracle.preprocess(oracle.Scene(a), cam, gs.default_config(mode=gs.GSC_MODE_REF))["colors"][0]
    assert ref[1] == pytest.approx(0.5) and ref[2] == pytest.approx(0.5)
    assert ref[0] != pytest.approx(0.5)
    assert full[1] != pytest.approx(0.5)


@pytest.mark.parametrize("seed", [1, 2])
def test_oracle_contributing_lists_render_identically(oracle, seed):
    """Dropping the pairs the exact whole-tile test rejects changes no pixel."""
    a = gs.synthetic_arrays(4000, seed)
    a["log_scale"] = (a["log_scale"] + np.float32(0.8)).astype(np.float32)  # larger footprints
    cam = gs.make_camera(97, 75, (0.3, -0.2, 3.0)).to_struct()
    sc = oracle.Scene(a)
    ref = oracle.forward_pipeline(sc, cam, gs.default_config(binning=_abi.GSC_BIN_REFERENCE))
    con = oracle.forward_pipeline(sc, cam, gs.default_config(binning=_abi.GSC_BIN_CONTRIBUTING))
    assert 0 < con["sorted_keys"].size < 0.9 * ref["sorted_keys"].size
    for k in ("image", "n_contrib", "final_T"):
        np.testing.assert_array_equal(con[k], ref[k], err_msg=k)


def test_oracle_contributing_lists_adversarial(oracle):
    """Gaussians at the edge of the cull: opacities just above alpha_min,
    strongly elongated conics, means on tile borders. No pixel may change."""
    rng = np.random.default_rng(7)
    n = 6000
    a = gs.synthetic_arrays(n, 7)
    cam = gs.make_camera(96, 80, (0.0, 0.0, 3.0))
    # opacity in (1/255, 3/255]: logit = ln(o / (1 - o))
    o = rng.uniform(1.0001 / 255, 3.0 / 255, n)
    a["logit_opacity"][:, 0] = np.log(o / (1 - o)).astype(np.float32)
    # elongated: one axis 20x another
    a["log_scale"][:, 0] = rng.uniform(-4.0, -2.5, n).astype(np.float32)
    a["log_scale"][:, 1] = (a["log_scale"][:, 0] - np.float32(3.0)).astype(np.float32)
    a["position"][:, 2] = rng.uniform(-0.2, 0.2, n).astype(np.float32)
    sc = oracle.Scene(a)
    cs = cam.to_struct()
    ref = oracle.forward_pipeline(sc, cs, gs.default_config(binning=_abi.GSC_BIN_REFERENCE))
    con = oracle.forward_pipeline(sc, cs, gs.default_config(binning=_abi.GSC_BIN_CONTRIBUTING))
    assert con["sorted_keys"].size < ref["sorted_keys"].size
    for k in ("image", "n_contrib", "final_T"):
        np.testing.assert_array_equal(con[k], ref[k], err_msg=k)


@pytest.mark.parametrize("n,begin,end", [(1, 0, 64), (1000, 0, 64), (300_001, 0, 45), (1 << 20, 8, 40)])
def test_oracle_sort_is_numpys_stable_sort(oracle, n, begin, end):
    """The oracle's pair sort (parallel chunks + stable merges) against
    numpy's stable argsort of the same key bits, duplicates included."""
    rng = np.random.default_rng(n)
    keys = rng.integers(0, 2**63, n, dtype=np.uint64) * np.uint64(2) + rng.integers(0, 2, n, dtype=np.uint64)
    keys[: n // 3] = keys[n // 3: 2 * (n // 3)]
    vals = np.arange(n, dtype=np.uint32)
    oracle.set_threads(8)
    try:
        k, v = oracle.sort_pairs(keys, vals, begin, end)
    finally:
        oracle.set_threads(1)
    sel = (keys >> np.uint64(begin)) & np.uint64((1 << (end - begin)) - 1 if end - begin < 64 else 2**64 - 1)
    order = np.argsort(sel, kind="stable")
    np.testing.assert_array_equal(v, vals[order])
    np.testing.assert_array_equal(k, keys[order])
