"""Host-side logic: camera conventions, the parameter arena, bench helpers."""
import math

import numpy as np
import pytest


def test_look_at_is_opencv(gs):
    cam = gs.make_camera(200, 100, (0.0, 0.0, 4.0))
    W = cam.world_to_camera
    # the target projects to the principal point, in front of the camera
    p = W @ np.array([0, 0, 0, 1.0])
    assert p[2] == pytest.approx(4.0) and abs(p[0]) < 1e-12 and abs(p[1]) < 1e-12
    # world +Y (up) maps to image -y (rows grow downward); +X to image +x
    assert (W @ np.array([0, 1, 0, 1.0]))[1] < 0
    assert (W @ np.array([1, 0, 0, 1.0]))[0] > 0
    np.testing.assert_allclose(cam.position, [0, 0, 4], atol=1e-12)
    k = cam.intrinsics
    assert k.fx == pytest.approx(100 / math.tan(math.radians(30)))
    assert k.fy == k.fx and k.cx == 100 and k.cy == 50
    s = cam.to_struct()
    assert s.width == 200 and s.tan_fov_x == pytest.approx(math.tan(math.radians(30)), rel=1e-6)


def test_look_at_straight_down(gs):
    cam = gs.make_camera(64, 64, (0.0, 5.0, 0.0))  # forward parallel to world up
    R = cam.world_to_camera[:3, :3]
    np.testing.assert_allclose(R @ R.T, np.eye(3), atol=1e-12)


def test_gaussian_arena_layout(gs):
    import torch
    a = gs.synthetic_arrays(7, 3)
    g = gs.Gaussian3D(a, device="cpu")
    assert g.arena.numel() >= 7 * 59
    for name, t in zip(("position", "log_scale", "rotation", "logit_opacity", "sh_coeffs"), g.parameters()):
        assert t.data_ptr() % 16 == 0
        np.testing.assert_array_equal(t.numpy(), a[name].reshape(t.shape))
    v = g.views_of(torch.arange(g.arena.numel(), dtype=torch.float32))
    assert v["rotation"].shape == (7, 4) and v["sh_coeffs"].shape == (7, 16, 3)


def test_synthetic_distributions(gs):
    a = gs.synthetic_arrays(200000, 5, extent=3.0)
    assert np.abs(a["position"]).max() <= 3.0
    assert a["log_scale"].mean() == pytest.approx(-4.5, abs=0.01)
    assert a["log_scale"].std() == pytest.approx(0.5, abs=0.01)
    np.testing.assert_allclose(np.linalg.norm(a["rotation"], axis=1), 1.0, rtol=1e-5)
    assert a["sh_coeffs"][:, 0].std() == pytest.approx(0.5, abs=0.01)
    assert a["sh_coeffs"][:, 1:].std() == pytest.approx(0.1, abs=0.01)


def test_bench_work_model():
    import bench
    assert bench.sort_bytes_per_pair(45) == 8 + 24 * 6
    assert bench.sort_bytes_per_pair(13, 4) == 4 + 16 * 2
    # histogram read, 16 B per pass, the last pass writing 4 B ids (+ 4 B keys)
    assert bench.packed_sort_bytes(32, hi=True) == 8 + 16 * 4
    assert bench.packed_sort_bytes(13, hist=False) == 16 + 12
    w = bench.stage_work(1000, 5000, 5000, 10 ** 6, 8160, 45)
    assert w["adam"] == ("hbm", 1652 * 1000)
    assert w["preprocess"][1] == (236 + 88) * 1000
    w8 = bench.stage_work(1000, 5000, 5000, 10 ** 6, 8160, 45, batch=8)
    assert w8["preprocess"] == ("hbm", (236 / 8 + 88) * 1000)
    assert w8["preprocess_bwd"] == ("hbm", (3 * 236 / 8 + 36) * 1000)
    # batched depth words: 28 + 3 bits (4 passes); tile sort: digits counted by emission
    assert w8["sort"] == ("hbm", (8 + 16 * 3 + 12) * 1000 + (16 + 12) * 5000)
    assert w8["ranges"] == ("hbm", 8 * 8160)
    # Adam: once per step over every parameter, shared by the step's views
    assert bench.stage_work(1000, 1, 1, 1, 8160, 45, views_per_step=4)["adam"] == ("hbm", 1652 * 1000 / 4)
    # occluded binning: the binned pairs are sorted, the later slice gathers again,
    # two slices of ranges and the kept ids copied
    wo = bench.stage_work(1000, 2000, 300, 10 ** 6, 8160, 45, batch=8, occluded=True)
    assert wo["sort"][1] == (8 + 16 * 3 + 12) * 1000 + (16 + 12) * 2000
    assert wo["emit"][1] == 36 * 1000 + 8 * 2000
    assert wo["scan"][1] == 20 * 1000 + 36 * 800
    assert wo["ranges"][1] == 8 * 8160 * 2 + 8 * 300 + 8 * 8160
    # with the per-tile cut both slices count over every position
    wc = bench.stage_work(1000, 2000, 300, 10 ** 6, 8160, 45, batch=8, occluded=True, tile_cut=True)
    assert wc["scan"][1] == 2 * 48 * 1000 and wc["emit"][1] == 8 * 1000 + 8 * 2000
    r = bench.rooflines({"adam": {"ms": 2.0, "calls": 1, "kernels": 1}}, {"adam": ("hbm", 1e9)},
                        {"hbm_gbs": 1000.0}, 2)
    assert r["adam"]["achieved"] == 1000.0 and r["adam"]["ms_per_view"] == 1.0
