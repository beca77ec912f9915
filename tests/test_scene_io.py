"""Scene I/O: COLMAP text/binary models, CameraSet.from_colmap,
Gaussian3D.from_points, PLY and PNG round trips (host code; one GPU test
trains on a loaded scene)."""
import math
import struct
import zlib

import numpy as np
import pytest

from helpers import gs

sio = gs.scene_io


def model(n_views=5, n_points=200, seed=0):
    cams = [gs.make_camera(64 + 8 * i, 48 + 4 * i, tuple(e)) for i, e in
            enumerate(gs.sphere_poses(n_views, 4.0, seed=seed))]
    ccams, imgs = sio.colmap_model_of(cams)
    rng = np.random.default_rng(seed)
    xyz = rng.uniform(-1, 1, (n_points, 3))
    rgb = rng.integers(0, 256, (n_points, 3)).astype(np.uint8)
    return cams, ccams, imgs, (xyz, rgb)


def reference_w2c(q, t):
    """COLMAPImage#world_to_camera (colmap_loader.cr:74-138) restated."""
    qw, qx, qy, qz = q
    n = math.sqrt(qw * qw + qx * qx + qy * qy + qz * qz)
    w, x, y, z = qw / n, qx / n, qy / n, qz / n
    r = [1.0 - 2.0 * (y * y + z * z), 2.0 * (x * y - z * w), 2.0 * (x * z + y * w),
         2.0 * (x * y + z * w), 1.0 - 2.0 * (x * x + z * z), 2.0 * (y * z - x * w),
         2.0 * (x * z - y * w), 2.0 * (y * z + x * w), 1.0 - 2.0 * (x * x + y * y)]
    m = np.zeros(16, np.float32)
    for i in range(3):
        for j in range(3):
            m[i * 4 + j] = np.float32(r[i * 3 + j])
        m[i * 4 + 3] = np.float32(t[i])
    m[15] = 1
    return m.reshape(4, 4)


@pytest.mark.parametrize("fmt", ["text", "binary"])
def test_colmap_round_trip(tmp_path, fmt):
    cams, ccams, imgs, pts = model()
    (sio.save_colmap_text if fmt == "text" else sio.save_colmap_binary)(tmp_path, ccams, imgs, pts)
    L = gs.load_colmap(str(tmp_path))
    assert sorted(L.cameras) == [c.id for c in ccams] and sorted(L.images) == [i.id for i in imgs]
    for c in ccams:
        assert L.cameras[c.id].params == c.params and L.cameras[c.id].model == "PINHOLE"
    for im in imgs:
        li = L.images[im.id]
        assert li.q == im.q and li.t == im.t and li.name == im.name and li.camera_id == im.camera_id
        np.testing.assert_array_equal(li.world_to_camera(), reference_w2c(im.q, im.t))
    np.testing.assert_array_equal(L.points_xyz, pts[0])
    np.testing.assert_array_equal(L.points_rgb, pts[1])
    np.testing.assert_array_equal(L.colors_tensor().numpy(), pts[1].astype(np.float32) / np.float32(255))
    loaded = L.gs_cameras()
    for c, lc in zip(cams, loaded):
        np.testing.assert_allclose(lc.world_to_camera, c.world_to_camera, atol=1e-6)
        np.testing.assert_allclose(lc.position, c.position, atol=1e-5)
        assert lc.intrinsics.fx == np.float32(c.intrinsics.fx)


def test_colmap_text_edge_cases(tmp_path):
    (tmp_path / "cameras.txt").write_text(
        "# c\n1 SIMPLE_RADIAL 100 80 90.0 50.0 40.0 0.01\n2 WEIRD_MODEL 10 10 5 6 7 8\n")
    # image 1 has no 2D points (empty line); image 2 has four (12 fields)
    (tmp_path / "images.txt").write_text(
        "# i\n1 1 0 0 0 0.1 0.2 0.3 1 a.png\n\n"
        "2 0.5 0.5 0.5 0.5 1 2 3 2 b.png\n1.0 2.0 -1 3.0 4.0 -1 5.0 6.0 7 8.0 9.0 -1\n")
    L = gs.load_colmap(str(tmp_path))
    assert sorted(L.images) == [1, 2] and L.images[2].name == "b.png"
    k = L.cameras[1].intrinsics()
    assert (k.fx, k.fy, k.cx, k.cy) == (90.0, 90.0, 50.0, 40.0)
    assert L.cameras[2].model == "PINHOLE"   # unknown name -> PINHOLE, as the reference
    assert len(L.points_xyz) == 0 and len(L.gs_cameras()) == 2
    # CameraSet.from_colmap knows only PINHOLE / SIMPLE_PINHOLE intrinsics
    cs = gs.CameraSet.from_colmap(str(tmp_path / "images.txt"), str(tmp_path / "cameras.txt"))
    assert len(cs) == 0
    (tmp_path / "cameras.txt").write_text("1 SIMPLE_RADIAL 100 80 90.0 50.0 40.0 0.01\n"
                                          "2 PINHOLE 10 10 5 6 7 8\n")
    cs = gs.CameraSet.from_colmap(str(tmp_path / "images.txt"), str(tmp_path / "cameras.txt"))
    assert len(cs) == 1 and cs[0].image_path == "b.png" and cs[0].intrinsics.fy == 6.0


def test_colmap_binary_model_table(tmp_path):
    """OPENCV_FISHEYE (id 5) has 8 parameters in COLMAP's table."""
    cams = [sio.COLMAPCamera(1, "OPENCV_FISHEYE", 10, 10, [1, 2, 3, 4, 5, 6, 7, 8]),
            sio.COLMAPCamera(2, "SIMPLE_PINHOLE", 10, 10, [9, 5, 5])]
    imgs = [sio.COLMAPImage(1, 2, "x.png", 1, 0, 0, 0, 0, 0, 0)]
    sio.save_colmap_binary(tmp_path, cams, imgs)
    L = gs.load_colmap(str(tmp_path))
    assert L.cameras[1].params == [1, 2, 3, 4, 5, 6, 7, 8] and L.cameras[2].params == [9, 5, 5]
    raw = bytearray((tmp_path / "cameras.bin").read_bytes())
    struct.pack_into("<i", raw, 12, 99)
    (tmp_path / "cameras.bin").write_bytes(bytes(raw))
    with pytest.raises(ValueError):
        gs.load_colmap(str(tmp_path))


def test_camera_set_from_colmap_fp32(tmp_path):
    cams, ccams, imgs, _ = model(3)
    sio.save_colmap_text(tmp_path, ccams, imgs)
    cs = gs.CameraSet.from_colmap(str(tmp_path / "images.txt"), str(tmp_path / "cameras.txt"))
    assert len(cs) == 3
    for c, lc in zip(cams, cs):
        np.testing.assert_allclose(lc.world_to_camera, c.world_to_camera, atol=2e-6)


def test_from_points_and_ply_round_trip(tmp_path):
    rng = np.random.default_rng(1)
    pts = rng.uniform(-1, 1, (50, 3)).astype(np.float32)
    col = rng.random((50, 3), dtype=np.float32)
    g = sio.from_points(pts, col, device="cpu")
    np.testing.assert_array_equal(g.position.numpy(), pts)
    np.testing.assert_array_equal(g.sh_coeffs[:, 0, :].numpy(), col / sio.SH_C0)
    assert float(g.sh_coeffs[:, 1:, :].abs().sum()) == 0.0
    assert np.all(g.log_scale.numpy() == -3.0) and np.all(g.logit_opacity.numpy() == 0.0)
    np.testing.assert_array_equal(g.rotation.numpy(), np.tile([1, 0, 0, 0], (50, 1)))
    h = gs.Gaussian3D(gs.synthetic_arrays(77, 3), device="cpu")
    sio.save_ply(h, str(tmp_path / "g.ply"))
    h2 = sio.load_ply(str(tmp_path / "g.ply"), device="cpu")
    for f in ("position", "log_scale", "rotation", "logit_opacity", "sh_coeffs"):
        np.testing.assert_array_equal(getattr(h2, f).numpy(), getattr(h, f).numpy(), err_msg=f)
    head = (tmp_path / "g.ply").read_bytes()[:2000].decode("latin1")
    assert "property float f_rest_44" in head and "element vertex 77" in head
    # channel-major f_rest: f_rest_15 is coefficient 1 of green
    raw = (tmp_path / "g.ply").read_bytes()
    data = np.frombuffer(raw[raw.index(b"end_header\n") + 11:], "<f4").reshape(77, 62)
    np.testing.assert_array_equal(data[:, 9 + 15], h.sh_coeffs[:, 1, 1].numpy())


def _png_filtered(a, filters):
    """PNG encoder applying the given per-row filter types (PNG 1.2, 6.3)."""
    h, w, ch = a.shape
    rows = a.reshape(h, w * ch).astype(np.int32)
    out = []
    prev = np.zeros(w * ch, np.int32)
    for y in range(h):
        f, r = filters[y % len(filters)], rows[y]
        left = np.concatenate([np.zeros(ch, np.int32), r[:-ch]])
        ul = np.concatenate([np.zeros(ch, np.int32), prev[:-ch]])
        if f == 0:
            e = r
        elif f == 1:
            e = r - left
        elif f == 2:
            e = r - prev
        elif f == 3:
            e = r - ((left + prev) >> 1)
        else:
            p = left + prev - ul
            pa, pb, pc = np.abs(p - left), np.abs(p - prev), np.abs(p - ul)
            e = r - np.where((pa <= pb) & (pa <= pc), left, np.where(pb <= pc, prev, ul))
        out.append(np.concatenate([[f], e & 255]).astype(np.uint8))
        prev = r
    body = zlib.compress(np.concatenate(out).tobytes())

    def chunk(t, b):
        return struct.pack(">I", len(b)) + t + b + struct.pack(">I", zlib.crc32(t + b) & 0xFFFFFFFF)
    ctype = {1: 0, 2: 4, 3: 2, 4: 6}[ch]
    return (b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, ctype, 0, 0, 0))
            + chunk(b"IDAT", body) + chunk(b"IEND", b""))


@pytest.mark.parametrize("ch", [1, 2, 3, 4])
def test_png_round_trip_all_filters(tmp_path, ch):
    a = np.random.default_rng(ch).integers(0, 256, (13, 11, ch)).astype(np.uint8)
    p = tmp_path / "f.png"
    p.write_bytes(_png_filtered(a, [0, 1, 2, 3, 4]))
    img = gs.load_png(str(p))
    assert (img.width, img.height, img.channels) == (11, 13, ch)
    np.testing.assert_array_equal(img.data, a)
    gs.save_png(str(tmp_path / "g.png"), a)
    np.testing.assert_array_equal(gs.load_png(str(tmp_path / "g.png")).data, a)
    np.testing.assert_array_equal(img.to_tensor().numpy(), a.astype(np.float32) / np.float32(255))


@pytest.mark.gpu
def test_train_on_loaded_colmap_scene(cuda, tmp_path):
    """A COLMAP scene written to disk, loaded back, initialised from its points
    and trained for a few steps on targets rendered from a reference scene."""
    import torch
    trainer = __import__("importlib").import_module("crystal-gausplat_b200.trainer")
    cams, ccams, imgs, (xyz, rgb) = model(4, 3000, seed=5)
    ccams = [sio.COLMAPCamera(c.id, c.model, 96, 80, [83.1, 83.1, 48.0, 40.0]) for c in ccams]
    sio.save_colmap_binary(tmp_path, ccams, imgs, (xyz, rgb))
    L = gs.load_colmap(str(tmp_path))
    views = L.gs_cameras()
    truth = gs.Gaussian3D(gs.synthetic_arrays(3000, 9))
    targets = [gs.Rasterizer.forward(truth, v)[0].clone() for v in views]
    g = sio.from_points(L.points_tensor(), L.colors_tensor())
    g.log_scale.fill_(-4.0)
    tr = trainer.DataParallelTrainer(g, views, gs.default_config())
    losses = [float(tr.step(lambda v: targets[v])) for _ in range(20)]
    assert losses[-1] < losses[0]
    sio.save_png(str(tmp_path / "r.png"), gs.Rasterizer.forward(g, views[0])[0].clamp(0, 1).cpu())
    assert gs.load_png(str(tmp_path / "r.png")).data.shape == (80, 96, 3)


def literal_resize_target(a, dw, dh, dc):
    """ImageIO.resize (image_io.cr:289-335) + to_tensor, in numpy fp32 scalars."""
    f = np.float32
    sh, sw, sc = a.shape
    if (sw, sh) == (dw, dh):
        return a[:, :, :dc].astype(np.float32) / f(255)
    out = np.zeros((dh, dw, dc), np.float32)
    kx, ky = f(sw) / f(dw), f(sh) / f(dh)
    for y in range(dh):
        for x in range(dw):
            sx = min(max(f(f(f(x) + f(0.5)) * kx) - f(0.5), f(0)), f(sw - 1))
            sy = min(max(f(f(f(y) + f(0.5)) * ky) - f(0.5), f(0)), f(sh - 1))
            x0, y0 = min(max(int(sx), 0), sw - 1), min(max(int(sy), 0), sh - 1)
            x1, y1 = min(x0 + 1, sw - 1), min(y0 + 1, sh - 1)
            fx, fy = f(sx - f(x0)), f(sy - f(y0))
            for c in range(dc):
                v00, v10, v01, v11 = (f(a[y0, x0, c]), f(a[y0, x1, c]), f(a[y1, x0, c]), f(a[y1, x1, c]))
                v0 = f(f(v00 * f(f(1) - fx)) + f(v10 * fx))
                v1 = f(f(v01 * f(f(1) - fx)) + f(v11 * fx))
                v = f(f(v0 * f(f(1) - fy)) + f(v1 * fy))
                out[y, x, c] = f(int(min(max(v, f(0)), f(255)))) / f(255)
    return out


@pytest.mark.parametrize("shape,dst", [((13, 17, 4), (17, 13, 3)), ((13, 17, 3), (9, 5, 3)),
                                       ((8, 6, 1), (23, 19, 1)), ((7, 9, 4), (9, 7, 4))])
def test_image_target_oracle_is_the_literal_resize(oracle, shape, dst):
    a = np.random.default_rng(sum(shape)).integers(0, 256, shape).astype(np.uint8)
    dw, dh, dc = dst
    np.testing.assert_array_equal(oracle.image_to_target(a, dw, dh, dc),
                                  literal_resize_target(a, dw, dh, dc))


@pytest.mark.gpu
@pytest.mark.parametrize("shape,dst", [((1080, 1920, 4), (1920, 1080, 3)), ((1080, 1920, 3), (960, 540, 3)),
                                       ((301, 207, 4), (640, 480, 3)), ((5, 3, 1), (2, 1, 1))])
def test_cuda_image_target_bit_exact(cuda, oracle, shape, dst):
    from helpers import host
    a = np.random.default_rng(sum(shape)).integers(0, 256, shape).astype(np.uint8)
    dw, dh, dc = dst
    t = sio.image_to_target(a, dw, dh, dc)
    np.testing.assert_array_equal(host(t), oracle.image_to_target(a, dw, dh, dc))
