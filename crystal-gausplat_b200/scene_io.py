"""Scene I/O on the host: the COLMAP loader (src/utils/colmap_loader.cr,
CameraSet.from_colmap in src/gaussian_splatting/camera.cr:288-358),
Gaussian3D.from_points (gaussian.cr:86-116), 8-bit PNG images
(src/utils/image_io.cr's Image, whose loader is macOS ImageIO) and the
Gaussian PLY layout that 3DGS viewers read.

COLMAP follows its published sparse-model format: the camera-model table with
the standard ids and parameter counts (the reference maps id 5 to
FULL_OPENCV's 12 parameters, which misreads OPENCV_FISHEYE files), and an
image's 2D-point line may be empty (the reference drops empty lines before
pairing, which shifts every later image). Intrinsics take fx, fy, cx, cy
from the parameters exactly as COLMAPCamera#to_gs_camera does; distortion
is ignored, as there.
"""
import math
import os
import struct
import zlib

import numpy as np

from .camera import Camera, CameraIntrinsics

# (name, id, number of parameters, focal layout): "f" = f, cx, cy; "fxfy" = fx, fy, cx, cy
COLMAP_MODELS = (
    ("SIMPLE_PINHOLE", 0, 3, "f"), ("PINHOLE", 1, 4, "fxfy"), ("SIMPLE_RADIAL", 2, 4, "f"),
    ("RADIAL", 3, 5, "f"), ("OPENCV", 4, 8, "fxfy"), ("OPENCV_FISHEYE", 5, 8, "fxfy"),
    ("FULL_OPENCV", 6, 12, "fxfy"), ("FOV", 7, 5, "fxfy"), ("SIMPLE_RADIAL_FISHEYE", 8, 4, "f"),
    ("RADIAL_FISHEYE", 9, 5, "f"), ("THIN_PRISM_FISHEYE", 10, 12, "fxfy"),
)
MODEL_BY_NAME = {m[0]: m for m in COLMAP_MODELS}
MODEL_BY_ID = {m[1]: m for m in COLMAP_MODELS}


class COLMAPCamera:
    def __init__(self, id, model, width, height, params):
        self.id, self.model = int(id), model
        self.width, self.height = int(width), int(height)
        self.params = [float(p) for p in params]

    def intrinsics(self):
        p = self.params
        if MODEL_BY_NAME[self.model][3] == "f":
            fx = fy = p[0]
            cx, cy = p[1], p[2]
        else:
            fx, fy, cx, cy = p[0], p[1], p[2], p[3]
        f32 = np.float32
        return CameraIntrinsics(self.width, self.height, f32(fx), f32(fy), f32(cx), f32(cy))

    def to_gs_camera(self, world_to_camera):
        """COLMAPCamera#to_gs_camera (colmap_loader.cr:31-55)."""
        cam = Camera(self.intrinsics())
        cam.set_world_to_camera(world_to_camera)
        return cam


class COLMAPImage:
    def __init__(self, id, camera_id, name, qw, qx, qy, qz, tx, ty, tz):
        self.id, self.camera_id, self.name = int(id), int(camera_id), name
        self.q = (float(qw), float(qx), float(qy), float(qz))
        self.t = (float(tx), float(ty), float(tz))

    def rotation_matrix(self):
        """Normalised quaternion -> R in float64, rounded to fp32 (colmap_loader.cr:74-99)."""
        qw, qx, qy, qz = self.q
        n = math.sqrt(qw * qw + qx * qx + qy * qy + qz * qz)
        w, x, y, z = qw / n, qx / n, qy / n, qz / n
        R = np.array([
            [1.0 - 2.0 * (y * y + z * z), 2.0 * (x * y - z * w), 2.0 * (x * z + y * w)],
            [2.0 * (x * y + z * w), 1.0 - 2.0 * (x * x + z * z), 2.0 * (y * z - x * w)],
            [2.0 * (x * z - y * w), 2.0 * (y * z + x * w), 1.0 - 2.0 * (x * x + y * y)]])
        return R.astype(np.float32)

    def world_to_camera(self):
        """[R | t; 0 0 0 1] in fp32 (colmap_loader.cr:112-138)."""
        m = np.zeros((4, 4), np.float32)
        m[:3, :3] = self.rotation_matrix()
        m[:3, 3] = np.array(self.t, np.float64).astype(np.float32)
        m[3, 3] = 1.0
        return m

    def camera_center(self):
        """C = -R^T t (colmap_loader.cr:141-152)."""
        R = self.rotation_matrix().astype(np.float64)
        return tuple(-(R.T @ np.array(self.t)))


class COLMAPPoint3D:
    __slots__ = ("id", "xyz", "rgb", "error", "track_length")

    def __init__(self, id, xyz, rgb, error, track_length):
        self.id, self.xyz, self.rgb = int(id), xyz, rgb
        self.error, self.track_length = float(error), int(track_length)


class COLMAPLoader:
    """COLMAPLoader (colmap_loader.cr:171-436): text first, then binary."""

    def __init__(self, path):
        self.path = path
        self.cameras = {}
        self.images = {}
        self.points_xyz = np.zeros((0, 3), np.float64)
        self.points_rgb = np.zeros((0, 3), np.uint8)
        self.points_error = np.zeros(0, np.float64)
        self.points_id = np.zeros(0, np.int64)
        self.points_track_length = np.zeros(0, np.int32)

    def load(self):
        j = lambda f: os.path.join(self.path, f)  # noqa: E731
        if os.path.exists(j("cameras.txt")):
            self._cameras_txt(j("cameras.txt"))
            self._images_txt(j("images.txt"))
            if os.path.exists(j("points3D.txt")):
                self._points_txt(j("points3D.txt"))
        elif os.path.exists(j("cameras.bin")):
            self._cameras_bin(j("cameras.bin"))
            self._images_bin(j("images.bin"))
            if os.path.exists(j("points3D.bin")):
                self._points_bin(j("points3D.bin"))
        else:
            raise FileNotFoundError(f"No COLMAP data found in {self.path}")
        return self

    # -- outputs ------------------------------------------------------------
    @property
    def points3d(self):
        return [COLMAPPoint3D(i, tuple(x), tuple(int(c) for c in rgb), e, t) for i, x, rgb, e, t in
                zip(self.points_id, self.points_xyz, self.points_rgb, self.points_error,
                    self.points_track_length)]

    def gs_cameras(self):
        """One Camera per image whose camera id is known, in image-id order."""
        out = []
        for iid in sorted(self.images):
            img = self.images[iid]
            cam = self.cameras.get(img.camera_id)
            if cam is None:
                continue
            c = cam.to_gs_camera(img.world_to_camera())
            c.image_path = img.name
            out.append(c)
        return out

    def points_tensor(self, device="cpu"):
        import torch
        return torch.from_numpy(self.points_xyz.astype(np.float32)).to(device)

    def colors_tensor(self, device="cpu"):
        """RGB / 255 in fp32 (colmap_loader.cr:237-251)."""
        import torch
        return torch.from_numpy(self.points_rgb.astype(np.float32) / np.float32(255.0)).to(device)

    # -- text ---------------------------------------------------------------
    def _cameras_txt(self, path):
        with open(path) as f:
            for line in f:
                line = line.strip()
                if not line or line.startswith("#"):
                    continue
                p = line.split()
                if len(p) < 5:
                    continue
                model = p[1] if p[1] in MODEL_BY_NAME else "PINHOLE"
                self.cameras[int(p[0])] = COLMAPCamera(int(p[0]), model, int(p[2]), int(p[3]),
                                                       [float(v) for v in p[4:]])

    def _images_txt(self, path):
        with open(path) as f:
            lines = [ln.rstrip("\n") for ln in f if not ln.startswith("#")]
        # Records are line pairs; the 2D-point line may be empty. Trailing blank lines end it.
        while lines and not lines[-1].strip():
            lines.pop()
        i = 0
        while i < len(lines):
            p = lines[i].split()
            if len(p) < 10:
                if not p:
                    i += 1
                    continue
                break
            self.images[int(p[0])] = COLMAPImage(int(p[0]), int(p[8]), p[9], *map(float, p[1:8]))
            i += 2

    def _points_txt(self, path):
        ids, xyz, rgb, err, tl = [], [], [], [], []
        with open(path) as f:
            for line in f:
                line = line.strip()
                if not line or line.startswith("#"):
                    continue
                p = line.split()
                if len(p) < 8:
                    continue
                ids.append(int(p[0]))
                xyz.append((float(p[1]), float(p[2]), float(p[3])))
                rgb.append((int(p[4]), int(p[5]), int(p[6])))
                err.append(float(p[7]))
                tl.append((len(p) - 8) // 2)
        self._set_points(ids, xyz, rgb, err, tl)

    def _set_points(self, ids, xyz, rgb, err, tl):
        self.points_id = np.asarray(ids, np.int64)
        self.points_xyz = np.asarray(xyz, np.float64).reshape(-1, 3)
        self.points_rgb = np.asarray(rgb, np.uint8).reshape(-1, 3)
        self.points_error = np.asarray(err, np.float64)
        self.points_track_length = np.asarray(tl, np.int32)

    # -- binary (little endian) ----------------------------------------------
    def _cameras_bin(self, path):
        b = open(path, "rb").read()
        (n,), o = struct.unpack_from("<Q", b, 0), 8
        for _ in range(n):
            cid, mid, w, h = struct.unpack_from("<iiQQ", b, o)
            o += 24
            if mid not in MODEL_BY_ID:
                raise ValueError(f"{path}: unknown COLMAP camera model id {mid}")
            name, _, npar, _ = MODEL_BY_ID[mid]
            params = struct.unpack_from(f"<{npar}d", b, o)
            o += 8 * npar
            self.cameras[cid] = COLMAPCamera(cid, name, w, h, params)

    def _images_bin(self, path):
        b = open(path, "rb").read()
        (n,), o = struct.unpack_from("<Q", b, 0), 8
        for _ in range(n):
            iid, qw, qx, qy, qz, tx, ty, tz, cid = struct.unpack_from("<i7di", b, o)
            o += 64
            end = b.index(b"\0", o)
            name = b[o:end].decode()
            o = end + 1
            (np2d,) = struct.unpack_from("<Q", b, o)
            o += 8 + 24 * np2d
            self.images[iid] = COLMAPImage(iid, cid, name, qw, qx, qy, qz, tx, ty, tz)

    def _points_bin(self, path):
        b = open(path, "rb").read()
        (n,), o = struct.unpack_from("<Q", b, 0), 8
        ids, xyz, rgb, err, tl = [], [], [], [], []
        rec = struct.Struct("<Q3d3BdQ")
        for _ in range(n):
            pid, x, y, z, r, g, bl, e, t = rec.unpack_from(b, o)
            o += rec.size + 8 * t
            ids.append(pid)
            xyz.append((x, y, z))
            rgb.append((r, g, bl))
            err.append(e)
            tl.append(t)
        self._set_points(ids, xyz, rgb, err, tl)


def rotation_to_quaternion(R):
    """(w, x, y, z) of a rotation matrix (Shepperd's method), w >= 0."""
    R = np.asarray(R, np.float64)
    tr = R[0, 0] + R[1, 1] + R[2, 2]
    if tr > 0:
        s = math.sqrt(tr + 1.0) * 2
        q = (0.25 * s, (R[2, 1] - R[1, 2]) / s, (R[0, 2] - R[2, 0]) / s, (R[1, 0] - R[0, 1]) / s)
    elif R[0, 0] > R[1, 1] and R[0, 0] > R[2, 2]:
        s = math.sqrt(1.0 + R[0, 0] - R[1, 1] - R[2, 2]) * 2
        q = ((R[2, 1] - R[1, 2]) / s, 0.25 * s, (R[0, 1] + R[1, 0]) / s, (R[0, 2] + R[2, 0]) / s)
    elif R[1, 1] > R[2, 2]:
        s = math.sqrt(1.0 + R[1, 1] - R[0, 0] - R[2, 2]) * 2
        q = ((R[0, 2] - R[2, 0]) / s, (R[0, 1] + R[1, 0]) / s, 0.25 * s, (R[1, 2] + R[2, 1]) / s)
    else:
        s = math.sqrt(1.0 + R[2, 2] - R[0, 0] - R[1, 1]) * 2
        q = ((R[1, 0] - R[0, 1]) / s, (R[0, 2] + R[2, 0]) / s, (R[1, 2] + R[2, 1]) / s, 0.25 * s)
    return q if q[0] >= 0 else tuple(-v for v in q)


def colmap_model_of(cameras, names=None):
    """COLMAP cameras + images describing Camera objects (one PINHOLE each)."""
    cams, imgs = [], []
    for i, c in enumerate(cameras):
        k = c.intrinsics
        cams.append(COLMAPCamera(i + 1, "PINHOLE", k.width, k.height, [k.fx, k.fy, k.cx, k.cy]))
        w2c = np.asarray(c.world_to_camera, np.float64)
        q = rotation_to_quaternion(w2c[:3, :3])
        name = names[i] if names else f"view_{i:05d}.png"
        imgs.append(COLMAPImage(i + 1, i + 1, name, *q, *w2c[:3, 3]))
    return cams, imgs


def load_colmap(path):
    """Utils.load_colmap (colmap_loader.cr:438-442)."""
    return COLMAPLoader(path).load()


def save_colmap_text(path, cameras, images, points=None):
    """Write cameras.txt / images.txt / points3D.txt. cameras: list of
    COLMAPCamera; images: list of COLMAPImage; points: (xyz [N,3], rgb [N,3] u8)."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "cameras.txt"), "w") as f:
        f.write("# Camera list with one line of data per camera:\n")
        for c in cameras:
            f.write(f"{c.id} {c.model} {c.width} {c.height} " + " ".join(repr(float(p)) for p in c.params) + "\n")
    with open(os.path.join(path, "images.txt"), "w") as f:
        f.write("# Image list with two lines of data per image:\n")
        for im in images:
            f.write(f"{im.id} " + " ".join(repr(float(v)) for v in im.q + im.t) + f" {im.camera_id} {im.name}\n\n")
    if points is not None:
        xyz, rgb = points
        with open(os.path.join(path, "points3D.txt"), "w") as f:
            f.write("# 3D point list with one line of data per point:\n")
            for i, (p, c) in enumerate(zip(xyz, rgb)):
                f.write(f"{i + 1} {float(p[0])!r} {float(p[1])!r} {float(p[2])!r} {c[0]} {c[1]} {c[2]} 0.5\n")


def save_colmap_binary(path, cameras, images, points=None):
    """The same model as cameras.bin / images.bin / points3D.bin."""
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "cameras.bin"), "wb") as f:
        f.write(struct.pack("<Q", len(cameras)))
        for c in cameras:
            f.write(struct.pack("<iiQQ", c.id, MODEL_BY_NAME[c.model][1], c.width, c.height))
            f.write(struct.pack(f"<{len(c.params)}d", *c.params))
    with open(os.path.join(path, "images.bin"), "wb") as f:
        f.write(struct.pack("<Q", len(images)))
        for im in images:
            f.write(struct.pack("<i7di", im.id, *im.q, *im.t, im.camera_id))
            f.write(im.name.encode() + b"\0")
            f.write(struct.pack("<Q", 1) + struct.pack("<ddq", 1.0, 2.0, -1))
    if points is not None:
        xyz, rgb = points
        with open(os.path.join(path, "points3D.bin"), "wb") as f:
            f.write(struct.pack("<Q", len(xyz)))
            for i, (p, c) in enumerate(zip(xyz, rgb)):
                f.write(struct.pack("<Q3d3BdQ", i + 1, *map(float, p), *map(int, c), 0.5, 2))
                f.write(struct.pack("<iiii", 1, 0, 2, 0))


# ---- Gaussians from points, PLY ----------------------------------------------

SH_C0 = np.float32(0.28209479177387814)


def from_points(points, colors=None, device="cuda"):
    """Gaussian3D.from_points (gaussian.cr:86-116) with Gaussian3D.new's
    defaults (gaussian.cr:58-83): log-scale -3, identity rotation, logit 0,
    SH N(0,1) * 0.1 (seeded here), DC = colour / C0 when colours are given."""
    from .gaussian import SH_COEFFS, Gaussian3D
    pts = np.asarray(points.cpu() if hasattr(points, "cpu") else points, np.float32).reshape(-1, 3)
    n = pts.shape[0]
    rng = np.random.default_rng(0)
    sh = (rng.standard_normal((n, SH_COEFFS, 3), dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    if colors is not None:
        col = np.asarray(colors.cpu() if hasattr(colors, "cpu") else colors, np.float32).reshape(-1, 3)
        sh = np.zeros((n, SH_COEFFS, 3), np.float32)
        sh[:, 0, :] = col / SH_C0
    rot = np.zeros((n, 4), np.float32)
    rot[:, 0] = 1.0
    arrays = {"position": pts, "log_scale": np.full((n, 3), -3.0, np.float32), "rotation": rot,
              "logit_opacity": np.zeros((n, 1), np.float32), "sh_coeffs": sh}
    return Gaussian3D(arrays, device)


def _ply_names():
    names = ["x", "y", "z", "nx", "ny", "nz", "f_dc_0", "f_dc_1", "f_dc_2"]
    names += [f"f_rest_{i}" for i in range(45)]
    names += ["opacity", "scale_0", "scale_1", "scale_2", "rot_0", "rot_1", "rot_2", "rot_3"]
    return names


def save_ply(gaussians, path):
    """Binary little-endian PLY in the 3DGS layout: position, zero normals, SH
    DC, the 45 higher-order coefficients channel-major (all of R, then G, then
    B), logit opacity, log-scales, rotation (w, x, y, z)."""
    g = gaussians
    n = g.count
    sh = g.sh_coeffs.detach().cpu().numpy().reshape(n, 16, 3)
    cols = [g.position.detach().cpu().numpy().reshape(n, 3), np.zeros((n, 3), np.float32), sh[:, 0, :],
            sh[:, 1:, :].transpose(0, 2, 1).reshape(n, 45),
            g.logit_opacity.detach().cpu().numpy().reshape(n, 1),
            g.log_scale.detach().cpu().numpy().reshape(n, 3), g.rotation.detach().cpu().numpy().reshape(n, 4)]
    data = np.ascontiguousarray(np.concatenate(cols, axis=1).astype("<f4"))
    header = "ply\nformat binary_little_endian 1.0\n" + f"element vertex {n}\n"
    header += "".join(f"property float {name}\n" for name in _ply_names()) + "end_header\n"
    with open(path, "wb") as f:
        f.write(header.encode("ascii"))
        f.write(data.tobytes())


def load_ply(path, device="cuda"):
    """Inverse of save_ply (any property order; missing SH rest -> 0)."""
    from .gaussian import Gaussian3D
    with open(path, "rb") as f:
        raw = f.read()
    end = raw.index(b"end_header\n") + len(b"end_header\n")
    header = raw[:end].decode("ascii").splitlines()
    if "format binary_little_endian 1.0" not in header:
        raise ValueError("only binary_little_endian PLY is supported")
    n, props = 0, []
    for ln in header:
        p = ln.split()
        if p[:2] == ["element", "vertex"]:
            n = int(p[2])
        elif p[:1] == ["property"]:
            if p[1] not in ("float", "float32"):
                raise ValueError(f"unsupported PLY property type {p[1]}")
            props.append(p[2])
    data = np.frombuffer(raw, "<f4", count=n * len(props), offset=end).reshape(n, len(props))
    col = {name: data[:, i] for i, name in enumerate(props)}
    get = lambda k: col[k] if k in col else np.zeros(n, np.float32)  # noqa: E731
    sh = np.zeros((n, 16, 3), np.float32)
    for c in range(3):
        sh[:, 0, c] = get(f"f_dc_{c}")
        for k in range(15):
            sh[:, 1 + k, c] = get(f"f_rest_{c * 15 + k}")
    arrays = {"position": np.stack([get("x"), get("y"), get("z")], 1),
              "log_scale": np.stack([get(f"scale_{i}") for i in range(3)], 1),
              "rotation": np.stack([get(f"rot_{i}") for i in range(4)], 1),
              "logit_opacity": get("opacity").reshape(n, 1), "sh_coeffs": sh}
    return Gaussian3D({k: np.ascontiguousarray(v, np.float32) for k, v in arrays.items()}, device)


# ---- 8-bit PNG (Image of src/utils/image_io.cr) -------------------------------

class Image:
    """width x height x channels uint8, row-major (image_io.cr:72-130)."""

    def __init__(self, width, height, channels, data):
        self.width, self.height, self.channels = int(width), int(height), int(channels)
        self.data = np.ascontiguousarray(data, np.uint8).reshape(self.height, self.width, self.channels)

    def to_tensor(self, device="cpu"):
        """[H, W, C] fp32 = byte / 255 (image_io.cr:83-97)."""
        import torch
        return torch.from_numpy(self.data.astype(np.float32) / np.float32(255.0)).to(device)

    def to_target(self, width=None, height=None, channels=3, device="cuda", out=None):
        """The training target on the GPU: the bytes are uploaded and resized
        (ImageIO.resize) + normalised by gsc_image_to_target."""
        return image_to_target(self.data, width or self.width, height or self.height, channels,
                               device, out)


def image_to_target(data, width, height, channels=3, device="cuda", out=None):
    """[height, width, channels] fp32 target from an [h, w, c] uint8 array or
    CUDA tensor (gsc_image_to_target)."""
    import ctypes as C

    import torch

    from ._abi import check, lib
    from .rasterizer import context
    src = data if isinstance(data, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(data))
    src = src.to(device, non_blocking=True).contiguous()
    assert src.dtype == torch.uint8 and src.dim() == 3
    sh, sw, sc = src.shape
    out = torch.empty(height, width, channels, device=src.device) if out is None else out
    check(lib().gsc_image_to_target(context(src.device), C.c_void_p(src.data_ptr()), sw, sh, sc,
                                    C.c_void_p(out.data_ptr()), width, height, channels),
          "gsc_image_to_target")
    return out


def _paeth(a, b, c):
    p = a + b - c
    pa, pb, pc = abs(p - a), abs(p - b), abs(p - c)
    return np.where((pa <= pb) & (pa <= pc), a, np.where(pb <= pc, b, c))


def load_png(path):
    """8-bit grey / grey+alpha / RGB / RGBA, non-interlaced PNG (the PNG 1.2
    specification: zlib IDAT stream, per-row filters 0-4)."""
    raw = open(path, "rb").read()
    if raw[:8] != b"\x89PNG\r\n\x1a\n":
        raise ValueError(f"{path}: not a PNG")
    o, idat, hdr = 8, [], None
    while o < len(raw):
        (ln,), typ = struct.unpack_from(">I", raw, o), raw[o + 4:o + 8]
        body = raw[o + 8:o + 8 + ln]
        o += 12 + ln
        if typ == b"IHDR":
            hdr = struct.unpack(">IIBBBBB", body)
        elif typ == b"IDAT":
            idat.append(body)
        elif typ == b"IEND":
            break
    w, h, depth, ctype, _, _, interlace = hdr
    ch = {0: 1, 4: 2, 2: 3, 6: 4}.get(ctype)
    if depth != 8 or ch is None or interlace:
        raise ValueError(f"{path}: only 8-bit non-interlaced grey/RGB(A) PNG is supported")
    buf = np.frombuffer(zlib.decompress(b"".join(idat)), np.uint8).reshape(h, 1 + w * ch)
    out = np.zeros((h, w * ch), np.int32)
    prev = np.zeros(w * ch, np.int32)
    for y in range(h):
        f, row = buf[y, 0], buf[y, 1:].astype(np.int32)
        if f == 0:
            cur = row
        elif f == 2:
            cur = (row + prev) & 255
        elif f in (1, 3, 4):
            cur = np.zeros_like(row)
            for x in range(w * ch):  # left neighbour dependency: serial
                a = cur[x - ch] if x >= ch else 0
                if f == 1:
                    pred = a
                elif f == 3:
                    pred = (a + prev[x]) >> 1
                else:
                    c = prev[x - ch] if x >= ch else 0
                    pred = int(_paeth(np.int32(a), np.int32(prev[x]), np.int32(c)))
                cur[x] = (row[x] + pred) & 255
        else:
            raise ValueError(f"{path}: bad PNG filter {f}")
        out[y] = cur
        prev = cur
    return Image(w, h, ch, out.astype(np.uint8))


def save_png(path, image):
    """Write an [H, W, C] uint8 array (or an fp32 array in [0, 1], rounded) as PNG."""
    a = np.asarray(image.cpu() if hasattr(image, "cpu") else image)
    if a.dtype != np.uint8:
        a = np.clip(np.rint(a.astype(np.float64) * 255.0), 0, 255).astype(np.uint8)
    if a.ndim == 2:
        a = a[:, :, None]
    h, w, ch = a.shape
    ctype = {1: 0, 2: 4, 3: 2, 4: 6}[ch]
    rows = np.concatenate([np.zeros((h, 1), np.uint8), a.reshape(h, w * ch)], axis=1)

    def chunk(t, body):
        return struct.pack(">I", len(body)) + t + body + struct.pack(">I", zlib.crc32(t + body) & 0xFFFFFFFF)
    with open(path, "wb") as f:
        f.write(b"\x89PNG\r\n\x1a\n")
        f.write(chunk(b"IHDR", struct.pack(">IIBBBBB", w, h, 8, ctype, 0, 0, 0)))
        f.write(chunk(b"IDAT", zlib.compress(rows.tobytes(), 6)))
        f.write(chunk(b"IEND", b""))
