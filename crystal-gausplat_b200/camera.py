"""Pinhole camera, mirroring src/gaussian_splatting/camera.cr.

Convention: world_to_camera is a ROW-major 4x4 (camera.cr:185-187) whose
rows are (right, down, forward) -- OpenCV, +Z into the scene -- because the
projection culls z <= near (gaussian.metal:160). The reference's look_at
builds a -Z-forward pose that this cull would reject entirely; look_at here
builds the OpenCV pose, as Camera#set_world_to_camera with a COLMAP pose
would (camera.cr:121-124, 341-353).
"""
import math

import numpy as np

from . import _abi


class CameraIntrinsics:
    """CameraIntrinsics (camera.cr:9-56)."""

    def __init__(self, width, height, fx, fy, cx, cy):
        self.width, self.height = int(width), int(height)
        self.fx, self.fy, self.cx, self.cy = float(fx), float(fy), float(cx), float(cy)

    @classmethod
    def from_fov(cls, width, height, fov_x, fov_y=None):
        """camera.cr:21-27: fx = W / (2 tan(fov_x/2)); fy = fx without fov_y; c = centre."""
        fx = width / (2.0 * math.tan(fov_x / 2.0))
        fy = height / (2.0 * math.tan(fov_y / 2.0)) if fov_y else fx
        return cls(width, height, fx, fy, width / 2.0, height / 2.0)

    @property
    def tan_half_fov_x(self):
        # tan(fov_x / 2) with fov_x = 2 atan(W / (2 fx)), camera.cr:30-41
        return self.width / (2.0 * self.fx)

    @property
    def tan_half_fov_y(self):
        return self.height / (2.0 * self.fy)


class Camera:
    """Camera (camera.cr:59-256): intrinsics + world_to_camera pose."""

    def __init__(self, intrinsics):
        self.intrinsics = intrinsics
        self.world_to_camera = np.eye(4, dtype=np.float64)

    @property
    def width(self):
        return self.intrinsics.width

    @property
    def height(self):
        return self.intrinsics.height

    def look_at(self, eye, target=(0.0, 0.0, 0.0), up=(0.0, 1.0, 0.0)):
        eye = np.asarray(eye, np.float64)
        f = np.asarray(target, np.float64) - eye
        f /= np.linalg.norm(f)
        up = np.asarray(up, np.float64)
        if abs(float(np.dot(f, up))) > 0.999:
            up = np.array([0.0, 0.0, 1.0])
        right = np.cross(f, up)
        right /= np.linalg.norm(right)
        down = np.cross(f, right)
        R = np.stack([right, down, f])
        w2c = np.eye(4)
        w2c[:3, :3] = R
        w2c[:3, 3] = -R @ eye
        self.world_to_camera = w2c
        return self

    def set_world_to_camera(self, matrix):
        self.world_to_camera = np.asarray(matrix, np.float64).reshape(4, 4).copy()
        return self

    @property
    def position(self):
        """Camera centre in world space (camera.cr:133-137)."""
        R = self.world_to_camera[:3, :3]
        t = self.world_to_camera[:3, 3]
        return -R.T @ t

    def to_struct(self):
        """The packed CameraParamsGPU block (rasterizer.cr:502-531)."""
        c = _abi.Camera()
        v = self.world_to_camera.astype(np.float32).reshape(-1)
        for i in range(16):
            c.view[i] = float(v[i])
        k = self.intrinsics
        c.fx, c.fy, c.cx, c.cy = (np.float32(k.fx), np.float32(k.fy), np.float32(k.cx), np.float32(k.cy))
        c.width, c.height = k.width, k.height
        c.tan_fov_x = np.float32(k.tan_half_fov_x)
        c.tan_fov_y = np.float32(k.tan_half_fov_y)
        p = self.position.astype(np.float32)
        for i in range(3):
            c.campos[i] = float(p[i])
        return c


def sphere_poses(n, radius, seed):
    """Camera centres uniform on a sphere (normalised N(0,1)^3), seeded."""
    rng = np.random.default_rng(seed)
    u = rng.standard_normal((n, 3))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    return u * radius


def orbit_poses(n, radius):
    """Centres on a circle of the XZ plane at y = 0, angle 2 pi k / n."""
    a = 2.0 * np.pi * np.arange(n) / n
    return np.stack([radius * np.sin(a), np.zeros(n), radius * np.cos(a)], axis=1)


def make_camera(width, height, eye, fov_x_deg=60.0, target=(0.0, 0.0, 0.0)):
    cam = Camera(CameraIntrinsics.from_fov(width, height, math.radians(fov_x_deg)))
    return cam.look_at(eye, target)


class CameraSet(list):
    """CameraSet (camera.cr:259-286): a list of cameras."""

    def sample(self, rng=None):
        rng = rng or np.random.default_rng()
        return self[int(rng.integers(len(self)))]

    @classmethod
    def from_colmap(cls, images_txt_path, cameras_txt_path):
        """CameraSet.from_colmap (camera.cr:288-358): PINHOLE / SIMPLE_PINHOLE
        intrinsics; the pose quaternion is normalised and turned into R in fp32
        arithmetic, as there. Images are read as COLMAP's line pairs (the
        second, 2D-point line of each record is skipped even when it is empty
        or has ten or more fields)."""
        f32 = np.float32
        intr = {}
        with open(cameras_txt_path) as f:
            for line in f:
                if line.startswith("#") or not line.strip():
                    continue
                p = line.split()
                if len(p) < 5:
                    continue
                w, h = int(p[2]), int(p[3])
                if p[1] == "PINHOLE":
                    intr[int(p[0])] = CameraIntrinsics(w, h, f32(p[4]), f32(p[5]), f32(p[6]), f32(p[7]))
                elif p[1] == "SIMPLE_PINHOLE":
                    intr[int(p[0])] = CameraIntrinsics(w, h, f32(p[4]), f32(p[4]), f32(p[5]), f32(p[6]))
        out = cls()
        with open(images_txt_path) as f:
            lines = [ln for ln in f if not ln.startswith("#")]
        i = 0
        while i < len(lines):
            p = lines[i].split()
            if not p:
                i += 1
                continue
            i += 2
            if len(p) < 10 or int(p[8]) not in intr:
                continue
            w, x, y, z = (f32(v) for v in p[1:5])
            n = f32(np.sqrt(f32(f32(f32(w * w) + f32(x * x)) + f32(y * y)) + f32(z * z)))
            w, x, y, z = w / n, x / n, y / n, z / n
            one, two = f32(1), f32(2)
            R = [one - two * y * y - two * z * z, two * x * y - two * z * w, two * x * z + two * y * w,
                 two * x * y + two * z * w, one - two * x * x - two * z * z, two * y * z - two * x * w,
                 two * x * z - two * y * w, two * y * z + two * x * w, one - two * x * x - two * y * y]
            m = np.zeros((4, 4), np.float32)
            m[:3, :3] = np.array(R, np.float32).reshape(3, 3)
            m[:3, 3] = [f32(p[5]), f32(p[6]), f32(p[7])]
            m[3, 3] = 1
            cam = Camera(intr[int(p[8])]).set_world_to_camera(m)
            cam.image_path = p[9]
            out.append(cam)
        return out
