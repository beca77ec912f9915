"""Gaussian3D trainable state (src/gaussian_splatting/gaussian.cr:19-147) and
the seeded synthetic scenes the benchmark configurations name.

Layout (drop-in with the reference): position [N,3], log_scale [N,3],
rotation [N,4] as (w,x,y,z), logit_opacity [N,1], sh_coeffs [N,16,3]
(coefficient-major, channel-minor), row-major fp32. On the device the five
tensors are views into one contiguous arena [N*59] (three float4-aligned
blocks), so gradients, Adam moments and the data-parallel all-reduce each
work on one flat buffer.
"""
import numpy as np

SH_DEGREE = 3
SH_COEFFS = (SH_DEGREE + 1) ** 2
FLOATS_PER_GAUSSIAN = 3 + 3 + 4 + 1 + SH_COEFFS * 3  # 59
FIELDS = (("position", 3), ("log_scale", 3), ("rotation", 4), ("logit_opacity", 1),
          ("sh_coeffs", SH_COEFFS * 3))


def field_offsets(n):
    """Offsets (floats) of each field in the arena; each starts 16-byte aligned."""
    offs, o = {}, 0
    for name, w in FIELDS:
        offs[name] = o
        o += ((n * w + 3) // 4) * 4
    return offs, o


def synthetic_arrays(n, seed, extent=1.0):
    """Seeded host arrays with the distributions of every benchmark config:
    means U[-extent, extent]^3; log-scales N(-4.5, 0.5); rotations normalised
    N(0,1)^4; logit opacity N(0,1); SH DC N(0, 0.5), higher orders N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    pos = rng.uniform(-extent, extent, (n, 3)).astype(np.float32)
    log_scale = (rng.standard_normal((n, 3), dtype=np.float32) * np.float32(0.5)
                 - np.float32(4.5)).astype(np.float32)
    q = rng.standard_normal((n, 4), dtype=np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    logit = rng.standard_normal((n, 1), dtype=np.float32)
    sh = rng.standard_normal((n, SH_COEFFS, 3), dtype=np.float32) * np.float32(0.1)
    sh[:, 0, :] *= np.float32(5.0)  # DC: N(0, 0.5)
    return {"position": pos, "log_scale": log_scale, "rotation": q.astype(np.float32),
            "logit_opacity": logit, "sh_coeffs": sh.astype(np.float32)}


class Gaussian3D:
    """The five parameter tensors, as views of one device arena."""

    def __init__(self, arrays, device="cuda", count=None):
        import torch
        n = int(arrays["position"].shape[0]) if arrays is not None else int(count)
        self.count = n
        offs, total = field_offsets(n)
        self.offsets = offs
        self.arena = torch.zeros(total, dtype=torch.float32, device=device)
        for name, w in FIELDS:
            view = self.arena[offs[name]:offs[name] + n * w]
            if arrays is not None:
                view.copy_(torch.as_tensor(np.ascontiguousarray(arrays[name]).reshape(-1)))
            shape = (n, SH_COEFFS, 3) if name == "sh_coeffs" else (n, w)
            setattr(self, name, view.view(*shape))

    @classmethod
    def empty(cls, n, device="cuda"):
        """A zero-filled set of n Gaussians (the destination of densification)."""
        return cls(None, device, count=n)

    def rebind_arena(self, arena):
        """Use `arena` (same size and layout, e.g. in symmetric memory) for the parameters."""
        assert arena.numel() == self.arena.numel()
        self.arena = arena
        for name, t in self.views_of(arena).items():
            setattr(self, name, t)

    @classmethod
    def synthetic(cls, n, seed, extent=1.0, device="cuda"):
        return cls(synthetic_arrays(n, seed, extent), device)

    def parameters(self):
        """Gaussian3D#parameters order (gaussian.cr:145-147)."""
        return [self.position, self.log_scale, self.rotation, self.logit_opacity, self.sh_coeffs]

    def new_arena_like(self):
        import torch
        return torch.zeros_like(self.arena)

    def views_of(self, arena):
        """Field views of another arena with this layout (gradients, moments)."""
        out = {}
        n = self.count
        for name, w in FIELDS:
            v = arena[self.offsets[name]:self.offsets[name] + n * w]
            out[name] = v.view(n, SH_COEFFS, 3) if name == "sh_coeffs" else v.view(n, w)
        return out

    def scale(self):
        """Gaussian3D#scale: exp(log_scale) (gaussian.cr:119-129)."""
        return self.log_scale.exp()

    def opacity(self):
        """Gaussian3D#opacity: sigmoid(logit_opacity) (gaussian.cr:132-142)."""
        return self.logit_opacity.sigmoid()
