"""crystal-gausplat_b200: the Gaussian-splatting rasterizer hot path of
crystal-gausplat on B200 (sm_100a) behind the reference's API.

The compute is libgsplat_cuda.so (csrc/, C ABI in include/gsplat_cuda.h);
this package is its Python host side: Camera, Gaussian3D, Rasterizer,
RasterizerContext, GPURadixSort, Adam, l1_with_grad, and the view-sharded
data-parallel trainer. Import it with importlib.import_module("crystal-gausplat_b200").
"""
from . import _abi
from ._abi import GSC_MODE_FULL, GSC_MODE_REF, GscError, default_config
from .camera import Camera, CameraIntrinsics, CameraSet, make_camera, orbit_poses, sphere_poses
from .gaussian import Gaussian3D, synthetic_arrays
from . import scene_io
from .scene_io import (COLMAPLoader, Image, load_colmap, load_ply, load_png, save_ply,
                       save_png)

try:
    from .rasterizer import (GPURadixSort, Rasterizer, RasterizerContext, RasterizerGradients,
                             context, sync)
    from .optim import Adam, l1_with_grad
    from . import loss as Loss
    from .densify import (GradientAccumulator, densify_and_prune, densify_apply, densify_plan,
                          reset_opacity)
    from .trainer import DataParallelTrainer, Trainer, TrainerConfig, TrainStats
except ImportError:  # torch missing: camera/generator helpers stay usable
    pass


def build(force=False):
    from .build import build as _b
    return _b(force=force)
