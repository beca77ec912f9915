"""ctypes binding of libgsplat_cuda.so (include/gsplat_cuda.h).

This is the same binding a Crystal `lib GSCuda ... end` block declares; the
Python side exists for tests, the benchmark and Python users. There is no
fallback: if the library is missing or fails to load, importing the
rasterizer raises.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# GSC_LIBRARY: another build of the same library (e.g. a variant being measured)
LIB_PATH = os.environ.get("GSC_LIBRARY") or os.path.join(HERE, "libgsplat_cuda.so")

GSC_OK = 0
GSC_ERR_INVALID = -1
GSC_ERR_CUDA = -2
GSC_ERR_CAPACITY = -3
GSC_ERR_TIMEOUT = -4
GSC_ERR_NOMEM = -5
GSC_ERR_NODEVICE = -6
GSC_ERR_UNSUPPORTED = -7

GSC_MODE_FULL = 0
GSC_MODE_REF = 1

GSC_MAX_BATCH_VIEWS = 8

GSC_BIN_REFERENCE = 0
GSC_BIN_CONTRIBUTING = 1
GSC_BIN_OCCLUDED = 2

GSC_STATIC_SORT_MAX_PAIRS = 262144

GSC_FRAME_SPLATS = 0
GSC_FRAME_KEYS = 1
GSC_FRAME_VALUES = 2
GSC_FRAME_RANGES = 3
GSC_FRAME_IMAGE = 4
GSC_FRAME_FINAL_T = 5
GSC_FRAME_LAST = 6
GSC_FRAME_N_CONTRIB = 7
GSC_FRAME_GRAD2D = 8

P = C.c_void_p


class Camera(C.Structure):
    """gsc_camera == the reference's packed CameraParamsGPU (176 bytes)."""
    _fields_ = [("view", C.c_float * 16), ("proj", C.c_float * 16),
                ("fx", C.c_float), ("fy", C.c_float), ("cx", C.c_float), ("cy", C.c_float),
                ("width", C.c_int32), ("height", C.c_int32),
                ("tan_fov_x", C.c_float), ("tan_fov_y", C.c_float),
                ("campos", C.c_float * 3), ("_pad", C.c_float)]


class RasterConfig(C.Structure):
    _fields_ = [("mode", C.c_int32), ("sh_degree", C.c_int32), ("t_stop", C.c_float),
                ("alpha_min", C.c_float), ("alpha_max", C.c_float), ("lowpass", C.c_float),
                ("fov_cull", C.c_float), ("near_z", C.c_float), ("far_z", C.c_float),
                ("background", C.c_float * 3), ("binning", C.c_int32)]


class Gaussians(C.Structure):
    _fields_ = [("position", P), ("log_scale", P), ("rotation", P), ("logit_opacity", P),
                ("sh", P), ("count", C.c_int64)]


class GaussianGrads(C.Structure):
    _fields_ = [("position", P), ("log_scale", P), ("rotation", P), ("logit_opacity", P),
                ("sh", P)]


class Projected(C.Structure):
    _fields_ = [(name, P) for name in ("splats", "mean2d", "cov2d", "conic", "depth", "radius",
                                       "colors", "opacity", "tiles_touched", "cov3d")]


class Grads2D(C.Structure):
    _fields_ = [("mean2d", P), ("cov2d", P), ("opacity", P), ("colors", P)]


class AdamGroup(C.Structure):
    _fields_ = [("param", P), ("grad", P), ("m", P), ("v", P), ("numel", C.c_int64),
                ("lr", C.c_float), ("weight_decay", C.c_float)]


class GaussiansOut(C.Structure):
    _fields_ = [("position", P), ("log_scale", P), ("rotation", P), ("logit_opacity", P), ("sh", P)]


GSC_DENSIFY_CLONE = 1
GSC_DENSIFY_SPLIT = 2
GSC_DENSIFY_PRUNE = 4


class DpAdamArgs(C.Structure):
    _fields_ = [("nranks", C.c_int32), ("rank", C.c_int32),
                ("peer_grads", P * 8), ("peer_params", P * 8), ("m", P), ("v", P),
                ("ngroups", C.c_int32), ("offset", C.c_int64 * 8), ("numel", C.c_int64 * 8),
                ("lr", C.c_float * 8), ("weight_decay", C.c_float * 8),
                ("beta1", C.c_float), ("beta2", C.c_float), ("eps", C.c_float), ("step", C.c_int32),
                ("grad_scale", C.c_float), ("mc_grads", P), ("mc_params", P)]


class DpBarrierArgs(C.Structure):
    _fields_ = [("nranks", C.c_int32), ("rank", C.c_int32), ("peer_flags", P * 8),
                ("epoch", C.c_uint32), ("timeout_us", C.c_int32)]


assert C.sizeof(Camera) == 176, C.sizeof(Camera)

_SIGS = {
    "gsc_version": (C.c_int, []),
    "gsc_last_error": (C.c_char_p, []),
    "gsc_raster_config_default": (None, [C.POINTER(RasterConfig)]),
    "gsc_init": (C.c_int, [C.c_int, C.POINTER(P)]),
    "gsc_destroy": (C.c_int, [P]),
    "gsc_set_stream": (C.c_int, [P, P]),
    "gsc_sync": (C.c_int, [P]),
    "gsc_alloc": (C.c_int, [P, C.c_size_t, C.POINTER(P)]),
    "gsc_free": (C.c_int, [P, P]),
    "gsc_memcpy_h2d": (C.c_int, [P, P, P, C.c_size_t]),
    "gsc_memcpy_d2h": (C.c_int, [P, P, P, C.c_size_t]),
    "gsc_memset": (C.c_int, [P, P, C.c_int, C.c_size_t]),
    "gsc_preprocess": (C.c_int, [P, C.POINTER(Gaussians), C.POINTER(Camera), C.POINTER(RasterConfig),
                                 C.POINTER(Projected)]),
    "gsc_bin": (C.c_int, [P, C.c_int64, P, C.c_int32, C.c_int32, P, P, C.c_int64,
                          C.POINTER(C.c_int64)]),
    "gsc_sort_pairs_u64": (C.c_int, [P, P, P, C.c_int64, C.c_int, C.c_int]),
    "gsc_sort_pairs_u64_static": (C.c_int, [P, P, C.c_int64, C.c_int, C.c_int, P]),
    "gsc_sort_pairs_u64_static_status": (C.c_int, [P]),
    "gsc_selftest_wait_timeout": (C.c_int, [P, C.c_int32]),
    "gsc_tile_ranges": (C.c_int, [P, P, C.c_int64, C.c_int32, P]),
    "gsc_composite_forward": (C.c_int, [P, P, P, P, C.c_int32, C.c_int32, C.POINTER(RasterConfig),
                                        P, P, P, P]),
    "gsc_composite_backward": (C.c_int, [P, P, P, P, C.c_int32, C.c_int32, C.POINTER(RasterConfig),
                                         P, P, P, C.c_float, P, P, P, P]),
    "gsc_preprocess_backward": (C.c_int, [P, C.POINTER(Gaussians), C.POINTER(Camera),
                                          C.POINTER(RasterConfig), P, C.POINTER(GaussianGrads),
                                          C.POINTER(Grads2D)]),
    "gsc_l1_loss_grad": (C.c_int, [P, P, P, C.c_int64, C.c_float, P, P]),
    "gsc_adam_step": (C.c_int, [P, C.POINTER(AdamGroup), C.c_int32, C.c_float, C.c_float,
                                C.c_float, C.c_int32, C.c_float]),
    "gsc_dp_adam_step": (C.c_int, [P, C.POINTER(DpAdamArgs)]),
    "gsc_dp_barrier": (C.c_int, [P, C.POINTER(DpBarrierArgs)]),
    "gsc_ssim_loss_grad": (C.c_int, [P, P, P, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_int32,
                                     P, P, P]),
    "gsc_combined_loss_grad": (C.c_int, [P, P, P, C.c_int32, C.c_int32, C.c_int32, C.c_float,
                                         C.c_int32, P, P]),
    "gsc_mse_loss_grad": (C.c_int, [P, P, P, C.c_int64, P, P]),
    "gsc_image_to_target": (C.c_int, [P, P, C.c_int32, C.c_int32, C.c_int32, P, C.c_int32,
                                      C.c_int32, C.c_int32]),
    "gsc_grad_accumulate": (C.c_int, [P, P, C.c_int32, C.c_int64, P, P]),
    "gsc_densify_plan": (C.c_int, [P, C.POINTER(Gaussians), P, P, C.c_float, C.c_float, C.c_float,
                                   P, C.POINTER(C.c_int64)]),
    "gsc_densify_apply": (C.c_int, [P, C.POINTER(Gaussians), P, C.POINTER(GaussiansOut), C.c_float,
                                    C.c_float, C.c_uint64]),
    "gsc_reset_opacity": (C.c_int, [P, P, C.c_int64, C.c_float]),
    "gsc_frame_create": (C.c_int, [P, C.POINTER(P)]),
    "gsc_frame_destroy": (C.c_int, [P]),
    "gsc_frame_set_tile_hint": (C.c_int, [P, P, C.c_int64, C.c_int32]),
    "gsc_rasterize_forward": (C.c_int, [P, P, C.POINTER(Gaussians), C.POINTER(Camera),
                                        C.POINTER(RasterConfig), P, P, P, C.POINTER(C.c_int64)]),
    "gsc_rasterize_backward": (C.c_int, [P, P, C.POINTER(Gaussians), C.POINTER(Camera),
                                         C.POINTER(RasterConfig), P, P, C.c_float, P,
                                         C.POINTER(GaussianGrads), C.POINTER(Grads2D)]),
    "gsc_rasterize_forward_batch": (C.c_int, [P, C.POINTER(P), C.POINTER(Camera), C.c_int32,
                                              C.POINTER(Gaussians), C.POINTER(RasterConfig),
                                              C.POINTER(P), C.POINTER(C.c_int64)]),
    "gsc_rasterize_backward_batch": (C.c_int, [P, C.POINTER(P), C.POINTER(Camera), C.c_int32,
                                               C.POINTER(Gaussians), C.POINTER(RasterConfig),
                                               C.POINTER(GaussianGrads)]),
    "gsc_frame_get": (C.c_int, [P, C.c_int, C.POINTER(P), C.POINTER(C.c_int64)]),
    "gsc_profile_enable": (C.c_int, [P, C.c_int]),
    "gsc_profile_read": (C.c_int, [P, C.POINTER(C.c_double), C.POINTER(C.c_int64),
                                   C.POINTER(C.c_int64), C.c_int]),
    "gsc_kernel_count": (C.c_int64, [P]),
    "gsc_profile_pairs": (C.c_int, [P, C.POINTER(C.c_uint64), C.c_int]),
    "gsc_profile_pge": (C.c_int, [P, C.POINTER(C.c_uint64), C.c_int]),
}

STAGES = ("preprocess", "scan", "emit", "sort", "ranges", "composite_fwd", "composite_bwd",
          "preprocess_bwd", "adam", "l1")

EXPORTED = tuple(_SIGS)

_lib = None


class GscError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"{msg} (status {code})")
        self.code = code


def lib():
    """Load libgsplat_cuda.so once; raise if it is missing (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run __graft_entry__.build() "
                              "or python crystal-gausplat_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc, what=""):
    if rc != GSC_OK:
        msg = lib().gsc_last_error().decode(errors="replace")
        raise GscError(rc, f"{what}: {msg}" if what else msg)
    return rc


def default_config(mode=GSC_MODE_FULL, sh_degree=3, background=(0.0, 0.0, 0.0), t_stop=None,
                   binning=None):
    """gsc_raster_config_default with overrides (binning: GSC_BIN_*, default OCCLUDED)."""
    cfg = RasterConfig()
    lib().gsc_raster_config_default(C.byref(cfg))
    if binning is not None:
        cfg.binning = binning
    cfg.mode = mode
    cfg.sh_degree = sh_degree
    for i in range(3):
        cfg.background[i] = background[i]
    if t_stop is not None:
        cfg.t_stop = t_stop
    return cfg
