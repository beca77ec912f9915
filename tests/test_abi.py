"""The C-ABI library loads without a GPU, exports every entry point that
include/gsplat_cuda.h declares, and its argument checks and error reporting
work on the host (no compute call needs a GPU here)."""
import ctypes as C
import os
import re

import pytest

from helpers import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "gsplat_cuda.h")


def declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"GSC_API\s+[\w\s\*]+?\b(gsc_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = declared()
    assert "gsc_rasterize_forward" in names and "gsc_sort_pairs_u64_static" in names
    assert len(names) >= 30


def test_library_exports_every_declared_symbol():
    lib = C.CDLL(_abi.LIB_PATH)
    missing = [n for n in declared() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert sorted(_abi.EXPORTED) == declared()


def test_struct_layouts():
    # gsc_camera is byte-for-byte the reference's packed CameraParamsGPU.
    assert C.sizeof(_abi.Camera) == 176
    assert _abi.Camera.fx.offset == 128 and _abi.Camera.campos.offset == 160
    assert C.sizeof(_abi.RasterConfig) == 13 * 4
    assert C.sizeof(_abi.Gaussians) == 6 * 8
    assert C.sizeof(_abi.AdamGroup) == 6 * 8


def test_default_config_is_the_reference_constants():
    cfg = _abi.default_config()
    assert cfg.mode == _abi.GSC_MODE_FULL and cfg.sh_degree == 3
    assert cfg.t_stop == pytest.approx(1e-3) and cfg.alpha_min == pytest.approx(1 / 255)
    assert cfg.alpha_max == pytest.approx(0.99) and cfg.lowpass == pytest.approx(0.3)
    assert cfg.fov_cull == pytest.approx(1.3) and cfg.near_z == pytest.approx(0.01)
    assert cfg.far_z == pytest.approx(1000.0)


def test_argument_errors_without_a_gpu():
    lib = _abi.lib()
    assert lib.gsc_version() == 1
    # null context / bad arguments are rejected before touching CUDA
    assert lib.gsc_sort_pairs_u64(None, None, None, 10, 0, 64) == _abi.GSC_ERR_INVALID
    assert b"null" in lib.gsc_last_error()
    assert lib.gsc_sync(None) == _abi.GSC_ERR_INVALID
    assert lib.gsc_sort_pairs_u64_static(None, None, -1, 0, 64, None) == _abi.GSC_ERR_INVALID
    assert lib.gsc_sort_pairs_u64_static(None, None, 1 << 20, 0, 64, None) == _abi.GSC_ERR_INVALID
    assert lib.gsc_sort_pairs_u64_static(None, None, 1, 0, 64, None) == _abi.GSC_OK  # n <= 1: no work
    g = _abi.AdamGroup()
    assert lib.gsc_adam_step(None, C.byref(g), 1, 0.9, 0.999, 1e-8, 1, 1.0) == _abi.GSC_ERR_INVALID


def test_init_without_a_device_reports_nodevice():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    h = C.c_void_p()
    rc = _abi.lib().gsc_init(0, C.byref(h))
    assert rc == _abi.GSC_ERR_NODEVICE
    assert h.value is None
    with pytest.raises(_abi.GscError):
        _abi.check(rc, "gsc_init")


def test_selftest_argument_checks():
    lib = _abi.lib()
    assert lib.gsc_selftest_wait_timeout(None, 10) == _abi.GSC_ERR_INVALID


def test_dp_barrier_argument_checks():
    lib = _abi.lib()
    b = _abi.DpBarrierArgs()
    b.nranks, b.rank, b.timeout_us = 2, 0, 0
    assert lib.gsc_dp_barrier(None, C.byref(b)) == _abi.GSC_ERR_INVALID
