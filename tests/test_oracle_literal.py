"""The oracle's fused expression forms against the reference's literal ones.

The oracle (and the CUDA kernels, bit for bit) evaluate the compositing power
as fma(dy dy, -C/2, fma(dx dy, -B, dx dx (-A/2))) with a precomputed conic and
accumulate colour with fused multiply-adds. The reference writes
power = -0.5 (dx dx inv_xx + 2 dx dy inv_xy + dy dy inv_yy) with the inverse
recomputed per pixel, and colour += T alpha c (gaussian.metal:403-436).
gso_composite_forward_literal restates those forms. On config 0 of the
benchmark (100k Gaussians, 256x256) the two agree within the image bar
(1e-5 relative) at every pixel where both accept the same Gaussians. A pixel
where some Gaussian's alpha (or the transmittance) lies within rounding of
its threshold can accept one Gaussian more or less under either form; such
pixels must be rare (at most 5 of the 65,536) and differ by at most one
threshold-level contribution: (alpha_min + t_stop) times the largest colour
or background magnitude. So the fused forms are a rounding-level
reformulation of the reference, not a different algorithm."""
import numpy as np
import pytest

from helpers import _abi, gs, rel_err

IMG_RTOL = 1e-5


@pytest.mark.parametrize("seed", [0, 1, 2])
@pytest.mark.parametrize("background", [(0.0, 0.0, 0.0), (0.1, 0.2, 0.3)])
def test_fused_forward_equals_literal_reference_forms_c0(oracle, seed, background):
    arrays = gs.synthetic_arrays(100_000, seed)
    cam = gs.make_camera(256, 256, (0.0, 0.0, 4.0)).to_struct()
    cfg = gs.default_config(binning=_abi.GSC_BIN_REFERENCE, background=background)
    ref = oracle.forward_pipeline(oracle.Scene(arrays), cam, cfg)
    img, nc, fT = oracle.composite_forward_literal(256, 256, ref["ranges"], ref["sorted_vals"],
                                                   ref["pre"], cfg)
    assert ref["sorted_keys"].size > 100_000
    check_literal(ref, img, nc, fT, cfg)


def check_literal(ref, img, nc, fT, cfg):
    same = (ref["n_contrib"] == nc) & (np.abs(ref["final_T"] - fT) <= IMG_RTOL * np.abs(ref["final_T"]))
    flips = int((~same).sum())
    assert flips <= 5, flips
    assert rel_err(ref["image"][same], img[same], 1e-6) <= IMG_RTOL
    if flips:
        cmax = max(float(np.abs(ref["pre"]["colors"]).max()), max(abs(b) for b in cfg.background))
        bound = (cfg.alpha_min + cfg.t_stop) * cmax
        assert float(np.abs(ref["image"][~same] - img[~same]).max()) <= bound


@pytest.mark.parametrize("t_stop", [1e-3, 1e-4])
def test_fused_forward_equals_literal_reference_forms_t_stop(oracle, t_stop):
    """Also at the north star's T < 1e-4 stop, on a denser view."""
    arrays = gs.synthetic_arrays(100_000, 5)
    cam = gs.make_camera(256, 256, (0.0, 0.0, 3.0)).to_struct()
    cfg = gs.default_config(binning=_abi.GSC_BIN_REFERENCE, t_stop=t_stop)
    ref = oracle.forward_pipeline(oracle.Scene(arrays), cam, cfg)
    img, nc, fT = oracle.composite_forward_literal(256, 256, ref["ranges"], ref["sorted_vals"],
                                                   ref["pre"], cfg)
    check_literal(ref, img, nc, fT, cfg)
