"""Committed golden fixtures (tests/golden/make_golden.py): the oracle must
reproduce them bit for bit (CPU), and the CUDA path must match them with the
parity bars (GPU) without running the oracle."""
import glob
import os

import numpy as np
import pytest

from helpers import R, _abi, gs, host, to_dev

HERE = os.path.dirname(os.path.abspath(__file__))
FIXTURES = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))


def load(path):
    z = np.load(path)
    arrays = {k[3:]: z[k] for k in z.files if k.startswith("in_")}
    cam = gs.make_camera(int(z["W"]), int(z["H"]), tuple(z["eye"]))
    cfg = gs.default_config(mode=int(z["mode"]), background=(0.05, 0.1, 0.15),
                            binning=_abi.GSC_BIN_REFERENCE)
    return z, arrays, cam, cfg


def test_fixtures_exist():
    assert len(FIXTURES) == 4


@pytest.mark.parametrize("path", FIXTURES, ids=os.path.basename)
def test_oracle_reproduces_golden(oracle, path):
    z, arrays, cam, cfg = load(path)
    cs = cam.to_struct()
    np.testing.assert_array_equal(np.float32(list(cs.view)), z["view"])
    sc = oracle.Scene(arrays)
    fw = oracle.forward_pipeline(sc, cs, cfg)
    for k in ("sorted_keys", "sorted_vals", "ranges", "image", "n_contrib", "final_T"):
        np.testing.assert_array_equal(fw[k], z[k], err_msg=k)
    W, H = int(z["W"]), int(z["H"])
    g2d, loss = oracle.composite_backward(W, H, fw["ranges"], fw["sorted_vals"], fw["pre"], cfg,
                                          fw["final_T"], fw["last"], image=fw["image"],
                                          target=z["target"], l1_scale=1.0 / z["target"].size)
    grads, _ = oracle.preprocess_backward(sc, cs, cfg, g2d)
    for k, v in grads.items():
        np.testing.assert_array_equal(v, z[f"grad_{k}"], err_msg=k)
    assert loss == float(z["loss"])


@pytest.mark.gpu
@pytest.mark.parametrize("path", FIXTURES, ids=os.path.basename)
def test_cuda_matches_golden(cuda, path):
    from test_gpu_parity import GRAD_RTOL, grad_close
    z, arrays, cam, cfg = load(path)
    g = gs.Gaussian3D(arrays)
    img, ctx = gs.Rasterizer.forward(g, cam, config=cfg)
    np.testing.assert_array_equal(host(img), z["image"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_KEYS, np.uint64), z["sorted_keys"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_VALUES, np.uint32), z["sorted_vals"])
    np.testing.assert_array_equal(ctx.get(_abi.GSC_FRAME_RANGES, np.uint32), z["ranges"])
    grads = gs.Rasterizer.backward(None, g, cam, ctx, target=to_dev(z["target"]),
                                   l1_scale=1.0 / z["target"].size)
    R.sync()
    pairs = {"position": grads.dL_dposition, "log_scale": grads.dL_dlog_scale,
             "rotation": grads.dL_drotation, "logit_opacity": grads.dL_dlogit_opacity,
             "sh_coeffs": grads.dL_dsh}
    for k, t in pairs.items():
        assert grad_close(host(t), z[f"grad_{k}"]) <= GRAD_RTOL, k
