"""Regenerates tests/golden/*.npz: small seeded views run through the CPU
oracle (inputs and every output the parity tests compare). The reference
(Crystal + Metal) cannot run here and ships no vectors for this path, so
these fixtures pin the oracle against regressions and give the GPU tests a
fixed answer that needs no oracle at run time.

    python tests/golden/make_golden.py
"""
import importlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

CASES = {  # name: (n, W, H, eye, seed)
    "view_a": (300, 48, 40, (0.0, 0.0, 4.0), 11),
    "view_b": (800, 70, 50, (2.0, 1.0, -3.0), 12),
}


def make(name, mode):
    gs = importlib.import_module("crystal-gausplat_b200")
    from oracle import oracle as O
    O.set_threads(1)
    n, W, H, eye, seed = CASES[name]
    arrays = gs.synthetic_arrays(n, seed)
    cam = gs.make_camera(W, H, eye)
    cs = cam.to_struct()
    cfg = gs.default_config(mode=mode, background=(0.05, 0.1, 0.15),
                            binning=gs._abi.GSC_BIN_REFERENCE)  # the reference lists
    sc = O.Scene(arrays)
    fw = O.forward_pipeline(sc, cs, cfg)
    target = np.random.default_rng(seed + 1).uniform(0, 1, (H, W, 3)).astype(np.float32)
    scale = 1.0 / target.size
    g2d, loss = O.composite_backward(W, H, fw["ranges"], fw["sorted_vals"], fw["pre"], cfg,
                                     fw["final_T"], fw["last"], image=fw["image"], target=target,
                                     l1_scale=scale)
    grads, _ = O.preprocess_backward(sc, cs, cfg, g2d)
    out = {f"in_{k}": v for k, v in arrays.items()}
    out.update(eye=np.float64(eye), W=W, H=H, mode=mode, target=target,
               view=np.float32(list(cs.view)), sorted_keys=fw["sorted_keys"], sorted_vals=fw["sorted_vals"],
               ranges=fw["ranges"], image=fw["image"], n_contrib=fw["n_contrib"], final_T=fw["final_T"],
               loss=np.float64(loss), **{f"grad_{k}": v for k, v in grads.items()})
    return out


def main():
    for name in CASES:
        for mode, tag in ((0, "full"), (1, "ref")):
            np.savez_compressed(os.path.join(HERE, f"{name}_{tag}.npz"), **make(name, mode))
            print("wrote", name, tag)


if __name__ == "__main__":
    main()
