"""Densification and pruning: the oracle against a literal restatement of the
reference's densify_and_prune! (src/gaussian_splatting/trainer.cr:293-392,
gaussian.cr:150-271) on the CPU, and the CUDA path against the oracle bit
for bit on the GPU."""
import math

import numpy as np
import pytest

from helpers import _abi, gs, host, scene, to_dev

GRAD_T, SIZE_T, OP_T = 0.0002, 0.01, 0.005
LN16 = np.float32(math.log(1.6))
CLONE, SPLIT, PRUNE = _abi.GSC_DENSIFY_CLONE, _abi.GSC_DENSIFY_SPLIT, _abi.GSC_DENSIFY_PRUNE
FIELDS = ("position", "log_scale", "rotation", "logit_opacity", "sh_coeffs")


def densify_case(n, seed, prune_frac=0.1, log_scale_shift=0.0):
    """A scene whose accumulated gradients and opacities hit every category."""
    rng = np.random.default_rng(seed)
    a = scene(n, seed)
    a["log_scale"] = (a["log_scale"] + np.float32(log_scale_shift)).astype(np.float32)
    lo = rng.random(n) < prune_frac
    a["logit_opacity"][lo, 0] = np.float32(-8.0)  # sigmoid(-8) = 3.4e-4 < 0.005
    accum = (rng.random(n, dtype=np.float32) * np.float32(0.004)).astype(np.float32)
    count = rng.integers(0, 8, n).astype(np.int32)
    return a, accum, count


def reference_plan(a, accum, count):
    """densify_and_prune!'s loop (trainer.cr:304-325), literally."""
    to_clone, to_split, to_prune = [], [], set()
    n = a["position"].shape[0]
    for i in range(n):
        avg = np.float32(0.0) if count[i] == 0 else np.float32(accum[i] / np.float32(count[i]))
        s = oracle_expf(a["log_scale"][i])
        max_scale = max(s[0], max(s[1], s[2]))
        if avg > np.float32(GRAD_T):
            (to_split if max_scale > np.float32(SIZE_T) else to_clone).append(i)
        lg = np.float32(a["logit_opacity"][i, 0])
        op = np.float32(1.0) / (np.float32(1.0) + oracle_expf(np.array([-lg], np.float32))[0])
        if op < np.float32(OP_T):
            to_prune.add(i)
    return to_clone, to_split, to_prune


oracle_expf = None


@pytest.fixture(autouse=True)
def _expf(oracle):
    global oracle_expf
    oracle_expf = oracle.expf


def test_grad_accumulate_oracle(oracle):
    rng = np.random.default_rng(3)
    n = 1000
    d = rng.standard_normal((n, 9)).astype(np.float32)
    acc = rng.random(n, dtype=np.float32)
    cnt = rng.integers(0, 5, n).astype(np.int32)
    a2, c2 = acc.copy(), cnt.copy()
    oracle.grad_accumulate(d, a2, c2)
    expect = acc + np.sqrt(d[:, 0] * d[:, 0] + d[:, 1] * d[:, 1])
    np.testing.assert_array_equal(a2, expect)
    np.testing.assert_array_equal(c2, cnt + 1)


@pytest.mark.parametrize("seed", [1, 2])
def test_plan_matches_reference_loop(oracle, seed):
    a, accum, count = densify_case(3000, seed, log_scale_shift=0.5)
    flags, counts = oracle.densify_plan(oracle.Scene(a), accum, count, GRAD_T, SIZE_T, OP_T)
    to_clone, to_split, to_prune = reference_plan(a, accum, count)
    assert to_clone and to_split and to_prune
    assert list(np.nonzero(flags & CLONE)[0]) == to_clone
    assert list(np.nonzero(flags & SPLIT)[0]) == to_split
    assert set(np.nonzero(flags & PRUNE)[0].tolist()) == to_prune
    kept = sum(1 for i in range(3000) if i not in to_prune and i not in set(to_split))
    assert counts == (kept, len(to_clone), len(to_split))


def test_apply_clone_and_prune_equals_reference(oracle):
    """No splits: the reference's clone_gaussians + concat! + remove! order is
    exactly [kept][clones]; every field but the clone noise matches."""
    a, accum, count = densify_case(2000, 5, log_scale_shift=-3.0)
    sc = oracle.Scene(a)
    flags, counts = oracle.densify_plan(sc, accum, count, GRAD_T, SIZE_T, OP_T)
    assert counts[1] > 0 and counts[2] == 0
    out = oracle.densify_apply(sc, flags, 0.001, LN16, seed=9)
    to_clone, _, to_prune = reference_plan(a, accum, count)
    # reference: concat!(clone_gaussians(to_clone)) then remove!(to_prune) on
    # the concatenated set, whose first n rows are the originals.
    rows = [i for i in range(2000) if i not in to_prune] + to_clone
    for f in ("log_scale", "rotation", "logit_opacity", "sh_coeffs"):
        np.testing.assert_array_equal(out[f], a[f].reshape(2000, -1)[rows].reshape(out[f].shape))
    kept = counts[0]
    np.testing.assert_array_equal(out["position"][:kept], a["position"][rows[:kept]])
    d = out["position"][kept:] - a["position"][to_clone]
    assert np.all(np.abs(d) <= np.float32(0.001) * 1.0001)
    assert np.std(d) > 1e-4  # the noise is there


def test_apply_split_equals_reference(oracle):
    """No pruning: split_gaussians! removes the originals and appends two halves."""
    a, accum, count = densify_case(2000, 6, prune_frac=0.0, log_scale_shift=1.5)
    a["logit_opacity"][:] = np.float32(1.0)
    sc = oracle.Scene(a)
    flags, counts = oracle.densify_plan(sc, accum, count, GRAD_T, SIZE_T, OP_T)
    assert counts[2] > 0
    out = oracle.densify_apply(sc, flags, 0.001, LN16, seed=4)
    to_clone, to_split, _ = reference_plan(a, accum, count)
    kept, nc, ns = counts
    split_set = set(to_split)
    rows = [i for i in range(2000) if i not in split_set] + to_clone + to_split + to_split
    for f in ("rotation", "logit_opacity", "sh_coeffs"):
        np.testing.assert_array_equal(out[f], a[f].reshape(2000, -1)[rows].reshape(out[f].shape))
    ls = a["log_scale"][to_split] - LN16
    np.testing.assert_array_equal(out["log_scale"][kept + nc:kept + nc + ns], ls)
    np.testing.assert_array_equal(out["log_scale"][kept + nc + ns:], ls)
    bound = oracle_expf(ls[:, 0]) * np.float32(0.5) * np.float32(0.5)
    for h in range(2):
        blk = out["position"][kept + nc + h * ns:kept + nc + (h + 1) * ns]
        assert np.all(np.abs(blk - a["position"][to_split]) <= bound[:, None] * 1.0001)


def test_plan_never_prunes_everything(oracle):
    a = scene(500, 1)
    a["logit_opacity"][:] = np.float32(-9.0)
    flags, counts = oracle.densify_plan(oracle.Scene(a), np.zeros(500, np.float32),
                                        np.zeros(500, np.int32), GRAD_T, SIZE_T, OP_T)
    assert counts == (500, 0, 0) and not np.any(flags & PRUNE)


def test_apply_is_seeded(oracle):
    a, accum, count = densify_case(1000, 8, log_scale_shift=0.5)
    sc = oracle.Scene(a)
    flags, _ = oracle.densify_plan(sc, accum, count, GRAD_T, SIZE_T, OP_T)
    o1 = oracle.densify_apply(sc, flags, 0.001, LN16, seed=1)
    o2 = oracle.densify_apply(sc, flags, 0.001, LN16, seed=1)
    o3 = oracle.densify_apply(sc, flags, 0.001, LN16, seed=2)
    np.testing.assert_array_equal(o1["position"], o2["position"])
    assert not np.array_equal(o1["position"], o3["position"])


# ---------------------------------------------------------------- GPU parity

def _gpu_accum(accum, count):
    acc = gs.GradientAccumulator(accum.size)
    acc.position_grad_accum.copy_(to_dev(accum))
    acc.position_grad_count.copy_(to_dev(count))
    return acc


@pytest.mark.gpu
@pytest.mark.parametrize("n,seed,shift", [(1, 1, 0.0), (255, 2, 0.5), (257, 3, 0.5),
                                          (100_000, 4, 0.5), (1_000_003, 5, 0.8)])
def test_cuda_densify_bit_exact(cuda, oracle, n, seed, shift):
    a, accum, count = densify_case(n, seed, log_scale_shift=shift)
    sc = oracle.Scene(a)
    flags_o, counts_o = oracle.densify_plan(sc, accum, count, GRAD_T, SIZE_T, OP_T)
    out_o = oracle.densify_apply(sc, flags_o, 0.001, LN16, seed=seed)
    g = gs.Gaussian3D(a)
    acc = _gpu_accum(accum, count)
    flags, counts = gs.densify_plan(g, acc, GRAD_T, SIZE_T, OP_T)
    assert counts == counts_o
    np.testing.assert_array_equal(host(flags), flags_o)
    out = gs.densify_apply(g, flags, counts, 0.001, 1.6, seed=seed)
    assert out.count == sum(counts_o[:2]) + 2 * counts_o[2]
    for f in FIELDS:
        np.testing.assert_array_equal(host(getattr(out, f)).reshape(out_o[f].shape), out_o[f],
                                      err_msg=f)


@pytest.mark.gpu
def test_cuda_grad_accumulate_and_reset(cuda, oracle):
    import torch
    rng = np.random.default_rng(7)
    n = 300_001
    acc0 = rng.random(n, dtype=np.float32)
    cnt0 = rng.integers(0, 5, n).astype(np.int32)
    d2 = rng.standard_normal((n, 2)).astype(np.float32)
    acc = _gpu_accum(acc0, cnt0)
    acc.accumulate(to_dev(d2))
    a2, c2 = acc0.copy(), cnt0.copy()
    oracle.grad_accumulate(d2, a2, c2)
    np.testing.assert_array_equal(host(acc.position_grad_accum), a2)
    np.testing.assert_array_equal(host(acc.position_grad_count), c2)
    acc.resize(10)
    assert acc.count == 10
    g = gs.Gaussian3D(scene(1000, 1))
    gs.reset_opacity(g, -1.0)
    torch.cuda.synchronize()
    assert torch.all(g.logit_opacity == -1.0)


@pytest.mark.gpu
def test_cuda_densify_after_training(cuda):
    """A few real views: accumulate screen-space gradients, densify, render the new set."""
    import torch
    cam = gs.make_camera(128, 128, (0.0, 0.0, 4.0))
    g = gs.Gaussian3D(scene(20_000, 11))
    target = torch.rand(128, 128, 3, device="cuda")
    acc = gs.GradientAccumulator(g.count)
    for _ in range(3):
        img, ctx = gs.Rasterizer.forward(g, cam)
        grads = gs.Rasterizer.backward(None, g, cam, ctx, target=target)
        acc.accumulate(grads)
    assert int(acc.position_grad_count.min()) == 3
    g2 = gs.densify_and_prune(g, acc, grad_threshold=1e-7)
    assert g2.count > g.count and acc.count == g2.count
    assert int(acc.position_grad_count.sum()) == 0
    img2, _ = gs.Rasterizer.forward(g2, cam)
    torch.cuda.synchronize()
    assert torch.isfinite(img2).all()
    gs.Adam.for_gaussians(g2, gs.RasterizerGradients(g2)).step()
