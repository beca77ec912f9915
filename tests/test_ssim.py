"""SSIM, combined L1 + SSIM and MSE losses (src/ops/loss.cr:59-296).

CPU: the oracle's REF SSIM equals a literal restatement of Loss.ssim
(loss.cr:117-186) bit for bit; the oracle's FULL value and gradient match a
float64 torch autograd of the same definition. GPU: the CUDA path equals the
oracle bit for bit (maps, gradients) and within 1e-6 relative on the
double-summed loss values; at 1080p it matches float64 autograd within 1e-4.
"""
import numpy as np
import pytest

from helpers import _abi, gs, host, to_dev

FULL, REF = _abi.GSC_MODE_FULL, _abi.GSC_MODE_REF
VALUE_RTOL = 1e-6   # loss values: double sums cast to fp32 (GPU vs oracle)
GRAD_RTOL = 1e-4    # fp32 analytic gradient vs float64 autograd


def images(h, w, c=3, seed=0, corr=0.7):
    rng = np.random.default_rng(seed)
    t = rng.random((h, w, c), dtype=np.float32)
    p = (corr * t + (1 - corr) * rng.random((h, w, c), dtype=np.float32)).astype(np.float32)
    return p, t


def literal_ssim_map(oracle, pred, target, win=11):
    """Loss.ssim's loops (loss.cr:127-185) in numpy float32 scalars."""
    f = np.float32
    c = win // 2
    vals = []
    for y in range(win):
        for x in range(win):
            dx, dy = x - c, y - c
            vals.append(f(-(dx * dx + dy * dy)) / (f(2.0) * f(1.5) * f(1.5)))
    w = oracle.expf(np.array(vals, np.float32))
    s = f(0.0)
    for v in w:
        s = f(s + v)
    w = (w / s).astype(np.float32)
    H, W, C = pred.shape
    out = np.zeros_like(pred)
    C1, C2 = f(0.01) * f(0.01), f(0.03) * f(0.03)
    for ch in range(C):
        for y in range(c, H - c):
            for x in range(c, W - c):
                px = pred[y - c:y + c + 1, x - c:x + c + 1, ch].reshape(-1)
                py = target[y - c:y + c + 1, x - c:x + c + 1, ch].reshape(-1)
                mx = my = sx = sy = sxy = f(0.0)
                for k in range(win * win):
                    mx = f(mx + f(w[k] * px[k]))
                    my = f(my + f(w[k] * py[k]))
                for k in range(win * win):
                    a, b = f(px[k] - mx), f(py[k] - my)
                    sx = f(sx + f(f(w[k] * a) * a))
                    sy = f(sy + f(f(w[k] * b) * b))
                    sxy = f(sxy + f(f(w[k] * a) * b))
                num = f(f(f(f(2.0) * mx) * my) + C1) * f(f(f(2.0) * sxy) + C2)
                den = f(f(f(mx * mx) + f(my * my)) + C1) * f(f(sx + sy) + C2)
                out[y, x, ch] = f(num / den)
    return out


def torch_ssim64(pred, target, win=11):
    """Mean SSIM of the separable definition in float64 (valid region)."""
    import torch
    k = torch.arange(win, dtype=torch.float64) - win // 2
    g = torch.exp(-(k * k) / 4.5)
    g = (g / g.sum()).to(pred.device)
    C = pred.shape[2]
    x = pred.permute(2, 0, 1).unsqueeze(1)
    y = target.permute(2, 0, 1).unsqueeze(1)
    kh, kv = g.view(1, 1, 1, win), g.view(1, 1, win, 1)

    def blur(z):
        return torch.nn.functional.conv2d(torch.nn.functional.conv2d(z, kh), kv)
    mx, my = blur(x), blur(y)
    sxx, syy, sxy = blur(x * x) - mx * mx, blur(y * y) - my * my, blur(x * y) - mx * my
    c1, c2 = 0.01 ** 2, 0.03 ** 2
    s = ((2 * mx * my + c1) * (2 * sxy + c2)) / ((mx * mx + my * my + c1) * (sxx + syy + c2))
    return s.mean()


def test_ref_ssim_is_the_literal_reference(oracle):
    p, t = images(17, 21, 3, seed=1)
    out, _, smap = oracle.loss_grad(p, t, 11, REF, want_grad=False, want_map=True)
    lit = literal_ssim_map(oracle, p, t)
    np.testing.assert_array_equal(smap, lit)
    assert out[2] == np.float32(lit[5:-5, 5:-5].astype(np.float64).mean())


def test_full_value_and_gradient_vs_float64_autograd(oracle):
    import torch
    p, t = images(40, 33, 3, seed=2)
    out, grad, _ = oracle.loss_grad(p, t, 11, FULL, w_l1=0.0, w_ssim=1.0)
    pt = torch.from_numpy(p).double().requires_grad_(True)
    s = torch_ssim64(pt, torch.from_numpy(t).double())
    (1.0 - s).backward()
    assert abs(float(out[2]) - s.item()) <= 1e-6 * abs(s.item())
    g64 = pt.grad.numpy()
    err = np.abs(grad - g64).max() / np.abs(g64).max()
    assert err <= GRAD_RTOL, err
    # REF and FULL agree on the value to fp32 rounding.
    ref, _, _ = oracle.loss_grad(p, t, 11, REF, want_grad=False)
    assert abs(float(ref[2]) - float(out[2])) <= 1e-5


def test_combined_composition(oracle):
    p, t = images(24, 30, 3, seed=3)
    lam = np.float32(0.2)
    for mode in (REF, FULL):
        o, g, _ = oracle.loss_grad(p, t, 11, mode, w_l1=np.float32(1) - lam, w_ssim=lam)
        o_s, g_s, _ = oracle.loss_grad(p, t, 11, mode, w_l1=0.0, w_ssim=1.0)
        d = p - t
        n = np.float32(p.size)
        l1d = (np.sign(d).astype(np.float32) / n).astype(np.float32)
        expect = ((np.float32(1) - lam) * l1d + lam * g_s).astype(np.float32)
        np.testing.assert_array_equal(g, expect)
        assert o[1] == np.float32(np.abs(d).astype(np.float64).sum() / p.size)
        assert o[0] == (np.float32(1) - lam) * o[1] + lam * (np.float32(1) - o[2])
    # REF surrogate gradient of the SSIM term (loss.cr:208-212).
    _, g_ref, _ = oracle.loss_grad(p, t, 11, REF, w_l1=0.0, w_ssim=1.0)
    np.testing.assert_array_equal(g_ref, (np.float32(2) * (p - t) / np.float32(p.size)) * np.float32(1))


def test_image_smaller_than_window(oracle):
    p, t = images(8, 9, 3, seed=4)
    for mode in (REF, FULL):
        o, g, _ = oracle.loss_grad(p, t, 11, mode, w_l1=0.8, w_ssim=0.2)
        assert o[2] == 0.0 and o[0] == np.float32(0.8) * o[1] + np.float32(0.2)
        assert np.all(np.isfinite(g))


def test_mse_oracle(oracle):
    p, t = images(13, 11, 3, seed=5)
    o, g = oracle.mse_loss_grad(p, t)
    d = p - t
    assert o[0] == np.float32((d * d).astype(np.float64).sum() / d.size)
    np.testing.assert_array_equal(g, np.float32(2) * d / np.float32(d.size))


# ---------------------------------------------------------------- GPU parity

@pytest.mark.gpu
@pytest.mark.parametrize("h,w,c,win", [(16, 16, 3, 11), (37, 53, 3, 11), (64, 80, 1, 7),
                                       (130, 97, 4, 15), (9, 40, 3, 11), (256, 192, 3, 11)])
@pytest.mark.parametrize("mode", [REF, FULL])
def test_cuda_ssim_bit_exact(cuda, oracle, h, w, c, win, mode):
    import torch
    p, t = images(h, w, c, seed=h * w + c)
    o_out, o_grad, o_map = oracle.loss_grad(p, t, win, mode, w_l1=0.0, w_ssim=1.0, want_map=True)
    pd, td = to_dev(p), to_dev(t)
    smap = torch.zeros_like(pd)
    loss, grad = gs.Loss.ssim_loss_with_grad(pd, td, win, mode, ssim_map=smap)
    np.testing.assert_array_equal(host(smap), o_map)
    np.testing.assert_array_equal(host(grad), o_grad)
    assert abs(float(loss) - float(o_out[0])) <= VALUE_RTOL * max(1.0, abs(float(o_out[0])))


@pytest.mark.gpu
@pytest.mark.parametrize("mode", [REF, FULL])
def test_cuda_combined_bit_exact(cuda, oracle, mode):
    p, t = images(120, 136, 3, seed=7)
    lam = np.float32(0.2)
    o_out, o_grad, _ = oracle.loss_grad(p, t, 11, mode, w_l1=np.float32(1) - lam, w_ssim=lam)
    loss, grad = gs.Loss.combined_with_grad(to_dev(p), to_dev(t), 0.2, mode)
    np.testing.assert_array_equal(host(grad), o_grad)
    assert abs(float(loss) - float(o_out[0])) <= VALUE_RTOL * abs(float(o_out[0]))
    mse, mg = gs.Loss.mse_with_grad(to_dev(p), to_dev(t))
    m_out, m_grad = oracle.mse_loss_grad(p, t)
    np.testing.assert_array_equal(host(mg), m_grad)
    assert abs(float(mse) - float(m_out[0])) <= VALUE_RTOL * float(m_out[0])
    assert abs(gs.Loss.psnr(to_dev(p), to_dev(t)) - 10 * np.log10(1.0 / float(m_out[0]))) < 1e-4


@pytest.mark.gpu
def test_cuda_ssim_1080p_vs_float64_autograd(cuda):
    """Full-size image: the fp32 CUDA gradient against float64 autograd."""
    import torch
    torch.manual_seed(0)
    t = torch.rand(1080, 1920, 3, device="cuda")
    p = (0.7 * t + 0.3 * torch.rand(1080, 1920, 3, device="cuda")).contiguous()
    loss, grad = gs.Loss.ssim_loss_with_grad(p, t)
    p64 = p.double().requires_grad_(True)
    s = torch_ssim64(p64, t.double())
    (1.0 - s).backward()
    assert abs(float(loss) - (1.0 - s.item())) <= 1e-5
    err = float((grad.double() - p64.grad).abs().max() / p64.grad.abs().max())
    assert err <= GRAD_RTOL, err


@pytest.mark.gpu
def test_trainer_combined_loss(cuda):
    """Trainer with Trainer#train_step's combined loss: gradients equal the
    explicit loss -> dL/dimage -> backward chain, and the loss decreases."""
    import torch
    trainer = __import__("importlib").import_module("crystal-gausplat_b200.trainer")
    from helpers import scene
    cams = [gs.make_camera(96, 80, tuple(e)) for e in gs.sphere_poses(3, 4.0, seed=1)]
    targets = [torch.rand(80, 96, 3, device="cuda") for _ in cams]
    cfg = gs.default_config()
    g = gs.Gaussian3D(scene(6000, 3))
    g_ref = gs.Gaussian3D(scene(6000, 3))
    tr = trainer.DataParallelTrainer(g, cams, cfg, loss="combined", lambda_ssim=0.2)
    tr.zero()
    for v in range(len(cams)):
        tr.view_fwd_bwd(v, targets[v])
    tr.flush()
    grads = gs.RasterizerGradients(g_ref, screen=False)
    for v, cam in enumerate(cams):
        img, ctx = gs.Rasterizer.forward(g_ref, cam, config=cfg)
        _, dimg = gs.Loss.combined_with_grad(img, targets[v], 0.2)
        gs.Rasterizer.backward(dimg, g_ref, cam, ctx, grads=grads, config=cfg)
    torch.cuda.synchronize()
    from test_gpu_parity import GRAD_RTOL as G_RTOL, grad_close  # atomics: order-dependent sums
    assert grad_close(host(tr.grads.arena), host(grads.arena)) <= G_RTOL
    tr.reduce_and_step()
    losses = [float(tr.step(lambda v: targets[v])) for _ in range(15)]
    assert losses[-1] < losses[0]
