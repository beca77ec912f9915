"""Pins the oracle's FULL-mode gradients with float64 central finite
differences of an independent numpy restatement of the forward pass.

The discrete decisions of the forward (culling, radius, tile lists, which
pixel-Gaussian pairs pass the alpha and transmittance tests) are frozen at
the unperturbed point, exactly as the analytic backward treats them, so the
finite differences of the frozen model are the analytic gradient.
"""
import numpy as np
import pytest

SH_C0 = 0.28209479177387814
SH_C1 = 0.4886025119029199
SH_C2 = [1.0925484305920792, -1.0925484305920792, 0.31539156525252005, -1.0925484305920792,
         0.5462742152960396]
SH_C3 = [-0.5900435899266435, 2.890611442640554, -0.4570457994644658, 0.3731763325901154,
         -0.4570457994644658, 1.445305721320277, -0.5900435899266435]


def sh_basis(d):
    x, y, z = d[:, 0], d[:, 1], d[:, 2]
    xx, yy, zz = x * x, y * y, z * z
    b = [np.full_like(x, SH_C0), -SH_C1 * y, SH_C1 * z, -SH_C1 * x,
         SH_C2[0] * x * y, SH_C2[1] * y * z, SH_C2[2] * (2 * zz - xx - yy), SH_C2[3] * x * z,
         SH_C2[4] * (xx - yy),
         SH_C3[0] * y * (3 * xx - yy), SH_C3[1] * x * y * z, SH_C3[2] * y * (4 * zz - xx - yy),
         SH_C3[3] * z * (2 * zz - 3 * xx - 3 * yy), SH_C3[4] * x * (4 * zz - xx - yy),
         SH_C3[5] * z * (xx - yy), SH_C3[6] * x * (xx - 3 * yy)]
    return np.stack(b, axis=1)  # [N,16]


def quat_R(q):
    q = q / np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    R = np.empty((q.shape[0], 3, 3))
    R[:, 0, 0] = 1 - 2 * (y * y + z * z); R[:, 0, 1] = 2 * (x * y - z * w); R[:, 0, 2] = 2 * (x * z + y * w)
    R[:, 1, 0] = 2 * (x * y + z * w); R[:, 1, 1] = 1 - 2 * (x * x + z * z); R[:, 1, 2] = 2 * (y * z - x * w)
    R[:, 2, 0] = 2 * (x * z - y * w); R[:, 2, 1] = 2 * (y * z + x * w); R[:, 2, 2] = 1 - 2 * (x * x + y * y)
    return R


def project(P, cam):
    W = np.array(cam.view, np.float64).reshape(4, 4)
    V = W[:3, :3]
    s = np.exp(P["log_scale"])
    R = quat_R(P["rotation"])
    M = R * s[:, None, :]
    Sigma = M @ np.transpose(M, (0, 2, 1))
    pc = P["position"] @ V.T + W[:3, 3]
    x, y, z = pc.T
    fx, fy = cam.fx, cam.fy
    px = fx * x / z + cam.cx
    py = fy * y / z + cam.cy
    J = np.zeros((len(z), 2, 3))
    J[:, 0, 0] = fx / z; J[:, 0, 2] = -fx * x / z ** 2
    J[:, 1, 1] = fy / z; J[:, 1, 2] = -fy * y / z ** 2
    C = V[None] @ Sigma @ V.T[None]
    cov2 = J @ C @ np.transpose(J, (0, 2, 1))
    cov2[:, 0, 0] += 0.3
    cov2[:, 1, 1] += 0.3
    conic = np.linalg.inv(cov2)
    campos = np.array(cam.campos, np.float64)
    v = campos[None] - P["position"]
    d = v / np.linalg.norm(v, axis=1, keepdims=True)
    raw = np.einsum("nk,nkc->nc", sh_basis(d), P["sh"].reshape(-1, 16, 3)) + 0.5
    col = np.maximum(raw, 0.0)
    op = 1.0 / (1.0 + np.exp(-P["logit_opacity"].reshape(-1)))
    return px, py, z, conic, col, op


def render(P, cam, lists, masks, W, H):
    """Composite with the frozen tile lists / contribution masks."""
    px, py, z, conic, col, op = project(P, cam)
    img = np.zeros((H, W, 3))
    for (tx, ty), ids in lists.items():
        xs = np.arange(tx * 16, min(W, tx * 16 + 16))
        ys = np.arange(ty * 16, min(H, ty * 16 + 16))
        gx, gy = np.meshgrid(xs + 0.5, ys + 0.5)
        T = np.ones_like(gx)
        C = np.zeros(gx.shape + (3,))
        for g in ids:
            dx, dy = gx - px[g], gy - py[g]
            A, B, Cc = conic[g, 0, 0], conic[g, 0, 1], conic[g, 1, 1]
            power = -0.5 * (A * dx * dx + 2 * B * dx * dy + Cc * dy * dy)
            alpha = op[g] * np.exp(power) * masks[(tx, ty, g)]
            C += (T * alpha)[..., None] * col[g]
            T = T * (1 - alpha)
        img[ys[0]:ys[-1] + 1, xs[0]:xs[-1] + 1] = C
    return img


@pytest.mark.parametrize("seed", [3, 4])
def test_full_mode_gradients_match_finite_differences(gs, oracle, seed):
    W = H = 32
    n = 12
    rng = np.random.default_rng(seed)
    arrays = gs.synthetic_arrays(n, seed, extent=0.5)
    arrays["log_scale"][:] = rng.normal(-2.3, 0.2, (n, 3)).astype(np.float32)
    arrays["logit_opacity"][:] = rng.normal(-0.5, 0.4, (n, 1)).astype(np.float32)
    cam = gs.make_camera(W, H, (0.3, -0.2, 3.0)).to_struct()
    cfg = gs.default_config(t_stop=1e-6)
    sc = oracle.Scene(arrays)
    fw = oracle.forward_pipeline(sc, cam, cfg)
    pre = fw["pre"]
    lists, masks = {}, {}
    ranges = fw["ranges"].reshape(-1, 2)
    tiles_x = (W + 15) // 16
    for t in range(ranges.shape[0]):
        ids = [int(g) for g in fw["sorted_vals"][ranges[t, 0]:ranges[t, 1]]]
        tx, ty = t % tiles_x, t // tiles_x
        lists[(tx, ty)] = ids
        xs = np.arange(tx * 16, min(W, tx * 16 + 16))
        ys = np.arange(ty * 16, min(H, ty * 16 + 16))
        gx, gy = np.meshgrid(xs + 0.5, ys + 0.5)
        for g in ids:
            mx, my = pre["mean2d"][g]
            a, b, c = pre["cov2d"][g].astype(np.float64)
            det = a * c - b * b
            A, B, Cc = c / det, -b / det, a / det
            dx, dy = gx - mx, gy - my
            power = -0.5 * (A * dx * dx + 2 * B * dx * dy + Cc * dy * dy)
            alpha = pre["opacity"][g] * np.exp(power)
            masks[(tx, ty, g)] = ((power <= 0) & (alpha >= 1 / 255)).astype(np.float64)
    assert np.max(pre["opacity"]) < 0.99
    wts = rng.standard_normal((H, W, 3))
    P = {"position": arrays["position"].astype(np.float64), "log_scale": arrays["log_scale"].astype(np.float64),
         "rotation": arrays["rotation"].astype(np.float64),
         "logit_opacity": arrays["logit_opacity"].astype(np.float64),
         "sh": arrays["sh_coeffs"].astype(np.float64).reshape(n, 48)}
    img64 = render(P, cam, lists, masks, W, H)
    np.testing.assert_allclose(img64, fw["image"], atol=2e-5)
    g2d, _ = oracle.composite_backward(W, H, fw["ranges"], fw["sorted_vals"], pre, cfg, fw["final_T"],
                                       fw["last"], dL_dimage=wts.astype(np.float32))
    grads, _ = oracle.preprocess_backward(sc, cam, cfg, g2d)
    name_map = {"position": "position", "log_scale": "log_scale", "rotation": "rotation",
                "logit_opacity": "logit_opacity", "sh": "sh_coeffs"}
    for key, gname in name_map.items():
        ana = grads[gname].reshape(-1).astype(np.float64)
        fd = np.zeros_like(ana)
        flat = P[key].reshape(-1)
        for j in range(flat.size):
            h = 1e-5
            old = flat[j]
            flat[j] = old + h
            lp = float(np.sum(wts * render(P, cam, lists, masks, W, H)))
            flat[j] = old - h
            lm = float(np.sum(wts * render(P, cam, lists, masks, W, H)))
            flat[j] = old
            fd[j] = (lp - lm) / (2 * h)
        err = np.linalg.norm(ana - fd) / max(np.linalg.norm(fd), 1e-12)
        assert err < 2e-3, (key, err)
