"""The reference's single-view Trainer loop (src/gaussian_splatting/trainer.cr:
15-57, 125-420): configuration defaults on the CPU; on the GPU a short run with
densification, pruning and an opacity reset inside the schedule."""
import numpy as np
import pytest

from helpers import gs, scene


def test_trainer_config_defaults_are_the_reference():
    c = gs.TrainerConfig()
    assert (c.iterations, c.densify_from, c.densify_until, c.densify_interval) == (30000, 500, 15000, 100)
    assert (c.opacity_reset_interval, c.prune_interval) == (3000, 100)
    assert c.lrs() == {"position": 0.00016, "log_scale": 0.005, "rotation": 0.001,
                       "logit_opacity": 0.05, "sh_coeffs": 0.0025}
    assert (c.lambda_ssim, c.densify_grad_threshold, c.densify_size_threshold,
            c.opacity_threshold) == (0.2, 0.0002, 0.01, 0.005)
    assert str(gs.TrainStats(3, 0.5, 20.0, 10)) == "Iter 3: loss=0.5000, PSNR=20.00dB, gaussians=10"


@pytest.mark.gpu
def test_trainer_loop_densifies_and_resets(cuda):
    import torch
    cams = gs.CameraSet(gs.make_camera(96, 80, tuple(e)) for e in gs.sphere_poses(4, 4.0, seed=2))
    truth = gs.Gaussian3D(scene(4000, 5))
    for c in cams:
        c.image = gs.Rasterizer.forward(truth, c)[0].clone()
    g = gs.Gaussian3D(scene(3000, 6))
    cfg = gs.TrainerConfig(iterations=12, densify_from=4, densify_until=10, densify_interval=4,
                           densify_grad_threshold=1e-6, opacity_reset_interval=11)
    tr = gs.Trainer(g, cams, cfg, seed=1)
    stats = []
    tr.train(stats.append)
    torch.cuda.synchronize()
    assert len(stats) == 12 and all(np.isfinite(s.loss) and s.loss > 0 for s in stats)
    counts = [s.num_gaussians for s in stats]
    assert counts[0] == 3000 and counts[-1] != 3000  # densified at steps 4 and 8
    assert tr.gaussians.count == tr.grad_accum.count
    assert torch.all(tr.gaussians.logit_opacity == -1.0)  # reset after step 11
