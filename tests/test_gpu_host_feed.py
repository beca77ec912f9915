"""The host-fed training step (DataParallelTrainer.step_from_host with a
HostTargetFeeder, the bench's end-to-end path): targets copied from pinned
host memory on a side stream, several views ahead, each waited for only
before the backward that reads it. It must see the same targets as the
device-fed step: same loss, same gradients up to the order of the
backward's atomic adds."""
import importlib

import numpy as np
import pytest

from helpers import R, _abi, gs, host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("depth", [1, 3, 8])
def test_host_fed_views_match_device_fed(cuda, depth):
    trainer_mod = importlib.import_module("crystal-gausplat_b200.trainer")
    W, H, V = 128, 96, 11
    arrays = gs.synthetic_arrays(20_000, 0x7C0400)
    eyes = gs.sphere_poses(V, 4.0, 0x7C0401)
    cams = [gs.make_camera(W, H, tuple(e)) for e in eyes]
    targets = [np.random.default_rng(500 + v).random((H, W, 3), dtype=np.float32) for v in range(V)]
    pinned = cuda.from_numpy(np.stack(targets)).pin_memory()
    dev_t = [cuda.from_numpy(t).cuda() for t in targets]
    cfg = gs.default_config(binning=_abi.GSC_BIN_OCCLUDED)

    def grads_of(feed):
        g = gs.Gaussian3D(arrays)
        tr = trainer_mod.DataParallelTrainer(g, cams, cfg, batch_views=4)
        out = []
        for _ in range(2):  # the second pass reuses the feeder's slots and the views' tile cuts
            tr.zero()
            feed(tr)
            tr.flush()
            R.sync()
            out.append((float(tr.loss.item()), host(tr.grads.arena).copy()))
        return out

    def device_fed(tr):
        for v in range(V):
            tr.view_fwd_bwd(v, dev_t[v])

    feeder = trainer_mod.HostTargetFeeder(pinned, "cuda", depth=depth)
    assert len(feeder.bufs) == depth

    def host_fed(tr):
        feeder.run(range(V), lambda k, t, ready: tr.view_fwd_bwd(k, t, ready))

    ref = grads_of(device_fed)
    got = grads_of(host_fed)
    for (l0, g0), (l1, g1) in zip(ref, got):
        assert abs(l1 - l0) <= 1e-6 * abs(l0), (l0, l1)
        assert np.linalg.norm(g1 - g0) <= 1e-5 * np.linalg.norm(g0)
