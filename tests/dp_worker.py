"""Worker processes for the gloo data-parallel tests (CPU ranks; the oracle
computes the per-view gradients, torch.distributed does the exchange)."""
import importlib
import os
import sys
from datetime import timedelta

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def scene():
    gs = importlib.import_module("crystal-gausplat_b200")
    arrays = gs.synthetic_arrays(400, 21)
    eyes = gs.sphere_poses(6, 4.0, 22)
    cams = [gs.make_camera(48, 32, tuple(e)) for e in eyes]
    targets = [np.random.default_rng(100 + v).uniform(0, 1, (32, 48, 3)).astype(np.float32)
               for v in range(len(cams))]
    return gs, arrays, cams, targets


def view_grads(arrays, cams, targets, views):
    """Sum of the oracle gradients of `views`, flattened in arena field order."""
    gs = importlib.import_module("crystal-gausplat_b200")
    from oracle import oracle as O
    O.set_threads(1)
    sc = O.Scene(arrays)
    cfg = gs.default_config()
    total = None
    for v in views:
        _, g, _, _ = O.render_view(sc, cams[v].to_struct(), cfg, targets[v], 1.0 / targets[v].size)
        flat = np.concatenate([g[k].reshape(-1) for k in ("position", "log_scale", "rotation",
                                                           "logit_opacity", "sh_coeffs")])
        total = flat if total is None else total + flat
    return total


def dp_rank(rank, world, port, out_dir, fail_rank=-1):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    trainer = importlib.import_module("crystal-gausplat_b200.trainer")
    gs, arrays, cams, targets = scene()
    lo, hi = trainer.shard(len(cams), rank, world)
    local = view_grads(arrays, cams, targets, range(lo, hi))
    if rank == fail_rank:
        # this rank dies between steps, before the exchange
        os._exit(3)
    t = torch.from_numpy(local)
    try:
        dist.all_reduce(t)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), t.numpy())
        status = "ok"
    except Exception as e:  # the surviving rank learns of the failure here
        status = "error: " + type(e).__name__
    with open(os.path.join(out_dir, f"rank{rank}.status"), "w") as f:
        f.write(status)
    if status == "ok":
        dist.destroy_process_group()


def gpu_rank(rank, world, port, out_dir, steps=2):
    """One GPU rank: the same training steps with the NCCL exchange and with the
    fused exchange (gsc_dp_adam_step); saves the final parameter arenas."""
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=timedelta(seconds=60))
    gs = importlib.import_module("crystal-gausplat_b200")
    trainer = importlib.import_module("crystal-gausplat_b200.trainer")
    arrays = gs.synthetic_arrays(20000, 31)
    eyes = gs.sphere_poses(8, 4.0, 32)
    cams = [gs.make_camera(128, 96, tuple(e)) for e in eyes]
    targets = [torch.from_numpy(np.random.default_rng(200 + v).uniform(0, 1, (96, 128, 3))
                                .astype(np.float32)).to(dev) for v in range(len(cams))]
    cfg = gs.default_config()
    paths = {}
    # "fused": peer loads and stores; "multicast": the NVSwitch multicast
    # object where the box has one (else the same peer path)
    for mode, exchange, mc in (("nccl", "nccl", False), ("fused", "fused", False),
                               ("multicast", "fused", True)):
        g = gs.Gaussian3D(arrays, device=dev)
        tr = trainer.DataParallelTrainer(g, cams, cfg, process_group=dist.group.WORLD, exchange=exchange,
                                         multicast=mc)
        for _ in range(steps):
            tr.step(lambda v: targets[v])
        if exchange == "fused":
            tr.check()  # no cross-rank wait gave up
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"gpu_rank{rank}_{mode}.npy"), g.arena.detach().cpu().numpy().copy())
        paths[mode] = tr.exchange_path
    with open(os.path.join(out_dir, f"gpu_rank{rank}.status"), "w") as f:
        f.write("ok " + str(paths.get("multicast")))
    dist.barrier()
    dist.destroy_process_group()
