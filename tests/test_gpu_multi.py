"""Two-GPU test of the fused data-parallel exchange (gsc_dp_adam_step): after
two training steps the fused path -- over peer loads and stores, and over the
NVSwitch multicast object where the box has one -- leaves every replica with
identical parameters, equal (fp32 summation order aside) to all-reduce + Adam."""
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

import dp_worker

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_fused_exchange_matches_allreduce(tmp_path):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=dp_worker.gpu_rank, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        if p.is_alive():
            p.kill()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    n0, n1 = (np.load(tmp_path / f"gpu_rank{r}_nccl.npy") for r in range(2))
    np.testing.assert_array_equal(n0, n1)
    scale = max(1.0, float(np.abs(n0).max()))
    for mode in ("fused", "multicast"):
        f0, f1 = (np.load(tmp_path / f"gpu_rank{r}_{mode}.npy") for r in range(2))
        np.testing.assert_array_equal(f0, f1)  # one writer per element: replicas identical
        # equal to all-reduce + Adam up to the fp32 order of the two-rank sum
        assert np.max(np.abs(f0 - n0)) <= 1e-5 * scale, mode
    path = (tmp_path / "gpu_rank0.status").read_text().split()[1]
    assert path in ("multimem", "peer")
    print("multicast exchange path:", path)
