"""Host logic of the view-sharded data-parallel step on CPU ranks (gloo):
sharding + gradient all-reduce equals the single-process sum over all views,
and a rank that dies before the exchange is reported to the survivor as an
error instead of a hang."""
import multiprocessing as mp
import os
import socket

import numpy as np

import dp_worker


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def run(world, tmp_path, fail_rank=-1, timeout=120):
    ctx = mp.get_context("spawn")
    port = free_port()
    procs = [ctx.Process(target=dp_worker.dp_rank, args=(r, world, port, str(tmp_path), fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
            p.join()
    return procs


def test_sharding_and_allreduce_match_single_process(tmp_path):
    import importlib
    trainer = importlib.import_module("crystal-gausplat_b200.trainer")
    assert [trainer.shard(6, r, 4) for r in range(4)] == [(0, 1), (1, 3), (3, 4), (4, 6)]
    procs = run(2, tmp_path)
    assert all(p.exitcode == 0 for p in procs)
    gs, arrays, cams, targets = dp_worker.scene()
    ref = dp_worker.view_grads(arrays, cams, targets, range(len(cams)))
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}.npy")
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-6 * np.abs(ref).max())


def test_rank_failure_is_reported_not_hung(tmp_path):
    procs = run(2, tmp_path, fail_rank=1, timeout=90)
    assert procs[1].exitcode == 3
    status = (tmp_path / "rank0.status").read_text()
    assert status.startswith("error"), status


def test_multicast_address_of_a_tensor_in_a_symmetric_buffer():
    """The fused exchange's multicast form: the tensor's offset inside its
    symmetric-memory buffer carried onto the buffer's multicast address, and
    0 (the peer form) when the buffer has no multicast object."""
    import importlib
    trainer = importlib.import_module("crystal-gausplat_b200.trainer")

    class Tensor:
        def __init__(self, p):
            self.p = p

        def data_ptr(self):
            return self.p

    class Handle:
        def __init__(self, mc, rank=1):
            self._mc, self.rank = mc, rank
            self.buffer_ptrs = [0x1000, 0x20000]

        @property
        def multicast_ptr(self):
            if isinstance(self._mc, Exception):
                raise self._mc
            return self._mc

    assert trainer._multicast_ptr(Tensor(0x20000 + 256), Handle(0x7000000)) == 0x7000000 + 256
    assert trainer._multicast_ptr(Tensor(0x20000), Handle(0)) == 0
    assert trainer._multicast_ptr(Tensor(0x20000), Handle(RuntimeError("no multicast"))) == 0
    assert trainer.MULTICAST_MIN_RANKS == 4
