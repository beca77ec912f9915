"""Failure detection on the GPU without a GPU fault: the sort's bounded
look-back wait is made to run out (its predecessor never publishes), the
kernel finishes, the host reads the timeout through gsc_sync, and the context
stays usable. The static sort's status query reports a clean run."""
import ctypes as C

import numpy as np
import pytest

from helpers import R, _abi, u32_dev, u32_host, u64_dev, u64_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("spin_limit", [1, 300])
def test_lookback_wait_gives_up_and_context_survives(cuda, spin_limit):
    lib = _abi.lib()
    ctx = R.context()
    assert lib.gsc_sync(ctx) == _abi.GSC_OK
    assert lib.gsc_selftest_wait_timeout(ctx, spin_limit) == _abi.GSC_OK
    assert lib.gsc_sync(ctx) == _abi.GSC_ERR_TIMEOUT
    assert b"gave up" in lib.gsc_last_error()
    assert lib.gsc_sync(ctx) == _abi.GSC_OK  # the flag was cleared
    # the context still sorts correctly afterwards
    rng = np.random.default_rng(spin_limit)
    keys = rng.integers(0, 2**63, 100_000, dtype=np.uint64)
    vals = np.arange(keys.size, dtype=np.uint32)
    dk, dv = u64_dev(keys), u32_dev(vals)
    _abi.check(lib.gsc_sort_pairs_u64(ctx, R.ptr(dk), R.ptr(dv), keys.size, 0, 64))
    assert lib.gsc_sync(ctx) == _abi.GSC_OK
    order = np.argsort(keys, kind="stable")
    np.testing.assert_array_equal(u64_host(dk), keys[order])
    np.testing.assert_array_equal(u32_host(dv), vals[order])


def _barrier_args(flags_a, flags_b, epoch, timeout_us):
    b = _abi.DpBarrierArgs()
    b.nranks, b.rank = 2, 0
    b.peer_flags[0] = flags_a.data_ptr()  # this rank's own flag array
    b.peer_flags[1] = flags_b.data_ptr()  # stands in for the peer's array
    b.epoch, b.timeout_us = epoch, timeout_us
    return b


def test_dp_barrier_times_out_without_a_peer_and_skips_the_exchange(cuda):
    """A peer that never arrives: the barrier's wait runs out (its flag is
    never set), the fused exchange that follows touches nothing, and the host
    reads GSC_ERR_TIMEOUT; the context stays usable."""
    lib = _abi.lib()
    ctx = R.context()
    flags_a = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    flags_b = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    assert lib.gsc_sync(ctx) == _abi.GSC_OK
    b = _barrier_args(flags_a, flags_b, 1, 2000)
    _abi.check(lib.gsc_dp_barrier(ctx, C.byref(b)))
    # a one-rank-shard exchange over local arenas: must be skipped
    n = 4096
    params = cuda.ones(n, device="cuda")
    grads = cuda.ones(n, device="cuda")
    m = cuda.zeros(n, device="cuda")
    v = cuda.zeros(n, device="cuda")
    a = _abi.DpAdamArgs()
    a.nranks, a.rank = 2, 0
    for p in range(2):
        a.peer_grads[p], a.peer_params[p] = grads.data_ptr(), params.data_ptr()
    a.m, a.v, a.ngroups = m.data_ptr(), v.data_ptr(), 1
    a.offset[0], a.numel[0], a.lr[0] = 0, n, 0.1
    a.beta1, a.beta2, a.eps, a.step, a.grad_scale = 0.9, 0.999, 1e-8, 1, 1.0
    _abi.check(lib.gsc_dp_adam_step(ctx, C.byref(a)))
    assert lib.gsc_sync(ctx) == _abi.GSC_ERR_TIMEOUT
    assert int(flags_b[0].item()) == 1          # the signal to the peer was published
    assert float(params.min()) == 1.0 and float(params.max()) == 1.0  # nothing updated
    assert lib.gsc_sync(ctx) == _abi.GSC_OK


def test_dp_barrier_passes_when_the_peer_has_arrived(cuda):
    lib = _abi.lib()
    ctx = R.context()
    flags_a = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    flags_b = cuda.zeros(2, dtype=cuda.int32, device="cuda")
    for epoch in (1, 2, 3):
        flags_a[1] = epoch  # the peer's signal for this epoch is already there
        b = _barrier_args(flags_a, flags_b, epoch, 1_000_000)
        _abi.check(lib.gsc_dp_barrier(ctx, C.byref(b)))
        assert lib.gsc_sync(ctx) == _abi.GSC_OK
        assert int(flags_b[0].item()) == epoch
