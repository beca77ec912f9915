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
