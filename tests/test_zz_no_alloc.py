"""gsc_sort_pairs_u64_static: the sort for callers that cannot allocate device
memory (their own pool owns all of it, or they must not take the driver's
allocation locks, or they have no gsc_ctx). It must give exactly what
gsc_sort_pairs_u64 gives -- keys and values bit-exact, the bar of every sort
test here -- on two calls in a row through the shared fixed scratch array,
report a clean device status after each, change neither the free device
memory nor torch's allocation, and refuse sizes beyond its limit. This file sorts last so that a run that
stops at the first failure has already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import R, _abi, u32_dev, u32_host, u64_dev, u64_host

pytestmark = pytest.mark.gpu


def _pairs(n, seed, tiles=8160):
    rng = np.random.default_rng(seed)
    t = rng.integers(0, tiles, n, dtype=np.uint64)
    d = rng.uniform(0.5, 10.0, n).astype(np.float32).view(np.uint32).astype(np.uint64)
    keys = (t << np.uint64(32)) | d
    keys[: n // 8] = keys[n // 8: 2 * (n // 8)]  # duplicates: stability matters
    return keys, np.arange(n, dtype=np.uint32)


def test_static_sort_matches_context_sort_twice(cuda):
    lib = _abi.lib()
    stream = C.c_void_p(cuda.cuda.current_stream().cuda_stream)
    cases = ((_abi.GSC_STATIC_SORT_MAX_PAIRS, 1, 0, 45), (70001, 2, 0, 64))
    # Every buffer is made before the measured calls, so a change of free
    # device memory or of torch's allocation during them would be the sort's.
    inputs = []
    for n, seed, begin, end in cases:
        keys, vals = _pairs(n, seed)
        ref_k, ref_v = u64_dev(keys), u32_dev(vals)
        _abi.check(lib.gsc_sort_pairs_u64(R.context(), R.ptr(ref_k), R.ptr(ref_v), n, begin, end))
        inputs.append((keys, vals, ref_k, ref_v, u64_dev(keys), u32_dev(vals)))
    # one warm-up call on a buffer of its own (the first call on a device may
    # load the device code and reserve the array)
    wk, wv = u64_dev(inputs[1][0]), u32_dev(inputs[1][1])
    _abi.check(lib.gsc_sort_pairs_u64_static(R.ptr(wk), R.ptr(wv), 70001, 0, 64, stream))
    assert lib.gsc_sort_pairs_u64_static_status(stream) == _abi.GSC_OK
    cuda.cuda.synchronize()
    free0 = cuda.cuda.mem_get_info()[0]
    alloc0 = cuda.cuda.memory_allocated()
    # Two calls in a row with different sizes and bit ranges: the second must
    # not see anything the first left in the shared array.
    for (n, seed, begin, end), (keys, vals, ref_k, ref_v, got_k, got_v) in zip(cases, inputs):
        _abi.check(lib.gsc_sort_pairs_u64_static(R.ptr(got_k), R.ptr(got_v), n, begin, end, stream))
        assert lib.gsc_sort_pairs_u64_static_status(stream) == _abi.GSC_OK, lib.gsc_last_error()
        assert cuda.cuda.mem_get_info()[0] == free0
        assert cuda.cuda.memory_allocated() == alloc0
        np.testing.assert_array_equal(u64_host(got_k), u64_host(ref_k))
        np.testing.assert_array_equal(u32_host(got_v), u32_host(ref_v))
        order = np.argsort(keys if end == 64 else keys & np.uint64((1 << end) - 1), kind="stable")
        np.testing.assert_array_equal(u32_host(got_v), vals[order])


def test_static_sort_rejects_oversize(cuda):
    lib = _abi.lib()
    n = _abi.GSC_STATIC_SORT_MAX_PAIRS + 1
    rc = lib.gsc_sort_pairs_u64_static(None, None, n, 0, 64, None)
    assert rc == _abi.GSC_ERR_INVALID
    assert b"exceeds" in lib.gsc_last_error()
