"""sm100_argmax_noalloc: the argmax entry point that allocates no device memory.

It exists for callers that cannot call cudaMalloc: a plugin whose device
memory belongs to a host framework's allocator, a service that fixes its
memory plan at start-up and allocates nothing after it, a process whose
device budget is spent.  Its scratch is a fixed array inside the library (at most
SM100_ARGMAX_NOALLOC_MAX_ROWS = 64 rows per call).  Its ids must equal those
of the allocating entry point sm100_argmax, exactly (argmax is index work),
on two calls in a row (the shared array keeps the previous call's contents).

This file is named to be collected last, so that a run that stops at the
first failure has already run every other test; it also passes alone in a
fresh process (the device fixture initialises the backend)."""
import numpy as np
import pytest

from thvm_b200 import _lib as L

pytestmark = pytest.mark.gpu


def _rows(seed, M, N):
    x = np.random.default_rng(seed).standard_normal((M, N)).astype(np.float32)
    x[0, 5] = x[0, N - 3] = x[0].max() + 2.0     # a tie: the first index wins
    x[M - 1, :] = -1.5                           # a constant row: index 0
    return x


def test_noalloc_argmax_matches_allocating_entry_point(device):
    lib = device.lib
    N = 50257
    out_ref = device.alloc(4 * 64)
    out_na = device.alloc(4 * 64)
    for call, (seed, M) in enumerate(((1, 7), (2, 64))):   # two calls in a row
        x = _rows(seed, M, N)
        xb = device.upload(x)
        assert lib.sm100_argmax(device.dptr(xb), M, N, 0, device.dptr(out_ref), None, device.stream) == 0
        assert lib.sm100_argmax_noalloc(device.dptr(xb), M, N, 0, device.dptr(out_na), None, device.stream) == 0, \
            lib.sm100_last_error()
        device.sync()
        ref = device.read(out_ref, np.int32, (M,))
        got = device.read(out_na, np.int32, (M,))
        assert np.array_equal(got, ref), (call, got, ref)
        assert np.array_equal(got, np.argmax(x, axis=1))


def test_noalloc_argmax_bump_and_limit(device):
    lib = device.lib
    x = device.upload(_rows(3, 2, 1000))
    out = device.alloc(8)
    pos = device.upload(np.array([10], np.int32))
    assert lib.sm100_argmax_noalloc(device.dptr(x), 2, 1000, 0, device.dptr(out), device.dptr(pos), device.stream) == 0
    device.sync()
    assert device.read(pos, np.int32, (1,))[0] == 11
    rc = lib.sm100_argmax_noalloc(device.dptr(x), 65, 1000, 0, device.dptr(out), None, device.stream)
    assert rc == L.ERR_ARG
    assert b"64 rows" in lib.sm100_last_error()
