"""The custom-kernel ABI on the device (sm100_custom_program / _dispatch): raw
CUDA-C programs compiled once by NVRTC for sm_100a and launched over backend
buffers, with the eager and capture-and-replay contract of the reference's
tests/test_custom_kernel_cuda.c: an eager kernel, an eager two-kernel chain
through a scratch buffer, the chain captured into a CUDA graph and replayed
three times over inputs rewritten in place, and a kernel with two outputs
under capture / replay; plus the primary-output rebinding and
registration caching."""
from ctypes import c_uint32

import numpy as np
import pytest

from thvm_b200 import _lib as L

pytestmark = pytest.mark.gpu

SRC_ADDONE = b'''extern "C" __global__ void addone(const float *x, float *y) {
  unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 8) y[i] = x[i] + 1.0f;
}
'''
SRC_DOUBLE = b'''extern "C" __global__ void dbl(const float *x, float *s) {
  unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 8) s[i] = x[i] * 2.0f;
}
'''
SRC_ADD3 = b'''extern "C" __global__ void add3(const float *s, float *y) {
  unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 8) y[i] = s[i] + 3.0f;
}
'''
SRC_TWO_OUT = b'''extern "C" __global__ void twoout(const float *x, float *y1, float *y2) {
  unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < 8) { y1[i] = x[i] + 1.0f; y2[i] = x[i] * 10.0f; }
}
'''
SRC_SHARED = b'''extern "C" __global__ void revsum(const float *x, float *y) {
  extern __shared__ float buf[];
  const unsigned n = 16384;
  for (unsigned i = threadIdx.x; i < n; i += blockDim.x) buf[i] = x[i];
  __syncthreads();
  for (unsigned i = threadIdx.x; i < n; i += blockDim.x) y[i] = buf[n - 1 - i] + buf[i];
}
'''

N = 8
GRID, BLOCK = (c_uint32 * 3)(1, 1, 1), (c_uint32 * 3)(N, 1, 1)


def _prog(lib, name, src, grid=GRID, block=BLOCK, shared=0):
    pid = lib.sm100_custom_program(name, src, grid, block, shared)
    assert pid > 0, lib.sm100_last_error()
    return pid


def _fire(lib, pid, ids, out_slot=1, out_id=0):
    arr = (c_uint32 * len(ids))(*ids)
    L.check(lib.sm100_custom_dispatch(pid, arr, len(ids), out_slot, out_id), "custom_dispatch")


def test_custom_eager_chain_and_graph_replays(device):
    dev, lib = device, device.lib
    xv = np.arange(N, dtype=np.float32)
    x, y = dev.upload(xv), dev.upload(np.zeros(N, np.float32))
    k_add = _prog(lib, b"addone", SRC_ADDONE)
    _fire(lib, k_add, [x, y])
    np.testing.assert_array_equal(dev.read(y), xv + 1.0)
    # the same program registered again is the same id: compiled once
    assert _prog(lib, b"addone", SRC_ADDONE) == k_add
    # eager two-kernel chain through a scratch buffer
    cx, scratch, cy = dev.upload(xv), dev.upload(np.zeros(N, np.float32)), dev.upload(np.zeros(N, np.float32))
    k_dbl, k_add3 = _prog(lib, b"dbl", SRC_DOUBLE), _prog(lib, b"add3", SRC_ADD3)
    _fire(lib, k_dbl, [cx, scratch])
    _fire(lib, k_add3, [scratch, cy])
    np.testing.assert_array_equal(dev.read(cy), xv * 2.0 + 3.0)
    # the chain captured once, replayed three times over inputs rewritten in place
    slot = dev.new_graph_slot()
    dev.capture_begin(slot)
    _fire(lib, k_dbl, [cx, scratch])
    _fire(lib, k_add3, [scratch, cy])
    dev.capture_end(slot)
    for rep in (1, 2, 3):
        xv = (10 * rep + np.arange(N)).astype(np.float32)
        dev.write(cx, xv)
        dev.write(scratch, np.full(N, -999.0, np.float32))
        dev.write(cy, np.full(N, -999.0, np.float32))
        dev.replay(slot)
        np.testing.assert_array_equal(dev.read(scratch), xv * 2.0)
        np.testing.assert_array_equal(dev.read(cy), xv * 2.0 + 3.0)
    dev.drop(slot)
    # two outputs under capture / replay
    mx, y1, y2 = dev.upload(xv), dev.upload(np.zeros(N, np.float32)), dev.upload(np.zeros(N, np.float32))
    k_two = _prog(lib, b"twoout", SRC_TWO_OUT)
    slot = dev.new_graph_slot()
    dev.capture_begin(slot)
    _fire(lib, k_two, [mx, y1, y2])
    dev.capture_end(slot)
    for rep in (1, 2, 3):
        xv = (7 * rep + np.arange(N)).astype(np.float32)
        dev.write(mx, xv)
        dev.replay(slot)
        np.testing.assert_array_equal(dev.read(y1), xv + 1.0)
        np.testing.assert_array_equal(dev.read(y2), xv * 10.0)
    dev.drop(slot)
    for b in (x, y, cx, scratch, cy, mx, y1, y2):
        dev.free(b)


def test_custom_out_rebinding_and_large_shared(device):
    """A non-zero out_buf_id replaces the primary output slot's buffer; a
    program asking for 64 KiB of dynamic shared memory gets the opt-in."""
    dev, lib = device, device.lib
    xv = np.arange(N, dtype=np.float32)
    x, y, other = dev.upload(xv), dev.upload(np.zeros(N, np.float32)), dev.upload(np.zeros(N, np.float32))
    k_add = _prog(lib, b"addone", SRC_ADDONE)
    _fire(lib, k_add, [x, y], out_slot=1, out_id=other)
    np.testing.assert_array_equal(dev.read(other), xv + 1.0)
    np.testing.assert_array_equal(dev.read(y), np.zeros(N, np.float32))
    n = 16384
    v = np.random.default_rng(0).standard_normal(n).astype(np.float32)
    xs, ys = dev.upload(v), dev.upload(np.zeros(n, np.float32))
    k = _prog(lib, b"revsum", SRC_SHARED, (c_uint32 * 3)(1, 1, 1), (c_uint32 * 3)(256, 1, 1), n * 4)
    _fire(lib, k, [xs, ys])
    np.testing.assert_array_equal(dev.read(ys), v[::-1] + v)
    for b in (x, y, other, xs, ys):
        dev.free(b)
