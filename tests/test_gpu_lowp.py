"""bf16 and block-scaled fp8 e4m3 weights on the sm_100a linear kernel,
through the C ABI, against the CPU oracle (oracle.linear_bf16 / linear_fp8bs:
the reference's f32 Linear loop over the widened weights).  BASELINE config 2:
x[1, 4096] against W (11008 x 4096), bf16 and e4m3 with one f32 scale per
128 x 128 block (scales uniform in [0.5, 2]); plus ragged shapes.  The kernel
accumulates in f32 in another order (and scales 16-term partials), so the
bound is |dev - ref| <= 1e-4 * (|ref| + rms(ref))."""
import numpy as np
import pytest

import oracle as O
from thvm_b200 import _lib as L
from thvm_b200.gpt2 import make_op

pytestmark = pytest.mark.gpu


def close(dev, ref, tol=1e-4):
    dev, ref = np.asarray(dev, np.float64), np.asarray(ref, np.float64)
    assert dev.shape == ref.shape
    scale = np.sqrt(np.mean(ref * ref)) + np.abs(ref)
    err = np.abs(dev - ref) - tol * scale
    assert err.max() <= 0, f"max excess {err.max()}"


def inputs(M, K, N, seed):
    rng = np.random.default_rng(seed)
    x = O.bf16_to_f32(O.to_bf16(rng.standard_normal((M, K)).astype(np.float32)))
    return rng, x


@pytest.mark.parametrize("M,K,N", [(1, 4096, 11008), (2, 4096, 11008), (3, 1000, 700), (1, 136, 129)])
def test_linear_bf16(device, M, K, N):
    rng, x = inputs(M, K, N, 11)
    wb = O.to_bf16(rng.standard_normal((N, K)).astype(np.float32))
    y = device.alloc(M * N * 4)
    op = make_op(L.K_LINEAR, y, {0: device.upload(x), 1: device.upload(wb)}, m=M, n=N, k=K)
    op.kernel.dtype = L.DT_BF16
    device.dispatch(op.kernel, op.in_ids, op.out_id)
    device.sync()
    close(device.read(y, np.float32, (M, N)), O.linear_bf16(x, wb))


@pytest.mark.parametrize("M,K,N", [(1, 4096, 11008), (4, 4096, 11008), (2, 1000, 700), (1, 144, 130)])
def test_linear_fp8_block_scaled(device, M, K, N):
    rng, x = inputs(M, K, N, 12)
    w8 = O.to_fp8e4m3(rng.standard_normal((N, K)).astype(np.float32))
    sc = rng.uniform(0.5, 2.0, ((N + 127) // 128, (K + 127) // 128)).astype(np.float32)
    y = device.alloc(M * N * 4)
    op = make_op(L.K_LINEAR, y, {0: device.upload(x), 1: device.upload(w8), 6: device.upload(sc)}, m=M, n=N, k=K)
    op.kernel.dtype = L.DT_FP8E4M3
    device.dispatch(op.kernel, op.in_ids, op.out_id)
    device.sync()
    close(device.read(y, np.float32, (M, N)), O.linear_fp8bs(x, w8, sc))
