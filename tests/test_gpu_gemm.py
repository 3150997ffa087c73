"""The tcgen05 bf16 GEMM (sm100_gemm_bf16: C = A . B^T, f32 accumulate)
through the C ABI against the CPU oracle (oracle.gemm_bf16: bf16 products in
f32, one accumulator in k order).  M = N = K = 4096 and
M = 8192, N = K = 4096, N(0,1) inputs; at those sizes 96 seeded rows are
checked against the oracle (the oracle's full product takes minutes).  The
tensor cores accumulate in another order: |dev - ref| <= 1e-4 (|ref| + rms)."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def close(dev, ref, tol=1e-4):
    dev, ref = np.asarray(dev, np.float64), np.asarray(ref, np.float64)
    scale = np.sqrt(np.mean(ref * ref)) + np.abs(ref)
    err = np.abs(dev - ref) - tol * scale
    assert err.max() <= 0, f"max excess {err.max()} at {np.unravel_index(err.argmax(), err.shape)}"


def run_gemm(device, a, b, M, N, K):
    from thvm_b200 import _lib as L
    pa, pb = device.upload(a), device.upload(b)
    c = device.alloc(M * N * 4)
    L.check(device.lib.sm100_gemm_bf16(device.dptr(pa), device.dptr(pb), device.dptr(c), M, N, K, device.stream),
            "gemm_bf16")
    device.sync()
    assert device.lib.sm100_gemm_status() == 0
    out = device.read(c, np.float32, (M, N))
    for bid in (pa, pb, c):
        device.free(bid)
    return out


def operands(M, N, K, seed):
    rng = np.random.default_rng(seed)
    a = O.to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    b = O.to_bf16(rng.standard_normal((N, K)).astype(np.float32))
    return a, b


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (128, 256, 192), (256, 512, 256), (384, 768, 1024)])
def test_gemm_small(device, M, N, K):
    a, b = operands(M, N, K, M + N + K)
    close(run_gemm(device, a, b, M, N, K), O.gemm_bf16(a, b))


@pytest.mark.parametrize("M,N,K", [(4096, 4096, 4096), (8192, 4096, 4096)])
def test_gemm_config2_rows(device, M, N, K):
    a, b = operands(M, N, K, 2)
    c = run_gemm(device, a, b, M, N, K)
    rows = np.sort(np.random.default_rng(3).choice(M, 96, replace=False))
    close(c[rows], O.gemm_bf16(a[rows], b))


def test_gemm_rejects_ragged_shapes(device):
    from thvm_b200 import _lib as L
    assert device.lib.sm100_gemm_bf16(None, None, None, 100, 256, 64, device.stream) == L.ERR_ARG
