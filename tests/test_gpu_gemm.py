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


@pytest.mark.parametrize("M,N,K,flags,use_bias,use_res", [
    (300, 104, 200, 0, True, True),        # ragged M, N, K (N, K multiples of 8)
    (208, 960, 320, 2, True, False),       # the prompt pass's qkv product shape class, bf16 out
    (256, 1280, 320, 3, True, False),      # + GELU, bf16 out
    (520, 808, 800, 0, False, True),       # K = 800 (6400 split 8 ways), in-place residual
])
def test_gemm_ep_matches_oracle(device, M, N, K, flags, use_bias, use_res):
    """sm100_gemm_bf16_ep: the product, then + bias, GELU, + residual and the
    bf16 store of round to nearest even, against the oracle's product with
    the same epilogue in f32 (GELU: oracle.gelu, the reference's tanh form);
    bf16 outputs within one bf16 step of the oracle's f32 value."""
    from thvm_b200 import _lib as L
    a, b = operands(M, N, K, M + N + K + flags)
    rng = np.random.default_rng(7)
    bias = rng.standard_normal(N).astype(np.float32) if use_bias else None
    res = rng.standard_normal((M, N)).astype(np.float32) if use_res else None
    ref = O.gemm_bf16(a, b)
    if bias is not None:
        ref = ref + bias
    if flags & L.GEMM_GELU:
        ref = O.gelu(ref)
    if res is not None:
        ref = ref + res
    out_bf16 = bool(flags & L.GEMM_OUT_BF16)
    pa, pb = device.upload(a), device.upload(b)
    pbias = device.upload(bias) if bias is not None else None
    c = device.upload(res) if (res is not None and not out_bf16) else device.alloc(M * N * (2 if out_bf16 else 4))
    pres = c if (res is not None and not out_bf16) else (device.upload(res) if res is not None else None)
    dp = lambda bid: device.dptr(bid) if bid is not None else None
    for _ in range(2):   # twice: the second call must not depend on the first (the in-place residual aside)
        if pres is not None and pres == c:
            device.write(c, res)
        L.check(device.lib.sm100_gemm_bf16_ep(dp(pa), dp(pb), dp(c), M, N, K, dp(pbias), dp(pres), flags,
                                              device.stream), "gemm_bf16_ep")
        device.sync()
        assert device.lib.sm100_gemm_status() == 0
        if out_bf16:
            got = O.bf16_to_f32(device.read(c, np.uint16, (M, N)))
            step = np.abs(ref) * 2.0 ** -8
            excess = np.abs(got - ref) - (step + 1e-4 * (np.sqrt(np.mean(ref * ref)) + np.abs(ref)))
            assert excess.max() <= 0, excess.max()
        else:
            close(device.read(c, np.float32, (M, N)), ref)
    for bid in {pa, pb, pbias, c, pres} - {None}:
        device.free(bid)


def test_gemm_ep_rejects_bad_shapes(device):
    from thvm_b200 import _lib as L
    lib = device.lib
    assert lib.sm100_gemm_bf16_ep(None, None, None, 128, 256, 64, None, None, 0, device.stream) == L.ERR_ARG
    a = device.alloc(1 << 16)
    p = device.dptr(a)
    assert lib.sm100_gemm_bf16_ep(p, p, p, 16, 100, 64, None, None, 0, device.stream) == L.ERR_ARG   # N % 8
    assert lib.sm100_gemm_bf16_ep(p, p, p, 16, 104, 60, None, None, 0, device.stream) == L.ERR_ARG   # K % 8
    assert lib.sm100_gemm_bf16_ep(p, p, p, 16, 104, 64, None, p, 2, device.stream) == L.ERR_ARG     # bf16 in place
    assert lib.sm100_gemm_bf16_ep(p, p, p, 16, 104, 64, None, None, 4, device.stream) == L.ERR_ARG  # unknown flag
    device.free(a)


@pytest.mark.parametrize("M,N,K,ep", [(2048, 4864, 512, False), (2000, 4856, 520, True), (4096, 4096, 1024, False)])
def test_gemm_partial_rounds_match_oracle(device, M, N, K, ep):
    """Shapes whose 256 x 256 tiles do not fill whole rounds of the 148 SMs
    (152, 152 and 256 tiles: a last round of 128-row halves, or of whole
    tiles), twice in a row, 96 seeded rows against the oracle; the second
    case ragged in M, N and K with the fused epilogue (bias, GELU, bf16
    out)."""
    from thvm_b200 import _lib as L
    a, b = operands(M, N, K, 11 + M + N + K)
    rows = np.sort(np.random.default_rng(3).choice(M, 96, replace=False))
    ref = O.gemm_bf16(a[rows], b)
    bias = np.random.default_rng(8).standard_normal(N).astype(np.float32) if ep else None
    if ep:
        ref = O.gelu(ref + bias)
    pa, pb = device.upload(a), device.upload(b)
    pbias = device.upload(bias) if ep else None
    c = device.alloc(M * N * (2 if ep else 4))
    for _ in range(2):
        if ep:
            L.check(device.lib.sm100_gemm_bf16_ep(device.dptr(pa), device.dptr(pb), device.dptr(c), M, N, K,
                                                  device.dptr(pbias), None, L.GEMM_GELU | L.GEMM_OUT_BF16,
                                                  device.stream), "gemm_bf16_ep")
        else:
            L.check(device.lib.sm100_gemm_bf16(device.dptr(pa), device.dptr(pb), device.dptr(c), M, N, K,
                                               device.stream), "gemm_bf16")
        device.sync()
        assert device.lib.sm100_gemm_status() == 0
        if ep:
            got = O.bf16_to_f32(device.read(c, np.uint16, (M, N)))[rows]
            excess = np.abs(got - ref) - (np.abs(ref) * 2.0 ** -8 + 1e-4 * (np.sqrt(np.mean(ref * ref)) + np.abs(ref)))
            assert excess.max() <= 0, excess.max()
        else:
            close(device.read(c, np.float32, (M, N))[rows], ref)
    for bid in (pa, pb, c) + ((pbias,) if ep else ()):
        device.free(bid)
