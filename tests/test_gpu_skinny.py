"""The skinny tcgen05 GEMM of batched decode (sm100_skinny_bf16: Y = epi(X W^T),
X [M <= 32, K] and W [N, K] bf16, f32 accumulate) through the C ABI against the
CPU oracle (oracle.gemm_bf16: bf16 products in f32) with the epilogue applied
in the reference's order (bias, tanh GELU as oracle.gelu, residual).  Shapes:
the GPT-2-XL projections of BASELINE config 3 at batch 16 (c_attn 1600 -> 4800,
c_proj 1600 -> 1600, c_fc 1600 -> 6400, mlp proj 6400 -> 1600), ragged M / N /
K, and M = 32.  The tensor cores sum in another order: |dev - ref| <= 1e-4
(|ref| + rms)."""
import ctypes

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu


def close(dev, ref, tol=1e-4):
    dev, ref = np.asarray(dev, np.float64), np.asarray(ref, np.float64)
    scale = np.sqrt(np.mean(ref * ref)) + np.abs(ref)
    err = np.abs(dev - ref) - tol * scale
    assert err.max() <= 0, f"max excess {err.max()} at {np.unravel_index(err.argmax(), err.shape)}"


def bf16_to_f32(b):
    return (b.astype(np.uint32) << 16).view(np.float32)


def run(device, x, w, bias=None, residual=None, flags=0, kv=None, pos=None, kv_ctx=0, repeat=1, accumulate=1):
    from thvm_b200 import _lib as L
    M, K = x.shape
    N = w.shape[0]
    ids = {"x": device.upload(x), "w": device.upload(w)}
    if bias is not None:
        ids["bias"] = device.upload(bias)
    out_bytes = M * N * (2 if flags & L.SK_OUT_BF16 else 4)
    ids["y"] = device.upload(residual.copy()) if residual is not None else device.alloc(out_bytes)
    ids["ws"] = device.alloc(device.lib.sm100_skinny_ws_bytes(M))
    ids["counters"] = device.alloc(((N + 127) // 128) * 4)
    device.lib.sm100_buf_zero(ids["counters"])
    if kv is not None:
        ids["kv_cache"] = device.upload(kv)
        ids["pos"] = device.upload(np.array([pos], np.int32))
    a = L.Sm100SkinnyArgs()
    for k, v in ids.items():
        setattr(a, k, device.dptr(v))
    if residual is not None and not flags & L.SK_ACCUM:
        a.residual = a.y
    a.M, a.N, a.K, a.flags, a.kv_ctx = M, N, K, flags, kv_ctx
    for _ in range(repeat):
        if residual is not None:
            device.write(ids["y"], residual)
        for _ in range(accumulate):
            L.check(device.lib.sm100_skinny_bf16(ctypes.byref(a), device.stream), "skinny")
    device.sync()
    assert device.lib.sm100_skinny_status() == 0
    if flags & L.SK_OUT_BF16:
        y = bf16_to_f32(device.read(ids["y"], np.uint16, (M, N)))
    else:
        y = device.read(ids["y"], np.float32, (M, N))
    kv_out = device.read(ids["kv_cache"], np.uint16, kv.shape) if kv is not None else None
    for v in ids.values():
        device.free(v)
    return y, kv_out


def operands(M, N, K, seed):
    rng = np.random.default_rng(seed)
    x = O.to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    w = O.to_bf16((0.02 * rng.standard_normal((N, K))).astype(np.float32))
    b = (0.02 * rng.standard_normal(N)).astype(np.float32)
    return x, w, b


@pytest.mark.parametrize("M,N,K", [(16, 4800, 1600), (16, 1600, 1600), (16, 6400, 1600), (16, 1600, 6400),
                                   (5, 300, 200), (1, 128, 64), (32, 1000, 512), (23, 2000, 1032)])
def test_skinny_plain(device, M, N, K):
    x, w, _ = operands(M, N, K, M + N + K)
    y, _ = run(device, x, w)
    close(y, O.gemm_bf16(x, w))


def test_skinny_epilogues(device):
    """bias + GELU to bf16 (the c_fc shape), and bias + residual in place (the projections);
    repeated launches reuse the tile counters."""
    from thvm_b200 import _lib as L
    M, N, K = 16, 6400, 1600
    x, w, b = operands(M, N, K, 1)
    y, _ = run(device, x, w, bias=b, flags=L.SK_GELU | L.SK_OUT_BF16, repeat=3)
    ref = O.gelu(O.gemm_bf16(x, w) + b)
    close(y, bf16_to_f32(O.to_bf16(ref)), tol=1e-2)   # bf16 output: half an ulp of 2^-8
    M, N, K = 16, 1600, 6400
    x, w, b = operands(M, N, K, 2)
    res = np.random.default_rng(3).standard_normal((M, N)).astype(np.float32)
    y, _ = run(device, x, w, bias=b, residual=res, flags=L.SK_RESIDUAL, repeat=2)
    close(y, O.gemm_bf16(x, w) + b + res)


def test_skinny_kv_append(device):
    """The fused qkv projection writes its k / v thirds into the bf16 cache row pos."""
    from thvm_b200 import _lib as L
    M, C, K, ctx, pos = 16, 1600, 1600, 64, 37
    x, w, b = operands(M, 3 * C, K, 4)
    kv = np.zeros((2, M, ctx, C), np.uint16)
    y, kv_out = run(device, x, w, bias=b, flags=L.SK_KV, kv=kv, pos=pos, kv_ctx=ctx)
    ref = O.gemm_bf16(x, w) + b
    close(y, ref)
    np.testing.assert_array_equal(kv_out[0, :, pos], O.to_bf16(y[:, C:2 * C]))
    np.testing.assert_array_equal(kv_out[1, :, pos], O.to_bf16(y[:, 2 * C:]))
    assert not kv_out[:, :, :pos].any() and not kv_out[:, :, pos + 1:].any()


def test_skinny_accumulate(device):
    """SM100_SK_ACCUM: y += X W^T + bias, twice over the same y (the bias once per call)."""
    from thvm_b200 import _lib as L
    M, N, K = 16, 1600, 6400
    x, w, b = operands(M, N, K, 6)
    y0 = np.random.default_rng(7).standard_normal((M, N)).astype(np.float32)
    y, _ = run(device, x, w, bias=b, residual=y0, flags=L.SK_ACCUM, repeat=1, accumulate=2)
    close(y, y0 + 2 * (O.gemm_bf16(x, w) + b))


def test_skinny_x_gelu(device):
    """SM100_SK_X_GELU: the f32 operand enters the product as bf16(gelu(x)) (the MLP down-projection)."""
    from thvm_b200 import _lib as L
    for M, N, K in ((16, 1600, 6400), (5, 300, 520)):
        rng = np.random.default_rng(K)
        xf = rng.standard_normal((M, K)).astype(np.float32)
        _, w, b = operands(M, N, K, 8)
        y0 = np.zeros((M, N), np.float32)
        y, _ = run(device, xf, w, bias=b, residual=y0, flags=L.SK_ACCUM | L.SK_X_GELU)
        close(y, O.gemm_bf16(O.to_bf16(O.gelu(xf)), w) + b)


@pytest.mark.parametrize("M,N,K", [(16, 4800, 1600), (16, 6400, 1600), (16, 50257, 1600), (7, 640, 320)])
def test_skinny_x_layernorm(device, M, N, K):
    """SM100_SK_X_LN: the f32 operand enters the product as bf16(LayerNorm(x) * g + b), computed
    inside the GEMM (the ln_1 / ln_2 / ln_f before c_attn, c_fc and lm_head).  A LayerNorm output
    one f32 rounding from a bf16 tie may round the other way: 1e-3 of the scale."""
    import ctypes as C
    from thvm_b200 import _lib as L
    rng = np.random.default_rng(M + N)
    xf = (rng.standard_normal((M, K)) * 3 + 0.5).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    bb = (0.1 * rng.standard_normal(K)).astype(np.float32)
    _, w, b = operands(M, N, K, 9)
    ids = {"x": device.upload(xf), "w": device.upload(w), "bias": device.upload(b), "y": device.alloc(M * N * 4),
           "ws": device.alloc(device.lib.sm100_skinny_ws_bytes(M)), "counters": device.alloc(((N + 127) // 128) * 4),
           "g": device.upload(g), "bb": device.upload(bb)}
    a = L.Sm100SkinnyArgs()
    for k in ("x", "w", "bias", "y", "ws", "counters"):
        setattr(a, k, device.dptr(ids[k]))
    a.ln_g, a.ln_b, a.eps = device.dptr(ids["g"]), device.dptr(ids["bb"]), 1e-5
    a.M, a.N, a.K, a.flags = M, N, K, L.SK_X_LN
    L.check(device.lib.sm100_skinny_bf16(C.byref(a), device.stream), "skinny")
    device.sync()
    assert device.lib.sm100_skinny_status() == 0
    y = device.read(ids["y"], np.float32, (M, N))
    for v in ids.values():
        device.free(v)
    ln = O.layernorm(xf, g, bb, 1e-5)
    close(y, O.gemm_bf16(O.to_bf16(ln), w) + b, tol=1e-3)


def test_skinny_rejects(device):
    from thvm_b200 import _lib as L
    a = L.Sm100SkinnyArgs()
    a.M, a.N, a.K = 33, 128, 64
    assert device.lib.sm100_skinny_bf16(ctypes.byref(a), device.stream) == L.ERR_ARG
