"""Each sm_100a kernel through the C ABI (sm100_dispatch_kernel over buffer
ids) against the reference's outputs (tests/golden/ops.npz) and the CPU oracle
on seeded inputs.  float32 tolerance: |dev - ref| <= 1e-4 * |ref| + 1e-5
(elementwise steps are the reference's own IEEE
operations, only reduction order differs).  Index results are exact."""
import numpy as np
import pytest

import oracle as O
from thvm_b200 import _lib as L
from thvm_b200.gpt2 import make_op

pytestmark = pytest.mark.gpu

RTOL, ATOL = 1e-4, 1e-5


def close(dev, ref):
    dev, ref = np.asarray(dev, np.float64), np.asarray(ref, np.float64)
    assert dev.shape == ref.shape
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(dev), fin)
    err = np.abs(dev[fin] - ref[fin]) - (RTOL * np.abs(ref[fin]) + ATOL)
    assert err.max(initial=-1) <= 0, f"max excess {err.max()}"


def run(device, op):
    device.dispatch(op.kernel, op.in_ids, op.out_id)
    device.sync()


@pytest.mark.parametrize("name", ["lin_a", "lin_b", "lin_c"])
@pytest.mark.parametrize("flags", [0, L.LIN_GELU])
def test_linear_bias(device, golden_ops, name, flags):
    g = golden_ops
    x, w, b = g[name + "_x"], g[name + "_w"], g[name + "_b"]
    M, K, N = x.size // x.shape[-1], x.shape[-1], w.shape[0]
    y = device.alloc(M * N * 4)
    run(device, make_op(L.K_LINEAR, y, {0: device.upload(x), 1: device.upload(w), 2: device.upload(b)},
                        flags=flags, m=M, n=N, k=K))
    ref = g[name + "_y"].reshape(M, N)
    if flags & L.LIN_GELU:
        ref = O.gelu(ref)
    close(device.read(y, np.float32, (M, N)), ref)


@pytest.mark.parametrize("M,K,N", [(1, 768, 2304), (1, 3072, 768), (1, 768, 50257), (16, 768, 3072),
                                   (5, 1600, 6400), (3, 36, 10)])
def test_linear_ln_residual(device, M, K, N):
    rng = np.random.default_rng(M * 7 + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    b = (rng.standard_normal(N) * 0.02).astype(np.float32)
    g_ = rng.standard_normal(K).astype(np.float32)
    be = rng.standard_normal(K).astype(np.float32)
    r = rng.standard_normal((M, N)).astype(np.float32)
    y = device.upload(r)
    run(device, make_op(L.K_LINEAR, y, {0: device.upload(x), 1: device.upload(w), 2: device.upload(b),
                                        3: device.upload(g_), 4: device.upload(be), 5: y},
                        flags=L.LIN_LN | L.LIN_RESIDUAL, m=M, n=N, k=K, eps=1e-5))
    ref = r + O.linear(O.layernorm(x, g_, be), w, b)
    close(device.read(y, np.float32, (M, N)), ref)


def test_linear_kv_append(device):
    rng = np.random.default_rng(3)
    d, ctx, T, pos = 96, 32, 3, 7
    x = rng.standard_normal((T, d)).astype(np.float32)
    w = (rng.standard_normal((3 * d, d)) * 0.05).astype(np.float32)
    cache = device.alloc(2 * ctx * d * 4)
    posb = device.upload(np.array([pos], np.int32))
    y = device.alloc(T * 3 * d * 4)
    run(device, make_op(L.K_LINEAR, y, {0: device.upload(x), 1: device.upload(w), 7: posb, 8: cache},
                        flags=L.LIN_KV_APPEND, m=T, n=3 * d, k=d, max_ctx=ctx))
    qkv = device.read(y, np.float32, (T, 3 * d))
    close(qkv, O.linear(x, w))
    c = device.read(cache, np.float32, (2, ctx, d))
    assert np.array_equal(c[0, pos:pos + T], qkv[:, d:2 * d])
    assert np.array_equal(c[1, pos:pos + T], qkv[:, 2 * d:])
    assert not c[:, :pos].any() and not c[:, pos + T:].any()


@pytest.mark.parametrize("name", ["ln_a", "ln_b", "ln_c"])
def test_layernorm(device, golden_ops, name):
    g = golden_ops
    x = g[name + "_x"]
    D = x.shape[-1]
    y = device.alloc(x.nbytes)
    run(device, make_op(L.K_LAYERNORM, y, {0: device.upload(x), 1: device.upload(g[name + "_w"]),
                                           2: device.upload(g[name + "_b"])}, m=x.size // D, k=D, eps=1e-5))
    close(device.read(y, np.float32, x.shape), g[name + "_y"])


def test_rmsnorm(device):
    x = np.random.default_rng(5).standard_normal((7, 2048)).astype(np.float32)
    w = np.random.default_rng(6).standard_normal(2048).astype(np.float32)
    y = device.alloc(x.nbytes)
    run(device, make_op(L.K_RMSNORM, y, {0: device.upload(x), 1: device.upload(w)}, m=7, k=2048, eps=1e-6))
    close(device.read(y, np.float32, x.shape), O.rmsnorm(x, w, 1e-6))


def test_softmax_masked(device, golden_ops):
    x = golden_ops["sm_x"]
    y = device.alloc(x.nbytes)
    run(device, make_op(L.K_SOFTMAX, y, {0: device.upload(x)}, m=x.shape[0], k=x.shape[1]))
    close(device.read(y, np.float32, x.shape), golden_ops["sm_y"])


def test_gelu_matches_reference_bits(device, golden_ops):
    """GELU is elementwise in the reference's op order with its xexp2, so the
    device result is bit-identical."""
    x = golden_ops["gelu_x"]
    y = device.alloc(x.nbytes)
    run(device, make_op(L.K_GELU, y, {0: device.upload(x)}, m=1, k=x.size))
    assert np.array_equal(device.read(y, np.float32, x.shape), golden_ops["gelu_y"])


def _attention(device, q, k, v, pos, T, causal_rows=True):
    """q [T, H, hd]; k, v [L, H, hd] written into a cache at rows 0..L-1."""
    H, hd = q.shape[1], q.shape[2]
    Lk = k.shape[0]
    ctx = max(64, Lk)
    cache = np.zeros((2, ctx, H * hd), np.float32)
    cache[0, :Lk] = k.reshape(Lk, -1)
    cache[1, :Lk] = v.reshape(Lk, -1)
    out = device.alloc(T * H * hd * 4)
    run(device, make_op(L.K_ATTENTION, out, {0: device.upload(q.reshape(T, -1)), 1: device.upload(cache),
                                             7: device.upload(np.array([pos], np.int32))},
                        m=T, heads=H, head_dim=hd, max_ctx=ctx, scale=float(1 / np.sqrt(hd))))
    return device.read(out, np.float32, (T, H, hd))


@pytest.mark.parametrize("name", ["sdpa_dec", "sdpa_dec1"])
def test_attention_decode(device, golden_ops, name):
    g = golden_ops
    q, k, v = g[name + "_q"][0], g[name + "_k"][0], g[name + "_v"][0]   # [H, L, hd]
    Lk = k.shape[1]
    y = _attention(device, q.transpose(1, 0, 2), k.transpose(1, 0, 2), v.transpose(1, 0, 2), Lk - 1, 1)
    close(y.transpose(1, 0, 2)[None], g[name + "_y"])


def test_attention_prompt_causal(device, golden_ops):
    g = golden_ops
    q, k, v = g["sdpa_mask_q"][0], g["sdpa_mask_k"][0], g["sdpa_mask_v"][0]   # [H, 16, 64]
    y = _attention(device, q.transpose(1, 0, 2), k.transpose(1, 0, 2), v.transpose(1, 0, 2), 0, 16)
    close(y.transpose(1, 0, 2)[None], g["sdpa_mask_y"])


def test_attention_long_context(device):
    rng = np.random.default_rng(11)
    H, hd, Lk = 12, 64, 1000
    q = rng.standard_normal((1, H, hd)).astype(np.float32)
    k = rng.standard_normal((Lk, H, hd)).astype(np.float32)
    v = rng.standard_normal((Lk, H, hd)).astype(np.float32)
    y = _attention(device, q, k, v, Lk - 1, 1)
    ref = O.sdpa(q.transpose(1, 0, 2), k.transpose(1, 0, 2), v.transpose(1, 0, 2))   # [H, 1, hd]
    close(y.transpose(1, 0, 2), ref)


def test_embedding_exact(device, golden_ops):
    g = golden_ops
    w, idx = g["emb_w"], g["emb_idx"].reshape(-1)
    y = device.alloc(idx.size * w.shape[1] * 4)
    run(device, make_op(L.K_EMBEDDING, y, {0: device.upload(w), 1: device.upload(idx)},
                        m=idx.size, n=w.shape[0], k=w.shape[1]))
    assert np.array_equal(device.read(y, np.float32, g["emb_y"].shape), g["emb_y"])


def test_embedding_plus_position(device):
    rng = np.random.default_rng(2)
    wte = rng.standard_normal((50, 24)).astype(np.float32)
    wpe = rng.standard_normal((40, 24)).astype(np.float32)
    idx = np.array([3, 49, 0], np.int32)
    y = device.alloc(3 * 24 * 4)
    run(device, make_op(L.K_EMBEDDING, y, {0: device.upload(wte), 1: device.upload(idx), 2: device.upload(wpe),
                                           7: device.upload(np.array([5], np.int32))}, m=3, n=50, k=24))
    assert np.array_equal(device.read(y, np.float32, (3, 24)), wte[idx] + wpe[5:8])


def test_argmax_exact_with_ties(device, golden_ops):
    x = golden_ops["am_x"]
    out = device.alloc(4 * x.shape[0])
    run(device, make_op(L.K_ARGMAX, out, {0: device.upload(x)}, m=x.shape[0], n=x.shape[1]))
    assert np.array_equal(device.read(out, np.int32, (x.shape[0],)), golden_ops["am_y"])


def test_argmax_vocab_and_bump(device):
    rng = np.random.default_rng(9)
    x = rng.standard_normal((3, 50257)).astype(np.float32)
    x[2, 50256] = x[2, 17] = 9.0
    out = device.alloc(12)
    pos = device.upload(np.array([41], np.int32))
    for _ in range(2):   # the completion counter resets between launches
        run(device, make_op(L.K_ARGMAX, out, {0: device.upload(x), 7: pos}, m=3, n=50257))
        assert np.array_equal(device.read(out, np.int32, (3,)), O.argmax(x))
    assert device.read(pos, np.int32, (1,))[0] == 43


def test_scatter_rows_exact(device):
    dst = device.upload(np.zeros((10, 3), np.float32))
    src = np.arange(12, dtype=np.float32).reshape(4, 3)
    idx = np.array([7, -1, 2, 10], np.int32)   # out-of-range ids are skipped
    run(device, make_op(L.K_SCATTER, dst, {0: device.upload(src), 1: device.upload(idx)}, m=4, n=10, k=3))
    ref = np.zeros((10, 3), np.float32)
    ref[7], ref[2] = src[0], src[2]
    assert np.array_equal(device.read(dst, np.float32, (10, 3)), ref)


def test_kv_append_and_pos_add(device):
    d, ctx = 8, 6
    cache = device.alloc(2 * ctx * d * 4)
    k = np.arange(16, dtype=np.float32).reshape(2, 8)
    v = -k
    pos = device.upload(np.array([3], np.int32))
    run(device, make_op(L.K_KV_APPEND, cache, {0: device.upload(k), 1: device.upload(v), 7: pos},
                        m=2, k=d, max_ctx=ctx))
    c = device.read(cache, np.float32, (2, ctx, d))
    assert np.array_equal(c[0, 3:5], k) and np.array_equal(c[1, 3:5], v)
    run(device, make_op(L.K_POS_ADD, pos, {}, pos=5))
    assert device.read(pos, np.int32, (1,))[0] == 8


def test_gather_strided_exact(device):
    src = np.arange(4 * 5 * 6, dtype=np.float32).reshape(4, 5, 6)
    s = device.upload(src)
    view = src.transpose(2, 0, 1)[1:, :, ::2]
    dst = device.alloc(view.nbytes)
    device.gather_strided(dst, s, dims=view.shape, strides=(1, 30, 12), offset=1)
    assert np.array_equal(device.read(dst, np.float32, view.shape), view)


def test_dispatch_rejects_dead_buffer(device):
    k = make_op(L.K_GELU, 0, {0: 123456}, m=1, k=4)
    with pytest.raises(L.Sm100Error):
        device.dispatch(k.kernel, k.in_ids, k.out_id)
