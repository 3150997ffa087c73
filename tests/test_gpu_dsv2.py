"""The batched MoE decode step of the DeepSeek-V2-Lite-shaped model (BASELINE
config 5) on one GPU (thvm_b200.dsv2.DSModel, expert-parallel degree 1)
against the CPU oracle (oracle.DSModel, orc_ds_step) on a reduced model
(2 layers: one dense, one MoE with 8 fp8 experts, top-3, 2 shared halves;
d 512, 4 heads, kv_lora 128, nope 32, rope 16, v 32; vocab 1000; batch 32):
6 prompt positions and 8 decode steps, both sides fed the oracle's ids.
The north star's fp8 / bf16 gates: logits within 2e-2 of the row scale and
top-1 agreement >= 99 %; the compressed KV cache rows of layer 0 within two
bf16 ulps, deeper layers within four (their inputs carry the bf16
pipeline's rounding differences)."""
import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, dim=512, heads=4, kv_lora=128, d_nope=32, d_rope=16, d_v=32, n_exp=8, top_k=3, moe_inter=128,
           dense_inter=256, n_dense=1, n_shared=2, vocab=1000, max_ctx=64, batch=32)


def f32(b):
    return (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def test_ds_decode_matches_oracle():
    import torch
    from thvm_b200.dsv2 import DSConfig, DSModel, ep_shard, ds_weights, yarn_tables
    cfg = DSConfig(**CFG)
    w = ds_weights(cfg, seed=0)
    dev = DSModel(cfg, w, ep_shard(cfg, 0, 1))
    cos, sin = yarn_tables(cfg.d_rope, cfg.max_ctx)
    ref = O.DSModel(cfg, w, cos, sin)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, (cfg.batch, 6)).astype(np.int32)
    tok = prompt[:, 0]
    agree, total, worst = 0, 0, 0.0
    for pos in range(14):
        dev.tok.copy_(torch.from_numpy(tok))
        dev.step()
        torch.cuda.synchronize()
        lg, nxt = ref.step(tok, pos)
        dl = dev.logits.cpu().numpy()
        worst = max(worst, float((np.abs(dl - lg).max(1) / np.abs(lg).max(1)).max()))
        agree += int((dev.tok.cpu().numpy() == nxt).sum())
        total += cfg.batch
        assert int(dev.pos.item()) == pos + 1
        tok = prompt[:, pos + 1] if pos + 1 < prompt.shape[1] else nxt
    assert worst <= 2e-2, worst
    assert agree / total >= 0.99, agree / total
    assert dev.lib.sm100_ds_status() == 0
    for l in range(cfg.n_layers):
        # layer 0's rows see identical inputs: a bf16 operand one rounding apart moves a value by
        # an ulp of its input, which the rotary can leave in a near-cancelled output (hence the
        # floor in units of the rms); deeper layers inherit the bf16 pipeline's differences
        rel, floor = (2.0 ** -6, 2.0 ** -6) if l == 0 else (2.0 ** -5, 2.0 ** -5)
        for mine, theirs in ((dev.cache_c[l], ref.cache_c[l]), (dev.cache_pe[l], ref.cache_pe[l])):
            a = f32(mine.cpu().numpy().view(np.uint16)[:, :14])
            r = f32(theirs[:, :14])
            excess = np.abs(a - r) - (rel * np.abs(r) + floor * np.sqrt(np.mean(r * r)))
            assert excess.max() <= 0, (l, excess.max())


def test_ds_route_matches_oracle_rule():
    """The routing kernel alone: softmax, top-K with ties to the lowest id, expert-major slots,
    then the shared experts' slots."""
    import ctypes
    import torch
    from thvm_b200 import _lib as L
    lib = L.lib()
    B, E, K = 32, 64, 6
    rng = np.random.default_rng(2)
    logits = rng.standard_normal((B, E)).astype(np.float32)
    logits[0, 5] = logits[0, 9] = logits[0].max() + 1.0   # a tie: 5 before 9
    d = lambda a: torch.from_numpy(a).cuda()
    lg = d(logits)
    sel, wsel = torch.zeros(B * K, dtype=torch.int32, device="cuda"), torch.zeros(B * K, device="cuda")
    NS = 2
    off = torch.zeros(E + NS + 1, dtype=torch.int32, device="cuda")
    stok, sw = torch.zeros(B * (K + NS), dtype=torch.int32, device="cuda"), torch.zeros(B * (K + NS), device="cuda")
    L.check(lib.sm100_ds_route(lg.data_ptr(), E, K, B, 0, E, NS, sel.data_ptr(), wsel.data_ptr(), off.data_ptr(),
                               stok.data_ptr(), sw.data_ptr(), ctypes.c_void_p(0)), "ds_route")
    torch.cuda.synchronize()
    p = np.exp(logits - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    ref = np.argsort(-p, axis=1, kind="stable")[:, :K]   # stable: ties keep the lower id first
    np.testing.assert_array_equal(sel.cpu().numpy().reshape(B, K), ref)
    np.testing.assert_allclose(wsel.cpu().numpy().reshape(B, K), np.take_along_axis(p, ref, 1), rtol=1e-5)
    o = off.cpu().numpy()
    assert o[0] == 0 and o[E] == B * K and o[-1] == B * (K + NS) and np.all(np.diff(o) >= 0)
    for e in range(E):
        toks = stok.cpu().numpy()[o[e]:o[e + 1]]
        np.testing.assert_array_equal(toks, np.nonzero((ref == e).any(1))[0])
    for k in range(NS):   # the shared experts: every token, weight 1
        np.testing.assert_array_equal(stok.cpu().numpy()[o[E + k]:o[E + k + 1]], np.arange(B))
        assert np.all(sw.cpu().numpy()[o[E + k]:o[E + k + 1]] == 1.0)
