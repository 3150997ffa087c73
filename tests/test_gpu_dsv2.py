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
    from thvm_b200.dsv2 import DSConfig, DSModel, ds_shard, ds_weights, shard_ds_weights, yarn_tables
    cfg = DSConfig(**CFG)
    w = ds_weights(cfg, seed=0)
    sh = ds_shard(cfg, 0, 1)
    dev = DSModel(cfg, shard_ds_weights(w, cfg, sh), sh)
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
    assert dev.status() == 0
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
    """The routing kernel alone against the oracle's orc_ds_route (the reference's rule: top-K of
    the logits with ties to the lowest id, softmax weights): an exact tie, two distinct logits
    with equal f32 probabilities (the larger logit wins), expert-major slots, then the shared
    experts' slots."""
    import ctypes
    import torch
    from thvm_b200 import _lib as L
    lib = L.lib()
    B, E, K = 32, 64, 6
    rng = np.random.default_rng(2)
    logits = rng.standard_normal((B, E)).astype(np.float32)
    logits[0, 5] = logits[0, 9] = logits[0].max() + 1.0   # a tie: 5 before 9
    logits[1] = -20.0                                        # equal probabilities, distinct logits
    logits[1, 0], logits[1, 1:5] = 6.0, 5.0
    logits[1, 7], logits[1, 40] = -2.0, np.nextafter(np.float32(-2.0), np.float32(0.0))
    d = lambda a: torch.from_numpy(a).cuda()
    lg = d(logits)
    sel, wsel = torch.zeros(B * K, dtype=torch.int32, device="cuda"), torch.zeros(B * K, device="cuda")
    NS = 2
    off = torch.zeros(E + NS + 1, dtype=torch.int32, device="cuda")
    stok, sw = torch.zeros(B * (K + NS), dtype=torch.int32, device="cuda"), torch.zeros(B * (K + NS), device="cuda")
    L.check(lib.sm100_ds_route(lg.data_ptr(), E, K, B, 0, E, NS, sel.data_ptr(), wsel.data_ptr(), off.data_ptr(),
                               stok.data_ptr(), sw.data_ptr(), ctypes.c_void_p(0)), "ds_route")
    torch.cuda.synchronize()
    ref, ref_w = O.ds_route(logits, K)
    assert ref[0, 0] == 5 and ref[1, 5] == 40   # a top-K of probabilities would take 7
    np.testing.assert_array_equal(sel.cpu().numpy().reshape(B, K), ref)
    np.testing.assert_allclose(wsel.cpu().numpy().reshape(B, K), ref_w, rtol=1e-5)
    o = off.cpu().numpy()
    assert o[0] == 0 and o[E] == B * K and o[-1] == B * (K + NS) and np.all(np.diff(o) >= 0)
    for e in range(E):
        toks = stok.cpu().numpy()[o[e]:o[e + 1]]
        np.testing.assert_array_equal(toks, np.nonzero((ref == e).any(1))[0])
    for k in range(NS):   # the shared experts: every token, weight 1
        np.testing.assert_array_equal(stok.cpu().numpy()[o[E + k]:o[E + k + 1]], np.arange(B))
        assert np.all(sw.cpu().numpy()[o[E + k]:o[E + k + 1]] == 1.0)


def test_ds_router_route_matches_oracle_rule():
    """The router product and the routing in one launch (sm100_ds_router_route):
    its logits within 1e-5 of the f64 product of the bf16 operands, its
    choices the oracle's rule on those logits, the slot lists as
    sm100_ds_route builds them from the same logits, twice in a row (the
    launch leaves its CTA counter at zero)."""
    import ctypes
    import torch
    from thvm_b200 import _lib as L
    lib = L.lib()
    B, E, K, D, NS = 32, 64, 6, 2048, 2
    g = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.randn(B, D, generator=g, device="cuda")).to(torch.bfloat16)
    w = (torch.randn(E, D, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    z = lambda n, dt=torch.float32: torch.zeros(n, dtype=dt, device="cuda")
    logits, counter = z(B * E), z(1, torch.int32)
    outs = [(z(B * K, torch.int32), z(B * K), z(E + NS + 1, torch.int32), z(B * (K + NS), torch.int32),
             z(B * (K + NS))) for _ in range(2)]
    for sel, wsel, off, stok, sw in outs:
        L.check(lib.sm100_ds_router_route(x.data_ptr(), w.data_ptr(), logits.data_ptr(), counter.data_ptr(), D, E, K,
                                          B, 0, E, NS, sel.data_ptr(), wsel.data_ptr(), off.data_ptr(),
                                          stok.data_ptr(), sw.data_ptr(), ctypes.c_void_p(0)), "ds_router_route")
    torch.cuda.synchronize()
    assert int(counter.item()) == 0
    lg = logits.cpu().numpy().reshape(B, E)
    want = x.double().cpu().numpy() @ w.double().cpu().numpy().T
    np.testing.assert_allclose(lg, want, rtol=0, atol=1e-5 * np.abs(want).max())
    ref, ref_w = O.ds_route(lg, K)
    ref_outs = (z(B * K, torch.int32), z(B * K), z(E + NS + 1, torch.int32), z(B * (K + NS), torch.int32),
                z(B * (K + NS)))
    L.check(lib.sm100_ds_route(logits.data_ptr(), E, K, B, 0, E, NS, *[t.data_ptr() for t in ref_outs],
                               ctypes.c_void_p(0)), "ds_route")
    torch.cuda.synchronize()
    for sel, wsel, off, stok, sw in outs:
        np.testing.assert_array_equal(sel.cpu().numpy().reshape(B, K), ref)
        np.testing.assert_allclose(wsel.cpu().numpy().reshape(B, K), ref_w, rtol=1e-5)
        for a, b in zip((sel, wsel, off, stok, sw), ref_outs):
            assert torch.equal(a, b)


def _experts_case(B, D, I, slots, seed):
    """sm100_ds_experts on explicit slot lists against the oracle's fp8 block-scaled linear."""
    import ctypes
    import torch
    from thvm_b200 import _lib as L
    from thvm_b200.dsv2 import _bf16, _fp8
    lib = L.lib()
    rng = np.random.default_rng(seed)
    E = len(slots)
    x = _bf16(rng.standard_normal((B, D), dtype=np.float32))
    w_gu = _fp8(rng.standard_normal((E, 2 * I, D), dtype=np.float32))
    s_gu = (rng.uniform(0.5, 2.0, (E, 2 * I // 128, D // 128)) * 0.02).astype(np.float32)
    w_d = _fp8(rng.standard_normal((E, D, I), dtype=np.float32))
    s_d = (rng.uniform(0.5, 2.0, (E, D // 128, I // 128)) * 0.02).astype(np.float32)
    off = np.concatenate([[0], np.cumsum([len(s) for s in slots])]).astype(np.int32)
    tok = np.concatenate([np.asarray(s, np.int32) for s in slots])
    wts = rng.uniform(0.1, 1.0, int(off[-1])).astype(np.float32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    t = {k: dev(v) for k, v in dict(x=x.view(np.int16), w_gu=w_gu, s_gu=s_gu, w_d=w_d, s_d=s_d, off=off, tok=tok,
                                      w=wts).items()}
    a = torch.zeros(int(off[-1]), I, dtype=torch.int16, device="cuda")
    y = torch.zeros(B, D, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    lib.sm100_ds_status()   # reading clears the sticky word: start from this call's own status
    L.check(lib.sm100_ds_experts(t["x"].data_ptr(), t["w_gu"].data_ptr(), t["s_gu"].data_ptr(), t["w_d"].data_ptr(),
                                 t["s_d"].data_ptr(), t["off"].data_ptr(), t["tok"].data_ptr(), t["w"].data_ptr(),
                                 a.data_ptr(), y.data_ptr(), E, D, I, ctypes.c_void_p(0)), "ds_experts")
    status = int(lib.sm100_ds_status())
    xf = O.bf16_to_f32(x)
    ref = np.zeros((B, D), np.float64)
    for e in range(E):
        for j in range(off[e], min(off[e + 1], off[e] + 32)):
            gu = O.linear_fp8bs(xf[tok[j]][None], w_gu[e], s_gu[e])[0].astype(np.float64)
            g, u = gu[:I], gu[I:]
            h = O.bf16_to_f32(_bf16((g / (1.0 + np.exp(-g)) * u).astype(np.float32)))
            ref[tok[j]] += wts[j] * O.linear_fp8bs(h[None], w_d[e], s_d[e])[0]
    return y.cpu().numpy(), ref, status


def test_ds_experts_match_oracle():
    """Routed slot lists of 10, 0, 15 and 32 tokens (an empty expert, a full
    N = 32 tile), D = 384 and I = 256 (3 and 2 k-blocks): the fp8 x fp8
    products (token rows split into e4m3 hi + lo) within 5e-3 of the largest
    output of the float64 oracle sum."""
    rng = np.random.default_rng(3)
    B = 32
    slots = [list(range(10)), [], sorted(rng.choice(B, 15, replace=False)), list(range(B))]
    y, ref, status = _experts_case(B, 384, 256, slots, 4)
    assert status == 0, status
    np.testing.assert_allclose(y, ref, rtol=0, atol=5e-3 * np.abs(ref).max())


def test_ds_experts_flags_more_than_32_slots():
    """An expert with 40 slots: the first 32 tokens are served and the status
    word carries SM100_DECODE_ERR_ARG (the MMA's N is 32)."""
    from thvm_b200 import _lib as L
    y, ref, status = _experts_case(40, 256, 128, [list(range(40))], 6)
    assert status & L.DECODE_ERR_ARG, status
    np.testing.assert_allclose(y[:32], ref[:32], rtol=0, atol=5e-3 * np.abs(ref).max())
    assert not np.any(y[32:])


@pytest.mark.parametrize("H", [16, 4, 2])
def test_ds_mla_post_is_post_then_mla(H):
    """sm100_ds_mla_post (the q / latent post-processing done inside the MLA
    group kernel, the current row walked from shared memory) against the two
    launches it replaces (sm100_ds_qkv_post, sm100_ds_mla) on the same inputs
    at the DeepSeek-V2-Lite MLA shapes: the attention output and both cache
    rows bit for bit, at positions 0, 1 and 37 (16, 4 and 2 heads: 4, 1 and 1
    sequences per CTA)."""
    import ctypes
    import torch
    from thvm_b200 import _lib as L
    from thvm_b200.dsv2 import yarn_tables
    lib = L.lib()
    B, DN, DR, DV, KV, ctx = 32, 128, 64, 128, 512, 64
    nq = H * (DN + DR)
    ld = nq + KV + DR
    g = torch.Generator(device="cuda").manual_seed(11)
    cos, sin = (torch.from_numpy(t).cuda() for t in yarn_tables(DR, ctx))
    gkv = torch.rand(KV, generator=g, device="cuda") + 0.5
    wuk = (torch.randn(H, DN, KV, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    wuv = (torch.randn(H, DV, KV, generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    cache0 = (torch.randn(B, ctx, KV, generator=g, device="cuda")).to(torch.bfloat16)
    pe0 = (torch.randn(B, ctx, DR, generator=g, device="cuda")).to(torch.bfloat16)
    scale = 0.1
    st = ctypes.c_void_p(0)
    for p in (0, 1, 37):
        qkva = torch.randn(B, ld, generator=g, device="cuda")
        pos = torch.tensor([p], dtype=torch.int32, device="cuda")
        outs = []
        for fused in (False, True):
            cc, cp = cache0.clone(), pe0.clone()
            qo = torch.zeros(B, nq, dtype=torch.bfloat16, device="cuda")
            o = torch.zeros(B, H * DV, dtype=torch.bfloat16, device="cuda")
            if fused:
                rc = lib.sm100_ds_mla_post(qkva.data_ptr(), ld, nq, gkv.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                           pos.data_ptr(), qo.data_ptr(), wuk.data_ptr(), wuv.data_ptr(),
                                           cc.data_ptr(), cp.data_ptr(), o.data_ptr(), B, H, DN, DR, DV, KV, ctx,
                                           1e-6, scale, st)
                L.check(rc, "ds_mla_post")
            else:
                q = qkva.data_ptr()
                L.check(lib.sm100_ds_qkv_post(q, q + 4 * nq, ld, gkv.data_ptr(), cos.data_ptr(), sin.data_ptr(),
                                              pos.data_ptr(), qo.data_ptr(), cc.data_ptr(), cp.data_ptr(), B, H, DN,
                                              DR, KV, ctx, 1e-6, st), "ds_qkv_post")
                L.check(lib.sm100_ds_mla(qo.data_ptr(), wuk.data_ptr(), wuv.data_ptr(), cc.data_ptr(), cp.data_ptr(),
                                         pos.data_ptr(), o.data_ptr(), B, H, DN, DR, DV, KV, ctx, scale, st), "ds_mla")
            torch.cuda.synchronize()
            outs.append((o, cc, cp))
        assert lib.sm100_ds_status() == 0
        for a, b in zip(*outs):
            assert torch.equal(a.view(torch.int16), b.view(torch.int16)), p
