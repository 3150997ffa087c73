"""The CPU oracle against the reference's own outputs (tests/golden/, made by
running the reference: tests/golden/make_golden.py).  Bit-exact: the oracle
restates the reference's float32 op order, its xexp2 and its serial sums."""
import numpy as np
import pytest

import oracle as O
from conftest import GOLDEN


@pytest.mark.parametrize("name", ["lin_a", "lin_b", "lin_c"])
def test_linear(golden_ops, name):
    g = golden_ops
    y = O.linear(g[name + "_x"], g[name + "_w"], g[name + "_b"])
    assert np.array_equal(y, g[name + "_y"])


@pytest.mark.parametrize("name", ["ln_a", "ln_b", "ln_c"])
def test_layernorm(golden_ops, name):
    g = golden_ops
    assert np.array_equal(O.layernorm(g[name + "_x"], g[name + "_w"], g[name + "_b"]), g[name + "_y"])


def test_softmax_with_masked_entries(golden_ops):
    g = golden_ops
    assert np.array_equal(O.softmax(g["sm_x"]), g["sm_y"])


def test_gelu(golden_ops):
    g = golden_ops
    assert np.array_equal(O.gelu(g["gelu_x"]), g["gelu_y"])


@pytest.mark.parametrize("name", ["sdpa_dec", "sdpa_dec1"])
def test_sdpa_decode(golden_ops, name):
    g = golden_ops
    assert np.array_equal(O.sdpa(g[name + "_q"], g[name + "_k"], g[name + "_v"]), g[name + "_y"])


def test_sdpa_causal(golden_ops):
    g = golden_ops
    y = O.sdpa(g["sdpa_causal_q"], g["sdpa_causal_k"], g["sdpa_causal_v"], causal=True)
    assert np.array_equal(y, g["sdpa_causal_y"])


def test_sdpa_additive_mask(golden_ops):
    g = golden_ops
    y = O.sdpa(g["sdpa_mask_q"], g["sdpa_mask_k"], g["sdpa_mask_v"], mask=g["sdpa_mask_m"])
    assert np.array_equal(y, g["sdpa_mask_y"])


def test_argmax_ties_first_index(golden_ops):
    g = golden_ops
    assert np.array_equal(O.argmax(g["am_x"]), g["am_y"])


def test_embedding_out_of_range_is_zero(golden_ops):
    g = golden_ops
    assert np.array_equal(O.embedding(g["emb_w"], g["emb_idx"]), g["emb_y"])


def test_gpt2_prompt_logits_and_64_tokens(golden_gpt2, gpt2_small_weights):
    from thvm_b200.synthetic import GPT2_SMALL
    g = golden_gpt2
    m = O.GPT2(GPT2_SMALL, gpt2_small_weights)
    tok, lg = m.forward(g["prompt"], 0, want_logits=True)
    assert tok == g["tokens"][0]
    assert np.array_equal(lg, g["logits_step0"])
    tok1, lg1 = m.forward([tok], len(g["prompt"]), want_logits=True)
    assert np.array_equal(lg1, g["logits_step1"])
    assert tok1 == g["tokens"][1]
    out = m.generate(g["prompt"], 64)
    assert np.array_equal(out, g["tokens"])


def test_planted_mistake_is_caught(golden_ops):
    """A wrong oracle must fail the comparison (the check is not vacuous)."""
    g = golden_ops
    y = O.linear(g["lin_b_x"], g["lin_b_w"], g["lin_b_b"])
    y[0, 0, 3] += 1e-6
    assert not np.array_equal(y, g["lin_b_y"])
    assert not np.array_equal(O.argmax(g["am_x"][:, ::-1].copy()), g["am_y"])


# ---- bf16 / fp8 e4m3 storage formats (tests/golden/dtypes.npz: the
# reference library's own conversions, bit for bit) ---------------------------

@pytest.fixture(scope="module")
def golden_dtypes():
    from conftest import GOLDEN
    return dict(np.load(GOLDEN / "dtypes.npz"))


def test_bf16_conversion_matches_reference(golden_dtypes):
    g = golden_dtypes
    x = g["x_bits"].view(np.float32)
    assert np.array_equal(O.to_bf16(x), g["bf16"])


def test_fp8e4m3_encode_matches_reference(golden_dtypes):
    g = golden_dtypes
    x = g["x_bits"].view(np.float32)
    assert np.array_equal(O.to_fp8e4m3(x), g["fp8e4m3"])


def test_fp8e4m3_decode_matches_reference(golden_dtypes):
    ref = golden_dtypes["fp8e4m3_decoded"]
    mine = O.fp8e4m3_to_f32(np.arange(256))
    assert np.array_equal(np.isnan(mine), np.isnan(ref))
    ok = ~np.isnan(ref)
    assert np.array_equal(mine[ok].view(np.uint32), ref[ok].view(np.uint32))


def test_lowp_linears_are_the_f32_loop_on_widened_weights():
    """The bf16 and block-scaled fp8 oracles are the reference's f32 Linear
    loop over the widened weights (for fp8: decoded * its block scale), bit
    for bit."""
    rng = np.random.default_rng(5)
    M, K, N = 2, 300, 260
    x = O.bf16_to_f32(O.to_bf16(rng.standard_normal((M, K)).astype(np.float32)))
    wb = O.to_bf16(rng.standard_normal((N, K)).astype(np.float32))
    assert np.array_equal(O.linear_bf16(x, wb), O.linear(x, O.bf16_to_f32(wb)))
    w8 = O.to_fp8e4m3(rng.standard_normal((N, K)).astype(np.float32))
    sc = rng.uniform(0.5, 2.0, ((N + 127) // 128, (K + 127) // 128)).astype(np.float32)
    wide = O.fp8e4m3_to_f32(w8) * np.repeat(np.repeat(sc, 128, 0), 128, 1)[:N, :K]
    assert np.array_equal(O.linear_fp8bs(x, w8, sc), O.linear(x, wide))
    a = O.to_bf16(rng.standard_normal((7, K)).astype(np.float32))
    assert np.array_equal(O.gemm_bf16(a, wb), O.linear(O.bf16_to_f32(a), O.bf16_to_f32(wb)))


# ---- DeepSeek-V2 decode ---------------------------------

def _bytesum(a):
    """The DSV2_DUMP fingerprint of a buffer: sum of byte[i] * (1 + (i & 7))."""
    b = np.frombuffer(np.ascontiguousarray(a).tobytes(), np.uint8).astype(np.uint64)
    return int((b * (1 + (np.arange(b.size) & 7)).astype(np.uint64)).sum())


@pytest.fixture(scope="module")
def golden_dsv2():
    g = dict(np.load(GOLDEN / "dsv2.npz"))
    cfg = O.DSREF_SMALL
    assert {k[4:]: int(v) for k, v in g.items() if k.startswith("cfg_")} == {k: int(v) for k, v in cfg.env().items()}
    return g, cfg


def test_ds_ref_step_is_the_reference_step_bit_for_bit(golden_dsv2):
    """orc_ds_ref_step against the reference's own decode bench run on the same
    pack (tests/golden/make_dsv2_golden.py): after the first step every
    DSV2_DUMP fingerprint (the last layer's qlat, attention weights, olat and o,
    the dense layer's gate / up outputs, each layer's cache row 0, the logits'
    bit sum) is identical; then the 8-id prompt fed token by token and 23
    greedy steps give the same 24 ids and the same printed top-2 logits."""
    g, cfg = golden_dsv2
    m = O.DSRef(cfg, O.ds_ref_weights(cfg, seed=int(g["seed"])))
    prompt = [int(t) for t in g["prompt"]]
    lg, nxt = m.step(prompt[0], 1)
    tr = m.trace
    mine = {"T_ql": tr["ql"], "T_sm": tr["sm"], "T_ol": tr["ol"], "T_ob": tr["ob"], "T_g1o": tr["g1o"],
            "T_u1o": tr["u1o"]}
    for name, want in zip(g["dump_names"], g["dump_sums"]):
        assert _bytesum(mine[str(name)]) == int(want), name
    assert [int(m.ckv[l, 0].astype(np.uint64).sum()) for l in range(cfg.n_layers)] == g["dump_ckv"].tolist()
    assert [int(m.kpe[l, 0].astype(np.uint64).sum()) for l in range(cfg.n_layers)] == g["dump_kpe"].tolist()
    assert int(lg.view(np.uint32).astype(np.uint64).sum()) == int(g["dump_logits_bitsum"])
    for i in range(1, len(prompt)):
        lg, nxt = m.step(prompt[i], i + 1)
    gen = [nxt]
    for i in range(1, len(g["gen_ids"])):
        lg, nxt = m.step(gen[-1], len(prompt) + i)
        gen.append(nxt)
        top = np.argsort(-lg, kind="stable")[:2]
        assert top.tolist() == g["top2_ids"][i - 1].tolist(), i
        assert [f"{float(lg[t]):.6f}" for t in top] == g["top2_txt"][i - 1].tolist(), i
    assert gen == g["gen_ids"].tolist()


def test_ds_batched_step_agrees_with_the_pinned_step():
    """The batched config-5 oracle (orc_ds_step: f32 residual, fp8 block-scaled
    experts, bf16 router) on the same model as the pinned reference step
    (expert weights chosen fp8-exact): per step logits within the north star's
    2e-2 of the row's largest, and the same greedy id at every step, over 8
    prompt positions and 24 greedy steps at batch 1."""
    cfg = O.DSREF_SMALL
    rw = O.ds_ref_weights(cfg, seed=3, fp8_experts=True)
    c5, w5 = O.ds_from_ref(cfg, rw)
    cos, sin = O.ds_rope_tables(cfg.d_rope, cfg.max_seq)
    mine, ref = O.DSModel(c5, w5, cos, sin), O.DSRef(cfg, rw)
    seq = np.random.default_rng(5).integers(0, cfg.vocab, 8).tolist()
    tok, worst = seq[0], 0.0
    for pos in range(32):
        lr, nr = ref.step(tok, pos + 1)
        lm, nm = mine.step(np.array([tok], np.int32), pos)
        worst = max(worst, float(np.abs(lm[0] - lr).max() / np.abs(lr).max()))
        assert int(nm[0]) == nr, pos
        tok = seq[pos + 1] if pos + 1 < len(seq) else nr
    assert worst <= 2e-2, worst


def test_ds_route_takes_top_k_of_logits():
    """The reference's routing rule: top-K over the router logits with ties to
    the lowest id, weights exp(l - max) / sum.  Two distinct logits whose
    probabilities are equal in f32 (both 8.0 below the max) resolve to the
    larger logit, where a top-K over probabilities would take the lower id."""
    g = np.full((2, 8), -20.0, np.float32)
    g[:, 0] = 6.0
    g[:, 1:5] = 5.0
    g[0, 5], g[0, 6] = -2.0, np.nextafter(np.float32(-2.0), np.float32(0.0))
    g[1, 5] = g[1, 6] = -2.0                         # an exact tie: the lower id
    sel, pr = O.ds_route(g, 6)
    assert sel[0].tolist() == [0, 1, 2, 3, 4, 6] and sel[1].tolist() == [0, 1, 2, 3, 4, 5]
    p = np.exp(g[0] - 6.0, dtype=np.float32)
    assert np.float32(g[0, 5] - 6.0) == np.float32(g[0, 6] - 6.0)   # equal probabilities
    np.testing.assert_allclose(pr[0], p[[0, 1, 2, 3, 4, 6]] / p.sum(), rtol=1e-6)


# ---- GPT-2-XL-shaped batched decode ---------------------

def test_xl_step_without_rounding_is_the_pinned_gpt2_forward():
    """orc_xl_step with its bf16 roundings off (f32 cache) is the f32 GPT-2
    forward pinned to the reference (orc_gpt2_forward) on the bf16-valued
    weights, bit for bit: logits and ids of two sequences decoded side by side
    over 12 positions (a prompt of 6 fed one id per step, then 6 greedy)."""
    from types import SimpleNamespace
    from thvm_b200.gpt2_xl import XLConfig, xl_weights
    cfg = XLConfig(n_layers=2, dim=128, heads=2, vocab=500, max_ctx=32, batch=2)
    w = xl_weights(cfg, seed=4)
    rng = np.random.default_rng(7)
    for k in w:   # LayerNorm affine parameters off their identity defaults
        if ".ln_" in k or k.startswith("ln_f"):
            w[k] = (w[k] + rng.uniform(-0.1, 0.1, w[k].shape)).astype(np.float32)
    xl = O.XLModel(cfg, w, exact=True)
    wide = lambda b: O.bf16_to_f32(b)
    names = {"attn.w": "attn.c_attn.weight", "attn.b": "attn.c_attn.bias", "proj.w": "attn.c_proj.weight",
             "proj.b": "attn.c_proj.bias", "fc.w": "mlp.c_fc.weight", "fc.b": "mlp.c_fc.bias",
             "p2.w": "mlp.c_proj.weight", "p2.b": "mlp.c_proj.bias", "ln_1.w": "ln_1.weight", "ln_1.b": "ln_1.bias",
             "ln_2.w": "ln_2.weight", "ln_2.b": "ln_2.bias"}
    g = {"wte.weight": wide(w["wte"]), "wpe.weight": wide(w["wpe"]), "lm_head.weight": wide(w["lm_head"]),
         "ln_f.weight": w["ln_f.w"], "ln_f.bias": w["ln_f.b"]}
    for i in range(cfg.n_layers):
        for a, b in names.items():
            v = w[f"h.{i}.{a}"]
            g[f"h.{i}.{b}"] = wide(v) if v.dtype == np.uint16 else v
    gc = SimpleNamespace(n_layers=cfg.n_layers, n_heads=cfg.heads, dim=cfg.dim, vocab=cfg.vocab,
                         max_ctx=cfg.max_ctx, norm_eps=cfg.norm_eps)
    refs = [O.GPT2(gc, g) for _ in range(cfg.batch)]
    prompt = rng.integers(0, cfg.vocab, (cfg.batch, 6)).astype(np.int32)
    tok = prompt[:, 0]
    for pos in range(12):
        lg, nxt = xl.step(tok, pos)
        for b, r in enumerate(refs):
            t, rl = r.forward([int(tok[b])], pos, want_logits=True)
            assert int(nxt[b]) == t
            assert np.array_equal(lg[b].view(np.uint32), rl.view(np.uint32)), (pos, b)
        tok = prompt[:, pos + 1] if pos + 1 < prompt.shape[1] else nxt
