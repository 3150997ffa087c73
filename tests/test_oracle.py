"""The CPU oracle against the reference's own outputs (tests/golden/, made by
running the reference: tests/golden/make_golden.py).  Bit-exact: the oracle
restates the reference's float32 op order, its xexp2 and its serial sums."""
import numpy as np
import pytest

import oracle as O


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
