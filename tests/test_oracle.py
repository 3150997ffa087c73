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
