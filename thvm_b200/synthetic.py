"""Seeded synthetic inputs for the decode workloads (no checkpoints, no network).

The GPT-2 decoder shape is the one `bench/gpt2/thvm_gpt2.py:27-128` builds with
`MODEL_PARAMS['gpt2']` (`thvm_gpt2.py:131-136`).  Parameters are generated in
the reference's `get_state_dict` key order (`py/thvm/nn_state.py:233`), which
for that Transformer is: wte, wpe, then per block c_attn w/b, c_proj w/b,
c_fc w/b, mlp c_proj w/b, ln_1 w/b, ln_2 w/b, then ln_f w/b and lm_head.
Every Linear weight, bias and embedding is N(0, 0.02) drawn from one
`numpy.random.default_rng(seed)` stream (float32 standard-normal draws times
float32(0.02)); LayerNorm weights are 1 and biases 0 and take no draws.
Prompts are `default_rng(1).integers(0, vocab, n)`.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


@dataclass(frozen=True)
class GPT2Config:
    n_layers: int = 12
    n_heads: int = 12
    dim: int = 768
    vocab: int = 50257
    max_ctx: int = 1024
    norm_eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def hidden(self) -> int:
        return 4 * self.dim


GPT2_SMALL = GPT2Config()
GPT2_XL = GPT2Config(n_layers=48, n_heads=25, dim=1600)


def gpt2_state_keys(cfg: GPT2Config) -> list[tuple[str, tuple[int, ...]]]:
    """(key, shape) in the reference's get_state_dict order; Linear weights
    are stored (out, in) as `py/thvm/nn.py:12-25` does."""
    d, h = cfg.dim, cfg.hidden
    keys: list[tuple[str, tuple[int, ...]]] = [
        ("wte.weight", (cfg.vocab, d)),
        ("wpe.weight", (cfg.max_ctx, d)),
    ]
    for i in range(cfg.n_layers):
        p = f"h.{i}."
        keys += [
            (p + "attn.c_attn.weight", (3 * d, d)), (p + "attn.c_attn.bias", (3 * d,)),
            (p + "attn.c_proj.weight", (d, d)), (p + "attn.c_proj.bias", (d,)),
            (p + "mlp.c_fc.weight", (h, d)), (p + "mlp.c_fc.bias", (h,)),
            (p + "mlp.c_proj.weight", (d, h)), (p + "mlp.c_proj.bias", (d,)),
            (p + "ln_1.weight", (d,)), (p + "ln_1.bias", (d,)),
            (p + "ln_2.weight", (d,)), (p + "ln_2.bias", (d,)),
        ]
    keys += [("ln_f.weight", (d,)), ("ln_f.bias", (d,)), ("lm_head.weight", (cfg.vocab, d))]
    return keys


def gpt2_weights(cfg: GPT2Config = GPT2_SMALL, seed: int = 0,
                 std: float = 0.02) -> dict[str, np.ndarray]:
    rng = np.random.default_rng(seed)
    out: dict[str, np.ndarray] = {}
    for key, shape in gpt2_state_keys(cfg):
        if ".ln_" in key or key.startswith("ln_f"):
            fill = 1.0 if key.endswith("weight") else 0.0
            out[key] = np.full(shape, fill, dtype=np.float32)
        else:
            out[key] = rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    return out


def prompt_tokens(n: int = 16, vocab: int = 50257, seed: int = 1) -> list[int]:
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]
