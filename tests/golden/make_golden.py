"""Generate the golden fixtures in tests/golden/ by running the REFERENCE itself.

This is test infrastructure, run where the reference checkout is present
(its location in $THVM_REF, else the build container's default):

    make -C oracle ref                  # builds oracle/_ref/libthvm_py.so
    python tests/golden/make_golden.py  # [ops] [gpt2]

It imports the reference's own Python package (`py/thvm`) over that CPU-only
library (through a directory of symlinks, oracle/_ref/py/thvm, so that the
package finds its library beside itself) and the reference's GPT-2 model code
(`bench/gpt2/thvm_gpt2.py`), runs them on seeded inputs, and writes:

  ops.npz      per-op inputs and outputs (linear, layernorm, softmax, gelu,
               scaled_dot_product_attention decode / causal / masked, argmax
               with ties, embedding incl. out-of-range ids).
  dtypes.npz   the reference's own storage conversions (src/dtype/fp_convert.c
               f32_to_bf16, src/dtype/fp8.c f32_to_fp8e4m3_sat and
               fp8e4m3_to_f32, called in its library) on f32 bit patterns:
               seeded normals, random bit patterns (NaN payloads, subnormals,
               infinities) and the e4m3 rounding / saturation edges; every e4m3
               code decoded.
  state.safetensors  a few seeded tensors of several dtypes written by the
               reference's own safe_save (the weight-file loader's fixture).
  state.pt, state_legacy.pt, torch_state.npz  a seeded state dict saved by
               torch.save in its zip and legacy formats, and what the
               reference's own torch_load reads from each (the checkpoint
               loader's fixture).
  gpt2.npz     GPT-2 small (12 layers, fp32, MAX_CONTEXT=1024) greedy decode:
               the 16 prompt ids, the 64 generated ids, per-step top-1 / top-2
               logits, and the full logits of the prompt step and the first
               decode step.
  gpt2_l2.npz  the same model cut to 2 layers: 16 prompt ids and 8 greedy ids
               (the reference-side router's end-to-end fixture).

Nothing under tests/ reads the reference at test time: only these files.
"""
from __future__ import annotations

import os
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
REF = Path(os.environ.get("THVM_REF", "/root/reference"))
OUT = Path(__file__).resolve().parent


def _ref_package() -> Path:
    """oracle/_ref/py/thvm: symlinks to the reference's py/thvm/*.py plus the
    library built by `make -C oracle ref`."""
    lib = REPO / "oracle" / "_ref" / "libthvm_py.so"
    if not lib.exists():
        raise SystemExit("build the reference first: make -C oracle ref")
    pkg = REPO / "oracle" / "_ref" / "py" / "thvm"
    pkg.mkdir(parents=True, exist_ok=True)
    for src in sorted((REF / "py" / "thvm").glob("*.py")):
        dst = pkg / src.name
        if not dst.is_symlink():
            dst.symlink_to(src)
    so = pkg / "libthvm_py.so"
    if not so.exists():
        so.symlink_to(lib)
    return pkg.parent


def _setup():
    os.environ.setdefault("DEV", "cpu")
    os.environ.setdefault("JIT", "0")
    os.environ["MAX_CONTEXT"] = "1024"
    sys.path[:0] = [str(_ref_package()), str(REF / "bench" / "gpt2"), str(REPO)]


def make_ops() -> None:
    from thvm import Tensor, dtypes

    rng = np.random.default_rng(1234)
    f32 = np.float32
    g: dict[str, np.ndarray] = {}

    def T(a):
        return Tensor(np.ascontiguousarray(a))

    # linear: x @ W^T + b with W (out, in), ragged K and N (py/thvm/nn.py:24-25)
    for name, (m, k, n) in {"lin_a": (1, 768, 320), "lin_b": (3, 37, 29),
                            "lin_c": (16, 100, 70)}.items():
        x = rng.standard_normal((1, m, k)).astype(f32)
        w = (rng.standard_normal((n, k)) * 0.02).astype(f32)
        b = (rng.standard_normal((n,)) * 0.02).astype(f32)
        g[name + "_x"], g[name + "_w"], g[name + "_b"] = x, w, b
        g[name + "_y"] = T(x).linear(T(w).transpose(), T(b)).numpy()

    # layernorm + affine (py/thvm/nn.py:160-164)
    for name, shape in {"ln_a": (1, 1, 768), "ln_b": (4, 3, 100), "ln_c": (16, 1600)}.items():
        x = (rng.standard_normal(shape) * 3 + 0.5).astype(f32)
        w = rng.standard_normal(shape[-1]).astype(f32)
        b = rng.standard_normal(shape[-1]).astype(f32)
        g[name + "_x"], g[name + "_w"], g[name + "_b"] = x, w, b
        g[name + "_y"] = (T(x).layernorm(axis=-1, eps=1e-5) * T(w) + T(b)).numpy()

    # softmax over the last axis, with -inf entries (masked scores)
    x = rng.standard_normal((5, 67)).astype(f32) * 4
    x[1, 10:] = -np.inf
    x[2, :3] = -np.inf
    g["sm_x"] = x
    g["sm_y"] = T(x).softmax(-1).numpy()

    # GELU, tanh form (src/nn/elementwise.c:27-34)
    x = np.concatenate([np.linspace(-12, 12, 2001), rng.standard_normal(999) * 3]).astype(f32)
    g["gelu_x"] = x
    g["gelu_y"] = T(x).gelu().numpy()

    # SDPA decode: one query row over L keys (GPT-2 decode shape)
    for name, (b, h, lq, lk, d) in {"sdpa_dec": (1, 12, 1, 37, 64),
                                   "sdpa_dec1": (1, 12, 1, 1, 64)}.items():
        q, k, v = (rng.standard_normal((b, h, n, d)).astype(f32) for n in (lq, lk, lk))
        g[name + "_q"], g[name + "_k"], g[name + "_v"] = q, k, v
        g[name + "_y"] = T(q).scaled_dot_product_attention(T(k), T(v)).numpy()

    # SDPA causal (is_causal) and with GPT-2's additive -inf triu mask
    q, k, v = (rng.standard_normal((2, 4, 33, 16)).astype(f32) for _ in range(3))
    g["sdpa_causal_q"], g["sdpa_causal_k"], g["sdpa_causal_v"] = q, k, v
    g["sdpa_causal_y"] = T(q).scaled_dot_product_attention(T(k), T(v), is_causal=True).numpy()
    s = 16
    q, k, v = (rng.standard_normal((1, 12, s, 64)).astype(f32) for _ in range(3))
    mask = Tensor.full((1, 1, s, s), float("-inf"), dtype=dtypes.float32).triu(1)
    g["sdpa_mask_q"], g["sdpa_mask_k"], g["sdpa_mask_v"] = q, k, v
    g["sdpa_mask_m"] = mask.numpy()
    g["sdpa_mask_y"] = T(q).scaled_dot_product_attention(T(k), T(v), mask).numpy()

    # argmax with ties (first index wins, py/thvm/tensor.py:998-1011)
    x = rng.standard_normal((4, 5003)).astype(f32)
    x[1, 7] = x[1, 4000] = x[1].max() + 1.0
    x[2, :] = 0.25
    x[3, 5002] = 100.0
    g["am_x"] = x
    g["am_y"] = T(x).argmax(-1).numpy()

    # embedding rows, including ids outside [0, vocab)
    w = rng.standard_normal((100, 16)).astype(f32)
    idx = np.array([[0, 5, 99, 17, 5, 100, -1]], dtype=np.int32)
    g["emb_w"], g["emb_idx"] = w, idx
    g["emb_y"] = T(w).embedding(Tensor(idx)).numpy()

    np.savez_compressed(OUT / "ops.npz", **g)
    print("wrote", OUT / "ops.npz", len(g), "arrays")


def make_gpt2(n_new: int = 64) -> None:
    import thvm_gpt2 as G
    from thvm import Tensor, Variable
    from thvm.nn.state import get_state_dict, load_state_dict
    from thvm_b200.synthetic import GPT2_SMALL, gpt2_state_keys, gpt2_weights, prompt_tokens

    cfg = GPT2_SMALL
    model = G.Transformer(**G.MODEL_PARAMS["gpt2"])
    ref_keys = [(k, tuple(v.shape)) for k, v in get_state_dict(model).items()]
    assert ref_keys == gpt2_state_keys(cfg), "state dict order differs from thvm_b200.synthetic"
    weights = gpt2_weights(cfg, seed=0)
    load_state_dict(model, {k: Tensor(v) for k, v in weights.items()}, verbose=False)

    captured = {}
    lm_head = model.lm_head

    def lm_head_tap(x):
        y = lm_head(x)
        captured["logits"] = y
        return y
    model.lm_head = lm_head_tap

    toks = prompt_tokens(16, cfg.vocab, seed=1)
    prompt = list(toks)
    top = []
    full = {}
    start_pos = 0
    t0 = time.time()
    for step in range(n_new):
        if start_pos == 0:
            tk = Tensor([toks])
        else:
            tk = Variable("tokens", 0, cfg.vocab - 1).bind(toks[start_pos])
        sp = Variable("start_pos", 1 if start_pos else 0, cfg.max_ctx - 1).bind(start_pos)
        nxt = model(tk, sp, 0.0).tolist()[0]
        logits = captured["logits"].numpy()[0, -1].astype(np.float32)
        order = np.argsort(-logits, kind="stable")
        top.append((int(order[0]), float(logits[order[0]]), int(order[1]), float(logits[order[1]])))
        if step in (0, 1, n_new - 1):
            full[f"logits_step{step}"] = logits
        assert int(order[0]) == nxt or logits[order[0]] == logits[nxt], (step, nxt, order[:2])
        start_pos = len(toks)
        toks.append(nxt)
        print(f"step {step:3d} tok {nxt:6d} margin {top[-1][1] - top[-1][3]:.4g} "
              f"{time.time() - t0:.1f}s", flush=True)

    np.savez_compressed(OUT / "gpt2.npz", prompt=np.array(prompt, np.int32),
                        tokens=np.array(toks[16:], np.int32),
                        top=np.array([(a, b, c, d) for a, b, c, d in top], np.float64),
                        **full)
    print("wrote", OUT / "gpt2.npz")


def make_gpt2_l2(n_new: int = 8) -> None:
    """gpt2_l2.npz: the same model code and weight generator cut to 2 layers
    (seed 0, the same 16 prompt ids), n_new greedy ids: the fixture of the
    reference-side router's end-to-end tests, which run this model through
    the reference's own package on the sm_100a device."""
    import thvm_gpt2 as G
    from thvm import Tensor, Variable
    from thvm.nn.state import load_state_dict
    from thvm_b200.synthetic import GPT2Config, gpt2_weights, prompt_tokens

    cfg = GPT2Config(n_layers=2)
    params = dict(G.MODEL_PARAMS["gpt2"], n_layers=2)
    model = G.Transformer(**params)
    load_state_dict(model, {k: Tensor(v) for k, v in gpt2_weights(cfg, seed=0).items()}, verbose=False)
    toks = prompt_tokens(16, cfg.vocab, seed=1)
    prompt = list(toks)
    start_pos = 0
    for _ in range(n_new):
        tk = Tensor([toks]) if start_pos == 0 else Variable("tokens", 0, cfg.vocab - 1).bind(toks[start_pos])
        sp = Variable("start_pos", 1 if start_pos else 0, cfg.max_ctx - 1).bind(start_pos)
        nxt = model(tk, sp, 0.0).tolist()[0]
        start_pos = len(toks)
        toks.append(nxt)
    np.savez_compressed(OUT / "gpt2_l2.npz", prompt=np.array(prompt, np.int32), tokens=np.array(toks[16:], np.int32))
    print("wrote", OUT / "gpt2_l2.npz", toks[16:])


def make_dtypes() -> None:
    """bf16 / fp8 e4m3 conversions of the reference library, bit for bit."""
    import ctypes
    lib = ctypes.CDLL(str(REPO / "oracle" / "_ref" / "libthvm_py.so"))
    lib.f32_to_bf16.restype = ctypes.c_uint16
    lib.f32_to_fp8e4m3_sat.restype = ctypes.c_uint8
    lib.fp8e4m3_to_f32.restype = ctypes.c_float
    lib.f32_to_bf16.argtypes = lib.f32_to_fp8e4m3_sat.argtypes = [ctypes.c_float]
    lib.fp8e4m3_to_f32.argtypes = [ctypes.c_uint8]
    rng = np.random.default_rng(7)
    edges = np.array([0.0, -0.0, np.inf, -np.inf, 448, 456, 464, 464.0001, 472, 480, -1000, 2 ** -10,
                      2 ** -9, 1.5 * 2 ** -10, 2.5 * 2 ** -9, 2 ** -6, 1.0625, 1.1875, 3e-38, 1e-45,
                      1.00390625, 1.0078125, 1.01171875], np.float32)
    x = np.concatenate([edges, -edges, rng.standard_normal(4096).astype(np.float32),
                        (rng.standard_normal(2048) * 64).astype(np.float32),
                        rng.integers(0, 2 ** 32, 4096, dtype=np.uint64).astype(np.uint32).view(np.float32)])
    # pass the exact f32 bits (a NaN payload survives: no Python float round trip)
    cf = [ctypes.c_float.from_buffer_copy(v.tobytes()) for v in x]
    bf16 = np.array([lib.f32_to_bf16(v) for v in cf], np.uint16)
    fp8 = np.array([lib.f32_to_fp8e4m3_sat(v) for v in cf], np.uint8)
    dec = np.array([lib.fp8e4m3_to_f32(i) for i in range(256)], np.float32)
    np.savez_compressed(OUT / "dtypes.npz", x_bits=x.view(np.uint32), bf16=bf16, fp8e4m3=fp8, fp8e4m3_decoded=dec)
    print("wrote", OUT / "dtypes.npz")


def state_tensors() -> dict:
    """The tensors of state.safetensors as numpy arrays (bf16 and fp8 as their
    raw codes): seeded, several dtypes and ranks, an empty one."""
    rng = np.random.default_rng(77)
    return {
        "wte.weight": rng.standard_normal((7, 5)).astype(np.float32),
        "h.0.attn.c_attn.bias": rng.standard_normal(12).astype(np.float32),
        "h.0.ln_1.weight": (rng.standard_normal(9) * 0.5).astype(np.float16),
        "experts.codes": rng.integers(0, 255, (3, 4, 2)).astype(np.uint8),
        "positions": rng.integers(-1000, 1000, (2, 3)).astype(np.int32),
        "lm_head.weight.bf16": rng.integers(0, 65535, (4, 6)).astype(np.uint16),
        "empty": np.zeros((0, 4), np.float32),
    }


def make_state() -> None:
    """state.safetensors, written by the reference's own safe_save
    (py/thvm/nn_state.py:64-85) from reference Tensors of several dtypes."""
    from thvm import Tensor, dtypes
    from thvm.nn_state import safe_save
    t = state_tensors()
    ts = {}
    for k, v in t.items():
        if k.endswith(".bf16"):
            ts[k] = Tensor(v.astype(np.int16)).bitcast(dtypes.bfloat16)
        elif k == "experts.codes":
            ts[k] = Tensor(v).bitcast(dtypes.fp8e4m3)
        else:
            ts[k] = Tensor(v)
    safe_save(ts, OUT / "state.safetensors", metadata={"format": "thvm", "note": "golden"})
    print("wrote", OUT / "state.safetensors")


def torch_state():
    """The state dict of state.pt / state_legacy.pt: seeded tensors of several
    dtypes and ranks, a transposed one and a permuted one (strides a
    permutation of row-major), a slice at a storage offset that shares its
    storage with another entry, a parameter, a 0-d and an empty tensor."""
    import torch
    rng = np.random.default_rng(78)
    base = torch.from_numpy(rng.standard_normal((6, 10)).astype(np.float32))
    return {
        "wte.weight": torch.from_numpy(rng.standard_normal((7, 5)).astype(np.float32)),
        "h.0.ln_1.weight": torch.from_numpy((rng.standard_normal(9) * 0.5).astype(np.float16)),
        "h.0.mlp.bf16": torch.from_numpy(rng.standard_normal((3, 4)).astype(np.float32)).bfloat16(),
        "double": torch.from_numpy(rng.standard_normal(4)),
        "positions": torch.from_numpy(rng.integers(-1000, 1000, (2, 3))),
        "ids32": torch.from_numpy(rng.integers(0, 50000, 6).astype(np.int32)),
        "codes": torch.from_numpy(rng.integers(0, 255, (3, 2)).astype(np.uint8)),
        "mask": torch.from_numpy(rng.integers(0, 2, 5).astype(bool)),
        "base": base,
        "base.rows": base[2:4],
        "lm_head.t": base.t(),
        "perm": torch.from_numpy(rng.standard_normal((2, 3, 4)).astype(np.float32)).permute(2, 0, 1),
        "param": torch.nn.Parameter(torch.from_numpy(rng.standard_normal((2, 2)).astype(np.float32))),
        "scalar": torch.tensor(3.5),
        "empty": torch.zeros(0, 4),
    }


def make_torch() -> None:
    """state.pt (torch.save's zip format) and state_legacy.pt (its legacy
    pickle format) of torch_state(), and torch_state.npz: what the
    reference's own torch_load (py/thvm/nn_state.py:123-230) reads from each,
    as numpy arrays under "zip/<name>" and "legacy/<name>"."""
    import torch
    from thvm.nn_state import torch_load
    sd = torch_state()
    torch.save(sd, OUT / "state.pt")
    torch.save(sd, OUT / "state_legacy.pt", _use_new_zipfile_serialization=False)
    out = {}
    for tag, fn in (("zip", "state.pt"), ("legacy", "state_legacy.pt")):
        for k, t in torch_load(OUT / fn).items():
            out[f"{tag}/{k}"] = t.numpy()
    np.savez(OUT / "torch_state.npz", **out)
    print("wrote", OUT / "state.pt", OUT / "state_legacy.pt", OUT / "torch_state.npz")


if __name__ == "__main__":
    which = sys.argv[1:] or ["ops", "gpt2", "gpt2_l2", "dtypes", "state", "torch"]
    if "dtypes" in which:
        make_dtypes()
    if "ops" in which or "gpt2" in which or "gpt2_l2" in which or "state" in which or "torch" in which:
        _setup()
    if "ops" in which:
        make_ops()
    if "gpt2" in which:
        make_gpt2()
    if "gpt2_l2" in which:
        make_gpt2_l2()
    if "state" in which:
        make_state()
    if "torch" in which:
        make_torch()
