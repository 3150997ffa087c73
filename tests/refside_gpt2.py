"""Runs the reference's own GPT-2 example (bench/gpt2/thvm_gpt2.py, through
the reference's own `thvm` Python package) on a build of the reference
runtime that carries this device's router (thvm_b200/refside, `make cpu` /
`make cuda`), and prints one JSON line: the greedy ids and the router's
counters.  A separate process per run: the package picks its device from
DEV at import.

    python tests/refside_gpt2.py <cpu|cuda> <n_layers> <n_new>
"""
import ctypes
import json
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]


def main() -> None:
    variant, n_layers, n_new = sys.argv[1], int(sys.argv[2]), int(sys.argv[3])
    pkg = REPO / "thvm_b200" / "refside" / "_build" / variant
    os.environ["DEV"] = "cuda" if variant == "cuda" else "cpu"
    os.environ.setdefault("JIT", "0")
    os.environ["MAX_CONTEXT"] = "1024"
    sys.path[:0] = [str(pkg), str(REPO)]
    import thvm_gpt2 as G
    from thvm import Tensor, Variable
    from thvm.nn.state import load_state_dict
    from thvm_b200.synthetic import GPT2Config, gpt2_weights, prompt_tokens

    cfg = GPT2Config(n_layers=n_layers)
    model = G.Transformer(**dict(G.MODEL_PARAMS["gpt2"], n_layers=n_layers))
    load_state_dict(model, {k: Tensor(v) for k, v in gpt2_weights(cfg, seed=0).items()}, verbose=False)
    toks = prompt_tokens(16, cfg.vocab, seed=1)
    start = 0
    for _ in range(n_new):
        tk = Tensor([toks]) if start == 0 else Variable("tokens", 0, cfg.vocab - 1).bind(toks[start])
        sp = Variable("start_pos", 1 if start else 0, cfg.max_ctx - 1).bind(start)
        nxt = model(tk, sp, 0.0).tolist()[0]
        start = len(toks)
        toks.append(int(nxt))
    lib = ctypes.CDLL(str(pkg / "thvm" / "libthvm_py.so"))
    st = (ctypes.c_uint64 * 7)()
    lib.py_sm100_ref_stats(st)
    keys = ["dispatch", "linear", "interp", "declined", "checked", "mismatch", "exact"]
    out = {"ids": toks[16:], **dict(zip(keys, map(int, st)))}
    if variant == "cuda":
        out["interp_status"] = int(lib.py_sm100_interp_status())
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
