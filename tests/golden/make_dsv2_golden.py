"""Generate tests/golden/dsv2.npz by running the REFERENCE's own DeepSeek-V2
decode bench (bench/dsv2_decode_bench.c) on its CPU backend.

    make -C oracle ref                      # builds oracle/_ref/dsv2_decode_bench
    python tests/golden/make_dsv2_golden.py

Steps: seeded weights in the reference's pack layout (oracle.ds_ref_weights,
shape oracle.DSREF_SMALL) are written as a DSV2PK01 pack; the bench runs with
DEV=cpu, DSV2_WEIGHTS=<pack>, DSV2_PROMPT_IDS=<8 seeded ids>, DSV2_COUNT=24,
DSV2_TOP2=1 and DSV2_DUMP=1 plus the DSV2_* shape knobs.  Its printed lines are
parsed into:

  prompt, gen_ids      the 8 prompt ids and the 24 greedy ids it generated
  top2_ids, top2_txt   per generated step 1..23 the top-2 ids and their logits
                       as printed ("%.6f")
  dump_*               the byte fingerprints DSV2_DUMP prints after the first
                       step (prompt id 0 at position 0): qlat, attention
                       weights, olat, o of the last layer, the dense layer's
                       gate / up outputs, per-layer cache row 0 sums, the
                       logits bit sum and logits[0..1]
  cfg_*, seed          the shape and the weight seed, so the test regenerates
                       the same weights

Nothing under tests/ runs the reference at test time: only this file does.
"""
from __future__ import annotations

import os
import re
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(REPO))
OUT = Path(__file__).resolve().parent / "dsv2.npz"
SEED, N_PROMPT, COUNT = 0, 8, 24


def main() -> None:
    import oracle as O
    exe = REPO / "oracle" / "_ref" / "dsv2_decode_bench"
    if not exe.exists():
        raise SystemExit("build the reference first: make -C oracle ref")
    cfg = O.DSREF_SMALL
    w = O.ds_ref_weights(cfg, seed=SEED)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, N_PROMPT).astype(np.int32)
    with tempfile.TemporaryDirectory() as td:
        pack = Path(td) / "dsv2_small.pack"
        O.write_dsv2_pack(pack, w)
        env = dict(os.environ, DEV="cpu", DSV2_WEIGHTS=str(pack), DSV2_COUNT=str(COUNT), DSV2_TOP2="1",
                   DSV2_DUMP="1", DSV2_PROMPT_IDS=",".join(map(str, prompt.tolist())), **cfg.env())
        r = subprocess.run([str(exe)], env=env, capture_output=True, text=True, timeout=600)
    if r.returncode != 0:
        raise SystemExit(f"reference run failed ({r.returncode}):\n{r.stdout}\n{r.stderr}")
    txt = r.stdout
    gen = [int(v) for v in re.search(r"thvm gen ids: \[([^\]]*)\]", txt).group(1).split(",")]
    top2 = re.findall(r"top2 step (\d+): tok=(-?\d+)\s+(-?\d+):(\S+)\s+(-?\d+):(\S+)\s+margin", txt)
    dumps = dict(re.findall(r"\[dump\] (T_\w+) bytesum=(\d+)", txt))
    layers = re.findall(r"\[dump\] l(\d+) ckv=(\d+) kpe=(\d+)", txt)
    lg = re.search(r"\[dump\] logits bitsum=(\d+) first2=(\S+) (\S+)", txt)
    out = {
        "seed": np.int64(SEED), "prompt": prompt, "gen_ids": np.array(gen, np.int32),
        "top2_ids": np.array([[int(t[2]), int(t[4])] for t in top2], np.int32),
        "top2_txt": np.array([[t[3], t[5]] for t in top2]),
        "dump_names": np.array(sorted(dumps)), "dump_sums": np.array([int(dumps[k]) for k in sorted(dumps)], np.uint64),
        "dump_ckv": np.array([int(t[1]) for t in layers], np.uint64),
        "dump_kpe": np.array([int(t[2]) for t in layers], np.uint64),
        "dump_logits_bitsum": np.uint64(int(lg.group(1))),
        "dump_logits_first2": np.array([float(lg.group(2)), float(lg.group(3))]),
    }
    for k, v in cfg.env().items():
        out["cfg_" + k] = np.int64(int(v))
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: gen ids {gen}")
    print(f"top2 rows {len(top2)}, dumps {sorted(dumps)}, layers {len(layers)}")


if __name__ == "__main__":
    main()
