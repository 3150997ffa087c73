"""The config-5 step with its host in C (sm100_ds_model_*, thvm_b200/csrc/
ds_host.c: weights from a .safetensors file or named device pointers,
backend buffers, the library's graph slots; no torch) against the Python
host (thvm_b200.dsv2.DSModel) on the reduced model of test_gpu_dsv2.py, both
fed the same teacher-forced ids: the same next ids every step, logits within
1e-3 of the row scale (the expert down projection adds with float atomics in
any order, so h differs in its last bits and a bf16 rounding of the next
norm's output can move by an ulp: ~1.5e-4 measured, far inside the 2e-2
gate), the position advanced once a step."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, dim=512, heads=4, kv_lora=128, d_nope=32, d_rope=16, d_v=32, n_exp=8, top_k=3, moe_inter=128,
           dense_inter=256, n_dense=1, n_shared=2, vocab=1000, max_ctx=64, batch=32)


def test_c_host_matches_the_python_host(tmp_path):
    import torch
    from thvm_b200.ds_host import CDSModel, save_ds_weights
    from thvm_b200.dsv2 import DSConfig, DSModel, ds_shard, ds_weights, shard_ds_weights
    cfg = DSConfig(**CFG)
    sh = ds_shard(cfg, 0, 1)
    w = shard_ds_weights(ds_weights(cfg, seed=0), cfg, sh)
    path = tmp_path / "ds.safetensors"
    save_ds_weights(path, cfg, w)
    ref = DSModel(cfg, w, sh)
    cm = CDSModel(cfg, path)
    # the same host over weights already on the device (the Python host's tensors)
    cp = CDSModel(cfg, {**ref.w, "cos": ref.cos, "sin": ref.sin})
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, (cfg.batch, 6)).astype(np.int32)
    tok = prompt[:, 0]
    worst = 0.0
    try:
        for pos in range(14):
            ref.tok.copy_(torch.from_numpy(tok))
            ref.step()
            got = cm.step(tok)
            want = ref.tok.cpu().numpy()
            np.testing.assert_array_equal(got, want, err_msg=f"position {pos}")
            np.testing.assert_array_equal(cp.step(tok), want, err_msg=f"position {pos} (device weights)")
            a, b = cm.logits(), ref.logits.cpu().numpy()
            worst = max(worst, float((np.abs(a - b).max(1) / np.abs(b).max(1)).max()))
            assert cm.pos == pos + 1
            tok = prompt[:, pos + 1] if pos + 1 < prompt.shape[1] else want
        assert worst <= 1e-3, worst
        assert ref.status() == 0
    finally:
        cm.close()
        cp.close()


def test_pure_c_program_decodes_the_python_hosts_ids(tmp_path):
    """thvm_b200/examples/ds_decode.c, compiled with gcc against the header
    and the library and run as its own process (no Python in it): its ids,
    prompt fed then greedy, equal the Python host's every step."""
    import shutil
    import subprocess
    from pathlib import Path
    import torch
    from thvm_b200.ds_host import save_ds_weights
    from thvm_b200.dsv2 import DSConfig, DSModel, ds_shard, ds_weights, shard_ds_weights
    root = Path(__file__).resolve().parents[1]
    cfg = DSConfig(**{**CFG, "batch": 4})
    sh = ds_shard(cfg, 0, 1)
    w = shard_ds_weights(ds_weights(cfg, seed=0), cfg, sh)
    path = tmp_path / "ds.safetensors"
    save_ds_weights(path, cfg, w)
    exe = tmp_path / "ds_decode"
    cc = shutil.which("gcc") or "gcc"
    subprocess.run([cc, "-std=c11", "-O2", f"-I{root / 'include'}", str(root / "thvm_b200/examples/ds_decode.c"),
                    f"-L{root / 'thvm_b200'}", "-lthvm_sm100", f"-Wl,-rpath,{root / 'thvm_b200'}", "-o", str(exe)],
                   check=True)
    np_, steps = 5, 12
    prompt = np.random.default_rng(4).integers(0, cfg.vocab, (cfg.batch, np_)).astype(np.int32)
    fields = [cfg.n_layers, cfg.dim, cfg.heads, cfg.kv_lora, cfg.d_nope, cfg.d_rope, cfg.d_v, cfg.n_exp, cfg.top_k,
              cfg.moe_inter, cfg.dense_inter, cfg.n_dense, cfg.n_shared, cfg.vocab, cfg.max_ctx, cfg.batch]
    args = [str(exe), str(path)] + [str(v) for v in fields] + [repr(cfg.eps), repr(cfg.scale), str(np_), str(steps)]
    args += [str(v) for v in prompt.reshape(-1)]
    r = subprocess.run(args, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    got = np.array([[int(v) for v in line.split()] for line in r.stdout.strip().splitlines()], np.int32)
    ref = DSModel(cfg, w, sh)
    out = None
    for t in range(steps):
        ref.tok.copy_(torch.from_numpy(prompt[:, t] if t < np_ else out))
        ref.step()
        out = ref.tok.cpu().numpy()
        np.testing.assert_array_equal(got[t], out, err_msg=f"step {t}")
    assert ref.status() == 0
