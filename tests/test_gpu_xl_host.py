"""The config-3 model with its host in C (sm100_xl_model_*, thvm_b200/csrc/
xl_host.c: weights from a .safetensors file or named device pointers,
backend buffers, the library's graph slots; no torch) against the Python
host (thvm_b200.gpt2_xl.XLModel) on the reduced model of test_gpu_xl.py:
the prompt pass and then decode steps, both hosts issuing the same kernels
in the same order, so the ids and logits agree exactly; the position after
the prompt and after each step."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_c_host_matches_the_python_host(tmp_path):
    import torch
    from thvm_b200.gpt2_xl import XLConfig, XLModel, shard_of, xl_weights
    from thvm_b200.weights import save_safetensors
    from thvm_b200.xl_host import CXLModel
    cfg = XLConfig(n_layers=2, dim=320, heads=5, vocab=1000, max_ctx=64, batch=16)
    w = xl_weights(cfg, seed=2)
    path = tmp_path / "xl.safetensors"
    save_safetensors(path, w)
    ref = XLModel(cfg, w, shard_of(cfg, 0, 1))
    cm = CXLModel(cfg, path)
    cp = CXLModel(cfg, dict(ref.w))   # the same host over the Python host's device tensors
    prompt = np.random.default_rng(6).integers(0, cfg.vocab, (cfg.batch, 11)).astype(np.int32)
    try:
        ref.prefill(prompt)
        want = ref.tok.cpu().numpy()
        np.testing.assert_array_equal(cm.prefill(prompt), want)
        np.testing.assert_array_equal(cp.prefill(prompt), want)
        np.testing.assert_array_equal(cm.logits(), ref.logits.cpu().numpy())
        assert cm.pos == 11 and cp.pos == 11
        for step in range(10):
            tok = want if step % 3 else np.random.default_rng(step).integers(0, cfg.vocab, cfg.batch).astype(np.int32)
            ref.tok.copy_(torch.from_numpy(tok))
            ref.step()
            want = ref.tok.cpu().numpy()
            np.testing.assert_array_equal(cm.step(tok), want, err_msg=f"step {step}")
            np.testing.assert_array_equal(cp.step(tok), want, err_msg=f"step {step} (device weights)")
            np.testing.assert_array_equal(cm.logits(), ref.logits.cpu().numpy(), err_msg=f"step {step}")
            assert cm.pos == 12 + step
    finally:
        cm.close()
        cp.close()


def test_pure_c_program_decodes_the_python_hosts_ids(tmp_path):
    """thvm_b200/examples/xl_decode.c, compiled with gcc against the header
    and the library and run as its own process (no Python in it): the ids
    of its prompt pass and of 6 greedy steps equal the Python host's."""
    import shutil
    import subprocess
    from pathlib import Path
    from thvm_b200.gpt2_xl import XLConfig, XLModel, shard_of, xl_weights
    from thvm_b200.weights import save_safetensors
    root = Path(__file__).resolve().parents[1]
    cfg = XLConfig(n_layers=2, dim=256, heads=4, vocab=1000, max_ctx=64, batch=4)
    w = xl_weights(cfg, seed=4)
    path = tmp_path / "xl.safetensors"
    save_safetensors(path, w)
    exe = tmp_path / "xl_decode"
    subprocess.run([shutil.which("gcc") or "gcc", "-std=c11", "-O2", f"-I{root / 'include'}",
                    str(root / "thvm_b200/examples/xl_decode.c"), f"-L{root / 'thvm_b200'}", "-lthvm_sm100",
                    f"-Wl,-rpath,{root / 'thvm_b200'}", "-o", str(exe)], check=True)
    np_, steps = 9, 6
    prompt = np.random.default_rng(7).integers(0, cfg.vocab, (cfg.batch, np_)).astype(np.int32)
    args = [str(exe), str(path)] + [str(v) for v in (cfg.n_layers, cfg.dim, cfg.heads, cfg.vocab, cfg.max_ctx,
                                                     cfg.batch)]
    args += [repr(cfg.norm_eps), str(np_), str(steps)] + [str(v) for v in prompt.reshape(-1)]
    r = subprocess.run(args, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    got = np.array([[int(v) for v in line.split()] for line in r.stdout.strip().splitlines()], np.int32)
    ref = XLModel(cfg, w, shard_of(cfg, 0, 1))
    ref.prefill(prompt)
    for t in range(steps + 1):
        if t:
            ref.step()
        np.testing.assert_array_equal(got[t], ref.tok.cpu().numpy(), err_msg=f"step {t}")
