"""The continuous-batching serve loop (thvm_b200.serve.Server, the reference's
DSV2_SERVE request loop, bench/dsv2_decode_bench.c:2760-2900) on the reduced
config-5 model of test_gpu_dsv2.py: four rows, requests of different prompt
lengths joining while others run, one stopped by its eos id, one admitted
into a row another request freed.  Every request's ids must be the base
greedy stream of that prompt (DSModel at batch 1: the prompt teacher-forced,
then its argmaxes)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, dim=512, heads=4, kv_lora=128, d_nope=32, d_rope=16, d_v=32, n_exp=8, top_k=3, moe_inter=128,
           dense_inter=256, n_dense=1, n_shared=2, vocab=1000, max_ctx=64)


def _base(m, prompt, n_new):
    import torch
    m.pos.zero_()
    out = []
    for t in range(len(prompt) + n_new - 1):
        if t < len(prompt):
            m.tok.copy_(torch.tensor([int(prompt[t])], dtype=torch.int32))
        m.step()
        if t + 1 >= len(prompt):
            out.append(int(m.tok.item()))
    return np.array(out, np.int32)


def test_serve_requests_match_their_base_streams():
    from thvm_b200.dsv2 import DSConfig, DSModel, ds_shard, ds_weights, shard_ds_weights
    from thvm_b200.serve import Server
    cfg1 = DSConfig(**CFG, batch=1)
    w = ds_weights(cfg1, seed=0)
    sh = ds_shard(cfg1, 0, 1)
    base_model = DSModel(cfg1, shard_ds_weights(w, cfg1, sh), sh)
    rng = np.random.default_rng(7)
    reqs = {"A": (rng.integers(0, 1000, 5), 10), "B": (rng.integers(0, 1000, 3), 6),
            "C": (rng.integers(0, 1000, 7), 8), "D": (rng.integers(0, 1000, 4), 9)}
    want = {k: _base(base_model, p, n) for k, (p, n) in reqs.items()}
    eos_c = int(want["C"][2])
    want["C"] = want["C"][:int(np.nonzero(want["C"] == eos_c)[0][0]) + 1]
    assert base_model.status() == 0

    cfg = DSConfig(**CFG, batch=4)
    srv = Server(cfg, shard_ds_weights(w, cfg, sh), sh)
    srv.capture()
    ids = {"A": srv.submit(*reqs["A"]), "B": srv.submit(*reqs["B"])}
    srv.run(4)
    ids["C"] = srv.submit(reqs["C"][0], reqs["C"][1], eos=eos_c)
    got, steps = {}, 0
    while srv.busy():
        srv.run(2)
        steps += 2
        assert steps < 200
        for rid, out in srv.poll().items():
            got[rid] = out
            if "D" not in ids:   # the first freed row takes the last request
                ids["D"] = srv.submit(*reqs["D"])
    for k, rid in ids.items():
        np.testing.assert_array_equal(got[rid], want[k], err_msg=k)
    assert srv.status() == 0
