"""Blind speculative decode of the batched MoE step (thvm_b200.spec.SpecDecoder,
the reference's DSV2_SPEC path: bench/dsv2_decode_bench.c:1110-1195) on the
reduced config-5 model of test_gpu_dsv2.py: 8 sequences of S = 4 verify rows
(32 rows, shared cache slots) against the base greedy stream of the same
model at batch 8 (one row per sequence).

  forced  drafts seeded with the base stream: every step commits S tokens
          (the acceptance-must-be-full gate) and the committed ids are the
          base stream;
  blind   drafts from the most recent bigram: the committed ids are the base
          stream, whatever the drafts were.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CFG = dict(n_layers=2, dim=512, heads=4, kv_lora=128, d_nope=32, d_rope=16, d_v=32, n_exp=8, top_k=3, moe_inter=128,
           dense_inter=256, n_dense=1, n_shared=2, vocab=1000, max_ctx=64)
N_SEQ, S, N_PROMPT, N_NEW = 8, 4, 6, 24


def _setup():
    from thvm_b200.dsv2 import DSConfig, ds_shard, ds_weights
    base_cfg = DSConfig(**CFG, batch=N_SEQ)
    w = ds_weights(base_cfg, seed=0)
    prompts = np.random.default_rng(5).integers(0, base_cfg.vocab, (N_SEQ, N_PROMPT)).astype(np.int32)
    return base_cfg, w, prompts, ds_shard(base_cfg, 0, 1)


def _base_stream(cfg, w, sh, prompts):
    """prompts teacher-forced, then N_NEW greedy ids, one row per sequence."""
    import torch
    from thvm_b200.dsv2 import DSModel, shard_ds_weights
    m = DSModel(cfg, shard_ds_weights(w, cfg, sh), sh)
    out = np.zeros((N_SEQ, N_PROMPT + N_NEW), np.int32)
    out[:, :N_PROMPT] = prompts
    for pos in range(N_PROMPT + N_NEW - 1):
        if pos < N_PROMPT:
            m.tok.copy_(torch.from_numpy(prompts[:, pos]))
        m.step()
        if pos + 1 >= N_PROMPT:
            out[:, pos + 1] = m.tok.cpu().numpy()
    torch.cuda.synchronize()
    assert m.status() == 0
    return out


def _spec(cfg, w, sh, forced):
    from thvm_b200.dsv2 import DSConfig, shard_ds_weights
    from thvm_b200.spec import SpecDecoder
    scfg = DSConfig(**CFG, batch=N_SEQ * S)
    return SpecDecoder(scfg, shard_ds_weights(w, scfg, sh), sh, N_SEQ, S, forced=forced)


def test_spec_forced_commits_s_per_step_and_the_base_stream():
    import torch
    cfg, w, prompts, sh = _setup()
    base = _base_stream(cfg, w, sh, prompts)
    sd = _spec(cfg, w, sh, forced=True)
    sd.prefill(prompts, seed_ids=base)
    sd.capture()
    want = N_PROMPT
    while want < N_PROMPT + N_NEW:
        sd.replay()
        torch.cuda.synchronize()
        want += S
        ids, ln = sd.stream_ids()
        assert np.all(ln == want), (ln, want)
    n = N_PROMPT + N_NEW
    np.testing.assert_array_equal(ids[:, :n], base)
    assert int(sd.committed.item()) == N_SEQ * (want - N_PROMPT)
    assert sd.status() == 0


def test_spec_blind_commits_the_base_stream():
    import torch
    cfg, w, prompts, sh = _setup()
    base = _base_stream(cfg, w, sh, prompts)
    sd = _spec(cfg, w, sh, forced=False)
    sd.prefill(prompts)
    sd.capture()
    steps = 0
    ids, ln = sd.stream_ids()
    while ln.min() < N_PROMPT + N_NEW:
        sd.replay()
        steps += 1
        assert steps <= N_NEW
        ids, ln = sd.stream_ids()
    n = N_PROMPT + N_NEW
    np.testing.assert_array_equal(ids[:, :n], base)
    assert int(sd.committed.item()) == int((ln - N_PROMPT).sum())
    assert sd.status() == 0
    print(f"blind: {steps} steps for {N_NEW}+ ids per sequence, {int(sd.committed.item())} committed")


def _draft_rule(ids, ln, S, ctx, forced):
    """The reference's draft_prep (bench/dsv2_decode_bench.c:1122-1170) per sequence."""
    P = ln - 1
    if P < 0 or P + S >= ctx:
        return None
    cand = [int(ids[P])]
    best = -1
    if not forced and P >= 1:
        for j in range(P - 1):
            if ids[j] == ids[P - 1] and ids[j + 1] == ids[P]:
                best = j
    for s in range(1, S):
        if forced:
            cand.append(int(ids[P + s]))
        else:
            cand.append(int(ids[best + 1 + s]) if best >= 0 and best + 1 + s <= P else -1)
    return cand


def test_spec_draft_and_accept_follow_the_reference_rule():
    """sm100_spec_draft / sm100_spec_accept on crafted streams: a repeated
    bigram (most recent match wins), no match (holes), a match too close to
    the end for every draft, a sequence whose window would pass the cache
    (left as it is, status 1); then acceptance of 0, 1 and S - 1 drafts."""
    import ctypes
    import torch
    from thvm_b200 import _lib as L
    lib = L.lib()
    ctx, S = 32, 4
    ids = np.zeros((5, ctx), np.int32)
    ln = np.array([12, 9, 10, 31, 11], np.int32)
    ids[0, :12] = [5, 6, 1, 2, 3, 4, 9, 1, 2, 7, 1, 2]                                    # (1, 2) at 2, 7 and P - 1 = 10
    ids[1, :9] = np.arange(100, 109)                                                      # no repeat
    ids[2, :10] = [4, 5, 6, 7, 8, 9, 4, 5, 4, 5]                                          # (4, 5) at 0, 6, 8: two drafts
    ids[3, :31] = 3
    ids[4, :20] = np.arange(200, 220)                                                     # forced run below
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    gi, gl = d(ids), d(ln)
    z = lambda n: torch.zeros(n, dtype=torch.int32, device="cuda")
    tok, cand, rp, rs = z(5 * S), z(5 * S), z(5 * S), z(5 * S)
    lib.sm100_spec_status()
    L.check(lib.sm100_spec_draft(gi.data_ptr(), gl.data_ptr(), 5, ctx, S, 0, tok.data_ptr(), cand.data_ptr(),
                                 rp.data_ptr(), rs.data_ptr(), ctypes.c_void_p(0)), "spec_draft")
    c = cand.cpu().numpy().reshape(5, S)
    for i in range(5):
        want = _draft_rule(ids[i], ln[i], S, ctx, False)
        P = ln[i] - 1
        if want is None:
            assert np.all(c[i] == -1) and np.all(rp.cpu().numpy().reshape(5, S)[i] == min(P, ctx - 1))
            continue
        np.testing.assert_array_equal(c[i], want)
        np.testing.assert_array_equal(tok.cpu().numpy().reshape(5, S)[i], [v if v >= 0 else ids[i, P] for v in want])
        np.testing.assert_array_equal(rp.cpu().numpy().reshape(5, S)[i], P + np.arange(S))
        np.testing.assert_array_equal(rs.cpu().numpy().reshape(5, S)[i], i)
    assert c[0].tolist() == [2, 7, 1, 2]      # the most recent (1, 2) before P is at 7
    assert c[1].tolist() == [108, -1, -1, -1]
    assert int(lib.sm100_spec_status()) == 1   # sequence 3: P + S >= ctx
    # forced drafts read the stream itself
    L.check(lib.sm100_spec_draft(gi.data_ptr(), gl.data_ptr(), 5, ctx, S, 1, tok.data_ptr(), cand.data_ptr(),
                                 rp.data_ptr(), rs.data_ptr(), ctypes.c_void_p(0)), "spec_draft")
    np.testing.assert_array_equal(cand.cpu().numpy().reshape(5, S)[4], ids[4, 10:14])
    lib.sm100_spec_status()
    # accept: am chosen so sequence 0 verifies no draft, 1 (holes) none, 2 one, 4 all
    am = np.full((5, S), -7, np.int32)
    c = cand.cpu().numpy().reshape(5, S)
    am[2, 0] = c[2, 1]
    am[4, :S - 1] = c[4, 1:]
    am[:, S - 1] = 999
    committed = torch.zeros(1, dtype=torch.int64, device="cuda")
    L.check(lib.sm100_spec_accept(gi.data_ptr(), gl.data_ptr(), 5, ctx, S, cand.data_ptr(), d(am).data_ptr(),
                                  committed.data_ptr(), ctypes.c_void_p(0)), "spec_accept")
    nid, nln = gi.cpu().numpy(), gl.cpu().numpy()
    ks = {0: 0, 1: 0, 2: 1, 4: S - 1}
    for i, k in ks.items():
        P = ln[i] - 1
        assert nln[i] == P + k + 2
        np.testing.assert_array_equal(nid[i, P + 1:P + 1 + k], c[i, 1:1 + k])
        assert nid[i, P + 1 + k] == am[i, k]
    assert nln[3] == ln[3] and np.array_equal(nid[3], ids[3])
    assert int(committed.item()) == sum(k + 1 for k in ks.values())
