"""Host logic of the tensor-parallel GPT-2-XL decode (thvm_b200.gpt2_xl) on the
CPU: the head / hidden / vocabulary split, that the shards' products
recombine into the full ones (Megatron column / row splits, rank 0 carrying
bias and residual), the (max, index) pick over vocabulary shards, and the
same recombination through torch.distributed (gloo, world size 2) as the
GPU ranks run it through NCCL."""
import numpy as np
import pytest

from thvm_b200.gpt2_xl import HEAD_DIM, XLConfig, shard_of, shard_weights, split_even, xl_weights

CFG = XLConfig(n_layers=1, dim=320, heads=5, vocab=1001, max_ctx=16, batch=4)


def f32(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


@pytest.mark.parametrize("n,parts", [(25, 1), (25, 2), (25, 4), (25, 8), (50257, 8), (6400, 8), (7, 7)])
def test_split_even(n, parts):
    rs = [split_even(n, parts, r) for r in range(parts)]
    assert rs[0][0] == 0 and rs[-1][1] == n
    assert all(rs[i][1] == rs[i + 1][0] for i in range(parts - 1))
    sizes = [hi - lo for lo, hi in rs]
    assert max(sizes) - min(sizes) <= 1


def test_shard_rejects_more_ranks_than_heads():
    with pytest.raises(ValueError):
        shard_of(CFG, 0, 6)


def tp_layer(w, cfg, world, x_attn_in, x_mlp_in, h):
    """The row-split projections as the ranks compute them: partials summed
    (the all-reduce), rank 0 adding bias and residual."""
    out_proj, out_p2 = np.zeros_like(h), np.zeros_like(h)
    qkv_cols = []
    for r in range(world):
        sh = shard_of(cfg, r, world)
        s = shard_weights(w, cfg, sh)
        c = slice(sh.h0 * HEAD_DIM, sh.h1 * HEAD_DIM)
        qkv_cols.append(x_attn_in @ f32(s["h.0.attn.w"]).T + s["h.0.attn.b"])
        part = x_attn_in[:, c] @ f32(s["h.0.proj.w"]).T
        out_proj += part + ((s["h.0.proj.b"] + h) if r == 0 else 0)
        f = slice(sh.f0, sh.f1)
        part = x_mlp_in[:, f] @ f32(s["h.0.p2.w"]).T
        out_p2 += part + ((s["h.0.p2.b"] + h) if r == 0 else 0)
    return qkv_cols, out_proj, out_p2


@pytest.mark.parametrize("world", [1, 2, 3, 5])
def test_shards_recombine(world):
    w = xl_weights(CFG, seed=3)
    rng = np.random.default_rng(0)
    B, D, F = CFG.batch, CFG.dim, CFG.hidden
    xa, xm, h = rng.standard_normal((B, D)), rng.standard_normal((B, F)), rng.standard_normal((B, D))
    qkv_cols, out_proj, out_p2 = tp_layer(w, CFG, world, xa, xm, h)
    full_qkv = xa @ f32(w["h.0.attn.w"]).T + w["h.0.attn.b"]
    for r, part in enumerate(qkv_cols):   # [q_r | k_r | v_r] are rank r's heads of q, k and v
        sh = shard_of(CFG, r, world)
        c = slice(sh.h0 * HEAD_DIM, sh.h1 * HEAD_DIM)
        C = sh.cols
        np.testing.assert_allclose(part[:, :C], full_qkv[:, c], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(part[:, C:2 * C], full_qkv[:, D:][:, c], rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(part[:, 2 * C:], full_qkv[:, 2 * D:][:, c], rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(out_proj, xa @ f32(w["h.0.proj.w"]).T + w["h.0.proj.b"] + h, rtol=1e-9, atol=1e-9)
    np.testing.assert_allclose(out_p2, xm @ f32(w["h.0.p2.w"]).T + w["h.0.p2.b"] + h, rtol=1e-9, atol=1e-9)


def pick(vals, idxs):
    """The device's xl_pick rule: the largest candidate, ties to the smaller index."""
    out = []
    for b in range(vals.shape[1]):
        best = 0
        for r in range(1, vals.shape[0]):
            if vals[r, b] > vals[best, b] or (vals[r, b] == vals[best, b] and idxs[r, b] < idxs[best, b]):
                best = r
        out.append(idxs[best, b])
    return np.array(out)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_vocab_split_argmax(world):
    rng = np.random.default_rng(world)
    V, B = 1001, 6
    logits = rng.standard_normal((B, V)).astype(np.float32)
    logits[0, 700] = logits[0, 10] = logits[0].max() + 1   # a tie across shards: the smaller index wins
    vals, idxs = np.zeros((world, B), np.float32), np.zeros((world, B), np.int64)
    for r in range(world):
        v0, v1 = split_even(V, world, r)
        part = logits[:, v0:v1]
        idxs[r] = part.argmax(1) + v0     # numpy argmax: first index of the maximum
        vals[r] = part.max(1)
    np.testing.assert_array_equal(pick(vals, idxs), logits.argmax(1))


_RANK_CODE = r"""
import os, sys
import numpy as np
import torch
import torch.distributed as dist
from thvm_b200.gpt2_xl import HEAD_DIM, XLConfig, shard_of, shard_weights, xl_weights
rank, world = int(sys.argv[1]), int(sys.argv[2])
dist.init_process_group("gloo", rank=rank, world_size=world)
CFG = XLConfig(n_layers=1, dim=320, heads=5, vocab=1001, max_ctx=16, batch=4)
f32 = lambda bits: (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
w = xl_weights(CFG, seed=3)
sh = shard_of(CFG, rank, world)
s = shard_weights(w, CFG, sh)
rng = np.random.default_rng(0)
B, D = CFG.batch, CFG.dim
xa, h = rng.standard_normal((B, D)), rng.standard_normal((B, D))
c = slice(sh.h0 * HEAD_DIM, sh.h1 * HEAD_DIM)
part = xa[:, c] @ f32(s["h.0.proj.w"]).T
if rank == 0:
    part = part + s["h.0.proj.b"] + h
t = torch.from_numpy(part)
dist.all_reduce(t)
ok = np.allclose(t.numpy(), xa @ f32(w["h.0.proj.w"]).T + w["h.0.proj.b"] + h, rtol=1e-9, atol=1e-9)
logits = rng.standard_normal((B, CFG.vocab)).astype(np.float32)
me_v = torch.from_numpy(logits[:, sh.v0:sh.v1].max(1).copy())
me_i = torch.from_numpy((logits[:, sh.v0:sh.v1].argmax(1) + sh.v0).astype(np.int64))
all_v, all_i = torch.zeros(world, B), torch.zeros(world, B, dtype=torch.int64)
dist.all_gather_into_tensor(all_v.view(-1), me_v)
dist.all_gather_into_tensor(all_i.view(-1), me_i)
av, ai = all_v.numpy(), all_i.numpy()
picked = []
for b in range(B):
    best = 0
    for r in range(1, world):
        if av[r, b] > av[best, b] or (av[r, b] == av[best, b] and ai[r, b] < ai[best, b]):
            best = r
    picked.append(ai[best, b])
ok = ok and np.array_equal(np.array(picked), logits.argmax(1))
dist.destroy_process_group()
sys.exit(0 if ok else 3)
"""


def test_tp_collectives_gloo():
    """Two CPU ranks run the row-split all-reduce and the shard pick through gloo."""
    import os
    import socket
    import subprocess
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), PYTHONPATH=str(root))
    procs = [subprocess.Popen([sys.executable, "-c", _RANK_CODE, str(r), "2"], cwd=root, env=env)
             for r in range(2)]
    codes = []
    for p in procs:
        try:
            codes.append(p.wait(timeout=180))
        except subprocess.TimeoutExpired:
            p.kill()
            codes.append(None)
    assert codes == [0, 0]
