"""Host logic of the sharded MoE decode (thvm_b200.dsv2) on
the CPU: every head, dense unit, expert, shared half and vocabulary row
belongs to exactly one rank; the shards' slices rebuild the full weights;
the row-split products (W_o by heads, the dense down projection by units)
summed over the ranks equal the full products, also when the sum is a
torch.distributed all-reduce over two gloo ranks as the GPU ranks run it
over NCCL."""
import os

import numpy as np
import pytest

from thvm_b200.dsv2 import DSConfig, ds_shard, ds_weights, shard_ds_weights

CFG = DSConfig(n_layers=2, dim=256, heads=4, kv_lora=128, d_nope=32, d_rope=16, d_v=32, n_exp=8, top_k=3,
               moe_inter=128, dense_inter=384, n_dense=1, n_shared=2, vocab=1001, max_ctx=16, batch=4)


def f64(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_every_unit_on_one_rank(world):
    shards = [ds_shard(CFG, r, world) for r in range(world)]
    for lo, hi, n in (("h0", "h1", CFG.heads), ("f0", "f1", CFG.dense_inter), ("e0", "e1", CFG.n_exp),
                      ("v0", "v1", CFG.vocab)):
        spans = [(getattr(s, lo), getattr(s, hi)) for s in shards]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert sorted(k for s in shards for k in s.shared) == list(range(CFG.n_shared))


def test_shard_rejects_more_ranks_than_heads():
    with pytest.raises(ValueError):
        ds_shard(CFG, 0, 8)


@pytest.mark.parametrize("world", [2, 4])
def test_shards_rebuild_the_weights(world):
    w = ds_weights(CFG, seed=3)
    s = [shard_ds_weights(w, CFG, ds_shard(CFG, r, world)) for r in range(world)]
    QS, NQ, DI = CFG.d_nope + CFG.d_rope, CFG.q_cols, CFG.dense_inter
    for l in range(CFG.n_layers):
        p = f"l{l}."
        nq = [ds_shard(CFG, r, world).heads * QS for r in range(world)]
        assert np.array_equal(np.concatenate([x[p + "w_qkva"][:n] for x, n in zip(s, nq)]), w[p + "w_qkva"][:NQ])
        for x, n in zip(s, nq):   # the latent block is on every rank
            assert np.array_equal(x[p + "w_qkva"][n:], w[p + "w_qkva"][NQ:])
        for k in ("w_uk", "w_uv"):
            assert np.array_equal(np.concatenate([x[p + k] for x in s]), w[p + k])
        assert np.array_equal(np.concatenate([x[p + "w_o"] for x in s], 1), w[p + "w_o"])
        if l < CFG.n_dense:
            g = [x[p + "d_gu"] for x in s]
            half = [a.shape[0] // 2 for a in g]
            assert np.array_equal(np.concatenate([a[:h] for a, h in zip(g, half)]), w[p + "d_gu"][:DI])
            assert np.array_equal(np.concatenate([a[h:] for a, h in zip(g, half)]), w[p + "d_gu"][DI:])
            assert np.array_equal(np.concatenate([x[p + "d_down"] for x in s], 1), w[p + "d_down"])
        else:
            for k in ("e_gu", "e_d", "e_gu_s", "e_d_s"):
                rows = {}
                for r, x in enumerate(s):
                    sh = ds_shard(CFG, r, world)
                    ids = list(range(sh.e0, sh.e1)) + [CFG.n_exp + q for q in sh.shared]
                    rows.update({e: x[p + k][i] for i, e in enumerate(ids)})
                assert sorted(rows) == list(range(CFG.n_exp + CFG.n_shared))
                for e, a in rows.items():
                    assert np.array_equal(a, w[p + k][e])
    assert np.array_equal(np.concatenate([x["lm_head"] for x in s]), w["lm_head"])


def _partials(w, rank, world, o, a):
    """Rank `rank`'s row-split partial sums of the o projection and the dense down projection."""
    sh = ds_shard(CFG, rank, world)
    x = shard_ds_weights(w, CFG, sh)
    DV = CFG.d_v
    po = o[:, sh.h0 * DV:sh.h1 * DV] @ f64(x["l0.w_o"]).T
    pd = a[:, sh.f0:sh.f1] @ f64(x["l0.d_down"]).T
    return po, pd


def test_row_split_partials_sum_to_the_full_products():
    w = ds_weights(CFG, seed=4)
    rng = np.random.default_rng(0)
    o = rng.standard_normal((CFG.batch, CFG.heads * CFG.d_v))
    a = rng.standard_normal((CFG.batch, CFG.dense_inter))
    for world in (2, 4):
        parts = [_partials(w, r, world, o, a) for r in range(world)]
        np.testing.assert_allclose(sum(p[0] for p in parts), o @ f64(w["l0.w_o"]).T, rtol=1e-12, atol=1e-12)
        np.testing.assert_allclose(sum(p[1] for p in parts), a @ f64(w["l0.d_down"]).T, rtol=1e-12, atol=1e-12)


def _gloo_rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = ds_weights(CFG, seed=4)
        rng = np.random.default_rng(0)
        o = rng.standard_normal((CFG.batch, CFG.heads * CFG.d_v))
        a = rng.standard_normal((CFG.batch, CFG.dense_inter))
        po, pd = _partials(w, rank, world, o, a)
        h = torch.from_numpy(po + pd)
        dist.all_reduce(h)
        if rank == 0:
            q.put(h.numpy())
    finally:
        dist.destroy_process_group()


def test_all_reduce_of_partials_over_gloo():
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 200
    ps = [ctx.Process(target=_gloo_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    w = ds_weights(CFG, seed=4)
    rng = np.random.default_rng(0)
    o = rng.standard_normal((CFG.batch, CFG.heads * CFG.d_v))
    a = rng.standard_normal((CFG.batch, CFG.dense_inter))
    np.testing.assert_allclose(got, o @ f64(w["l0.w_o"]).T + a @ f64(w["l0.d_down"]).T, rtol=1e-12, atol=1e-12)
