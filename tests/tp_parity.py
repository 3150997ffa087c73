"""Multi-rank parity of the sharded decode steps against the CPU oracle, one
process per GPU (run by tests/test_gpu_multi.py under torch.distributed.run):

  ds   config 5 (thvm_b200.dsv2.DSModel): heads, dense units, experts and
       vocabulary split over the ranks, the library's peer all-reduces of the
       residual (fused with the RMSNorm);
  xl   config 3 (thvm_b200.gpt2_xl.XLModel): Megatron column / row splits;
  spec speculative decode (forced drafts) and the serve loop over the split
       config-5 model, against its base greedy stream.

Each rank holds its shard of one seeded model, both sides are fed the
oracle's ids (teacher forcing), and rank 0 checks the gathered logits (within
2e-2 of each row's largest), the ids (top-1 agreement >= 99 %) and its cache
rows against the oracle.  Exit status 0 when every check passes.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 tests/tp_parity.py ds
"""
import datetime
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def gathered_logits(model, dist, world):
    """The full [B, V] logits from every rank's vocabulary rows [v0, v1)."""
    import torch
    # vocabulary shards can differ by one row: pad to the largest
    n = torch.tensor([model.logits.shape[1]], device="cuda")
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n)
    vmax = int(max(int(s.item()) for s in sizes))
    pad = torch.zeros(model.logits.shape[0], vmax, device="cuda")
    pad[:, :model.logits.shape[1]] = model.logits
    outs = [torch.zeros_like(pad) for _ in range(world)]
    dist.all_gather(outs, pad)
    return np.concatenate([o[:, :int(s.item())].cpu().numpy() for o, s in zip(outs, sizes)], 1)


def run_ds(rank, world, dist):
    import torch
    import oracle as O
    from thvm_b200.dsv2 import DSConfig, DSModel, ds_shard, ds_weights, shard_ds_weights, yarn_tables
    cfg = DSConfig(n_layers=2, dim=512, heads=4, kv_lora=128, d_nope=32, d_rope=16, d_v=32, n_exp=8, top_k=3,
                   moe_inter=128, dense_inter=256, n_dense=1, n_shared=2, vocab=1000, max_ctx=64, batch=32)
    w = ds_weights(cfg, seed=0)
    sh = ds_shard(cfg, rank, world)
    dev = DSModel(cfg, shard_ds_weights(w, cfg, sh), sh, dist.group.WORLD)
    ref = None
    if rank == 0:
        cos, sin = yarn_tables(cfg.d_rope, cfg.max_ctx)
        ref = O.DSModel(cfg, w, cos, sin)
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, (cfg.batch, 6)).astype(np.int32)
    tok = prompt[:, 0]
    agree, total, worst = 0, 0, 0.0
    for pos in range(12):
        dev.tok.copy_(torch.from_numpy(tok))
        dev.step()
        torch.cuda.synchronize()
        lg_all = gathered_logits(dev, dist, world)
        got = dev.tok.cpu().numpy()
        nxt = np.zeros(cfg.batch, np.int32)
        if rank == 0:
            lg, nxt = ref.step(tok, pos)
            worst = max(worst, float((np.abs(lg_all - lg).max(1) / np.abs(lg).max(1)).max()))
            agree += int((got == nxt).sum())
            total += cfg.batch
        t = torch.from_numpy(nxt).cuda()
        dist.broadcast(t, 0)
        nxt = t.cpu().numpy()
        tok = prompt[:, pos + 1] if pos + 1 < prompt.shape[1] else nxt
    status = dev.status()
    if rank == 0:
        print(f"ds world {world}: worst logit error {worst:.3e}, top-1 agreement {agree}/{total}, status {status}")
        assert worst <= 2e-2, worst
        assert agree / total >= 0.99, agree / total
        f32 = lambda b: (b.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        a = f32(dev.cache_c[0].cpu().numpy().view(np.uint16)[:, :12])
        r = f32(ref.cache_c[0][:, :12])
        excess = np.abs(a - r) - (2.0 ** -6 * np.abs(r) + 2.0 ** -6 * np.sqrt(np.mean(r * r)))
        assert excess.max() <= 0, excess.max()
    assert status == 0, status


def run_spec(rank, world, dist):
    """Speculative decode and the serve loop with the model split over the
    ranks: the committed streams (forced drafts: S per step) and a served
    request's ids equal the base greedy stream of the same split model."""
    import torch
    from thvm_b200.dsv2 import DSConfig, DSModel, ds_shard, ds_weights, shard_ds_weights
    from thvm_b200.serve import Server
    from thvm_b200.spec import SpecDecoder
    kw = dict(n_layers=2, dim=512, heads=4, kv_lora=128, d_nope=32, d_rope=16, d_v=32, n_exp=8, top_k=3,
              moe_inter=128, dense_inter=256, n_dense=1, n_shared=2, vocab=1000, max_ctx=64)
    n_seq, S, n_p, n_new = 4, 4, 6, 16
    base_cfg = DSConfig(**kw, batch=n_seq)
    w = ds_weights(base_cfg, seed=0)
    sh = ds_shard(base_cfg, rank, world)
    prompts = np.random.default_rng(5).integers(0, base_cfg.vocab, (n_seq, n_p)).astype(np.int32)
    m = DSModel(base_cfg, shard_ds_weights(w, base_cfg, sh), sh, dist.group.WORLD)
    base = np.zeros((n_seq, n_p + n_new), np.int32)
    base[:, :n_p] = prompts
    for pos in range(n_p + n_new - 1):
        if pos < n_p:
            m.tok.copy_(torch.from_numpy(prompts[:, pos]))
        m.step()
        if pos + 1 >= n_p:
            base[:, pos + 1] = m.tok.cpu().numpy()
    torch.cuda.synchronize()
    scfg = DSConfig(**kw, batch=n_seq * S)
    sd = SpecDecoder(scfg, shard_ds_weights(w, scfg, sh), sh, n_seq, S, group=dist.group.WORLD, forced=True)
    sd.prefill(prompts, seed_ids=base)
    sd.capture()
    want = n_p
    while want < n_p + n_new:
        sd.replay()
        want += S
        ids, ln = sd.stream_ids()
        assert np.all(ln == want), (ln, want)
    assert np.array_equal(ids[:, :n_p + n_new], base)
    # one request of the serve loop on a 2-row server
    vcfg = DSConfig(**kw, batch=2)
    srv = Server(vcfg, shard_ds_weights(w, vcfg, sh), sh, dist.group.WORLD)
    srv.capture()
    rid = srv.submit(prompts[1], n_new)
    got = {}
    for _ in range(64):
        srv.run(2)
        got.update(srv.poll())
        if not srv.busy():
            break
    assert np.array_equal(got[rid], base[1, n_p:]), (got.get(rid), base[1, n_p:])
    status = sd.status() | srv.status() | m.status()
    assert status == 0, status
    if rank == 0:
        print(f"spec world {world}: forced drafts committed {S} a step, the base stream; served request matches")


def run_xl(rank, world, dist):
    import torch
    import oracle as O
    from thvm_b200.gpt2_xl import XLConfig, XLModel, shard_of, shard_weights, xl_weights
    cfg = XLConfig(n_layers=2, dim=256, heads=4, vocab=1000, max_ctx=64, batch=16)
    w = xl_weights(cfg, seed=0)
    sh = shard_of(cfg, rank, world)
    dev = XLModel(cfg, shard_weights(w, cfg, sh), sh, dist.group.WORLD)
    ref = O.XLModel(cfg, w) if rank == 0 else None
    prompt = np.random.default_rng(1).integers(0, cfg.vocab, (cfg.batch, 8)).astype(np.int32)
    tok = prompt[:, 0]
    agree, total, worst = 0, 0, 0.0
    for pos in range(16):
        dev.tok.copy_(torch.from_numpy(tok))
        dev.step()
        torch.cuda.synchronize()
        lg_all = gathered_logits(dev, dist, world)
        got = dev.tok.cpu().numpy()
        nxt = np.zeros(cfg.batch, np.int32)
        if rank == 0:
            lg, nxt = ref.step(tok, pos)
            worst = max(worst, float((np.abs(lg_all - lg).max(1) / np.abs(lg).max(1)).max()))
            agree += int((got == nxt).sum())
            total += cfg.batch
        t = torch.from_numpy(nxt).cuda()
        dist.broadcast(t, 0)
        nxt = t.cpu().numpy()
        tok = prompt[:, pos + 1] if pos + 1 < prompt.shape[1] else nxt
    if rank == 0:
        print(f"xl world {world}: worst logit error {worst:.3e}, top-1 agreement {agree}/{total}")
        assert worst <= 2e-2, worst
        assert agree / total >= 0.99, agree / total
    # the prompt pass over the split model (row-split partial sums summed by an
    # NCCL all-reduce per block), then decode steps after it
    P = prompt.shape[1]
    dev2 = XLModel(cfg, shard_weights(w, cfg, sh), sh, dist.group.WORLD)
    ref2 = O.XLModel(cfg, w) if rank == 0 else None
    nxt = np.zeros(cfg.batch, np.int32)
    if rank == 0:
        for pos in range(P):
            lg, nxt = ref2.step(prompt[:, pos], pos)
    dev2.prefill(prompt)
    torch.cuda.synchronize()
    agree, total, worst = 0, 0, 0.0
    for step in range(7):
        if step:
            dev2.tok.copy_(torch.from_numpy(tok))
            dev2.step()
            torch.cuda.synchronize()
            if rank == 0:
                lg, nxt = ref2.step(tok, P + step - 1)
        lg_all = gathered_logits(dev2, dist, world)
        if rank == 0:
            worst = max(worst, float((np.abs(lg_all - lg).max(1) / np.abs(lg).max(1)).max()))
            agree += int((dev2.tok.cpu().numpy() == nxt).sum())
            total += cfg.batch
        t = torch.from_numpy(np.ascontiguousarray(nxt, np.int32)).cuda()
        dist.broadcast(t, 0)
        tok = t.cpu().numpy()
    if rank == 0:
        print(f"xl prefill world {world}: worst logit error {worst:.3e}, top-1 agreement {agree}/{total}")
        assert worst <= 2e-2, worst
        assert agree / total >= 0.99, agree / total
    dev.close()
    dev2.close()


def run_comm(rank, world, dist):
    """The peer collectives alone: the fused all-reduce + RMSNorm sums the
    ranks' rows in rank order (bit for bit what an f32 sum in that order
    gives), over several uses; the argmax pick takes the largest value, the
    smaller index on ties across ranks; the LayerNorm variant sums alike."""
    import torch
    from thvm_b200.comm import PeerComm
    B, D = 32, 2048
    comm = PeerComm(rank, world, D, dist.group.WORLD)
    g = torch.from_numpy(np.random.default_rng(9).uniform(0.5, 1.5, D).astype(np.float32)).cuda()
    y = torch.zeros(B, D, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for use in range(5):
        parts = [np.random.default_rng(100 * use + r).standard_normal((B, D)).astype(np.float32) for r in range(world)]
        h = torch.from_numpy(parts[rank].copy()).cuda()
        comm.allreduce_rmsnorm(h.data_ptr(), g.data_ptr(), y.data_ptr(), B, D, 1e-6, st)
        torch.cuda.synchronize()
        want = parts[0].copy()
        for r in range(1, world):
            want = want + parts[r]
        assert np.array_equal(h.cpu().numpy(), want), use
        # zero_rest: the same y, and zeros in h on the ranks other than 0
        y0 = y.clone()
        h = torch.from_numpy(parts[rank].copy()).cuda()
        comm.allreduce_rmsnorm(h.data_ptr(), g.data_ptr(), y.data_ptr(), B, D, 1e-6, st, zero_rest=True)
        torch.cuda.synchronize()
        assert torch.equal(y, y0)
        assert np.array_equal(h.cpu().numpy(), want if rank == 0 else np.zeros_like(want)), use
    val = torch.full((B,), float(rank % 2), device="cuda")            # ranks 1, 3, .. hold the maximum
    idx = torch.arange(B, dtype=torch.int32, device="cuda") + 1000 * (world - rank)   # the last of them the smallest index
    tok = torch.zeros(B, dtype=torch.int32, device="cuda")
    comm.pick(val.data_ptr(), idx.data_ptr(), B, tok.data_ptr(), st)
    torch.cuda.synchronize()
    best = max(r for r in range(world) if r % 2 == 1) if world > 1 else 0
    assert np.array_equal(tok.cpu().numpy(), np.arange(B) + 1000 * (world - best))
    # the LayerNorm variant: the same sum, y within a bf16 rounding of the f64 LayerNorm
    b = torch.from_numpy(np.random.default_rng(10).uniform(-0.5, 0.5, D).astype(np.float32)).cuda()
    parts = [np.random.default_rng(700 + r).standard_normal((B, D)).astype(np.float32) for r in range(world)]
    h = torch.from_numpy(parts[rank].copy()).cuda()
    comm.allreduce_layernorm(h.data_ptr(), g.data_ptr(), b.data_ptr(), y.data_ptr(), B, D, 1e-5, st)
    torch.cuda.synchronize()
    want = parts[0].copy()
    for r in range(1, world):
        want = want + parts[r]
    assert np.array_equal(h.cpu().numpy(), want)
    w64 = want.astype(np.float64)
    mu = w64.mean(1, keepdims=True)
    ref = (w64 - mu) / np.sqrt(((w64 - mu) ** 2).mean(1, keepdims=True) + 1e-5) * g.cpu().numpy() + b.cpu().numpy()
    np.testing.assert_allclose(y.float().cpu().numpy(), ref, rtol=2 ** -7, atol=2 ** -7)
    assert comm.status() == 0
    comm.close()
    if rank == 0:
        print(f"comm world {world}: five all-reduces bit-exact, pick ok")


def main():
    import torch
    import torch.distributed as dist
    which = sys.argv[1]
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    os.environ["THVM_SM100_DEVICE"] = str(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    try:
        {"ds": run_ds, "xl": run_xl, "comm": run_comm, "spec": run_spec}[which](rank, world, dist)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
