"""Blind speculative decode of the batched MoE step (the reference's DSV2_SPEC
path, bench/dsv2_decode_bench.c:1110-1195 and :2416-2510, there at batch 1):
n_seq sequences of S rows each.  Every step drafts S - 1 tokens per sequence
from the most recent earlier occurrence of its last bigram (or, forced, from
ids already seeded), verifies the pending token and the drafts in one forward
pass of n_seq * S rows (DSModel with shared cache slots: row i S + s at slot
i, position P + s), and commits the longest verified prefix plus the bonus
token (sm100_spec_draft / sm100_spec_accept).  Rows run the base step's
kernels, so the committed stream is the base greedy stream; the drafts only
decide how many positions a step commits.

The whole step is device-resident (no host round trip), so it is captured
once and replayed; the host reads the lengths and the committed-token counter
between bursts.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from .dsv2 import DSConfig, DSModel, DSShard


class SpecDecoder:
    def __init__(self, cfg: DSConfig, weights: dict, shard: DSShard, n_seq: int, S: int, group=None,
                 forced: bool = False):
        import torch
        if S < 1 or cfg.batch != n_seq * S:
            raise ValueError(f"batch {cfg.batch} must be n_seq {n_seq} x S {S}")
        self.torch, self.cfg, self.n_seq, self.S, self.forced = torch, cfg, n_seq, S, forced
        self.model = DSModel(cfg, weights, shard, group, n_slots=n_seq)
        self.lib = self.model.lib
        dev = self.model.h.device
        z = lambda *s: torch.zeros(*s, dtype=torch.int32, device=dev)
        self.ids, self.len = z(n_seq, cfg.max_ctx), z(n_seq)
        self.cand, self.row_pos, self.row_seq = z(cfg.batch), z(cfg.batch), z(cfg.batch)
        self.committed = torch.zeros(1, dtype=torch.int64, device=dev)
        self.model.use_rows(self.row_pos, self.row_seq, shared_slots=True)
        self.graph = None

    def _stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)

    def prefill(self, prompts: np.ndarray, seed_ids: np.ndarray | None = None):
        """Writes the cache rows of prompts [n_seq, n] (positions 0 .. n - 2;
        token n - 1 is left pending: len = n), S positions per forward pass.
        seed_ids [n_seq, m >= n] (forced drafts): the stream to seed, whose
        first n ids are the prompt."""
        torch = self.torch
        n = prompts.shape[1]
        if n < 2 or n + self.S >= self.cfg.max_ctx:
            raise ValueError(f"prompt of {n} ids (>= 2, < max_ctx - S)")
        seed = prompts if seed_ids is None else seed_ids
        if not np.array_equal(seed[:, :n], prompts):
            raise ValueError("seed_ids must start with the prompts")
        self.ids.zero_()
        self.ids[:, :seed.shape[1]] = torch.from_numpy(np.ascontiguousarray(seed, np.int32)).to(self.ids.device)
        slots = torch.arange(self.n_seq, dtype=torch.int32, device=self.ids.device).repeat_interleave(self.S)
        self.row_seq.copy_(slots)
        for p0 in range(0, n - 1, self.S):
            # row i S + s: position min(p0 + s, n - 2) of sequence i (repeats write the same row)
            pos = torch.clamp(torch.arange(self.S, dtype=torch.int32, device=self.ids.device) + p0, max=n - 2)
            self.row_pos.copy_(pos.repeat(self.n_seq))
            self.model.tok.copy_(self.ids[slots.long(), self.row_pos.long()])
            self.model.step()
        self.len.fill_(n)
        self.committed.zero_()

    def step(self):
        """One speculative step: draft, verify (n_seq * S rows), accept."""
        lib, st, c, m = self.lib, self._stream, self.cfg, self.model
        L.check(lib.sm100_spec_draft(self.ids.data_ptr(), self.len.data_ptr(), self.n_seq, c.max_ctx, self.S,
                                     int(self.forced), m.tok.data_ptr(), self.cand.data_ptr(), self.row_pos.data_ptr(),
                                     self.row_seq.data_ptr(), st()), "spec_draft")
        m.step()
        L.check(lib.sm100_spec_accept(self.ids.data_ptr(), self.len.data_ptr(), self.n_seq, c.max_ctx, self.S,
                                      self.cand.data_ptr(), m.tok.data_ptr(), self.committed.data_ptr(), st()),
                "spec_accept")
        m.launches += 2

    def capture(self):
        """Captures step() into a CUDA graph (after prefill, whose eager steps
        set up the model launches' attributes); replay() runs it."""
        torch = self.torch
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()

    def replay(self, n: int = 1):
        for _ in range(n):
            self.graph.replay()

    def status(self) -> int:
        return self.model.status() | (int(self.lib.sm100_spec_status()) << 16)

    def stream_ids(self) -> tuple[np.ndarray, np.ndarray]:
        """(ids [n_seq, max_ctx], len [n_seq]) on the host."""
        return self.ids.cpu().numpy(), self.len.cpu().numpy()
