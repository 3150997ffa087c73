"""A continuous-batching serve loop over the batched MoE step (the reference's
DSV2_SERVE request loop, bench/dsv2_decode_bench.c:2760-2900, which serves one
request at a time for tools/thvm_llm_service).

Each of the B rows is one request in its own cache slot at its own position
(DSModel.use_rows).  A step feeds every active row its next input (the next
prompt id while the prompt lasts, then its own last argmax) and
sm100_serve_advance does the per-row bookkeeping on the device, so the step
is one captured graph; requests join and leave between bursts of steps.

    srv = Server(cfg, weights, shard)
    rid = srv.submit(prompt_ids, max_new=64, eos=2)
    while srv.busy():
        srv.run(8)
        for rid, ids in srv.poll().items(): ...
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from .dsv2 import DSConfig, DSModel, DSShard


class Server:
    def __init__(self, cfg: DSConfig, weights: dict, shard: DSShard, group=None):
        import torch
        self.torch, self.cfg = torch, cfg
        self.model = DSModel(cfg, weights, shard, group)
        self.lib = self.model.lib
        dev = self.model.h.device
        B, ctx = cfg.batch, cfg.max_ctx
        z = lambda *s: torch.zeros(*s, dtype=torch.int32, device=dev)
        self.row_pos, self.row_seq = z(B), torch.arange(B, dtype=torch.int32, device=dev)
        self.prompt, self.out = z(B, ctx), z(B, ctx)
        self.plen, self.n_out, self.max_new, self.eos, self.active = z(B), z(B), z(B), z(B), z(B)
        self.model.use_rows(self.row_pos, self.row_seq, shared_slots=False)
        self.slot_of: dict[int, int] = {}   # request id -> row
        self.free = list(range(B))
        self.next_id = 0
        self.graph = None

    def _stream(self):
        return ctypes.c_void_p(self.torch.cuda.current_stream().cuda_stream)

    def submit(self, prompt, max_new: int, eos: int = -1) -> int:
        """Queues a request into a free row (raises when none is free);
        returns its id.  The row starts at position 0 with prompt[0]."""
        torch = self.torch
        prompt = np.asarray(prompt, np.int32)
        n = len(prompt)
        if not self.free:
            raise RuntimeError("no free row")
        if n < 1 or max_new < 1 or n + 1 >= self.cfg.max_ctx:
            raise ValueError(f"prompt of {n} ids, max_new {max_new} (cache of {self.cfg.max_ctx})")
        b = self.free.pop(0)
        dev = self.prompt.device
        self.prompt[b, :n] = torch.from_numpy(prompt).to(dev)
        for t, v in ((self.plen, n), (self.max_new, max_new), (self.eos, eos), (self.n_out, 0), (self.row_pos, 0),
                     (self.active, 1)):
            t[b] = v
        self.model.tok[b] = int(prompt[0])
        rid = self.next_id
        self.next_id += 1
        self.slot_of[rid] = b
        return rid

    def step(self):
        """One step of every row, then the rows' bookkeeping."""
        m, B = self.model, self.cfg.batch
        m.step()
        L.check(self.lib.sm100_serve_advance(self.row_pos.data_ptr(), m.tok.data_ptr(), m.tok.data_ptr(),
                                             self.prompt.data_ptr(), self.plen.data_ptr(), self.out.data_ptr(),
                                             self.n_out.data_ptr(), self.max_new.data_ptr(), self.eos.data_ptr(),
                                             self.active.data_ptr(), B, self.cfg.max_ctx, self._stream()),
                "serve_advance")
        m.launches += 1

    def capture(self):
        """One eager step with every row idle (sets the launches' attributes),
        then step() as a CUDA graph."""
        torch = self.torch
        if self.slot_of:
            raise RuntimeError("capture before the first submit")
        self.step()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step()

    def run(self, n: int = 1):
        for _ in range(n):
            if self.graph is not None:
                self.graph.replay()
            else:
                self.step()

    def busy(self) -> bool:
        return bool(self.slot_of)

    def poll(self) -> dict[int, np.ndarray]:
        """The requests that finished since the last poll: id -> generated ids
        (the eos id included when it stopped them); their rows are free."""
        active = self.active.cpu().numpy()
        done = {}
        for rid, b in list(self.slot_of.items()):
            if active[b] == 0:
                n = int(self.n_out[b].item())
                done[rid] = self.out[b, :n].cpu().numpy().copy()
                del self.slot_of[rid]
                self.free.append(b)
        return done

    def status(self) -> int:
        return self.model.status()
