"""GPT-2 decoding on the sm_100a device: the kernel schedule that thvm's
tensor track realizes for `bench/gpt2/thvm_gpt2.py` (tinygrad's gpt2.py),
expressed as Sm100Kernel dispatches and replayed as CUDA graphs.

Classes keep the reference model's names and call order (Attention,
FeedForward, TransformerBlock, Transformer: thvm_gpt2.py:27-128).  Each
__call__ appends the kernels the reference's schedule produces for that
module once the recognised shapes are routed to the device (the LayerNorm
folded into the following projection's prologue, bias / GELU / residual into
its epilogue, the KV-cache assign into the qkv projection's epilogue at the
device-resident position), so a decode step is:

  embedding(wte[tok] + wpe[pos])
  per block: ln_1+c_attn(+kv append) -> attention -> c_proj(+residual)
             -> ln_2+c_fc+gelu -> mlp.c_proj(+residual)
  ln_f+lm_head (last row) -> argmax (-> tok, pos += 1)

`start_pos` and the token live in device buffers, so one captured graph
serves every position (the TinyJit replay the reference runs, with its
Variable bound at run time instead of baked into the kernels).
"""
from __future__ import annotations

from dataclasses import dataclass

import ctypes

import numpy as np

from . import _lib as L
from ._lib import Sm100Kernel
from .device import Device
from .synthetic import GPT2Config

SLOT_X, SLOT_W, SLOT_B, SLOT_LNG, SLOT_LNB, SLOT_RES, SLOT_SCALE, SLOT_POS, SLOT_CACHE = range(9)


@dataclass
class Op:
    kernel: Sm100Kernel
    in_ids: list
    out_id: int


def make_op(kind: int, out_id: int, slots: dict, **fields) -> Op:
    """A descriptor whose slot s reads buffer slots[s] (in_buf_ids built here)."""
    ids, idx = [], {}
    for s, bid in slots.items():
        if bid is None:
            continue
        if bid not in idx:
            idx[bid] = len(ids)
            ids.append(bid)
        slots[s] = idx[bid]
    k = Sm100Kernel.make(kind, {s: v for s, v in slots.items() if v is not None}, **fields)
    return Op(k, ids, out_id)


class Linear:
    """nn.Linear (py/thvm/nn.py:12-25): y = x @ W^T + b with W (out, in)."""

    def __init__(self, dev: Device, w: np.ndarray, b: np.ndarray | None):
        self.out_f, self.in_f = w.shape
        self.w = dev.upload(w.astype(np.float32))
        self.b = dev.upload(b.astype(np.float32)) if b is not None else None


class LayerNorm:
    def __init__(self, dev: Device, g: np.ndarray, b: np.ndarray, eps: float):
        self.g, self.b, self.eps = dev.upload(g), dev.upload(b), eps


class Attention:
    def __init__(self, dev, cfg: GPT2Config, W: dict, p: str):
        self.c_attn = Linear(dev, W[p + "attn.c_attn.weight"], W[p + "attn.c_attn.bias"])
        self.c_proj = Linear(dev, W[p + "attn.c_proj.weight"], W[p + "attn.c_proj.bias"])
        self.n_heads, self.dim, self.head_dim = cfg.n_heads, cfg.dim, cfg.head_dim
        # cache_kv [2, max_ctx, H, hd] (thvm_gpt2.py:45-47, batch 1)
        self.cache_kv = dev.alloc(2 * cfg.max_ctx * cfg.dim * 4)
        self.max_ctx = cfg.max_ctx

    def __call__(self, ops, s, ln: LayerNorm, T: int):
        d = self.dim
        ops.append(make_op(L.K_LINEAR, s.qkv, {SLOT_X: s.x, SLOT_W: self.c_attn.w, SLOT_B: self.c_attn.b,
                                                SLOT_LNG: ln.g, SLOT_LNB: ln.b, SLOT_POS: s.pos,
                                                SLOT_CACHE: self.cache_kv},
                           flags=L.LIN_LN | L.LIN_KV_APPEND, m=T, n=3 * d, k=d, eps=ln.eps,
                           max_ctx=self.max_ctx))
        ops.append(make_op(L.K_ATTENTION, s.att, {0: s.qkv, 1: self.cache_kv, SLOT_POS: s.pos},
                           m=T, heads=self.n_heads, head_dim=self.head_dim, max_ctx=self.max_ctx,
                           ld_in=3 * d, scale=float(1.0 / np.sqrt(self.head_dim))))
        ops.append(make_op(L.K_LINEAR, s.x, {SLOT_X: s.att, SLOT_W: self.c_proj.w, SLOT_B: self.c_proj.b,
                                              SLOT_RES: s.x},
                           flags=L.LIN_RESIDUAL, m=T, n=d, k=d))


class FeedForward:
    def __init__(self, dev, cfg: GPT2Config, W: dict, p: str):
        self.c_fc = Linear(dev, W[p + "mlp.c_fc.weight"], W[p + "mlp.c_fc.bias"])
        self.c_proj = Linear(dev, W[p + "mlp.c_proj.weight"], W[p + "mlp.c_proj.bias"])

    def __call__(self, ops, s, ln: LayerNorm, T: int):
        d, h = self.c_fc.in_f, self.c_fc.out_f
        ops.append(make_op(L.K_LINEAR, s.fc, {SLOT_X: s.x, SLOT_W: self.c_fc.w, SLOT_B: self.c_fc.b,
                                               SLOT_LNG: ln.g, SLOT_LNB: ln.b},
                           flags=L.LIN_LN | L.LIN_GELU, m=T, n=h, k=d, eps=ln.eps))
        ops.append(make_op(L.K_LINEAR, s.x, {SLOT_X: s.fc, SLOT_W: self.c_proj.w, SLOT_B: self.c_proj.b,
                                              SLOT_RES: s.x},
                           flags=L.LIN_RESIDUAL, m=T, n=d, k=h))


class TransformerBlock:
    def __init__(self, dev, cfg: GPT2Config, W: dict, i: int):
        p = f"h.{i}."
        self.attn = Attention(dev, cfg, W, p)
        self.mlp = FeedForward(dev, cfg, W, p)
        self.ln_1 = LayerNorm(dev, W[p + "ln_1.weight"], W[p + "ln_1.bias"], cfg.norm_eps)
        self.ln_2 = LayerNorm(dev, W[p + "ln_2.weight"], W[p + "ln_2.bias"], cfg.norm_eps)

    def __call__(self, ops, s, T: int):
        # h = x + attn(ln_1(x)); h + mlp(ln_2(h))  (thvm_gpt2.py:77-79)
        self.attn(ops, s, self.ln_1, T)
        self.mlp(ops, s, self.ln_2, T)


class _State:
    """Device buffers of one decode stream (batch 1)."""

    def __init__(self, dev: Device, cfg: GPT2Config, max_tokens: int):
        d = cfg.dim
        self.max_tokens = max_tokens
        # io = [pos, tok[0..max_tokens)]: one 8-byte host write sets a step's
        # (start_pos, token) inputs.
        self.io = dev.alloc(4 + 4 * max_tokens)
        self.pos = dev.lib.sm100_buf_view(self.io, 0, 4)
        self.tok = dev.lib.sm100_buf_view(self.io, 4, 4 * max_tokens)
        self.x = dev.alloc(4 * max_tokens * d)
        self.qkv = dev.alloc(4 * max_tokens * 3 * d)
        self.att = dev.alloc(4 * max_tokens * d)
        self.fc = dev.alloc(4 * max_tokens * 4 * d)
        self.logits = dev.alloc(4 * cfg.vocab)
        self.start = dev.alloc(8)  # (token, position) a replayed generation restarts from


class Transformer:
    """GPT-2 decoder (thvm_gpt2.py:81-128) on the sm_100a device."""


    def __init__(self, cfg: GPT2Config, weights: dict, device: Device | None = None, max_prompt: int = 128,
                 fused: bool = True):
        self.cfg = cfg
        dev = self.dev = device or Device.get()
        self.wte = dev.upload(weights["wte.weight"])
        self.wpe = dev.upload(weights["wpe.weight"])
        self.h = [TransformerBlock(dev, cfg, weights, i) for i in range(cfg.n_layers)]
        self.ln_f = LayerNorm(dev, weights["ln_f.weight"], weights["ln_f.bias"], cfg.norm_eps)
        self.lm_head = Linear(dev, weights["lm_head.weight"], None)
        self.s = _State(dev, cfg, max_prompt)
        self._run_tokens = 0
        # graph slots of this model: one decode step; one whole generation
        self.GRAPH_STEP = dev.new_graph_slot()
        self.GRAPH_RUN = dev.new_graph_slot()
        self.fused = fused and self.fused_fits(cfg)
        if self.fused:
            self._build_fused()

    @staticmethod
    def fused_fits(cfg: GPT2Config) -> bool:
        """Shapes the fused decode-step kernel takes (include/thvm_sm100.h)."""
        return (cfg.n_layers <= L.DECODE_MAX_LAYERS and cfg.dim in (512, 768)
                and cfg.head_dim in (32, 64) and cfg.hidden == 4 * cfg.dim)

    def _build_fused(self) -> None:
        """The device-resident Sm100DecodeModel over this model's buffers."""
        cfg, dev, s = self.cfg, self.dev, self.s
        p = dev.dptr
        m = L.Sm100DecodeModel()
        m.n_layers, m.dim, m.hidden, m.vocab = cfg.n_layers, cfg.dim, cfg.hidden, cfg.vocab
        m.max_ctx, m.heads, m.head_dim, m.bump = cfg.max_ctx, cfg.n_heads, cfg.head_dim, 1
        m.eps, m.attn_scale = cfg.norm_eps, float(1.0 / np.sqrt(cfg.head_dim))
        m.wte, m.wpe = p(self.wte), p(self.wpe)
        m.ln_f_g, m.ln_f_b = p(self.ln_f.g), p(self.ln_f.b)
        # row-sliced weights block-transposed for the decode grid (one-time copies)
        def bt(w, kind: int, rows: int) -> int:
            out = dev.alloc(4 * rows * cfg.dim)
            L.check(dev.lib.sm100_decode_block_transpose(p(w), p(out), kind, cfg.dim, cfg.n_heads, cfg.vocab,
                                                         dev.stream), "decode_block_transpose")
            self.regrouped.append(out)
            return p(out)
        self.regrouped = []
        m.lm_head_bt = bt(self.lm_head.w, 2, cfg.vocab)
        for i, blk in enumerate(self.h):
            m.ln1_g[i], m.ln1_b[i] = p(blk.ln_1.g), p(blk.ln_1.b)
            m.w_qkv_bt[i], m.b_qkv[i] = bt(blk.attn.c_attn.w, 0, 3 * cfg.dim), p(blk.attn.c_attn.b)
            m.b_o[i] = p(blk.attn.c_proj.b)
            m.ln2_g[i], m.ln2_b[i] = p(blk.ln_2.g), p(blk.ln_2.b)
            m.w_fc_bt[i], m.b_fc[i] = bt(blk.mlp.c_fc.w, 1, cfg.hidden), p(blk.mlp.c_fc.b)
            m.b_p2[i] = p(blk.mlp.c_proj.b)
            m.kv_cache[i] = p(blk.attn.cache_kv)
        # the split projections regrouped once: c_proj per head, mlp.c_proj transposed
        for i, blk in enumerate(self.h):
            w_o_h, w_p2_t = dev.alloc(4 * cfg.dim * cfg.dim), dev.alloc(4 * cfg.hidden * cfg.dim)
            L.check(dev.lib.sm100_decode_regroup(p(blk.attn.c_proj.w), p(blk.mlp.c_proj.w), p(w_o_h), p(w_p2_t),
                                                 cfg.dim, cfg.n_heads, cfg.hidden, dev.stream), "decode_regroup")
            self.regrouped += [w_o_h, w_p2_t]
            m.w_o_h[i], m.w_p2_t[i] = p(w_o_h), p(w_p2_t)
        dev.sync()
        # the kernel's scratch words, zero-initialised: q/k/v of the new row, reduction sets
        self.words = [dev.alloc(8 * 3 * cfg.dim), dev.alloc(dev.lib.sm100_decode_red_bytes(cfg.n_layers, cfg.dim))]
        m.io = p(s.io)
        m.qkv_w, m.red_w = (p(b) for b in self.words)
        self.part = dev.alloc(dev.lib.sm100_decode_part_bytes())
        m.part_w = p(self.part)
        m.logits = p(s.logits)
        self.sync = dev.alloc(dev.lib.sm100_decode_sync_bytes())
        m.sync = p(self.sync)
        L.check(dev.lib.sm100_decode_prepare(ctypes.addressof(m)), "decode_prepare")
        self.desc = dev.alloc(ctypes.sizeof(m))
        L.check(dev.lib.sm100_buf_write(self.desc, ctypes.addressof(m), ctypes.sizeof(m)), "buf_write(desc)")
        self._desc_host = m
        self.fused_op = self.fused_tokens_op(1)

    def fused_tokens_op(self, n_tokens: int) -> Op:
        """The fused kernel over n greedy tokens (one launch)."""
        cfg = self.cfg
        return make_op(L.K_DECODE_STEP, self.s.io, {0: self.desc}, m=cfg.n_layers, k=cfg.dim,
                       heads=cfg.n_heads, ld_out=cfg.vocab, max_ctx=cfg.max_ctx, n=n_tokens)

    def set_trace(self, on: bool = True) -> None:
        """Record the fused kernel's per-CTA phase timeline (read_trace); the
        step graphs must be captured again after a change."""
        if not self.fused:
            raise ValueError("tracing is a feature of the fused decode step")
        m = self._desc_host
        if on:
            if not getattr(self, "trace", None):
                self.trace = self.dev.alloc(self.dev.lib.sm100_decode_trace_bytes(self.cfg.n_layers))
            m.trace = self.dev.dptr(self.trace)
        else:
            m.trace = None
        L.check(self.dev.lib.sm100_buf_write(self.desc, ctypes.addressof(m), ctypes.sizeof(m)), "buf_write(desc)")

    def read_trace(self) -> np.ndarray:
        """[grid, 3 n_layers + 1, 8] global-timer ns per CTA and step (the
        slots include/thvm_sm100.h lists for Sm100DecodeModel.trace)."""
        grid = self.dev.lib.sm100_decode_grid(self.cfg.n_heads, self.cfg.head_dim)
        n = grid * (3 * self.cfg.n_layers + 1) * 8
        return self.dev.read(self.trace, np.uint64, (n,)).reshape(grid, -1, 8)

    def step_ops(self) -> list:
        """The kernels of one decode step (T = 1, bump): the fused kernel, or
        the per-op schedule."""
        return [self.fused_op] if self.fused else self.forward_ops(1, bump=True)

    def decode_status(self, clear: bool = True) -> int:
        """The fused kernel's sticky status word (0 = no error)."""
        if not self.fused:
            return 0
        st = int(self.dev.read(self.sync, np.uint32, (4,))[2])
        if clear and st:
            # the status word only: sync[3] (the launch epoch) selects the
            # reduction set the next launch may use
            self.dev.write(self.sync, np.zeros(1, np.uint32), byte_off=8)
        return st

    # ---- the schedule ---------------------------------------------------
    def forward_ops(self, T: int, bump: bool) -> list:
        """Kernels of Transformer.forward over T new tokens at the device
        position (thvm_gpt2.py:91-124), ending in the greedy argmax."""
        cfg, s, ops = self.cfg, self.s, []
        ops.append(make_op(L.K_EMBEDDING, s.x, {0: self.wte, 1: s.tok, 2: self.wpe, SLOT_POS: s.pos},
                           dtype=L.DT_F32, m=T, n=cfg.vocab, k=cfg.dim))
        for blk in self.h:
            blk(ops, s, T)
        ops.append(make_op(L.K_LINEAR, s.logits, {SLOT_X: s.x, SLOT_W: self.lm_head.w,
                                                   SLOT_LNG: self.ln_f.g, SLOT_LNB: self.ln_f.b},
                           flags=L.LIN_LN, m=1, n=cfg.vocab, k=cfg.dim, row_off=T - 1, eps=cfg.norm_eps))
        ops.append(make_op(L.K_ARGMAX, s.tok, {0: s.logits, SLOT_POS: s.pos if bump else None},
                           m=1, n=cfg.vocab))
        return ops

    def _run(self, ops) -> None:
        for op in ops:
            self.dev.dispatch(op.kernel, op.in_ids, op.out_id)

    # ---- eager forward (one realize) ------------------------------------
    def forward(self, tokens, start_pos: int) -> int:
        """One realize of Transformer.forward: tokens at start_pos..; returns
        the greedy next id.  Leaves tok[0] = that id and pos = start_pos + T."""
        toks = np.asarray(tokens, np.int32).reshape(-1)
        T = toks.size
        if not 0 < T <= self.s.max_tokens or start_pos + T > self.cfg.max_ctx:
            raise ValueError(f"{T} tokens at {start_pos} do not fit")
        self.dev.write(self.s.tok, toks)
        self.dev.write(self.s.pos, np.array([start_pos], np.int32))
        self._run(self.forward_ops(T, bump=False))
        self.dev.write(self.s.pos, np.array([start_pos + T], np.int32))
        return int(self.dev.read(self.s.tok, np.int32, (1,))[0])

    def logits(self) -> np.ndarray:
        return self.dev.read(self.s.logits, np.float32, (self.cfg.vocab,))

    # ---- TinyJit replay ---------------------------------------------------
    def capture_step(self) -> None:
        """One decode step (T = 1) as a CUDA graph: reads tok[0] and pos,
        writes the next id to tok[0] and advances pos."""
        self.dev.capture_begin(self.GRAPH_STEP)
        try:
            self._run(self.step_ops())
        finally:
            self.dev.capture_end(self.GRAPH_STEP)

    def step(self, token: int | None = None, start_pos: int | None = None) -> None:
        """Replay the captured step; host inputs, when given, are written
        first (both together: one 8-byte copy)."""
        if token is not None and start_pos is not None:
            self.dev.write(self.s.io, np.array([start_pos, token], np.int32))
        elif token is not None:
            self.dev.write(self.s.tok, np.array([token], np.int32))
        elif start_pos is not None:
            self.dev.write(self.s.pos, np.array([start_pos], np.int32))
        self.dev.replay(self.GRAPH_STEP)

    def capture_run(self, n_tokens: int, token: int, start_pos: int) -> None:
        """n_tokens greedy decode steps as ONE graph that first restores
        (tok, pos) = (token, start_pos), so every replay regenerates the same
        stream: the decode loop of GPT2.generate (thvm_gpt2.py:195-220).
        Fused: the n tokens are one launch of the persistent kernel."""
        self.dev.write(self.s.start, np.array([token, start_pos], np.int32))
        self.dev.capture_begin(self.GRAPH_RUN)
        try:
            self.dev.copy_at(self.s.tok, 0, self.s.start, 4)
            self._copy_pos_from_start()
            if self.fused:
                self._run([self.fused_tokens_op(n_tokens)])
            else:
                ops = self.step_ops()
                for _ in range(n_tokens):
                    self._run(ops)
        finally:
            self.dev.capture_end(self.GRAPH_RUN)
        self._run_tokens = n_tokens

    def _copy_pos_from_start(self) -> None:
        # pos <- start[1]: a 4-byte device copy through a view of `start`
        v = self.dev.lib.sm100_buf_view(self.s.start, 4, 4)
        try:
            self.dev.copy_at(self.s.pos, 0, v, 4)
        finally:
            self.dev.free(v)

    def replay_run(self) -> None:
        self.dev.replay(self.GRAPH_RUN)

    def current_token(self) -> int:
        return int(self.dev.read(self.s.tok, np.int32, (1,))[0])

    def generate(self, prompt, n_new: int) -> list:
        """Greedy ids after the prompt (temperature 0): the prompt in one
        forward, then replays of the captured step (the host reads each id,
        as GPT2.generate's .tolist() does)."""
        out = [self.forward(prompt, 0)]
        self.capture_step()
        for _ in range(n_new - 1):
            self.step()
            out.append(self.current_token())
        return out
