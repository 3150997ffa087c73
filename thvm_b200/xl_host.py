"""The config-3 model with its host in C (include/thvm_sm100.h
sm100_xl_model_*, thvm_b200/csrc/xl_host.c): the prompt pass and the decode
step on one GPU, weights from a .safetensors file or named device pointers,
buffers and the captured step graph owned by the library; no torch.  This
module only wraps the C calls (thvm_b200.weights.save_safetensors writes the
file from thvm_b200.gpt2_xl.xl_weights as it is)."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from .gpt2_xl import XLConfig


class CXLModel:
    """weights: a .safetensors path, or a dict name -> device tensor (with
    data_ptr() and nbytes, kept alive by the caller) in xl_weights' names."""

    def __init__(self, cfg: XLConfig, weights):
        from .device import Device
        self.dev, self.cfg, self.lib = Device.get(), cfg, L.lib()
        c = L.Sm100XlCfg()
        for f, _ in L.Sm100XlCfg._fields_:
            setattr(c, f, getattr(cfg, f))
        self.slot = self.dev.new_graph_slot()
        self._m = ctypes.c_void_p()
        if isinstance(weights, dict):
            names = list(weights)
            arr_n = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
            arr_p = (ctypes.c_void_p * len(names))(*[weights[n].data_ptr() for n in names])
            arr_b = (ctypes.c_uint64 * len(names))(*[weights[n].nbytes for n in names])
            self._keep = weights
            L.check(self.lib.sm100_xl_model_open_ptrs(ctypes.byref(c), arr_n, arr_p, arr_b, len(names), self.slot,
                                                      ctypes.byref(self._m)), "xl_model_open_ptrs")
        else:
            L.check(self.lib.sm100_xl_model_open(ctypes.byref(c), str(weights).encode(), self.slot,
                                                 ctypes.byref(self._m)), "xl_model_open")

    def prefill(self, prompts: np.ndarray) -> np.ndarray:
        """prompts [batch, len] -> the first ids [batch]; position = len."""
        p = np.ascontiguousarray(prompts, np.int32)
        out = np.empty(self.cfg.batch, np.int32)
        L.check(self.lib.sm100_xl_model_prefill(self._m, p.ctypes.data, p.shape[1], out.ctypes.data),
                "xl_model_prefill")
        return out

    def step(self, tok=None) -> np.ndarray:
        """One decode step (tok: [batch] ids, None keeps the last choices)."""
        tin = None if tok is None else np.ascontiguousarray(tok, np.int32)
        out = np.empty(self.cfg.batch, np.int32)
        L.check(self.lib.sm100_xl_model_step(self._m, None if tin is None else tin.ctypes.data, out.ctypes.data),
                "xl_model_step")
        return out

    @property
    def pos(self) -> int:
        return int(self.lib.sm100_xl_model_pos(self._m))

    def logits(self) -> np.ndarray:
        bid = int(self.lib.sm100_xl_model_logits(self._m))
        return self.dev.read(bid, np.float32, (self.cfg.batch, self.cfg.vocab))

    def close(self):
        if self._m:
            self.lib.sm100_xl_model_close(self._m)
            self._m = ctypes.c_void_p()
            self.dev.drop(self.slot)
