"""The config-5 decode step with its host in C (include/thvm_sm100.h
sm100_ds_model_*, thvm_b200/csrc/ds_host.c): weights from a .safetensors
file or named device pointers, buffers and the captured step graph owned by
the library; no torch.  This module only writes the weight file and wraps
the C calls."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from .dsv2 import DSConfig, yarn_tables
from .weights import save_safetensors


def save_ds_weights(path, cfg: DSConfig, weights: dict[str, np.ndarray]) -> None:
    """One rank's weights (thvm_b200.dsv2.ds_weights / shard_ds_weights
    layout) plus the rotary tables, as the C host reads them."""
    cos, sin = yarn_tables(cfg.d_rope, cfg.max_ctx)
    save_safetensors(path, {**weights, "cos": cos.astype(np.float32), "sin": sin.astype(np.float32)})


class CDSModel:
    """weights: a .safetensors path (save_ds_weights), or a dict name ->
    device tensor (anything with data_ptr() and nbytes, e.g. torch tensors,
    kept alive by the caller) in the same names and layouts."""

    def __init__(self, cfg: DSConfig, weights):
        from .device import Device
        self.dev, self.cfg, self.lib = Device.get(), cfg, L.lib()
        c = L.Sm100DsCfg()
        for f, _ in L.Sm100DsCfg._fields_:
            setattr(c, f, getattr(cfg, f))
        self.slot = self.dev.new_graph_slot()
        self._m = ctypes.c_void_p()
        if isinstance(weights, dict):
            names = list(weights)
            arr_n = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
            arr_p = (ctypes.c_void_p * len(names))(*[weights[n].data_ptr() for n in names])
            arr_b = (ctypes.c_uint64 * len(names))(*[weights[n].nbytes for n in names])
            self._keep = weights
            L.check(self.lib.sm100_ds_model_open_ptrs(ctypes.byref(c), arr_n, arr_p, arr_b, len(names), self.slot,
                                                      ctypes.byref(self._m)), "ds_model_open_ptrs")
        else:
            L.check(self.lib.sm100_ds_model_open(ctypes.byref(c), str(weights).encode(), self.slot,
                                                 ctypes.byref(self._m)), "ds_model_open")

    def step(self, tok=None, read: bool = True) -> np.ndarray | None:
        """One step (tok: [batch] ids, None keeps the last step's choices);
        the next ids when read."""
        B = self.cfg.batch
        tin = None if tok is None else np.ascontiguousarray(tok, np.int32)
        out = np.empty(B, np.int32) if read else None
        L.check(self.lib.sm100_ds_model_step(self._m, None if tin is None else tin.ctypes.data,
                                             None if out is None else out.ctypes.data), "ds_model_step")
        return out

    @property
    def pos(self) -> int:
        return int(self.lib.sm100_ds_model_pos(self._m))

    def reset(self):
        L.check(self.lib.sm100_ds_model_reset(self._m), "ds_model_reset")

    def logits(self) -> np.ndarray:
        bid = int(self.lib.sm100_ds_model_logits(self._m))
        return self.dev.read(bid, np.float32, (self.cfg.batch, self.cfg.vocab))

    def close(self):
        if self._m:
            self.lib.sm100_ds_model_close(self._m)
            self._m = ctypes.c_void_p()
            self.dev.drop(self.slot)
