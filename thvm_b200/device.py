"""Python host mirror of the sm_100a Backend (include/thvm_sm100.h).

`Device` wraps the vtable entries one to one (buf_alloc / buf_write /
buf_read / buf_copy_at / dispatch_kernel / dispatch_end / graph capture and
replay), raising Sm100Error where the C entry returns a negative status, as
py/thvm's ctypes layer (py/thvm/thvm.py) wraps libthvm_py.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from ._lib import Sm100Kernel, Sm100View, check


class Device:
    _instance = None

    def __init__(self, host_memory: bool = False):
        lib = L.lib()
        if host_memory:
            lib.sm100_debug_host_memory(1)
        check(lib.sm100_init(), "sm100_init")
        self.lib = lib

    @classmethod
    def get(cls) -> "Device":
        if cls._instance is None or not L.lib().sm100_ready():
            cls._instance = Device()
        return cls._instance

    # ---- buffers ----------------------------------------------------------
    def alloc(self, nbytes: int) -> int:
        bid = self.lib.sm100_buf_alloc(int(nbytes))
        if bid == 0:
            raise L.Sm100Error(L.ERR_OOM, f"buf_alloc({nbytes})")
        return bid

    def upload(self, arr: np.ndarray) -> int:
        a = np.ascontiguousarray(arr)
        bid = self.alloc(a.nbytes)
        self.write(bid, a)
        return bid

    def write(self, bid: int, arr: np.ndarray, byte_off: int = 0) -> None:
        a = np.ascontiguousarray(arr)
        check(self.lib.sm100_buf_write_at(bid, byte_off, a.ctypes.data, a.nbytes), "buf_write_at")

    def read(self, bid: int, dtype=np.float32, shape=None) -> np.ndarray:
        n = self.lib.sm100_buf_nbytes(bid)
        dt = np.dtype(dtype)
        count = int(np.prod(shape)) if shape is not None else n // dt.itemsize
        out = np.empty(count, dt)
        check(self.lib.sm100_buf_read(bid, out.ctypes.data, out.nbytes), "buf_read")
        return out.reshape(shape) if shape is not None else out

    def copy_at(self, dst: int, dst_off: int, src: int, nbytes: int) -> None:
        check(self.lib.sm100_buf_copy_at(dst, dst_off, src, nbytes), "buf_copy_at")

    def free(self, bid: int) -> None:
        self.lib.sm100_buf_free(bid)

    def zero(self, bid: int) -> None:
        self.lib.sm100_buf_zero(bid)

    def dptr(self, bid: int) -> int:
        return self.lib.sm100_buf_dptr(bid) or 0

    # ---- dispatch ---------------------------------------------------------
    def dispatch(self, k: Sm100Kernel, in_ids, out_id: int) -> None:
        ids = (ctypes.c_uint32 * max(1, len(in_ids)))(*in_ids)
        check(self.lib.sm100_dispatch_kernel(ctypes.byref(k), ids, len(in_ids), out_id),
              f"dispatch_kernel(kind={k.kind})")

    def gather_strided(self, dst: int, src: int, dims, strides, offset: int = 0, elem_bytes: int = 4) -> None:
        v = Sm100View()
        v.ndim, v.elem_bytes, v.offset = len(dims), elem_bytes, offset
        for i, (d, s) in enumerate(zip(dims, strides)):
            v.dims[i], v.strides[i] = d, s
        check(self.lib.sm100_gather_strided(dst, src, ctypes.byref(v)), "gather_strided")

    def sync(self) -> None:
        self.lib.sm100_dispatch_end()
        msg = self.lib.sm100_last_error()
        if msg and msg.startswith(b"dispatch_end"):
            raise L.Sm100Error(L.ERR_CUDA, "dispatch_end")

    # ---- graphs (TinyJit replay) -----------------------------------------
    _next_slot = 0
    _free_slots: list = []

    def new_graph_slot(self) -> int:
        """A graph slot no other user of this Device holds (64 per process;
        drop() returns it)."""
        if Device._free_slots:
            return Device._free_slots.pop()
        if Device._next_slot >= 64:
            raise L.Sm100Error(L.ERR_STATE, "graph slots exhausted")
        Device._next_slot += 1
        return Device._next_slot - 1

    def capture_begin(self, slot: int) -> None:
        check(self.lib.sm100_graph_capture_begin(slot), "graph_capture_begin")

    def capture_end(self, slot: int) -> None:
        check(self.lib.sm100_graph_capture_end(slot), "graph_capture_end")

    def replay(self, slot: int) -> None:
        check(self.lib.sm100_graph_replay(slot), "graph_replay")

    def drop(self, slot: int) -> None:
        self.lib.sm100_graph_drop(slot)
        if slot not in Device._free_slots:
            Device._free_slots.append(slot)

    @property
    def stream(self) -> int:
        return self.lib.sm100_stream() or 0

    def launches(self) -> int:
        return int(self.lib.sm100_launch_count())
