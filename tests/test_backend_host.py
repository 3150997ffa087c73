"""Buffer-table semantics of the Backend vtable (include/thvm_sm100.h part 1),
run in host-memory mode on the CPU.  Each case runs in a fresh process because
the table is process-global and host mode must be chosen before sm100_init.

The contract is the reference CUDA backend's (src/backend/cuda/buf_*.c):
fresh buffers read as zeros, the freelist hands recycled storage to a NEW id
and kills the donor, views share storage and are never recycled, offset
writes are bounds-checked, jit-pinned buffers survive decref."""
import subprocess
import sys
import textwrap
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

PRELUDE = """
import numpy as np
from thvm_b200 import _lib as L
from thvm_b200.device import Device
d = Device(host_memory=True)
lib = d.lib
"""


def run(body: str):
    code = PRELUDE + textwrap.dedent(body)
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr


def test_alloc_zero_filled_and_roundtrip():
    run("""
    b = d.alloc(1000)
    assert lib.sm100_buf_nbytes(b) == 1000
    assert not d.read(b, np.uint8).any()
    x = np.arange(250, dtype=np.float32)
    d.write(b, x)
    assert np.array_equal(d.read(b, np.float32), x)
    assert lib.sm100_buf_refcount(b) == 1
    """)


def test_write_at_bounds_checked():
    run("""
    b = d.alloc(64)
    d.write(b, np.ones(4, np.float32), byte_off=48)
    assert d.read(b, np.float32)[12:].tolist() == [1, 1, 1, 1]
    try:
        d.write(b, np.ones(4, np.float32), byte_off=52)
        raise SystemExit("out-of-bounds write_at was accepted")
    except L.Sm100Error as e:
        assert "outside" in str(e)
    assert lib.sm100_buf_copy_at(b, 60, b, 8) != 0
    """)


def test_copy_at_kv_append():
    run("""
    cache = d.alloc(4 * 16 * 8)
    row = d.upload(np.full(8, 3.0, np.float32))
    for pos in (0, 5, 15):
        d.copy_at(cache, pos * 32, row, 32)
    c = d.read(cache, np.float32).reshape(16, 8)
    assert (c[[0, 5, 15]] == 3).all() and c.sum() == 3 * 8 * 3
    """)


def test_freelist_hands_storage_to_fresh_id():
    run("""
    a = d.alloc(4096)
    ptr = d.dptr(a)
    d.write(a, np.full(1024, 7, np.float32))
    lib.sm100_buf_freelist_push(a)
    assert lib.sm100_buf_refcount(a) == 0
    b = d.alloc(1000)               # best fit: reuses a's block
    assert b != a and d.dptr(b) == ptr
    assert d.dptr(a) == 0           # the donor id is dead
    assert not d.read(b, np.uint8).any()   # recycled storage is zeroed
    assert lib.sm100_buf_nbytes(b) == 1000
    """)


def test_freelist_best_fit_and_remove():
    run("""
    small, big = d.alloc(1024), d.alloc(65536)
    ps, pb = d.dptr(small), d.dptr(big)
    lib.sm100_buf_freelist_push(big)
    lib.sm100_buf_freelist_push(small)
    x = d.alloc(512)
    assert d.dptr(x) == ps           # smallest block that fits
    lib.sm100_buf_freelist_remove(big)
    assert lib.sm100_buf_refcount(big) == 1
    y = d.alloc(40000)
    assert d.dptr(y) != pb           # big was un-parked, not re-issued
    """)


def test_views_share_storage_and_are_not_recycled():
    run("""
    p = d.upload(np.arange(64, dtype=np.float32))
    v = lib.sm100_buf_view(p, 16, 32)
    assert v and lib.sm100_buf_storage_root(v) == p
    assert d.read(v, np.float32).tolist() == [4, 5, 6, 7, 8, 9, 10, 11]
    lib.sm100_buf_freelist_push(v)
    assert lib.sm100_buf_refcount(v) == 1   # views are never parked
    assert lib.sm100_buf_view(p, 240, 32) == 0   # outside the parent
    """)


def test_refcount_and_jit_pin():
    run("""
    a = d.alloc(16)
    lib.sm100_buf_incref(a)
    lib.sm100_buf_decref(a)
    assert d.dptr(a) != 0
    lib.sm100_buf_jit_pin(a)
    lib.sm100_buf_decref(a)
    assert d.dptr(a) != 0            # pinned: survives refcount 0
    lib.sm100_buf_jit_unpin(a)
    lib.sm100_buf_free(a)
    assert d.dptr(a) == 0
    live = lib.sm100_mem_live_bytes()
    b = d.alloc(1 << 20)
    assert lib.sm100_mem_live_bytes() == live + (1 << 20)
    assert lib.sm100_mem_peak_bytes() >= live + (1 << 20)
    """)


def test_byte_ceiling_and_dead_ids():
    run("""
    import os
    os.environ["THVM_MAX_BUF_BYTES"] = "4096"
    assert lib.sm100_buf_alloc(8192) == 0
    assert "THVM_MAX_BUF_BYTES" in lib.sm100_last_error().decode()
    assert lib.sm100_buf_read(0, None, 0) != 0
    assert lib.sm100_buf_read(12345, None, 0) != 0
    assert lib.sm100_buf_refcount(999) == 0
    """)


def test_host_mode_runs_no_kernels():
    run("""
    k = L.Sm100Kernel.make(L.K_GELU, {0: 0}, m=1, k=4)
    b = d.alloc(16)
    try:
        d.dispatch(k, [b], b)
        raise SystemExit("dispatch ran in host mode")
    except L.Sm100Error as e:
        assert e.code == L.ERR_UNSUPPORTED
    """)
