"""Weight files straight into device buffers (thvm_b200/weights.py over
sm100_safetensors_load / sm100_dsv2pack_load), on the CPU in host-memory
mode: the .safetensors file the reference's own safe_save wrote
(tests/golden/make_golden.py state) loads tensor for tensor, byte for byte,
with its dtypes and shapes and the __metadata__ entry skipped; a DSV2PK01
pack written by the oracle's pack writer loads likewise; malformed files are
rejected and leave no buffer behind."""
import subprocess
import sys
import textwrap
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]

PRELUDE = """
import numpy as np
from thvm_b200 import _lib as L
from thvm_b200.device import Device
from thvm_b200 import weights as W
d = Device(host_memory=True)
lib = d.lib
"""


def run(body: str):
    code = PRELUDE + textwrap.dedent(body)
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr


def test_safetensors_from_the_reference_loads_byte_for_byte():
    run("""
    import sys
    sys.path.insert(0, "tests/golden")
    from make_golden import state_tensors
    want = state_tensors()
    got = W.load_safetensors("tests/golden/state.safetensors")
    assert sorted(got) == sorted(want)
    tags = {"wte.weight": "F32", "h.0.attn.c_attn.bias": "F32", "h.0.ln_1.weight": "F16", "experts.codes": "F8_E4M3",
            "positions": "I32", "lm_head.weight.bf16": "BF16", "empty": "F32"}
    for k, v in want.items():
        t = got[k]
        assert t.dtype == tags[k] and t.shape == v.shape and t.nbytes == v.nbytes, (k, t)
        if v.size:
            assert np.array_equal(W.read(d, t).view(np.uint8), v.view(np.uint8)), k
    before = lib.sm100_buf_live_count()
    for t in got.values():
        lib.sm100_buf_free(t.buf_id)
    assert lib.sm100_buf_live_count() == before - len(got)
    """)


def test_dsv2_pack_loads_and_bad_files_leave_nothing():
    run("""
    import tempfile, os
    import oracle as O
    w = {"embed": (np.arange(24, dtype=np.uint16) * 7), "norm": np.linspace(-1, 1, 5, dtype=np.float32),
         "l0.wq": np.arange(6, dtype=np.uint16)}
    with tempfile.TemporaryDirectory() as td:
        p = os.path.join(td, "x.pack")
        O.write_dsv2_pack(p, w)
        got = W.load_dsv2_pack(p)
        assert sorted(got) == sorted(w)
        for k, v in w.items():
            t = got[k]
            assert t.dtype == ("BF16" if v.dtype == np.uint16 else "F32") and t.shape == (v.size,)
            assert np.array_equal(W.read(d, t), v)
        before = lib.sm100_buf_live_count()
        bad = os.path.join(td, "bad.safetensors")
        hdr = b'{"a":{"dtype":"F32","shape":[2],"data_offsets":[0,8]},"b":{"dtype":"F32","shape":[9],"data_offsets":[8,44]}}'
        open(bad, "wb").write(len(hdr).to_bytes(8, "little") + hdr + bytes(16))   # b's bytes run past the file
        try:
            W.load_safetensors(bad)
            raise SystemExit("a truncated file was accepted")
        except L.Sm100Error as e:
            assert "bad entry b" in str(e), e
        assert lib.sm100_buf_live_count() == before   # a's buffer was dropped again
        open(bad, "wb").write(b"DSV2PK01" + (5).to_bytes(8, "little"))
        try:
            W.load_dsv2_pack(bad)
            raise SystemExit("a bad pack was accepted")
        except L.Sm100Error:
            pass
    """)


def test_save_safetensors_round_trips_through_the_loader():
    """thvm_b200.weights.save_safetensors (the writer of the C host's weight
    files) -> sm100_safetensors_load: names, tags, shapes and bytes."""
    run("""
    import os, tempfile
    rng = np.random.default_rng(3)
    t = {"a": rng.standard_normal((3, 5)).astype(np.float32), "b.bf16": rng.integers(0, 65535, (7,), dtype=np.uint16),
         "c.fp8": rng.integers(0, 255, (2, 2, 4), dtype=np.uint8), "d": np.arange(6, dtype=np.int32)}
    with tempfile.TemporaryDirectory() as tmp:
        p = os.path.join(tmp, "w.safetensors")
        W.save_safetensors(p, t)
        got = W.load_safetensors(p)
    assert sorted(got) == sorted(t)
    for k, a in t.items():
        g = got[k]
        assert g.dtype == {"a": "F32", "b.bf16": "BF16", "c.fp8": "F8_E4M3", "d": "I32"}[k] and g.shape == a.shape
        assert np.array_equal(W.read(d, g), a)
    """)


def test_torch_checkpoints_load_as_the_reference_reads_them():
    """torch.save files (tests/golden/state.pt in the zip format,
    state_legacy.pt in the legacy pickle format) through sm100_torch_load:
    every tensor's elements equal what the reference's own torch_load read
    from the same file (tests/golden/torch_state.npz; it widens bf16 and f64
    to f32 and makes the 0-d tensor (1,)), and byte for byte what torch.load
    gives, shared storages, storage offsets, transposed and permuted strides
    included; the dtype tags are the storages' own; every buffer is freed."""
    run("""
    import torch
    gold = np.load("tests/golden/torch_state.npz")
    tags = {torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.float64: "F64",
            torch.int64: "I64", torch.int32: "I32", torch.uint8: "U8", torch.bool: "BOOL"}
    for fmt, fn in (("zip", "tests/golden/state.pt"), ("legacy", "tests/golden/state_legacy.pt")):
        got = W.load_torch(fn)
        want = torch.load(fn, weights_only=True)
        assert sorted(got) == sorted(want) == sorted(k.split("/", 1)[1] for k in gold.files if k.startswith(fmt))
        for k, t in want.items():
            t = t.detach().contiguous()
            e = got[k]
            assert e.dtype == tags[t.dtype] and e.shape == tuple(t.shape), (fmt, k, e)
            raw = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
            assert e.nbytes == raw.nbytes, (fmt, k)
            if not raw.size:
                continue
            back = W.read(d, e).reshape(-1)
            assert np.array_equal(back.view(np.uint8), raw.reshape(-1).view(np.uint8)), (fmt, k)
            ref = gold[f"{fmt}/{k}"].reshape(-1)
            mine = back
            if e.dtype == "BF16":
                mine = (back.astype(np.uint32) << 16).view(np.float32)
            elif e.dtype == "F64":
                mine = back.astype(np.float32)
            assert mine.dtype == ref.dtype and np.array_equal(mine, ref), (fmt, k)
        before = lib.sm100_buf_live_count()
        for t in got.values():
            lib.sm100_buf_free(t.buf_id)
        assert lib.sm100_buf_live_count() == before - len(got)
    """)


def test_torch_checkpoint_with_zip64_records_loads_the_same():
    """The members of state.pt rewritten with zip64 size fields (the records
    torch.save writes for large checkpoints) load to the same bytes."""
    run("""
    import os, tempfile, zipfile
    with tempfile.TemporaryDirectory() as td:
        p64 = os.path.join(td, "z64.pt")
        with zipfile.ZipFile("tests/golden/state.pt") as zin, zipfile.ZipFile(p64, "w", zipfile.ZIP_STORED) as zout:
            for i in zin.infolist():
                with zout.open(i.filename, "w", force_zip64=True) as f:
                    f.write(zin.read(i.filename))
        with open(p64, "rb") as f:
            assert bytes([1, 0, 16, 0]) in f.read()   # a zip64 extra field (id 1, 16 bytes)
        a, b = W.load_torch("tests/golden/state.pt"), W.load_torch(p64)
        assert sorted(a) == sorted(b)
        for k in a:
            assert a[k].shape == b[k].shape and a[k].dtype == b[k].dtype
            if a[k].nbytes:
                assert np.array_equal(W.read(d, a[k]).reshape(-1).view(np.uint8), W.read(d, b[k]).reshape(-1).view(np.uint8)), k
    """)


def test_bad_torch_checkpoints_are_refused_and_leave_nothing():
    """A truncated zip, a file that is neither format, a pickle whose
    storage is missing from the archive: refused with a message, no buffer
    left behind."""
    run("""
    import os, tempfile, zipfile
    raw = open("tests/golden/state.pt", "rb").read()
    with tempfile.TemporaryDirectory() as td:
        cases = {"trunc.pt": raw[: len(raw) // 2], "junk.pt": b"not a checkpoint" * 4}
        # the same archive without the first storage member
        with zipfile.ZipFile("tests/golden/state.pt") as zin, zipfile.ZipFile(os.path.join(td, "nostore.pt"), "w",
                                                                              zipfile.ZIP_STORED) as zout:
            for i in zin.infolist():
                if not i.filename.endswith("/data/0"):
                    zout.writestr(i, zin.read(i.filename))
        for name, b in cases.items():
            with open(os.path.join(td, name), "wb") as f:
                f.write(b)
        before = lib.sm100_buf_live_count()
        for name in list(cases) + ["nostore.pt"]:
            try:
                W.load_torch(os.path.join(td, name))
            except L.Sm100Error:
                pass
            else:
                raise AssertionError(name + " loaded")
            assert lib.sm100_last_error(), name
            assert lib.sm100_buf_live_count() == before, name
    """)
