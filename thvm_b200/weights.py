"""Weight files into device buffers (include/thvm_sm100.h sm100_safetensors_load,
sm100_dsv2pack_load, sm100_torch_load): the .safetensors files py/thvm's
safe_load / safe_save use (py/thvm/nn_state.py:44-85), the reference
DeepSeek-V2 bench's DSV2PK01 pack (bench/dsv2_decode_bench.c:229-262) and
torch.save checkpoints (torch_load, :123-230), mapped from disk and copied
once into backend buffers."""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib as L

_NP = {"F32": np.float32, "F16": np.float16, "BF16": np.uint16, "F64": np.float64, "I8": np.int8, "U8": np.uint8,
       "I16": np.int16, "U16": np.uint16, "I32": np.int32, "U32": np.uint32, "I64": np.int64, "U64": np.uint64,
       "BOOL": np.bool_, "F8_E4M3": np.uint8, "F8_E5M2": np.uint8}


@dataclass(frozen=True)
class DeviceTensor:
    """One tensor of a weight file in a backend buffer (bf16 / fp8 as raw codes)."""
    buf_id: int
    dtype: str
    shape: tuple
    nbytes: int

    @property
    def np_dtype(self):
        return np.dtype(_NP[self.dtype])


def _load(fn, path: str, cap: int) -> dict[str, DeviceTensor]:
    entries = (L.Sm100TensorEntry * cap)()
    n = ctypes.c_int32(0)
    L.check(fn(str(path).encode(), entries, cap, ctypes.byref(n)), "weights")
    out = {}
    for e in entries[:n.value]:
        out[e.name.decode()] = DeviceTensor(int(e.buf_id), e.dtype.decode(), tuple(e.shape[:e.ndim]), int(e.nbytes))
    return out


def load_safetensors(path, max_tensors: int = 4096) -> dict[str, DeviceTensor]:
    return _load(L.lib().sm100_safetensors_load, path, max_tensors)


def load_dsv2_pack(path, max_tensors: int = 4096) -> dict[str, DeviceTensor]:
    return _load(L.lib().sm100_dsv2pack_load, path, max_tensors)


def load_torch(path, max_tensors: int = 4096) -> dict[str, DeviceTensor]:
    """The tensors of a torch.save state dict (zip or legacy format; py/thvm's
    torch_load, py/thvm/nn_state.py:123-230), in their file types."""
    return _load(L.lib().sm100_torch_load, path, max_tensors)


def read(device, t: DeviceTensor) -> np.ndarray:
    """The tensor's bytes back from the device, shaped."""
    return device.read(t.buf_id, t.np_dtype, t.shape)


_TAG = {np.dtype(np.float32): "F32", np.dtype(np.uint16): "BF16", np.dtype(np.uint8): "F8_E4M3",
        np.dtype(np.int32): "I32", np.dtype(np.int64): "I64", np.dtype(np.float16): "F16"}


def save_safetensors(path, tensors: dict[str, np.ndarray]) -> None:
    """Writes tensors in the .safetensors layout load_safetensors reads (an
    8-byte little-endian header length, a JSON header of name -> {dtype,
    shape, data_offsets}, the raw bytes; py/thvm/nn_state.py:44-85).  uint16
    arrays are tagged BF16 (bf16 bits), uint8 arrays F8_E4M3 (e4m3 codes)."""
    import json
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        tag = _TAG.get(a.dtype)
        if tag is None:
            raise ValueError(f"{name}: dtype {a.dtype} has no safetensors tag here")
        header[name] = {"dtype": tag, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for b in blobs:
            f.write(b)
