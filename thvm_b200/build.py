"""Build libthvm_sm100.so in-tree: nvcc for the sm_100a kernels (.cu), gcc for
the C host runtime (.c), one shared library with the CUDA runtime linked
statically (so it does not depend on which libcudart another module loaded).

    python -m thvm_b200.build [--force]
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libthvm_sm100.so"
INCLUDE = PKG.parent / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]
CC_FLAGS = ["-std=c11", "-O2", "-fPIC", "-Wall", "-Wextra", "-Wno-unused-parameter"]


def _sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.c"))


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return src.stat().st_mtime > t or any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, force: bool) -> Path:
    obj = OBJ / (src.name + ".o")
    if not force and not _stale(obj, src, _headers()):
        return obj
    nvcc = str(CUDA_HOME / "bin" / "nvcc")
    if src.suffix == ".cu":
        cmd = [nvcc, *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
    else:
        cc = shutil.which(os.environ.get("CC", "gcc")) or "gcc"
        cmd = [cc, *CC_FLAGS, f"-I{CUDA_HOME / 'include'}", f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if r.stderr.strip() and os.environ.get("THVM_SM100_BUILD_VERBOSE"):
        sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        nvcc = str(CUDA_HOME / "bin" / "nvcc")
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs), "-lrt", "-ldl",
               "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        tmp.replace(LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
