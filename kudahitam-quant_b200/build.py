"""Build the engine's C-ABI shared library for sm_100a.

    python kudahitam-quant_b200/build.py        # -> kudahitam/_lib/libkudahitam.so

Every ``csrc/*.cu`` file is compiled by nvcc (in parallel, skipped when its
object is newer than the sources it depends on) and linked into one shared
library with the CUDA runtime linked statically, so the library travels as a
single file and binds to whatever CUDA context the caller (PyTorch) created.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = REPO / "include"
OBJ = PKG / "_build"
OUT = PKG / "kudahitam" / "_lib" / "libkudahitam.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-Wall", f"-I{INCLUDE}", f"-I{CSRC}"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and pathlib.Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _deps() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(nvcc: str, src: pathlib.Path, verbose: bool) -> pathlib.Path:
    obj = OBJ / (src.stem + ".o")
    newest = max([src.stat().st_mtime] + [p.stat().st_mtime for p in _deps()])
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> pathlib.Path:
    nvcc = _nvcc()
    OBJ.mkdir(parents=True, exist_ok=True)
    OUT.parent.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose), srcs))
    if OUT.exists() and OUT.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return OUT
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
