"""Build the engine's C-ABI shared library for sm_100a.

    python kudahitam-quant_b200/build.py        # -> kudahitam/_lib/libkudahitam.so
                                                #    kudahitam/_lib/libkh_torch.so

Every ``csrc/*.cu`` file is compiled by nvcc (in parallel, skipped when its
object is newer than the sources it depends on) and linked into one shared
library with the CUDA runtime linked statically, so the library travels as a
single file and binds to whatever CUDA context the caller (PyTorch) created.
``csrc/kh_torch.cpp`` (the torch.ops.kudahitam operators over that C ABI) is
compiled by g++ against PyTorch's headers into a second library that links
the first one (found beside it through its rpath).
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
TORCH_OUT = PKG / "kudahitam" / "_lib" / "libkh_torch.so"

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


def build_torch_ext(cuda_home: str) -> pathlib.Path:
    """g++ build of the torch.ops.kudahitam operators (csrc/kh_torch.cpp)."""
    src = CSRC / "kh_torch.cpp"
    newest = max(src.stat().st_mtime, OUT.stat().st_mtime,
                 *[p.stat().st_mtime for p in INCLUDE.glob("*.h")])
    if TORCH_OUT.exists() and TORCH_OUT.stat().st_mtime >= newest:
        return TORCH_OUT
    import torch
    tdir = pathlib.Path(torch.__file__).resolve().parent
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wno-unused-function",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-I{tdir / 'include'}", f"-I{tdir / 'include' / 'torch' / 'csrc' / 'api' / 'include'}",
           f"-I{cuda_home}/include", f"-I{INCLUDE}", str(src),
           "-o", str(TORCH_OUT.with_suffix(".so.tmp")),
           f"-L{tdir / 'lib'}", f"-L{OUT.parent}", "-lkudahitam", "-lc10", "-lc10_cuda",
           "-ltorch_cpu", "-ltorch", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"building kh_torch.cpp failed:\n{r.stdout}\n{r.stderr}")
    os.replace(TORCH_OUT.with_suffix(".so.tmp"), TORCH_OUT)
    return TORCH_OUT


def build(verbose: bool = False, torch_ext: bool = True) -> pathlib.Path:
    nvcc = _nvcc()
    OBJ.mkdir(parents=True, exist_ok=True)
    OUT.parent.mkdir(parents=True, exist_ok=True)
    srcs = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, verbose), srcs))
    if not (OUT.exists() and OUT.stat().st_mtime >= max(o.stat().st_mtime for o in objs)):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, OUT)
    if torch_ext:
        build_torch_ext(str(pathlib.Path(nvcc).resolve().parent.parent))
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
