"""Build the reference's own CUDA kernels for checking against on a GPU.

TEST INFRASTRUCTURE ONLY.  Compiles the reference's KudaHitamCUDA.cu from
where it lies (the reference tree is only read) together with ref_binding.cpp,
for sm_100a, into oracle/_ref/kh_ref.so.  The reference's own build
(torch.utils.cpp_extension.load into its own directory) is not used: it writes
into the reference tree.  Does nothing when the reference tree is absent (the
GPU machines run the prebuilt .so) or the output is newer than its sources.

    python oracle/build_ref.py REFERENCE_DIR
    KUDAHITAM_REFERENCE_DIR=... python oracle/build_ref.py

The reference tree's location is an argument (or the environment variable
KUDAHITAM_REFERENCE_DIR); without either, nothing is built.
"""
from __future__ import annotations

import os
import pathlib
import subprocess
import sys
import sysconfig

HERE = pathlib.Path(__file__).resolve().parent
OUT = HERE / "_ref" / "kh_ref.so"
ENV_VAR = "KUDAHITAM_REFERENCE_DIR"


def build(ref_dir: pathlib.Path | str | None = None) -> pathlib.Path | None:
    if ref_dir is None:
        ref_dir = os.environ.get(ENV_VAR)
    if not ref_dir:
        return OUT if OUT.exists() else None
    src = pathlib.Path(ref_dir) / "KudaHitamCUDA.cu"
    binding = HERE / "ref_binding.cpp"
    if not src.exists():
        return OUT if OUT.exists() else None
    if OUT.exists() and OUT.stat().st_mtime >= max(src.stat().st_mtime,
                                                   binding.stat().st_mtime,
                                                   pathlib.Path(__file__).stat().st_mtime):
        return OUT
    import torch
    import torch.utils.cpp_extension as ce
    OUT.parent.mkdir(parents=True, exist_ok=True)
    nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [f"-I{p}" for p in ce.include_paths(device_type="cuda")]
    incs.append(f"-I{sysconfig.get_paths()['include']}")
    common = ["-O3", "-std=c++17", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
              "-DTORCH_API_INCLUDE_EXTENSION_H", "-Xcompiler", "-fPIC", *incs]
    obj_cu = OUT.parent / "KudaHitamCUDA.o"
    obj_b = OUT.parent / "ref_binding.o"
    # the reference's own module is renamed so that kh_ref is the one imported;
    # the two translation units compile in parallel
    jobs = [
        subprocess.Popen([nvcc, "-gencode", "arch=compute_100a,code=sm_100a",
                          "-DTORCH_EXTENSION_NAME=kh_ref_reference_module",
                          "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
                          "-D__CUDA_NO_HALF2_OPERATORS__", *common, "-c", str(src), "-o",
                          str(obj_cu)]),
        subprocess.Popen(["g++", *[c for c in common if c != "-Xcompiler"],
                          "-DTORCH_EXTENSION_NAME=kh_ref", "-c", str(binding), "-o", str(obj_b)]),
    ]
    if any(j.wait() != 0 for j in jobs):
        raise RuntimeError("building the reference kernels failed")
    libs = [f"-L{p}" for p in ce.library_paths(device_type="cuda")]
    subprocess.run(["g++", "-shared", "-o", str(OUT), str(obj_cu), str(obj_b), *libs,
                    "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
                    "-ltorch_python", "-lcudart"], check=True)
    return OUT


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else None))
