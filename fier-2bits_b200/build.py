"""In-tree build of the Pop-KV B200 library.

  python fier-2bits_b200/build.py          # build what is out of date
  python fier-2bits_b200/build.py --force  # rebuild everything

Products (next to this file, under lib/):
  libpopkv_b200.so        C-ABI library: the sm_100a kernels (nvcc, no torch)
  _popkv_torch*.so        thin torch extension over the C ABI (pybind11 + ATen)

Both are plain shared objects loaded from this directory, so a copied tree
ships them as built.  Compiled for sm_100a only, without --use_fast_math
(IEEE division and square root in the kernels).
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIB = HERE / "lib"
ROOT = HERE.parent
INCLUDE = ROOT / "include"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_SOURCES = ["capi.cu", "pack.cu", "score.cu", "select.cu", "attention.cu", "decoder.cu"]
C_LIB = LIB / "libpopkv_b200.so"


def _torch_ext_path() -> Path:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return LIB / f"_popkv_torch{suffix}"


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_c_library(force: bool = False, verbose: bool = False) -> Path:
    deps = [CSRC / s for s in CUDA_SOURCES] + [CSRC / "common.cuh", CSRC / "score_core.cuh", INCLUDE / "popkv_b200.h"]
    if not force and not _stale(C_LIB, deps):
        return C_LIB
    LIB.mkdir(exist_ok=True)
    obj_dir = LIB / "obj"
    obj_dir.mkdir(exist_ok=True)
    objs, jobs = [], []
    headers = [CSRC / "common.cuh", CSRC / "score_core.cuh", INCLUDE / "popkv_b200.h"]
    for src in CUDA_SOURCES:
        obj = obj_dir / (Path(src).stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [CSRC / src, *headers]):
            jobs.append([NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                         "-Xptxas", "-warn-spills", f"-I{INCLUDE}", "-c", CSRC / src, "-o", obj])
    # The translation units are independent: compile them concurrently.
    procs = []
    for cmd in jobs:
        if verbose:
            print(" ".join(str(c) for c in cmd), flush=True)
        procs.append(subprocess.Popen([str(c) for c in cmd]))
    failed = [p.args for p in procs if p.wait() != 0]
    if failed:
        raise subprocess.CalledProcessError(1, failed[0])
    tmp = C_LIB.with_suffix(".so.tmp")
    _run([NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"], verbose)
    os.replace(tmp, C_LIB)
    return C_LIB


def build_torch_extension(force: bool = False, verbose: bool = False) -> Path:
    target = _torch_ext_path()
    src = CSRC / "torch_binding.cpp"
    deps = [src, INCLUDE / "popkv_b200.h", C_LIB]
    if not force and not _stale(target, deps):
        return target
    import torch
    from torch.utils import cpp_extension as ce

    includes = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"],
                                                        str(INCLUDE), str(CUDA_HOME / "include")]
    libdirs = ce.library_paths(device_type="cuda") + [str(LIB), str(CUDA_HOME / "lib64")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=_popkv_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{i}" for i in includes], src, "-o", target.with_suffix(".tmp"),
           *[f"-L{d}" for d in libdirs], "-lpopkv_b200", "-lc10", "-lc10_cuda", "-ltorch",
           "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python", "-lcudart",
           "-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    os.replace(target.with_suffix(".tmp"), target)
    return target


def build(force: bool = False, verbose: bool = False) -> None:
    build_c_library(force, verbose)
    build_torch_extension(force, verbose)


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
