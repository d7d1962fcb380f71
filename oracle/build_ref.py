"""Compile the reference's own CUDA extension -- TEST INFRASTRUCTURE ONLY.

Builds kw78999/FIER-2bits csrc/popkv_ext.cpp + csrc/popkv_ext.cu, unmodified and
read in place from the reference checkout, with the reference's own JIT flags
(-O3 --use_fast_math, popkv_cuda.py:16-22) for sm_100a, into
oracle/_ref/popkv_ext_ref*.so.  The GPU tests load it (when present) as the
golden for packed bitmasks, fp16 representatives and scores; nothing in the
shipped library uses it.

  python oracle/build_ref.py [<reference checkout>]
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "popkv_ext_ref"


def target() -> Path:
    return OUT / (NAME + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


def build(reference: str | Path, force: bool = False) -> Path | None:
    ref = Path(reference)
    cpp, cu = ref / "csrc" / "popkv_ext.cpp", ref / "csrc" / "popkv_ext.cu"
    if not (cpp.exists() and cu.exists()):
        return None
    out = target()
    if out.exists() and not force and out.stat().st_mtime > max(cpp.stat().st_mtime, cu.stat().st_mtime):
        return out
    import torch
    from torch.utils import cpp_extension as ce

    OUT.mkdir(exist_ok=True)
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"], str(cuda / "include")]
    libs = ce.library_paths(device_type="cuda") + [str(cuda / "lib64")]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = [f"-D_GLIBCXX_USE_CXX11_ABI={abi}", f"-DTORCH_EXTENSION_NAME={NAME}",
            "-DTORCH_API_INCLUDE_EXTENSION_H"]
    cu_obj, cpp_obj = OUT / "popkv_ext_cu.o", OUT / "popkv_ext_cpp.o"
    subprocess.run([str(cuda / "bin" / "nvcc"), "-gencode", "arch=compute_100a,code=sm_100a",
                    "-O3", "--use_fast_math", "-std=c++17", "-Xcompiler", "-fPIC", *defs,
                    *[f"-I{i}" for i in inc], "-c", str(cu), "-o", str(cu_obj)], check=True)
    subprocess.run(["g++", "-O3", "-std=c++17", "-fPIC", *defs, *[f"-I{i}" for i in inc],
                    "-c", str(cpp), "-o", str(cpp_obj)], check=True)
    subprocess.run(["g++", "-shared", "-o", str(out), str(cu_obj), str(cpp_obj),
                    *[f"-L{d}" for d in libs], "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu",
                    "-ltorch_cuda", "-ltorch_python", "-lcudart"], check=True)
    return out


def load():
    """Import the built reference extension, or None when it was not built."""
    out = target()
    if not out.exists():
        return None
    import importlib.machinery
    import importlib.util

    import torch  # noqa: F401  (loads libtorch before the extension)
    loader = importlib.machinery.ExtensionFileLoader(NAME, str(out))
    spec = importlib.util.spec_from_file_location(NAME, str(out), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else str(Path.home() / "reference"), force=True))
