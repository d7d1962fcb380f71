"""Loader of the in-tree native libraries (no JIT, no fallback).

``lib/libpopkv_b200.so`` (C ABI, sm_100a kernels) and ``lib/_popkv_torch*.so``
(torch front end) are built by ``build.py``.  ``extension()`` imports the torch
front end from this directory; it raises ``RuntimeError`` when no GPU is visible
(as the reference's loader does, popkv_cuda.py:14-15) or when the libraries were
not built -- there is no other code path to fall back to.
"""
from __future__ import annotations

import ctypes
import importlib.machinery
import importlib.util
import sysconfig
from functools import lru_cache
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_DIR = HERE / "lib"
C_LIBRARY = LIB_DIR / "libpopkv_b200.so"


def torch_extension_path() -> Path:
    return LIB_DIR / ("_popkv_torch" + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))


@lru_cache(maxsize=1)
def _load_torch_extension():
    path = torch_extension_path()
    if not path.exists() or not C_LIBRARY.exists():
        raise RuntimeError(
            f"Pop-KV native libraries are not built ({path.name}); run build.py in {HERE}")
    loader = importlib.machinery.ExtensionFileLoader("_popkv_torch", str(path))
    spec = importlib.util.spec_from_file_location("_popkv_torch", str(path), loader=loader)
    module = importlib.util.module_from_spec(spec)
    loader.exec_module(module)
    return module


def extension():
    """The torch front end; requires a CUDA device, like the reference."""
    if not torch.cuda.is_available():
        raise RuntimeError("Pop-KV CUDA scoring requires an NVIDIA GPU")
    return _load_torch_extension()


@lru_cache(maxsize=1)
def c_library() -> ctypes.CDLL:
    """The C-ABI library itself (loads without a GPU; calls need one)."""
    if not C_LIBRARY.exists():
        raise RuntimeError(f"{C_LIBRARY} is not built; run build.py in {HERE}")
    return ctypes.CDLL(str(C_LIBRARY))
