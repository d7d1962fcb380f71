"""The C-ABI library: loads without a GPU, exports every declared entry point, and
rejects bad arguments on the host before launching anything."""
import ctypes
import re
from pathlib import Path

import pytest

import _native

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "popkv_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(popkv_[a-z_0-9]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return _native.c_library()


def test_every_declared_symbol_is_exported(lib):
    names = declared_functions()
    assert "popkv_pack" in names and "popkv_sparse_attention" in names
    for name in names:
        assert hasattr(lib, name), f"{name} declared in {HEADER.name} but not exported"


def test_error_strings_and_version(lib):
    lib.popkv_error_string.restype = ctypes.c_char_p
    assert lib.popkv_error_string(0) == b"success"
    assert lib.popkv_error_string(2) == b"capacity exceeded"
    assert lib.popkv_version() >= 100


def _i64(*xs):
    return [ctypes.c_int64(x) for x in xs]


def test_pack_rejects_capacity_overflow_without_launching(lib):
    lib.popkv_last_error.restype = ctypes.c_char_p
    dummy = ctypes.c_void_p(16)
    rc = lib.popkv_pack(dummy, 2, *_i64(8, 40, 128, 40 * 128), dummy, dummy, dummy, dummy,
                        *_i64(32, 0), None, 0, None)
    assert rc == 2
    assert b"capacity" in lib.popkv_last_error()


def test_pack_rejects_bad_dtype_and_head_dim(lib):
    dummy = ctypes.c_void_p(16)
    assert lib.popkv_pack(dummy, 9, *_i64(1, 1, 64, 64), dummy, dummy, dummy, dummy,
                          *_i64(32, 0), None, 0, None) == 3
    assert lib.popkv_pack(dummy, 2, *_i64(1, 1, 300, 300), dummy, dummy, dummy, dummy,
                          *_i64(32, 0), None, 0, None) == 3


def test_select_rejects_budget_one(lib):
    dummy = ctypes.c_void_p(16)
    rc = lib.popkv_select(dummy, *_i64(4, 100, 100), None, ctypes.c_int64(0), ctypes.c_int64(1),
                          dummy, None, ctypes.c_int64(0), ctypes.c_int64(0), None, ctypes.c_size_t(0), None)
    assert rc == 1


def test_score_rejects_tokens_beyond_capacity(lib):
    dummy = ctypes.c_void_p(16)
    rc = lib.popkv_score(dummy, 2, *_i64(1, 32, 128), dummy, dummy, dummy, dummy,
                         *_i64(8, 64), 0, dummy, ctypes.c_int64(65), None, dummy,
                         ctypes.c_int64(65), None, 0, None)
    assert rc == 1


def test_attention_rejects_bad_group_and_small_workspace(lib):
    dummy = ctypes.c_void_p(256)
    # 12 query heads over 8 KV heads: not an integer group.
    rc = lib.popkv_sparse_attention(dummy, 2, *_i64(1, 12, 128), dummy, dummy, *_i64(8, 100), 0,
                                    None, None, None, *_i64(0, 16, 50), None, dummy, dummy,
                                    ctypes.c_size_t(1 << 20), ctypes.c_int64(0), None)
    assert rc == 3
    lib.popkv_sparse_attention_workspace_bytes.restype = ctypes.c_size_t
    need = lib.popkv_sparse_attention_workspace_bytes(*_i64(1, 32, 8, 128, 32768, 0))
    assert need > 0
    rc = lib.popkv_sparse_attention(dummy, 2, *_i64(1, 32, 128), dummy, dummy, *_i64(8, 40000), 0,
                                    None, None, None, *_i64(0, 4096, 32768), None, dummy, dummy,
                                    ctypes.c_size_t(need - 1), ctypes.c_int64(0), None)
    assert rc == 6
