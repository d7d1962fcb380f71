"""The allocation-free attention entry point against the regular one, through the C ABI.

popkv_sparse_attention_noalloc serves callers that may not allocate device memory
(an engine that owns every allocation, or code running while the engine holds its
allocator): it uses scratch built into the library instead of a workspace.  Two
calls in a row with different selections must both match popkv_sparse_attention
run with its own zeroed workspace -- the second call checks that scratch left by
the first is cleared.  This file is collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

import _native
import popkv_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
BF16 = 2


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def test_noalloc_matches_workspace_entry_point_twice():
    lib = _native.c_library()
    lib.popkv_last_error.restype = ctypes.c_char_p
    lib.popkv_sparse_attention_workspace_bytes.restype = ctypes.c_size_t
    I = ctypes.c_int64
    torch.cuda.init()
    g = torch.Generator().manual_seed(17)
    B, KVH, QH, D, L, budget = 1, 8, 32, 128, 4096, 1024
    kc = torch.randn(KVH, L + 1, D, generator=g).bfloat16().to(DEV)
    vc = torch.randn(KVH, L + 1, D, generator=g).bfloat16().to(DEV)
    ck = torch.randn(B, KVH, D, generator=g).bfloat16().to(DEV)
    cv = torch.randn(B, KVH, D, generator=g).bfloat16().to(DEV)
    need = lib.popkv_sparse_attention_workspace_bytes(I(B), I(QH), I(KVH), I(D), I(L), I(0))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        q = torch.randn(B, QH, D, generator=g).bfloat16().to(DEV)
        idx = torch.from_numpy(O.select(torch.randn(B * QH, L, generator=g).numpy(),
                                        budget=budget)).to(DEV)
        ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
        ref = torch.empty_like(q)
        got = torch.full_like(q, float("nan"))
        rc = lib.popkv_sparse_attention(_p(q), BF16, I(B), I(QH), I(D), _p(kc), _p(vc), I(KVH),
                                        I(L + 1), 0, _p(ck), _p(cv), _p(idx), I(budget), I(budget),
                                        I(L), None, _p(ref), _p(ws), ctypes.c_size_t(need), I(0),
                                        stream)
        assert rc == 0, lib.popkv_last_error()
        rc = lib.popkv_sparse_attention_noalloc(_p(q), BF16, I(B), I(QH), I(D), _p(kc), _p(vc),
                                                I(KVH), I(L + 1), 0, _p(ck), _p(cv), _p(idx),
                                                I(budget), I(budget), I(L), None, _p(got), I(0),
                                                stream)
        assert rc == 0, lib.popkv_last_error()
        torch.cuda.synchronize()
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= 2e-2, f"call {call}: max |err| {err}"


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _native.c_library()
    lib.popkv_last_error.restype = ctypes.c_char_p
    I = ctypes.c_int64
    dummy = ctypes.c_void_p(256)
    # 64 sequences x 8 KV heads x 128K tokens needs far more than the fixed scratch.
    rc = lib.popkv_sparse_attention_noalloc(dummy, BF16, I(64), I(32), I(128), dummy, dummy, I(8),
                                            I(131073), 1, None, None, dummy, I(4096), I(4096),
                                            I(131072), None, dummy, I(0), None)
    assert rc == 6
    assert b"scratch" in lib.popkv_last_error()
