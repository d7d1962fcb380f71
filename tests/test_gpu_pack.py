"""(a) key packer and (b) open-group append: bit-exact against the CPU oracle."""
import numpy as np
import pytest
import torch

import popkv
import popkv_cuda as pk
import popkv_oracle as O
from conftest import packed_numpy, synthetic_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("tokens,dim", [(1, 64), (31, 128), (32, 128), (33, 96), (37, 64),
                                        (100, 128), (257, 256), (45, 80), (64, 32)])
def test_pack_bit_exact(dtype, tokens, dim):
    k = synthetic_keys(3, tokens, dim, seed=tokens * 7 + dim, dtype=dtype)
    cap = tokens + 40
    got = pk.pack_keys(k.to(DEV), token_capacity=cap, with_thresholds=True)
    torch.cuda.synchronize()
    (ref, thr) = O.pack_keys(k.float().numpy(), capacity=cap, with_thresholds=True)
    gotn = packed_numpy(got[:4])
    for name, a, b in zip(("k_sign", "k_mag", "low", "delta"), gotn, ref):
        np.testing.assert_array_equal(a[:, :tokens], b[:, :tokens], err_msg=name)
    np.testing.assert_array_equal(got[4].cpu().numpy(), thr)


def test_pack_full_size_llama_layer():
    """configs[1] layer: 8 KV heads x 32768 tokens x 128, bf16 -- bit-exact."""
    k = synthetic_keys(8, 32768, 128, seed=0, dtype=torch.bfloat16)
    got = packed_numpy(pk.pack_keys(k.to(DEV), token_capacity=32768 + 256))
    ref = O.pack_keys(k.float().numpy(), capacity=32768 + 256)
    for name, a, b in zip(("k_sign", "k_mag", "low", "delta"), got, ref):
        np.testing.assert_array_equal(a[:, :32768], b[:, :32768], err_msg=name)


def test_pack_into_offset_and_errors():
    k = synthetic_keys(2, 20, 128, seed=5, dtype=torch.bfloat16).to(DEV)
    packed = pk.pack_keys(torch.zeros(2, 64, 128, dtype=torch.bfloat16, device=DEV), token_capacity=64)
    pk.pack_keys_into(k, packed, token_offset=32)
    ref = O.pack_keys(k.float().cpu().numpy(), capacity=64, token_offset=32)
    for a, b in zip(packed_numpy(packed), ref):
        np.testing.assert_array_equal(a[:, 32:52], b[:, 32:52])
    with pytest.raises(RuntimeError, match="capacity"):
        pk.pack_keys_into(k, packed, token_offset=50)
    with pytest.raises(ValueError):
        pk.pack_keys_into(k.transpose(1, 2), packed, token_offset=0)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("offset", [0, 3, 96])
def test_pack_many_groups_through_c_abi(dtype, offset):
    """Streaming packer through popkv_pack: more groups than CTAs (the stage ring
    wraps), a ragged last group, vector and scalar output stores, and 3 heads read
    with a head stride larger than tokens * head_dim."""
    import ctypes

    import _native

    lib = _native.c_library()
    lib.popkv_last_error.restype = ctypes.c_char_p
    H, T, D = 3, 32 * 700 + 13, 128
    full = synthetic_keys(H, T + 64, D, seed=11, dtype=dtype).to(DEV)
    cap = T + offset + 16
    packed = [torch.zeros(H, cap, D // 32, dtype=dt, device=DEV)
              for dt in (torch.int32, torch.int32, torch.float16, torch.float16)]
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]
    I = ctypes.c_int64
    ptr = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.popkv_pack(ptr(full), code, I(H), I(T), I(D), I((T + 64) * D), *map(ptr, packed),
                        I(cap), I(offset), None, 0,
                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, lib.popkv_last_error()
    torch.cuda.synchronize()
    ref = O.pack_keys(full[:, :T].float().cpu().numpy(), capacity=cap, token_offset=offset)
    for name, a, b in zip(("k_sign", "k_mag", "low", "delta"), packed_numpy(packed), ref):
        np.testing.assert_array_equal(a[:, offset:offset + T], b[:, offset:offset + T], err_msg=name)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_pack_special_values(dtype):
    """Subnormals, signed zeros, the largest finite values and constant channels:
    the paired 16-bit comparisons (v+v against max/min) must agree with the oracle's
    fp32 thresholds."""
    g = torch.Generator().manual_seed(5)
    finfo = torch.finfo(dtype)
    k = torch.randn(2, 96, 64, generator=g)
    k[:, ::3, 5] = 0.0
    k[:, 1::3, 5] = -0.0
    k[:, :, 7] = -0.0                                    # constant -0 channel
    k[:, :, 9] = 3.0                                     # constant channel
    k[:, ::2, 11] = finfo.max
    k[:, 1::2, 11] = -finfo.max
    k[:, :, 13] = finfo.max / 64 * torch.rand(2, 96, generator=g)
    sub = finfo.smallest_normal
    k[:, :, 17] = sub * torch.randint(-8, 9, (2, 96), generator=g) / 8   # subnormals / zeros
    k[:, :, 19] = sub * (1 + torch.rand(2, 96, generator=g))            # around the smallest normal
    k[:, :, 23] = -sub * torch.rand(2, 96, generator=g)
    k = k.to(dtype)
    got = pk.pack_keys(k.to(DEV), token_capacity=96, with_thresholds=True)
    torch.cuda.synchronize()
    (ref, thr) = O.pack_keys(k.float().numpy(), capacity=96, with_thresholds=True)
    for name, a, b in zip(("k_sign", "k_mag", "low", "delta"), packed_numpy(got[:4]), ref):
        np.testing.assert_array_equal(a, b, err_msg=name)
    np.testing.assert_array_equal(got[4].cpu().numpy(), thr)


def test_incremental_append_matches_full_pack():
    """build_popkv_cache + append_popkv over 70 tokens equals packing all of them at once."""
    k = synthetic_keys(4, 130, 128, seed=9, dtype=torch.bfloat16).to(DEV)
    cache = popkv.build_popkv_cache(k[:, :60].contiguous(), group_size=32, reserve_tokens=80)
    for t in range(60, 130):
        popkv.append_popkv(cache, k[:, t: t + 1])
        assert cache.token_count == t + 1
        assert cache.sealed_tokens == ((t + 1) // 32) * 32
        if t in (63, 64, 95, 100, 129):
            ref = O.pack_keys(k[:, : t + 1].float().cpu().numpy(), capacity=cache.capacity)
            for a, b in zip(packed_numpy(cache.packed), ref):
                np.testing.assert_array_equal(a[:, : t + 1], b[:, : t + 1])


def test_fused_append_writes_caches_and_repacks():
    B, H, D, cap = 2, 4, 128, 96
    k = synthetic_keys(B * H, 70, D, seed=3, dtype=torch.bfloat16).view(B, H, 70, D)
    v = synthetic_keys(B * H, 70, D, seed=4, dtype=torch.bfloat16).view(B, H, 70, D)
    kc = torch.zeros(B, H, cap, D, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    lens = [50, 61]
    for b in range(B):
        kc[b, :, : lens[b]] = k[b, :, : lens[b]].to(DEV)
        vc[b, :, : lens[b]] = v[b, :, : lens[b]].to(DEV)
    packed = tuple(torch.zeros(B, H, cap, 4, dtype=dt, device=DEV)
                   for dt in (torch.int32, torch.int32, torch.float16, torch.float16))
    seq_len = torch.tensor(lens, dtype=torch.int32, device=DEV)
    new_k = torch.stack([k[b, :, lens[b]] for b in range(B)]).to(DEV)
    new_v = torch.stack([v[b, :, lens[b]] for b in range(B)]).to(DEV)
    pk.append_keys(kc, vc, new_k, new_v, packed, position=0, seq_len=seq_len, kv_heads_per_seq=H)
    pk.advance(seq_len)
    torch.cuda.synchronize()
    assert seq_len.tolist() == [51, 62]
    got = packed_numpy(packed)
    for b in range(B):
        P = lens[b]
        torch.testing.assert_close(kc[b, :, P].cpu(), k[b, :, P])
        torch.testing.assert_close(vc[b, :, P].cpu(), v[b, :, P])
        g0 = (P // 32) * 32
        ref = O.pack_keys(k[b, :, g0: P + 1].float().numpy(), capacity=cap, token_offset=g0)
        for a, r in zip(got, ref):
            np.testing.assert_array_equal(a[b, :, g0: P + 1], r[:, g0: P + 1])
