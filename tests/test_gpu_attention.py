"""(f) fused gather + split-K attention against the exact oracle (fp64 accumulation).

Tolerance: 2e-2 absolute for bf16/fp16 caches (the path's stated bound), 1e-4 for
fp32 caches."""
import numpy as np
import pytest
import torch

import popkv_cuda as pk
import popkv_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = {torch.bfloat16: 2e-2, torch.float16: 2e-2, torch.float32: 1e-4}


def _case(B, KVH, QH, D, L, budget, dtype, seed, per_batch=False, dense=False, cur=True,
          lengths=None, splits=0):
    g = torch.Generator().manual_seed(seed)
    heads = B * KVH if per_batch else KVH
    cap = L + 3
    kc = torch.randn(heads, cap, D, generator=g).to(dtype)
    vc = torch.randn(heads, cap, D, generator=g).to(dtype)
    q = (torch.randn(B, QH, D, generator=g) * 2).to(dtype)
    ck = torch.randn(B, KVH, D, generator=g).to(dtype)
    cv = torch.randn(B, KVH, D, generator=g).to(dtype)
    lens = lengths or [L] * B
    idx = None
    if not dense:
        scores = torch.randn(B * QH, L, generator=g)
        idx = O.select(scores.numpy(), budget=budget, lengths=np.repeat(lens, QH))
    kdev = kc.view(B, KVH, cap, D) if per_batch else kc
    vdev = vc.view(B, KVH, cap, D) if per_batch else vc
    sl = torch.tensor(lens, dtype=torch.int32, device=DEV) if lengths else None
    out = pk.sparse_attention(q.to(DEV), kdev.to(DEV).contiguous(), vdev.to(DEV).contiguous(),
                              None if dense else torch.from_numpy(idx).to(DEV), budget=budget,
                              tokens=L, current_keys=ck.to(DEV) if cur else None,
                              current_values=cv.to(DEV) if cur else None, seq_len=sl,
                              splits=splits)
    ref = O.attention(q.float().numpy(), kc.float().numpy(), vc.float().numpy(),
                      head_to_kv=np.arange(QH) // (QH // KVH), lengths=lens, indices=idx,
                      budget=budget, cur_keys=ck.float().numpy() if cur else None,
                      cur_values=cv.float().numpy() if cur else None, cache_per_batch=per_batch,
                      kv_heads=KVH)
    err = np.abs(out.float().cpu().numpy() - ref).max()
    assert err <= TOL[dtype], f"max |err| {err}"
    return err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("D", [64, 96, 128, 256])
def test_attention_dtypes_and_head_dims(dtype, D):
    _case(1, 2, 8, D, 700, 128, dtype, seed=D)


@pytest.mark.parametrize("G", [1, 2, 4, 8, 16])
def test_attention_group_sizes(G):
    _case(1, 2, 2 * G, 128, 3000, 512, torch.bfloat16, seed=G)


@pytest.mark.parametrize("L,budget", [(1, 2), (3, 2), (40, 64), (4096, 1024), (32768, 4096)])
def test_attention_lengths(L, budget):
    _case(1, 8, 32, 128, L, budget, torch.bfloat16, seed=L)


def test_attention_dense_and_cache_current_row():
    _case(1, 2, 8, 128, 5000, 2, torch.bfloat16, seed=1, dense=True)
    _case(1, 2, 8, 128, 900, 64, torch.bfloat16, seed=2, cur=False)


def test_attention_per_batch_caches_and_lengths():
    _case(3, 2, 8, 128, 2000, 256, torch.bfloat16, seed=3, per_batch=True, lengths=[2000, 17, 999])


@pytest.mark.parametrize("splits,L", [(1, 2000), (3, 4000), (64, 4000)])
def test_attention_explicit_splits(splits, L):
    _case(1, 2, 8, 128, L, 512, torch.bfloat16, seed=splits, splits=splits)


def test_attention_rejects_overlong_segments():
    with pytest.raises(RuntimeError, match="segment longer"):
        _case(1, 2, 8, 128, 4000, 512, torch.bfloat16, seed=0, splits=1)


def test_attention_shape_changes_with_default_workspace():
    """Alternating sizes on the shared default workspace stay correct."""
    for L in (700, 3000, 700, 4096, 1500):
        _case(1, 2, 8, 128, L, 256, torch.bfloat16, seed=L)


def test_attention_workspace_reuse_is_clean():
    """Back-to-back calls sharing a workspace give identical results (masks, tickets reset)."""
    g = torch.Generator().manual_seed(7)
    KVH, QH, D, L, budget = 2, 8, 128, 3000, 256
    kc = torch.randn(KVH, L + 1, D, generator=g).bfloat16().to(DEV)
    vc = torch.randn(KVH, L + 1, D, generator=g).bfloat16().to(DEV)
    q = torch.randn(1, QH, D, generator=g).bfloat16().to(DEV)
    idx1 = torch.from_numpy(O.select(torch.randn(QH, L, generator=g).numpy(), budget=budget)).to(DEV)
    idx2 = torch.from_numpy(O.select(torch.randn(QH, L, generator=g).numpy(), budget=budget)).to(DEV)
    ws = pk.new_workspace(1, QH, KVH, D, L, DEV)
    a = pk.sparse_attention(q, kc, vc, idx1, budget=budget, tokens=L, workspace=ws)
    b = pk.sparse_attention(q, kc, vc, idx2, budget=budget, tokens=L, workspace=ws)
    a2 = pk.sparse_attention(q, kc, vc, idx1, budget=budget, tokens=L, workspace=ws)
    torch.testing.assert_close(a, a2, rtol=0, atol=0)
    assert not torch.equal(a, b)


def test_attention_accepts_reference_int64_unsorted_indices():
    """torch.topk(sorted=False) + _append_current output (int64, any order) works as is."""
    g = torch.Generator().manual_seed(8)
    KVH, QH, D, L, budget = 2, 8, 128, 1000, 100
    kc = torch.randn(KVH, L, D, generator=g).bfloat16()
    vc = torch.randn(KVH, L, D, generator=g).bfloat16()
    ck, cv = torch.randn(1, KVH, D, generator=g).bfloat16(), torch.randn(1, KVH, D, generator=g).bfloat16()
    q = torch.randn(1, QH, D, generator=g).bfloat16()
    scores = torch.randn(1, QH, L, generator=g)
    picked = torch.topk(scores, k=budget - 1, dim=-1, sorted=False).indices[0]
    idx = torch.cat([picked, torch.full((QH, 1), L)], dim=-1)
    out = pk.sparse_attention(q.to(DEV), kc.to(DEV), vc.to(DEV), idx.to(DEV), budget=budget,
                              tokens=L, current_keys=ck.to(DEV), current_values=cv.to(DEV))
    h2k = torch.arange(QH) // 4
    ks = torch.where(idx[..., None] == L, ck[0][h2k][:, None], kc[h2k[:, None], idx.clamp_max(L - 1)])
    vs = torch.where(idx[..., None] == L, cv[0][h2k][:, None], vc[h2k[:, None], idx.clamp_max(L - 1)])
    ref = torch.nn.functional.scaled_dot_product_attention(q[0].float()[:, None], ks.float(), vs.float())[:, 0]
    torch.testing.assert_close(out[0].float().cpu(), ref, atol=2e-2, rtol=0)


def test_premasked_attention_matches_index_path():
    """select writing the workspace bitmask + premasked attention == indices + scatter path."""
    g = torch.Generator().manual_seed(21)
    B, KVH, QH, D, L, budget = 2, 4, 16, 128, 20000, 2048
    kc = torch.randn(B, KVH, L + 1, D, generator=g).bfloat16().to(DEV)
    vc = torch.randn(B, KVH, L + 1, D, generator=g).bfloat16().to(DEV)
    q = torch.randn(B, QH, D, generator=g).bfloat16().to(DEV)
    ck = torch.randn(B, KVH, D, generator=g).bfloat16().to(DEV)
    cv = torch.randn(B, KVH, D, generator=g).bfloat16().to(DEV)
    scores = torch.randn(B * QH, L, generator=g).to(DEV)
    lens = torch.tensor([L, 9000], dtype=torch.int32, device=DEV)
    ws = pk.new_workspace(B, QH, KVH, D, L, DEV)
    for _ in range(2):  # the second round checks that the masks were cleared
        idx = pk.select(scores, budget=budget, tokens=L, seq_len=lens, rows_per_seq=QH,
                        attn_workspace=ws, attn_sizes=(B, QH, KVH, D, L, 0))
        got = torch.empty_like(q)
        pk.sparse_attention_premasked(q, kc, vc, tokens=L, current_keys=ck, current_values=cv,
                                      seq_len=lens, workspace=ws, out=got)
        ref = pk.sparse_attention(q, kc, vc, idx, budget=budget, tokens=L, current_keys=ck,
                                  current_values=cv, seq_len=lens)
        torch.testing.assert_close(got, ref, rtol=0, atol=0)
        scores = scores.roll(1, dims=1)
