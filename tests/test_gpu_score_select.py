"""Fused score + select (popkv_score_select) against the two-kernel form and the oracle.

One cluster per row scores its slices into shared memory and selects from there;
the indices and the attention head bitmask must equal popkv_score followed by
popkv_select bit for bit (and the oracle's select over the oracle's scores),
across cluster sizes (1..8 CTAs), both CTA widths (1024 and 512 threads), per-
sequence lengths, batched and shared caches, non-standard head maps, ties and
the k == L / k == 0 corners (reference popkv.py:587-600)."""
import numpy as np
import pytest
import torch

import popkv_cuda as pk
import popkv_oracle as O
from conftest import synthetic_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(B, KVH, QH, L, seed, dtype=torch.bfloat16, batched=True, cap_extra=40):
    g = torch.Generator().manual_seed(seed)
    H = B * KVH if batched else KVH
    k = synthetic_keys(H, L, 128, seed=seed, dtype=dtype)
    cap = L + cap_extra
    packed = pk.pack_keys(k.to(DEV), token_capacity=cap)
    if batched:
        packed = tuple(t.view(B, KVH, cap, 4) for t in packed)
    q = torch.randn(B, QH, 128, generator=g).to(dtype)
    return k, packed, q


def _two_kernel(q, packed, h2k, budget, L, seq_len=None, sizes=None, ws=None):
    B, QH = q.shape[:2]
    hist = pk.new_select_workspace(B * QH, L, q.device)
    scores = pk.score(q, packed, head_to_kv=h2k, tokens=L, seq_len=seq_len, hist=hist)
    return pk.select(scores.view(B * QH, L), budget=budget, tokens=L, seq_len=seq_len,
                     rows_per_seq=QH, attn_workspace=ws, attn_sizes=sizes or (), hist=hist)


@pytest.mark.parametrize("B,KVH,QH,L,budget", [
    (1, 8, 32, 32768, 4096),    # configs[1]: 4 CTAs per row
    (1, 2, 8, 5000, 512),       # few rows: 8 CTAs per row
    (2, 4, 16, 300, 64),        # short rows: 1 CTA
    (4, 8, 32, 131072, 4096),   # long batched rows: 512-thread CTAs, 8 per row
    (3, 2, 4, 2000, 2000),      # budget - 1 >= L: every token
    (2, 8, 32, 1, 8),           # L = 1
])
def test_fused_equals_two_kernel(B, KVH, QH, L, budget):
    k, packed, q = _case(B, KVH, QH, L, seed=L + B)
    qd = q.to(DEV)
    h2k = (torch.arange(QH) // (QH // KVH)).to(DEV)
    fused = pk.score_select(qd, packed, head_to_kv=h2k, budget=budget, tokens=L)
    ref = _two_kernel(qd, packed, h2k, budget, L)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(fused.cpu().numpy(), ref.cpu().numpy())


def test_fused_matches_oracle_with_lengths_masks_and_head_map():
    """Per-sequence lengths, a shared (unbatched) cache, a permuted head map, fp16
    queries, and the head bitmask consumed by the premasked attention."""
    B, KVH, QH, L, budget = 3, 4, 16, 9000, 700
    k, packed, q = _case(B, KVH, QH, L, seed=4, dtype=torch.float16, batched=False)
    h2k_np = np.array([(h * 5) % QH // (QH // KVH) for h in range(QH)])
    # Each KV head still serves QH/KVH query heads (needed by the head masks).
    assert sorted(np.bincount(h2k_np).tolist()) == [QH // KVH] * KVH
    h2k = torch.from_numpy(h2k_np).to(DEV)
    lens = torch.tensor([9000, 4321, 77], dtype=torch.int32, device=DEV)
    qd = q.to(DEV)
    got = pk.score_select(qd, packed, head_to_kv=h2k, budget=budget, tokens=L, seq_len=lens)
    ref = _two_kernel(qd, packed, h2k, budget, L, seq_len=lens)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())
    pn = tuple(t.cpu() for t in packed)
    pn = (pn[0].numpy(), pn[1].numpy(), pn[2].view(torch.int16).numpy().view(np.uint16),
          pn[3].view(torch.int16).numpy().view(np.uint16))
    for b, Lb in enumerate(lens.tolist()):
        sc = O.score(q[b: b + 1].float().numpy(), pn, head_to_kv=h2k_np, tokens=Lb)
        want = O.select(sc.reshape(QH, Lb), budget=budget)
        np.testing.assert_array_equal(got.cpu().numpy()[b * QH:(b + 1) * QH], want)


def test_fused_head_masks_equal_two_kernel():
    B, KVH, QH, L, budget = 2, 8, 32, 20000, 1024
    k, packed, q = _case(B, KVH, QH, L, seed=9)
    qd = q.to(DEV)
    h2k = (torch.arange(QH) // (QH // KVH)).to(DEV)
    sizes = (B, QH, KVH, 128, L, 0)
    ws_a = pk.new_workspace(B, QH, KVH, 128, L, DEV)
    ws_b = pk.new_workspace(B, QH, KVH, 128, L, DEV)
    a = pk.score_select(qd, packed, head_to_kv=h2k, budget=budget, tokens=L,
                        attn_workspace=ws_a, attn_sizes=sizes)
    b = _two_kernel(qd, packed, h2k, budget, L, sizes=sizes, ws=ws_b)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(a.cpu().numpy(), b.cpu().numpy())
    assert torch.equal(ws_a, ws_b)


def test_fused_ties_and_repeated_calls():
    """Constant keys (every score tied): the lowest indices win; two calls in a row
    give the same answer (no state carried between calls)."""
    B, KVH, QH, L, budget = 1, 2, 8, 40000, 300
    k = torch.ones(KVH, L, 128, dtype=torch.bfloat16)
    packed = pk.pack_keys(k.to(DEV), token_capacity=L + 8)
    q = torch.randn(B, QH, 128).bfloat16().to(DEV)
    h2k = (torch.arange(QH) // (QH // KVH)).to(DEV)
    for _ in range(2):
        got = pk.score_select(q, packed, head_to_kv=h2k, budget=budget, tokens=L).cpu().numpy()
        want = np.concatenate([np.arange(budget - 1), [L]])
        for r in range(B * QH):
            np.testing.assert_array_equal(got[r], want)


def test_fused_falls_back_for_other_head_dims():
    """head_dim 64 is not fused: with a score buffer and a workspace the call runs
    the two kernels; without them it is rejected."""
    B, KVH, QH, L, budget = 1, 2, 8, 1000, 100
    k = synthetic_keys(KVH, L, 64, seed=2, dtype=torch.bfloat16)
    packed = pk.pack_keys(k.to(DEV), token_capacity=L)
    q = torch.randn(B, QH, 64).bfloat16().to(DEV)
    h2k = (torch.arange(QH) // (QH // KVH)).to(DEV)
    with pytest.raises(RuntimeError, match="two-kernel"):
        pk.score_select(q, packed, head_to_kv=h2k, budget=budget, tokens=L)
    scores = torch.empty(B * QH, L, device=DEV)
    hist = pk.new_select_workspace(B * QH, L, DEV)
    got = pk.score_select(q, packed, head_to_kv=h2k, budget=budget, tokens=L, scores=scores, hist=hist)
    ref = _two_kernel(q, packed, h2k, budget, L)
    np.testing.assert_array_equal(got.cpu().numpy(), ref.cpu().numpy())
