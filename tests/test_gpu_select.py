"""(e) top-(budget-1) selection with the newest token reserved: bit-exact index sets
(ties to the lowest index) against the oracle; the reference's torch.topk agrees
as a set wherever the threshold is tie-free."""
import numpy as np
import pytest
import torch

import popkv_cuda as pk
import popkv_oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _check(scores: torch.Tensor, budget: int, lengths=None, rows_per_seq=0):
    tokens = scores.shape[-1]
    sl = None if lengths is None else torch.tensor(lengths, dtype=torch.int32, device=DEV)
    got = pk.select(scores.to(DEV), budget=budget, tokens=tokens, seq_len=sl,
                    rows_per_seq=rows_per_seq).cpu().numpy()
    rows = scores.shape[0]
    per_row = None if lengths is None else np.repeat(lengths, rows_per_seq)[:rows]
    ref = O.select(scores.numpy(), budget=budget, lengths=per_row)
    np.testing.assert_array_equal(got, ref)
    # The select-workspace path with an empty histogram (the top digit is then
    # counted inside select) gives the same rows and leaves the histogram zeroed.
    hist = pk.new_select_workspace(rows, tokens, DEV)
    got_ws = pk.select(scores.to(DEV), budget=budget, tokens=tokens, seq_len=sl,
                       rows_per_seq=rows_per_seq, hist=hist).cpu().numpy()
    np.testing.assert_array_equal(got_ws, ref)
    assert int(hist[: rows * 2048 * 4].abs().sum()) == 0
    return got


@pytest.mark.parametrize("L,budget", [(1, 2), (5, 2), (100, 17), (64, 65), (50, 51), (50, 4096),
                                      (1000, 128), (4096, 1024), (32768, 4096), (40000, 4096),
                                      (131072, 4096), (300000, 8192)])
def test_select_random(L, budget):
    g = torch.Generator().manual_seed(L + budget)
    scores = torch.randn(6, L, generator=g) * 5
    _check(scores, budget)


def test_select_matches_reference_topk_sets(golden):
    for case in ("select_L100_b17", "select_L64_b65", "select_L50_b51", "select_L300_b128"):
        scores = torch.from_numpy(golden[f"{case}/scores"][0])
        budget = int(case.split("_b")[1])
        got = _check(scores, budget)
        exp = golden[f"{case}/indices_sorted"]
        k = min(budget - 1, scores.shape[-1])
        np.testing.assert_array_equal(got[:, : k + 1], exp)


def test_select_ties_and_signed_zero():
    L = 5000
    scores = torch.zeros(4, L)
    scores[1, ::7] = 1.0               # ties above the threshold
    scores[2] = torch.randint(0, 3, (L,), generator=torch.Generator().manual_seed(1)).float()
    scores[3, ::2] = -0.0              # -0.0 ties with +0.0
    _check(scores, 300)


def test_select_quantised_scores_many_ties():
    g = torch.Generator().manual_seed(3)
    scores = (torch.randn(32, 32768, generator=g) * 4).round() / 4
    _check(scores, 4096)


def test_select_device_lengths():
    g = torch.Generator().manual_seed(4)
    scores = torch.randn(3 * 8, 20000, generator=g)
    _check(scores, 1024, lengths=[20000, 700, 1023], rows_per_seq=8)


def test_select_agrees_with_torch_topk_as_sets():
    g = torch.Generator().manual_seed(5)
    scores = torch.randn(32, 32768, generator=g)
    got = pk.select(scores.to(DEV), budget=4096).cpu()
    ref = torch.topk(scores.to(DEV), k=4095, dim=-1, sorted=False).indices.cpu()
    for r in range(32):
        assert set(got[r, :4095].tolist()) == set(ref[r].tolist())
        assert got[r, 4095] == 32768


def test_select_rejects_budget_one():
    with pytest.raises(ValueError):
        pk.select(torch.zeros(2, 10, device=DEV), budget=1)


@pytest.mark.parametrize("G,L", [(4, 32768), (4, 3000), (16, 20000), (8, 131072)])
def test_select_with_score_histogram_is_exact(G, L):
    """score(hist=...) -> select(hist=...) equals select without the histogram, and the
    histogram comes back zeroed (heads beyond 8 per KV head fall back inside select)."""
    from conftest import synthetic_keys
    KVH, D, budget = 2, 128, 4096
    QH = KVH * G
    k = synthetic_keys(KVH, L, D, seed=L, dtype=torch.bfloat16).to(DEV)
    q = synthetic_keys(1, QH, D, seed=L + 1, dtype=torch.bfloat16).to(DEV)
    h2k = (torch.arange(QH) // G).to(DEV)
    packed = pk.pack_keys(k)
    hist = pk.new_select_workspace(QH, L, DEV)
    for _ in range(2):
        scores = pk.score(q, packed, head_to_kv=h2k, tokens=L, hist=hist)
        got = pk.select(scores.view(QH, L), budget=budget, hist=hist)
        ref = pk.select(scores.view(QH, L), budget=budget)
        torch.testing.assert_close(got, ref, rtol=0, atol=0)
        assert int(hist[: QH * 2048 * 4].abs().sum()) == 0
        np.testing.assert_array_equal(ref.cpu().numpy(), O.select(scores.view(QH, L).cpu().numpy(), budget=budget))


@pytest.mark.parametrize("L,budget", [(3001, 2990), (33001, 33000), (40960, 40000)])
def test_select_threshold_among_negative_infinities(L, budget):
    """The k-th largest score is -inf (the lowest key bin): padding positions past L
    must not be counted as -inf scores."""
    g = torch.Generator().manual_seed(L)
    scores = torch.randn(3, L, generator=g)
    scores[:, ::2] = float("-inf")
    _check(scores, budget)


@pytest.mark.parametrize("B,L", [(10, 50000), (16, 131072)])
def test_select_many_rows_with_histogram_is_exact(B, L):
    """Batches whose rows fill the GPU many times over take the 512-thread cluster
    path (the configs[3] shape at B=16, L=128K): identical to the oracle's selection."""
    KVH, G, D, budget = 8, 4, 128, 4096
    QH = KVH * G
    g = torch.Generator(device=DEV).manual_seed(B)
    scores = (torch.randn(B * QH, L, generator=g, device=DEV) * 3).round(decimals=2) + 0.0  # ties; no -0
    hist = pk.new_select_workspace(B * QH, L, DEV)
    # The histogram the scorer would have built: counts of the top 11 key bits.
    u = scores.contiguous().view(torch.int32)
    key = torch.where(u < 0, ~u, u | torch.iinfo(torch.int32).min)
    top = ((key >> 21) & 0x7ff).long()
    h = torch.zeros(B * QH, 2048, dtype=torch.int64, device=DEV).scatter_add_(1, top, torch.ones_like(top))
    hist[: B * QH * 2048 * 4].view(torch.int32).copy_(h.view(-1).to(torch.int32))
    got = pk.select(scores, budget=budget, hist=hist)
    ref = pk.select(scores, budget=budget)
    torch.testing.assert_close(got, ref, rtol=0, atol=0)
    assert int(hist[: B * QH * 2048 * 4].abs().sum()) == 0
    rows = [0, B * QH // 2, B * QH - 1]
    np.testing.assert_array_equal(ref[rows].cpu().numpy(), O.select(scores[rows].cpu().numpy(), budget=budget))
