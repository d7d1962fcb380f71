"""Quest and FIER comparison methods (plain torch) against fixtures from the reference.

The fixtures in tests/golden/reference_baselines.npz come from the reference's own
``build_quest_cache`` / ``quest_scores`` / ``quest_indices`` / ``append_quest``
(popkv.py:150-207) and its FIER Triton kernels run by Triton's CPU interpreter
(fier_triton.py:18-128); tests/golden/make_golden_baselines.py made them.
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest
import torch

import fier_torch
import popkv

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_baselines.npz"


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _cases(prefix):
    names = sorted({k.split("/")[0] for k in np.load(GOLDEN).files})
    return [n for n in names if n.startswith(prefix)]


@pytest.mark.parametrize("name", _cases("quest"))
def test_quest_matches_reference_over_decode_steps(golden, name):
    kvh, qh, tokens, dim, page, budget, steps = (int(x) for x in golden[f"{name}/meta"])
    dtype = getattr(torch, str(golden[f"{name}/dtype"]))
    keys = torch.from_numpy(golden[f"{name}/keys"]).to(dtype)
    mapping = torch.arange(qh) // (qh // kvh)
    cache = popkv.build_quest_cache(keys, page_size=page, reserve_tokens=steps + page)
    n = tokens
    for s in range(steps):
        q = torch.from_numpy(golden[f"{name}/step{s}/queries"]).to(dtype)
        cur = torch.from_numpy(golden[f"{name}/step{s}/current"]).to(dtype)
        scores = popkv.quest_scores(q, cache, cur, mapping)
        np.testing.assert_allclose(scores.numpy(), golden[f"{name}/step{s}/scores"],
                                   rtol=1e-6, atol=1e-6)
        idx, valid = popkv.quest_indices(scores, num_tokens=n + 1, page_size=page, budget=budget)
        ref_idx = golden[f"{name}/step{s}/indices"]
        ref_valid = golden[f"{name}/step{s}/valid"]
        assert idx.shape == ref_idx.shape
        for r in range(qh):  # top-k order is unspecified: compare the valid sets
            ours = set(idx[r][valid[r]].tolist())
            theirs = set(ref_idx[r][ref_valid[r]].tolist())
            assert ours == theirs, (name, s, r)
            assert n in ours  # the newest token is always present
        popkv.append_quest(cache, cur[:, None])
        n += 1


def test_quest_bounds_dominate_exact_scores():
    """Quest's page score is an upper bound of every q.k in the page (tests/test_popkv.py:23-43)."""
    g = torch.Generator().manual_seed(0)
    keys = torch.randn(2, 64, 16, generator=g)
    q = torch.randn(4, 16, generator=g)
    mapping = torch.arange(4) // 2
    cache = popkv.build_quest_cache(keys, page_size=8, reserve_tokens=8)
    cur = torch.randn(2, 16, generator=g)
    bound = popkv.quest_scores(q, cache, cur, mapping)
    exact = torch.einsum("hd,htd->ht", q, keys.index_select(0, mapping))
    per_page = exact.view(4, 8, 8).amax(-1)
    assert torch.all(bound[:, :8] >= per_page - 1e-5)


@pytest.mark.parametrize("name", _cases("fier"))
def test_fier_pack_and_score_match_reference_kernels(golden, name):
    kvh, qh, tokens, dim, gs = (int(x) for x in golden[f"{name}/meta"])
    dtype = getattr(torch, str(golden[f"{name}/dtype"]))
    keys = torch.from_numpy(golden[f"{name}/keys"]).to(dtype).contiguous()
    q = torch.from_numpy(golden[f"{name}/queries"]).to(dtype)
    mapping = torch.arange(qh) // (qh // kvh)
    packed, mins, maxs = fier_torch.pack_keys(keys, group_size=gs)
    assert np.array_equal(packed.numpy(), golden[f"{name}/packed"])
    assert np.array_equal(mins.float().numpy(), golden[f"{name}/mins"])
    assert np.array_equal(maxs.float().numpy(), golden[f"{name}/maxs"])
    scores = fier_torch.score_packed_batched(q, packed, mins, maxs, mapping, tokens=tokens,
                                             group_size=gs)
    ref = golden[f"{name}/scores"]
    scale = np.abs(ref).max()
    np.testing.assert_allclose(scores.numpy(), ref, rtol=1e-5, atol=1e-5 * scale)


def test_fier_cache_stages_the_open_group_like_a_full_pack():
    g = torch.Generator().manual_seed(1)
    keys = torch.randn(2, 45, 64, generator=g)
    cur = torch.randn(2, 64, generator=g)
    mapping = torch.arange(4) // 2
    q = torch.randn(4, 64, generator=g)
    cache = popkv.build_fier_cache(keys, group_size=32, reserve_tokens=8)
    staged = popkv.fier_scores(q, cache, cur[:, None], mapping, num_tokens=46)
    full = fier_torch.score_tensors(q[None], torch.cat([keys, cur[:, None]], 1).contiguous(),
                                    head_to_kv=mapping, group_size=32)
    assert torch.allclose(staged, full, rtol=1e-6, atol=1e-6)
    popkv.append_fier(cache, cur[:, None])
    assert cache.token_count == 46 and cache.sealed_tokens == 32


def test_fier_rejects_bad_arguments():
    with pytest.raises(ValueError):
        fier_torch.pack_keys(torch.randn(4, 8), group_size=32)
    with pytest.raises(ValueError):
        fier_torch.pack_keys(torch.randn(1, 8, 4), group_size=0)
    assert math.isfinite(float(fier_torch.score_tensors(
        torch.randn(1, 2, 8), torch.randn(1, 5, 8), head_to_kv=torch.zeros(2, dtype=torch.long),
        group_size=32).sum()))
