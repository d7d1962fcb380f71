"""The CPU oracle, pinned against outputs of the reference's own code (CPU, no GPU needed).

tests/golden/reference_cpu.npz was produced by tests/golden/make_golden.py, which
imports the reference popkv.py and records popkv_reference_scores, torch.topk +
_append_current and gather_selected_kv + selected_attention on seeded inputs.
"""
import math

import numpy as np
import pytest
import torch

import popkv_oracle as O
import reconstruction as R

SCORE_CASES = ["ref_test_shape", "partial_word_d96", "llama_like_d128", "fp16_one_group",
               "single_token"]


@pytest.mark.parametrize("name", SCORE_CASES)
def test_oracle_scores_match_reference_readable_scores(golden, name):
    keys, queries = golden[f"{name}/keys"], golden[f"{name}/queries"]
    mapping, expected = golden[f"{name}/head_to_kv"], golden[f"{name}/scores"]
    got = O.score(queries, O.pack_keys(keys), head_to_kv=mapping, tokens=keys.shape[1])
    # The reference's own CUDA-vs-readable tolerance (tests/test_popkv.py:54).
    np.testing.assert_allclose(got, expected, atol=0.12, rtol=0.02)
    # Tighter: only fp16 rounding of the key representatives separates the two.
    scale = max(1.0, float(np.abs(expected).max()))
    assert float(np.abs(got - expected).max()) < 1e-3 * scale * 5


@pytest.mark.parametrize("name", SCORE_CASES)
def test_reconstruction_port_matches_reference(golden, name):
    keys, queries = golden[f"{name}/keys"], golden[f"{name}/queries"]
    mapping, expected = golden[f"{name}/head_to_kv"], golden[f"{name}/scores"]
    got = R.reconstruction_scores(torch.from_numpy(queries), torch.from_numpy(keys),
                                  head_to_kv=torch.from_numpy(mapping))
    np.testing.assert_allclose(got.numpy(), expected, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", SCORE_CASES)
def test_oracle_bitmasks_match_reconstruction_thresholds(golden, name):
    keys = golden[f"{name}/keys"]
    kvh, T, D = keys.shape
    (sign, mag, _, _), thr = O.pack_keys(keys, with_thresholds=True)
    k = torch.from_numpy(keys)
    groups = math.ceil(T / 32)
    for g in range(groups):
        blk = k[:, 32 * g: 32 * g + 32]
        np.testing.assert_array_equal(thr[:, g, :, 0], (blk.amin(1) * 0.5).numpy())
        np.testing.assert_array_equal(thr[:, g, :, 1], (blk.amax(1) * 0.5).numpy())
    words = (D + 31) // 32
    for t in range(T):
        g = t // 32
        v = k[:, t]
        s = v >= 0
        m = torch.where(s, v > torch.from_numpy(thr[:, g, :, 1]), v < torch.from_numpy(thr[:, g, :, 0]))
        for w in range(words):
            bits_s = sum(int(s[h, c]) << (c - 32 * w) for h in range(1) for c in range(32 * w, min(D, 32 * w + 32)))
            bits_m = sum(int(m[0, c]) << (c - 32 * w) for c in range(32 * w, min(D, 32 * w + 32)))
            assert (int(sign[0, t, w]) & 0xffffffff) == bits_s
            assert (int(mag[0, t, w]) & 0xffffffff) == bits_m


def _fp16_rn(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def test_oracle_representatives_follow_tree_order_sums():
    rng = np.random.default_rng(4)
    keys = rng.standard_normal((1, 32, 32)).astype(np.float32)
    sign, mag, low, delta = O.pack_keys(keys)
    mn, mx = keys[0].min(0) * np.float32(0.5), keys[0].max(0) * np.float32(0.5)
    for t in range(32):
        v = keys[0, t]
        m = np.where(v >= 0, v > mx, v < mn)
        lo = np.where(~m, np.abs(v), 0).astype(np.float32)
        hi = np.where(m, np.abs(v), 0).astype(np.float32)
        for off in (16, 8, 4, 2, 1):
            lo[:off] = lo[:off] + lo[off: 2 * off]
            hi[:off] = hi[:off] + hi[off: 2 * off]
        lc, hc = int((~m).sum()), int(m.sum())
        l = np.float32(lo[0] / np.float32(lc)) if lc else (np.float32(hi[0] / np.float32(hc)) if hc else np.float32(0))
        h = (np.float32(hi[0] / np.float32(hc)) if hc else l) if lc else l
        assert low[0, t, 0] == _fp16_rn(l)
        assert delta[0, t, 0] == _fp16_rn(np.float32(h - l))


@pytest.mark.parametrize("case", ["select_L100_b17", "select_L64_b65", "select_L50_b51",
                                  "select_L300_b128"])
def test_oracle_select_matches_reference_topk(golden, case):
    scores, expected = golden[f"{case}/scores"], golden[f"{case}/indices_sorted"]
    got = O.select(scores[0], budget=int(case.split("_b")[1]))
    L = scores.shape[-1]
    budget = int(case.split("_b")[1])
    k = min(budget - 1, L)
    np.testing.assert_array_equal(got[:, : k + 1], expected)
    assert (got[:, k + 1:] == -1).all()


def test_oracle_select_ties_go_to_lowest_index():
    scores = np.zeros((2, 10), np.float32)
    scores[0, [3, 7]] = 1.0
    scores[1, 5] = -0.0  # -0.0 ties with +0.0
    got = O.select(scores, budget=5)
    np.testing.assert_array_equal(got[0], [0, 1, 3, 7, 10])
    np.testing.assert_array_equal(got[1], [0, 1, 2, 3, 10])


def test_oracle_attention_matches_reference_gather_and_sdpa(golden):
    g = {k.split("/", 1)[1]: golden[k] for k in golden.files if k.startswith("attention/")}
    L = g["prefix_keys"].shape[1]
    idx = g["indices"].astype(np.int32)
    got = O.attention(g["queries"][None], g["prefix_keys"], g["prefix_values"],
                      head_to_kv=g["head_to_kv"], lengths=[L], indices=idx,
                      cur_keys=g["current_keys"][None], cur_values=g["current_values"][None])
    np.testing.assert_allclose(got[0], g["attention_fp32"], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(got[0], g["attention_bf16"], atol=2e-2)


def test_reconstruction_gather_matches_reference(golden):
    g = {k.split("/", 1)[1]: golden[k] for k in golden.files if k.startswith("attention/")}
    t = {k: torch.from_numpy(v) for k, v in g.items()}
    sk, sv = R.gather_rows(t["prefix_keys"], t["prefix_values"], t["current_keys"],
                           t["current_values"], t["indices"].long(), t["head_to_kv"].long())
    np.testing.assert_array_equal(sk.numpy(), g["selected_keys"])
    np.testing.assert_array_equal(sv.numpy(), g["selected_values"])
    out = R.attend(t["queries"], sk, sv)
    np.testing.assert_allclose(out.numpy(), g["attention_fp32"], atol=1e-5)
