"""Generate golden fixtures by running the reference's own Python code on the CPU.

Usage:  python tests/golden/make_golden.py <path-to-reference-checkout>

It imports the reference's ``popkv.py`` (kw78999/FIER-2bits) read-only and
records, for seeded inputs, the outputs of:

  popkv_reference_scores  (popkv.py:283-336)  readable reconstruction scores
  torch.topk + _append_current (popkv.py:594-600, 141-145) on tie-free scores
  gather_selected_kv + selected_attention (popkv.py:341-368)

The inputs are stored beside the outputs so the fixtures are self-contained
(``reference_cpu.npz``).  The committed file is what the tests read; this
script is only re-run to regenerate it.
"""
from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _inputs(seed, kvh, qh, tokens, dim, dtype, outliers=True):
    g = torch.Generator().manual_seed(seed)
    keys = torch.randn(kvh, tokens, dim, generator=g)
    queries = torch.randn(1, qh, dim, generator=g)
    if outliers:
        for h in range(kvh):
            ch = torch.randperm(dim, generator=g)[:4]
            keys[h, :, ch] *= 8.0
            queries[0, h * (qh // kvh):(h + 1) * (qh // kvh), ch] *= 8.0
    return keys.to(dtype), queries.to(dtype)


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    import popkv as ref  # the reference module, imported read-only

    out = {}
    cases = [
        # name, seed, kvh, qh, tokens, dim, dtype
        ("ref_test_shape", 11, 2, 8, 37, 64, torch.bfloat16),   # tests/test_popkv.py:49-51
        ("partial_word_d96", 5, 2, 8, 70, 96, torch.float32),
        ("llama_like_d128", 3, 2, 8, 161, 128, torch.bfloat16),
        ("fp16_one_group", 7, 1, 4, 32, 128, torch.float16),
        ("single_token", 9, 2, 4, 1, 64, torch.float32),
    ]
    for name, seed, kvh, qh, tokens, dim, dtype in cases:
        keys, queries = _inputs(seed, kvh, qh, tokens, dim, dtype)
        mapping = torch.arange(qh) // (qh // kvh)
        scores = ref.popkv_reference_scores(queries, keys, head_to_kv=mapping)
        out[f"{name}/keys"] = keys.float().numpy()
        out[f"{name}/queries"] = queries.float().numpy()
        out[f"{name}/dtype"] = np.array(str(dtype).split(".")[-1])
        out[f"{name}/head_to_kv"] = mapping.numpy()
        out[f"{name}/scores"] = scores.float().numpy()

    # Selection: reference topk + newest append on tie-free scores.
    g = torch.Generator().manual_seed(21)
    for L, budget in ((100, 17), (64, 65), (50, 51), (300, 128)):
        scores = torch.randperm(L * 4, generator=g)[: L * 4].float().view(1, 4, L) / 7.0
        picked = torch.topk(scores, k=min(budget - 1, L), dim=-1, sorted=False).indices[0]
        idx = ref._append_current(picked, L + 1)
        out[f"select_L{L}_b{budget}/scores"] = scores.numpy()
        out[f"select_L{L}_b{budget}/indices_sorted"] = np.concatenate(
            [np.sort(idx[:, :-1].numpy(), axis=1), idx[:, -1:].numpy()], axis=1)

    # Gather + attention.
    g = torch.Generator().manual_seed(33)
    kvh, qh, L, dim, budget = 2, 8, 90, 64, 24
    pk = torch.randn(kvh, L, dim, generator=g).bfloat16()
    pv = torch.randn(kvh, L, dim, generator=g).bfloat16()
    ck = torch.randn(kvh, dim, generator=g).bfloat16()
    cv = torch.randn(kvh, dim, generator=g).bfloat16()
    q = torch.randn(qh, dim, generator=g).bfloat16()
    mapping = torch.arange(qh) // (qh // kvh)
    picked = torch.stack([torch.randperm(L, generator=g)[: budget - 1] for _ in range(qh)])
    idx = ref._append_current(picked, L + 1)
    sk, sv = ref.gather_selected_kv(pk, pv, ck, cv, idx, mapping)
    att = ref.selected_attention(q, sk, sv, None)
    att32 = ref.selected_attention(q.float(), sk.float(), sv.float(), None)
    for key, val in (("prefix_keys", pk), ("prefix_values", pv), ("current_keys", ck),
                     ("current_values", cv), ("queries", q), ("head_to_kv", mapping),
                     ("indices", idx), ("selected_keys", sk), ("selected_values", sv),
                     ("attention_bf16", att), ("attention_fp32", att32)):
        out[f"attention/{key}"] = val.float().numpy() if val.is_floating_point() else val.numpy()

    np.savez_compressed(HERE / "reference_cpu.npz", **out)
    print("wrote", HERE / "reference_cpu.npz", len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(Path.home() / "reference"))
