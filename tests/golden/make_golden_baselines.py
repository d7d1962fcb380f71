"""Golden fixtures for the Quest and FIER comparison methods, from the reference's own code.

Usage:  TRITON_INTERPRET=1 python tests/golden/make_golden_baselines.py <path-to-reference-checkout>

* Quest: the reference's ``build_quest_cache`` / ``quest_scores`` / ``quest_indices`` /
  ``append_quest`` (popkv.py:150-207), run on the CPU over several decode steps.
* FIER: the reference's Triton kernels ``_group_minmax_kernel``, ``_pack_kernel`` and
  ``_score_kernel`` (fier_triton.py:18-128), run on the CPU by Triton's interpreter
  (TRITON_INTERPRET=1; the interpreter has no bf16, so fp32 and fp16 keys only).

Writes ``reference_baselines.npz`` beside this file (inputs stored with the outputs).
"""
from __future__ import annotations

import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def quest_cases(ref, out):
    cases = [
        # name, seed, kvh, qh, tokens, dim, page, budget, steps, dtype
        ("quest_ref_test", 3, 8, 32, 31, 16, 8, 16, 4, torch.bfloat16),  # tests/test_popkv.py:23-43
        ("quest_d64", 5, 2, 8, 100, 64, 16, 64, 5, torch.float32),
        ("quest_small_budget", 7, 2, 4, 40, 32, 8, 5, 3, torch.float16),
    ]
    for name, seed, kvh, qh, tokens, dim, page, budget, steps, dtype in cases:
        g = torch.Generator().manual_seed(seed)
        keys = torch.randn(kvh, tokens, dim, generator=g).to(dtype)
        mapping = torch.arange(qh) // (qh // kvh)
        cache = ref.build_quest_cache(keys, page_size=page, reserve_tokens=steps + page)
        out[f"{name}/keys"] = keys.float().numpy()
        out[f"{name}/meta"] = np.array([kvh, qh, tokens, dim, page, budget, steps])
        out[f"{name}/dtype"] = np.array(str(dtype).split(".")[-1])
        n = tokens
        for s in range(steps):
            q = torch.randn(qh, dim, generator=g).to(dtype)
            cur = torch.randn(kvh, dim, generator=g).to(dtype)
            scores = ref.quest_scores(q, cache, cur, mapping)
            idx, valid = ref.quest_indices(scores, num_tokens=n + 1, page_size=page, budget=budget)
            out[f"{name}/step{s}/queries"] = q.float().numpy()
            out[f"{name}/step{s}/current"] = cur.float().numpy()
            out[f"{name}/step{s}/scores"] = scores.numpy()
            out[f"{name}/step{s}/indices"] = idx.numpy()
            out[f"{name}/step{s}/valid"] = valid.numpy()
            ref.append_quest(cache, cur[:, None])
            n += 1


def fier_cases(out):
    import fier_triton as F
    cases = [
        # name, seed, kvh, qh, tokens, dim, group, dtype
        ("fier_f32_t70", 11, 2, 8, 70, 64, 32, torch.float32),
        ("fier_f16_t257", 12, 2, 8, 257, 128, 32, torch.float16),
        ("fier_f32_t5", 13, 1, 4, 5, 96, 32, torch.float32),
        ("fier_f32_g16", 14, 2, 4, 50, 64, 16, torch.float32),
    ]
    for name, seed, kvh, qh, tokens, dim, gs, dtype in cases:
        g = torch.Generator().manual_seed(seed)
        keys = torch.randn(kvh, tokens, dim, generator=g)
        for h in range(kvh):
            keys[h, :, torch.randperm(dim, generator=g)[:4]] *= 8.0
        keys = keys.to(dtype).contiguous()
        q = torch.randn(1, qh, dim, generator=g).to(dtype)
        mapping = torch.arange(qh) // (qh // kvh)
        groups, words = math.ceil(tokens / gs), math.ceil(tokens / 32)
        mins = torch.empty(kvh, groups, dim, dtype=dtype)
        maxs = torch.empty_like(mins)
        packed = torch.empty(kvh, dim, words, dtype=torch.int32)
        block_group = 1 << (gs - 1).bit_length()
        F._group_minmax_kernel[(kvh * groups * dim,)](
            keys, mins, maxs, tokens=tokens, head_dim=dim, num_groups=groups, group_size=gs,
            BLOCK_GROUP=block_group)
        F._pack_kernel[(kvh * dim * words,)](
            keys, mins, maxs, packed, tokens=tokens, head_dim=dim, num_groups=groups, words=words,
            group_size=gs)
        scores = torch.empty(1, qh, tokens)
        F._score_kernel[(math.ceil(tokens / 32), qh)](
            q, packed, mins, maxs, mapping, scores, tokens=tokens, q_heads=qh, head_dim=dim,
            num_groups=groups, words=words, group_size=gs, BLOCK_D=1 << (dim - 1).bit_length(),
            BLOCK_T=32)
        out[f"{name}/meta"] = np.array([kvh, qh, tokens, dim, gs])
        out[f"{name}/dtype"] = np.array(str(dtype).split(".")[-1])
        out[f"{name}/keys"] = keys.float().numpy()
        out[f"{name}/queries"] = q.float().numpy()
        out[f"{name}/packed"] = packed.numpy()
        out[f"{name}/mins"] = mins.float().numpy()
        out[f"{name}/maxs"] = maxs.float().numpy()
        out[f"{name}/scores"] = scores.numpy()


def main(reference: str) -> None:
    if os.environ.get("TRITON_INTERPRET") != "1":
        raise SystemExit("run with TRITON_INTERPRET=1 (FIER's Triton kernels run on the CPU)")
    sys.path.insert(0, reference)
    import popkv as ref  # the reference module, imported read-only

    out = {}
    quest_cases(ref, out)
    fier_cases(out)
    np.savez_compressed(HERE / "reference_baselines.npz", **out)
    print("wrote", HERE / "reference_baselines.npz", len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(Path.home() / "reference"))
