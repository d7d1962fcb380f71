"""Readable Pop-KV reconstruction path on the CPU -- TEST INFRASTRUCTURE ONLY.

A torch (CPU) restatement of the reference's own CPU path for one decode step:

  reconstruction_scores  popkv.py:283-336  popkv_reference_scores: explicit
                         q-hat / k-hat rebuilt from sign, magnitude and fp32
                         representatives, then a dot product scaled by 1/sqrt(D)
  topk_with_newest       popkv.py:594-600 torch.topk(sorted=False) + popkv.py:141-145
  gather_rows            popkv.py:341-357 gather_selected_kv
  attend                 popkv.py:360-368 selected_attention (SDPA)

It is the reference-semantics check for the CUDA path (at the reference
test's own tolerance, tests/test_popkv.py:54) and the timed CPU baseline of
``bench.py``.  It re-derives the packing of every key on every call, exactly
as the reference's CPU path does, so its "score" time includes packing.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def _word_representatives(x: torch.Tensor, magnitude: torch.Tensor):
    """Mean |x| of the low and high lanes of every 32-channel word (fp32).

    Same fallbacks as the reference: an empty side copies the other side.
    """
    dim = x.shape[-1]
    words = (dim + 31) // 32
    pad = words * 32 - dim
    absolute = x.abs()
    valid = torch.ones_like(magnitude)
    if pad:
        absolute = F.pad(absolute, (0, pad))
        magnitude = F.pad(magnitude, (0, pad), value=False)
        valid = F.pad(valid, (0, pad), value=False)
    shape = (*x.shape[:-1], words, 32)
    absolute, magnitude, valid = absolute.view(shape), magnitude.view(shape), valid.view(shape)
    high_lanes = magnitude & valid
    low_lanes = valid & ~magnitude
    n_low, n_high = low_lanes.sum(-1), high_lanes.sum(-1)
    low = (absolute * low_lanes).sum(-1) / n_low.clamp_min(1)
    high = (absolute * high_lanes).sum(-1) / n_high.clamp_min(1)
    low = torch.where(n_low > 0, low, high)
    high = torch.where(n_high > 0, high, low)
    return low, high


def _signed_reconstruction(x, sign, magnitude, low, high):
    dim = x.shape[-1]
    low_c = low.repeat_interleave(32, -1)[..., :dim]
    high_c = high.repeat_interleave(32, -1)[..., :dim]
    return torch.where(sign, 1.0, -1.0) * torch.where(magnitude, high_c, low_c)


def reconstruction_scores(queries: torch.Tensor, keys: torch.Tensor, *, head_to_kv: torch.Tensor,
                          group_size: int = 32) -> torch.Tensor:
    """queries [B, QH, D], keys [KVH, T, D] -> fp32 [B, QH, T]."""
    q = queries.float()
    q_neg = q.amin(-1, keepdim=True) * 0.5
    q_pos = q.amax(-1, keepdim=True) * 0.5
    q_sign = q >= 0
    q_mag = torch.where(q_sign, q > q_pos, q < q_neg)
    q_hat = _signed_reconstruction(q, q_sign, q_mag, *_word_representatives(q, q_mag))

    k = keys.float()
    kv_heads, tokens, dim = k.shape
    groups = math.ceil(tokens / group_size)
    pad = groups * group_size - tokens
    lo_src = F.pad(k, (0, 0, 0, pad), value=float("inf")) if pad else k
    hi_src = F.pad(k, (0, 0, 0, pad), value=float("-inf")) if pad else k
    g_min = lo_src.view(kv_heads, groups, group_size, dim).amin(2)
    g_max = hi_src.view(kv_heads, groups, group_size, dim).amax(2)
    which = torch.arange(tokens) // group_size
    k_neg, k_pos = g_min[:, which] * 0.5, g_max[:, which] * 0.5
    k_sign = k >= 0
    k_mag = torch.where(k_sign, k > k_pos, k < k_neg)
    k_low, k_high = _word_representatives(k, k_mag)
    h2k = head_to_kv.long().cpu()
    k_hat = _signed_reconstruction(
        k.index_select(0, h2k), k_sign.index_select(0, h2k), k_mag.index_select(0, h2k),
        k_low.index_select(0, h2k), k_high.index_select(0, h2k))
    return torch.einsum("bhd,htd->bht", q_hat, k_hat) / math.sqrt(dim)


def topk_with_newest(scores: torch.Tensor, *, budget: int, prefix_length: int) -> torch.Tensor:
    """[1, QH, L] scores -> int64 [QH, min(budget-1, L)+1]; last column is L."""
    picked = torch.topk(scores, k=min(budget - 1, prefix_length), dim=-1, sorted=False).indices[0]
    newest = torch.full((*picked.shape[:-1], 1), prefix_length, dtype=torch.long)
    return torch.cat([picked.long(), newest], dim=-1)


def gather_rows(prefix_keys, prefix_values, current_keys, current_values, indices, head_to_kv):
    """Materialised gather, index L taken from the current token's k/v."""
    prefix = int(prefix_keys.shape[1])
    clamped = indices.clamp_max(prefix - 1)
    heads = head_to_kv[:, None].expand_as(clamped)
    k_sel, v_sel = prefix_keys[heads, clamped], prefix_values[heads, clamped]
    is_current = indices.eq(prefix).unsqueeze(-1)
    k_cur = current_keys.index_select(0, head_to_kv)[:, None]
    v_cur = current_values.index_select(0, head_to_kv)[:, None]
    return torch.where(is_current, k_cur, k_sel), torch.where(is_current, v_cur, v_sel)


def attend(queries, keys, values):
    """queries [QH, D], keys/values [QH, n, D] -> [QH, D] (one query per head)."""
    return F.scaled_dot_product_attention(queries[None, :, None], keys[None], values[None],
                                          dropout_p=0.0, is_causal=False)[0, :, 0]


def decode_step(queries, prefix_keys, prefix_values, current_keys, current_values, *,
                head_to_kv, budget):
    """One layer of the reference CPU path. queries [QH, D]; caches [KVH, L, D]."""
    L = int(prefix_keys.shape[1])
    scores = reconstruction_scores(queries[None], prefix_keys, head_to_kv=head_to_kv)
    indices = topk_with_newest(scores, budget=budget, prefix_length=L)
    k_sel, v_sel = gather_rows(prefix_keys, prefix_values, current_keys, current_values,
                               indices, head_to_kv)
    return attend(queries, k_sel, v_sel), scores, indices
