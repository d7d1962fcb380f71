"""FIER's group-wise 1-bit key retrieval, in plain torch (no Triton).

Drop-in for the reference module ``fier_triton.py`` (kw78999/FIER-2bits): the same
``pack_keys`` / ``score_packed_batched`` / ``score_tensors`` signatures, layouts and
argument checks.  FIER is a comparison method of the reference, not the Pop-KV hot
path, so it is written with torch tensor ops on whatever device the inputs live on.

Layout (fier_triton.py:151-179):
  packed  int32 [KVH, D, ceil(T/32)]: bit (t % 32) of word t // 32 of channel d is
          key[t, d] >= (group_min + group_max) / 2 of t's group (fp32 compare);
  mins/maxs [KVH, ceil(T/group_size), D] in the key dtype: per-group channel extrema.
Score (fier_triton.py:80-128): sum_d q[d] * (bit ? max : min) in fp32.
"""
from __future__ import annotations

import math

import torch


def _validate_keys(keys: torch.Tensor, group_size: int) -> None:
    """Argument checks of fier_triton.py:131-141 (without its CUDA-only rule)."""
    if keys.ndim != 3:
        raise ValueError("keys must be [KVH, T, D]")
    if not keys.is_contiguous():
        raise ValueError("keys must be contiguous")
    if keys.shape[1] <= 0 or keys.shape[2] <= 0:
        raise ValueError("keys must have non-empty token and head dimensions")
    if group_size <= 0 or group_size > 1024:
        raise ValueError("group_size must be in [1, 1024]")


def group_extrema(keys: torch.Tensor, group_size: int):
    """Per-(head, group, channel) min and max over the group's tokens (partial last group)."""
    kvh, tokens, dim = keys.shape
    groups = math.ceil(tokens / group_size)
    pad = groups * group_size - tokens
    k = keys.float()
    lo_src = torch.nn.functional.pad(k, (0, 0, 0, pad), value=math.inf) if pad else k
    hi_src = torch.nn.functional.pad(k, (0, 0, 0, pad), value=-math.inf) if pad else k
    mins = lo_src.view(kvh, groups, group_size, dim).amin(dim=2)
    maxs = hi_src.view(kvh, groups, group_size, dim).amax(dim=2)
    return mins.to(keys.dtype), maxs.to(keys.dtype)


def _pack_bits(bits: torch.Tensor) -> torch.Tensor:
    """bool [KVH, T, D] -> int32 [KVH, D, ceil(T/32)] (token t -> bit t % 32)."""
    kvh, tokens, dim = bits.shape
    words = math.ceil(tokens / 32)
    pad = words * 32 - tokens
    b = bits.transpose(1, 2).to(torch.int64)
    if pad:
        b = torch.nn.functional.pad(b, (0, pad))
    weights = torch.bitwise_left_shift(torch.ones(32, dtype=torch.int64, device=bits.device),
                                       torch.arange(32, device=bits.device))
    word = (b.view(kvh, dim, words, 32) * weights).sum(-1)
    # Keep the low 32 bits as a signed int32 (bit 31 set -> negative).
    word = torch.where(word >= 2 ** 31, word - 2 ** 32, word)
    return word.to(torch.int32)


def pack_keys(keys: torch.Tensor, *, group_size: int):
    """Pack [KVH, T, D] keys and return (bits, group_min, group_max) (fier_triton.py:144-179)."""
    keys = keys.contiguous()
    _validate_keys(keys, int(group_size))
    tokens = int(keys.shape[1])
    mins, maxs = group_extrema(keys, int(group_size))
    group_of = torch.arange(tokens, device=keys.device) // int(group_size)
    # The midpoint is formed in the key dtype (the sum rounds to it, as the
    # reference's packer adds the two stored extrema), then compared in fp32.
    mid = ((mins + maxs) * 0.5).float()[:, group_of]
    return _pack_bits(keys.float() >= mid), mins, maxs


def score_packed_batched(queries: torch.Tensor, packed: torch.Tensor, mins: torch.Tensor,
                         maxs: torch.Tensor, head_to_kv: torch.Tensor, *, tokens: int,
                         group_size: int) -> torch.Tensor:
    """Dequantised scores for queries [B, QH, D] -> fp32 [B, QH, tokens] (fier_triton.py:182-249)."""
    if queries.ndim != 3 or packed.ndim != 3:
        raise ValueError("queries and packed keys must be rank 3")
    if queries.device != packed.device:
        raise RuntimeError("all FIER tensors must share a device")
    batch, q_heads, head_dim = (int(v) for v in queries.shape)
    if int(packed.shape[1]) != head_dim:
        raise ValueError("query/key head_dim mismatch")
    if mins.shape != maxs.shape or mins.ndim != 3:
        raise ValueError("group min/max tensors must have matching rank-3 shapes")
    if int(mins.shape[0]) != int(packed.shape[0]):
        raise ValueError("packed key and metadata KV-head counts differ")
    if tokens <= 0 or tokens > int(packed.shape[2]) * 32:
        raise ValueError("tokens is inconsistent with packed key storage")
    if int(mins.shape[1]) < math.ceil(tokens / group_size) or int(mins.shape[2]) != head_dim:
        raise ValueError("metadata capacity is inconsistent with tokens/group_size")
    if head_to_kv.numel() != q_heads:
        raise ValueError("head_to_kv must contain one entry per query head")
    h2k = head_to_kv.to(device=queries.device, dtype=torch.int64)
    t = torch.arange(tokens, device=queries.device)
    words = packed[:, :, t // 32]                                    # [KVH, D, T]
    bits = torch.bitwise_and(torch.bitwise_right_shift(words, (t % 32).to(torch.int32)), 1)
    g = t // group_size
    lo = mins[:, g].float().transpose(1, 2)                           # [KVH, D, T]
    hi = maxs[:, g].float().transpose(1, 2)
    deq = torch.where(bits != 0, hi, lo)                              # [KVH, D, T]
    per_head = deq.index_select(0, h2k)                               # [QH, D, T]
    return torch.einsum("bhd,hdt->bht", queries.float(), per_head)


def score_tensors(queries: torch.Tensor, keys: torch.Tensor, *, head_to_kv: torch.Tensor,
                  group_size: int) -> torch.Tensor:
    packed, mins, maxs = pack_keys(keys, group_size=group_size)
    return score_packed_batched(queries, packed, mins, maxs, head_to_kv,
                                tokens=int(keys.shape[1]), group_size=group_size)
