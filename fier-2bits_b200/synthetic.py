"""Seeded synthetic Llama-shaped caches and queries for the retrieval path.

Stand-in for the PG19 / LongBench inputs the reference measures on (those
datasets and checkpoints are not available offline).  Distribution:

* K, V, Q ~ N(0, 1);
* 4 fixed outlier channels per KV head (``randperm(D)[:4]``, drawn once per
  KV head; a query head reuses the channels of its KV head) scaled x8 before
  the rotary embedding;
* rotate-half RoPE with theta = 500000 (the Llama-3.1 base; the reference's
  _rotate_half/_apply_rope, popkv.py:389-398): keys at positions 0..L-1, the
  query (and the appended token) at position L, L+1, ...
"""
from __future__ import annotations

import torch

ROPE_THETA = 500000.0


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float = ROPE_THETA):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    ang = torch.cat([ang, ang], dim=-1)
    return ang.cos().float(), ang.sin().float()


def apply_rope(x: torch.Tensor, positions: torch.Tensor, theta: float = ROPE_THETA) -> torch.Tensor:
    """x [..., T, D] (float32) rotated at ``positions`` [T]."""
    cos, sin = rope_tables(positions, x.shape[-1], theta)
    cos, sin = cos.to(x.device), sin.to(x.device)
    half = x.shape[-1] // 2
    rotated = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rotated * sin


class SyntheticLayer:
    """Generator of one attention layer's K/V cache and decode-time inputs."""

    def __init__(self, *, kv_heads: int, q_heads: int, head_dim: int, seed: int = 0,
                 batch: int = 1, outliers: int = 4, outlier_scale: float = 8.0, device=None):
        self.kv_heads, self.q_heads, self.head_dim, self.batch = kv_heads, q_heads, head_dim, batch
        self.group = q_heads // kv_heads
        self.device = torch.device(device or "cpu")
        picker = torch.Generator().manual_seed(seed)
        scale = torch.ones(kv_heads, head_dim)
        for h in range(kv_heads):
            scale[h, torch.randperm(head_dim, generator=picker)[:outliers]] = outlier_scale
        self.gen = torch.Generator(device=self.device).manual_seed(seed + 1)
        self.kv_scale = scale.to(self.device)
        self.q_scale = scale.repeat_interleave(self.group, dim=0).to(self.device)

    def keys_values(self, tokens: int, start: int = 0):
        """float32 K, V of shape [batch, KVH, tokens, D] at positions start..start+tokens-1."""
        shape = (self.batch, self.kv_heads, tokens, self.head_dim)
        k = torch.randn(shape, generator=self.gen, device=self.device) * self.kv_scale[None, :, None, :]
        v = torch.randn(shape, generator=self.gen, device=self.device)
        pos = torch.arange(start, start + tokens)
        return apply_rope(k, pos), v

    def queries(self, position: int):
        """float32 queries [batch, QH, D] at ``position``."""
        q = torch.randn(self.batch, self.q_heads, 1, self.head_dim, generator=self.gen,
                        device=self.device)
        q = q * self.q_scale[None, :, None, :]
        return apply_rope(q, torch.tensor([position]))[:, :, 0]
