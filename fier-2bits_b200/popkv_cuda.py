"""Pop-KV CUDA entry points on B200 (sm_100a).

Drop-in for the reference module ``popkv_cuda.py`` (kw78999/FIER-2bits): the same
``pack_keys`` / ``pack_keys_into`` / ``score`` signatures, argument meaning and
errors (``ValueError`` for non-3-D, non-CUDA or non-contiguous inputs,
popkv_cuda.py:27-28,34-35,41-42; ``RuntimeError`` without a GPU, popkv_cuda.py:14-15;
``RuntimeError`` from the native checks, csrc/popkv_ext.cu:199-241), plus the rest
of the decode-time retrieval path as native kernels:

  append_keys        static-cache write + open-group re-pack   (popkv.py:270-280, 487-495)
  select             top-(budget-1) + newest token              (popkv.py:594-600, 141-145)
  sparse_attention   fused gather + exact split-K attention     (popkv.py:341-368)
  retrieve           score -> select -> sparse_attention

Every call is asynchronous on the current CUDA stream and goes through the thin
torch extension ``lib/_popkv_torch*.so`` over the C ABI ``libpopkv_b200.so``.
There is no CPU fallback: without the built extension or a GPU, calls raise.
"""
from __future__ import annotations

from typing import Sequence

import torch

from _native import extension

# Flag: divide like a --use_fast_math build of the reference extension (see the C header).
REFERENCE_DIVISION = 1
# Flag: score_select takes the two-kernel path (score buffer + select).
UNFUSED_SELECT = 2


def _packed(packed) -> Sequence[torch.Tensor]:
    if len(packed) != 4:
        raise ValueError("packed cache is (k_sign, k_mag, low, delta)")
    return packed


def pack_keys(keys: torch.Tensor, *, token_capacity: int | None = None, flags: int = 0,
              with_thresholds: bool = False):
    """Pack K sign/magnitude plus FP16 low/delta representatives (group size 32).

    keys [KV heads, tokens, head dim] (fp32/fp16/bf16) -> (k_sign int32, k_mag int32,
    low fp16, delta fp16), each [KV heads, token_capacity, ceil(D/32)].  With
    ``with_thresholds`` a fifth tensor [KVH, groups, D, 2] holds (min/2, max/2).
    """
    if keys.ndim != 3 or not keys.is_cuda or not keys.is_contiguous():
        raise ValueError("keys must be contiguous CUDA [KV heads, tokens, head dim]")
    capacity = int(keys.shape[1]) if token_capacity is None else int(token_capacity)
    return tuple(extension().pack(keys, capacity, int(flags), bool(with_thresholds)))


def pack_keys_into(keys: torch.Tensor, packed, *, token_offset: int, flags: int = 0) -> None:
    """Pack ``keys`` into rows token_offset.. of caller-owned packed tensors."""
    if keys.ndim != 3 or not keys.is_cuda or not keys.is_contiguous():
        raise ValueError("keys must be contiguous CUDA [KV heads, tokens, head dim]")
    extension().pack_into(keys, *_packed(packed), int(token_offset), int(flags))


def score(queries: torch.Tensor, packed, *, head_to_kv: torch.Tensor, tokens: int,
          flags: int = 0, seq_len: torch.Tensor | None = None,
          out: torch.Tensor | None = None, hist: torch.Tensor | None = None) -> torch.Tensor:
    """Return Pop-KV approximate QK scores for every query head and token.

    queries [B, QH, D]; packed [KVH, cap, W] (shared by the batch, as in the
    reference) or [B, KVH, cap, W] (one cache per sequence) -> fp32 [B, QH, tokens].
    ``hist`` (a select workspace from ``new_select_workspace(B*QH, tokens)``) collects
    each row's top-11-bit key histogram for ``select(hist=...)``, which consumes it.
    """
    if queries.ndim != 3 or not queries.is_cuda or not queries.is_contiguous():
        raise ValueError("queries must be contiguous CUDA [batch, query heads, head dim]")
    return extension().score(queries, *_packed(packed), head_to_kv.contiguous(), int(tokens),
                             int(flags), seq_len, out, hist)


def append_keys(key_cache: torch.Tensor, value_cache: torch.Tensor | None, new_keys,
                new_values, packed, *, position: int, seq_len: torch.Tensor | None = None,
                kv_heads_per_seq: int = 0, flags: int = 0) -> None:
    """Write the new token's k/v at ``position`` and re-pack its open 32-token group.

    key_cache/value_cache [..., heads, kv_capacity, D]; new_keys/new_values one row
    per cache head.  With ``seq_len`` (int32 device [B]) the position of sequence b
    is seq_len[b] and ``position`` is ignored.
    """
    if not key_cache.is_cuda or not key_cache.is_contiguous():
        raise ValueError("key_cache must be a contiguous CUDA tensor")
    extension().append(key_cache, value_cache, new_keys, new_values, *_packed(packed),
                       int(position), seq_len, int(kv_heads_per_seq), int(flags))


def select(scores: torch.Tensor, *, budget: int, tokens: int | None = None,
           seq_len: torch.Tensor | None = None, rows_per_seq: int = 0,
           out: torch.Tensor | None = None, attn_workspace: torch.Tensor | None = None,
           attn_sizes: tuple = (), hist: torch.Tensor | None = None) -> torch.Tensor:
    """Top-(budget-1) token indices per row plus the newest token.

    scores [..., L] fp32 -> int32 [rows, budget]: the min(budget-1, L) best tokens in
    ascending index order (ties to the lowest index), then L, then -1 padding.
    With ``attn_workspace`` (and ``attn_sizes`` = (batch, q_heads, kv_heads, head_dim,
    tokens, splits) of the attention call that will use it) the selection is also
    written as the workspace's token bitmask for ``sparse_attention_premasked``.
    """
    if not scores.is_cuda or scores.dtype != torch.float32:
        raise ValueError("scores must be a CUDA float32 tensor")
    if int(budget) <= 1:
        raise ValueError("budget must reserve at least one retrieved and one current token")
    tokens = int(scores.shape[-1]) if tokens is None else int(tokens)
    return extension().select(scores, int(budget), tokens, seq_len, int(rows_per_seq), out,
                              attn_workspace, [int(x) for x in attn_sizes], hist)


def score_select(queries: torch.Tensor, packed, *, head_to_kv: torch.Tensor, budget: int,
                 tokens: int, seq_len: torch.Tensor | None = None, out: torch.Tensor | None = None,
                 attn_workspace: torch.Tensor | None = None, attn_sizes: tuple = (),
                 scores: torch.Tensor | None = None, hist: torch.Tensor | None = None,
                 flags: int = 0) -> torch.Tensor:
    """``select(score(queries, packed))`` in one launch: int32 [B*QH, budget].

    Identical indices (and head bitmask with ``attn_workspace``) to the two calls.
    With head_dim 128 and bf16/fp16 queries no score buffer is written; other sizes
    fall back to score + select and need ``scores`` ([B*QH, >= tokens] fp32) and
    ``hist`` (a select workspace).
    """
    if queries.ndim != 3 or not queries.is_cuda or not queries.is_contiguous():
        raise ValueError("queries must be contiguous CUDA [batch, query heads, head dim]")
    if int(budget) <= 1:
        raise ValueError("budget must reserve at least one retrieved and one current token")
    return extension().score_select(queries, *_packed(packed), head_to_kv.contiguous(), int(budget),
                                    int(tokens), int(flags), seq_len, out, attn_workspace,
                                    [int(x) for x in attn_sizes], scores, hist)


def sparse_attention_premasked(queries, key_cache, value_cache, *, tokens: int, current_keys,
                               current_values, workspace, out, seq_len=None, splits: int = 0,
                               gather: "PeerGather | None" = None, layer: int = 0,
                               parity: int = 0, defer_wait: bool = False):
    """sparse_attention over the bitmask that ``select(attn_workspace=workspace)`` wrote.

    Batched caches [B, KVH, kv_cap, D]; queries/out [B, QH, D]; current rows [B, KVH, D].
    With ``gather`` (a :class:`PeerGather` of this rank), the output rows are also
    all-gathered over NVLink peer memory into ``gather.gathered[parity, layer]`` of
    every rank.  With ``defer_wait`` the call only publishes its arrival and
    ``gather.wait()`` (queued later on the stream) waits for all layers at once.
    """
    if gather is None:
        return extension().sparse_attention_premasked(queries, key_cache, value_cache, int(tokens),
                                                      current_keys, current_values, seq_len,
                                                      workspace, int(splits), out)
    return extension().sparse_attention_premasked(queries, key_cache, value_cache, int(tokens),
                                                  current_keys, current_values, seq_len,
                                                  workspace, int(splits), out,
                                                  gather.out_ptrs(layer, parity), gather.flag_ptrs(layer),
                                                  gather.rank, gather.sync[layer], bool(defer_wait))


class PeerGather:
    """Buffers of the fused peer all-gather (one process per GPU, one NVLink domain).

    ``gathered`` [2, layers, world * rows, head_dim] and the arrival words
    [layers, world] live in symmetric memory (every rank maps every rank's copy);
    ``sync`` [layers, 3] holds this rank's ticket / epoch / error words.  Two gathered
    buffers, used by alternate steps: a rank that runs ahead writes the next step's
    rows into the other buffer, never into the rows a slower peer may still be
    reading.  Built collectively by all ranks.
    """

    def __init__(self, layers: int, rows: int, head_dim: int, dtype, group=None):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer all-gather spans at most 8 ranks")
        dev = torch.device("cuda", torch.cuda.current_device())
        self.layers, self.rows, self.head_dim = int(layers), int(rows), int(head_dim)
        self.gathered = symm_mem.empty(2, layers, self.world * rows, head_dim, dtype=dtype, device=dev)
        self.flags = symm_mem.empty(layers, self.world, dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.gathered.zero_()
        torch.cuda.synchronize()
        group_name = group.group_name if group is not None else dist.group.WORLD.group_name
        self._hg = symm_mem.rendezvous(self.gathered, group_name)
        self._hf = symm_mem.rendezvous(self.flags, group_name)
        self.sync = torch.zeros(layers, 3, dtype=torch.int32, device=dev)
        self._layer_stride = self.world * rows * head_dim * self.gathered.element_size()
        self._flag_stride = self.world * 4

    @staticmethod
    def _peer_bases(handle, tensor, rank) -> list:
        off = tensor.data_ptr() - int(handle.buffer_ptrs[rank])  # the tensor's place in its buffer
        return [int(p) + off for p in handle.buffer_ptrs]

    def out_ptrs(self, layer: int, parity: int = 0) -> list:
        off = (int(parity) * self.layers + int(layer)) * self._layer_stride
        return [p + off for p in self._peer_bases(self._hg, self.gathered, self.rank)]

    def flag_ptrs(self, layer: int) -> list:
        return [p + layer * self._flag_stride for p in self._peer_bases(self._hf, self.flags, self.rank)]

    def push(self, out: torch.Tensor, layer: int, parity: int = 0) -> None:
        """All-gather ``out`` (this rank's [rows, head_dim] rows of ``layer``) by a
        separate one-CTA push kernel on the current stream; ``wait()`` completes it."""
        off = self.rank * self.rows * self.head_dim * self.gathered.element_size()
        extension().peer_push(out, [p + off for p in self.out_ptrs(layer, parity)],
                              self.flag_ptrs(layer), self.rank, self.sync[layer])

    def wait(self) -> None:
        """Queue the deferred wait for every layer's arrivals (current stream)."""
        extension().peer_wait(self.flags, self.sync)

    def errors(self) -> int:
        return int(self.sync[:, 2].sum().item())


def sparse_attention(queries: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                     indices: torch.Tensor | None, *, budget: int, tokens: int,
                     current_keys: torch.Tensor | None = None,
                     current_values: torch.Tensor | None = None,
                     seq_len: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                     splits: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
    """Exact attention of every query head over its selected tokens.

    queries [B, QH, D]; caches [KVH, kv_cap, D] (shared) or [B, KVH, kv_cap, D];
    indices int32 [B*QH, >= budget] (e.g. from ``select``; int64 is converted) or
    None for dense attention over tokens 0..L.  Token L is read from
    current_keys/current_values [B, KVH, D] when given.  Returns [B, QH, D].
    """
    if queries.ndim != 3 or not queries.is_cuda or not queries.is_contiguous():
        raise ValueError("queries must be contiguous CUDA [batch, query heads, head dim]")
    if indices is not None and indices.dtype != torch.int32:
        indices = indices.to(torch.int32)
    if indices is not None:
        indices = indices.contiguous()
    return extension().sparse_attention(queries, key_cache, value_cache, indices, int(budget),
                                        int(tokens), current_keys, current_values, seq_len,
                                        workspace, int(splits), out)


def new_select_workspace(rows: int, tokens: int, device) -> torch.Tensor:
    """Zero-filled select workspace shared by ``score(hist=)`` and ``select(hist=)``."""
    n = int(extension().select_workspace_bytes(int(rows), int(tokens)))
    return torch.zeros(n, dtype=torch.uint8, device=device)


def workspace_bytes(batch: int, q_heads: int, kv_heads: int, head_dim: int, tokens: int,
                    splits: int = 0) -> int:
    return int(extension().workspace_bytes(batch, q_heads, kv_heads, head_dim, tokens, splits))


def new_workspace(batch: int, q_heads: int, kv_heads: int, head_dim: int, tokens: int,
                  device, splits: int = 0) -> torch.Tensor:
    """Zero-filled attention workspace (the kernels keep it reusable)."""
    n = workspace_bytes(batch, q_heads, kv_heads, head_dim, tokens, splits)
    return torch.zeros(n, dtype=torch.uint8, device=device)


def advance(seq_len: torch.Tensor, increment: int = 1) -> None:
    extension().advance(seq_len, int(increment))


def retrieve(queries: torch.Tensor, packed, key_cache: torch.Tensor, value_cache: torch.Tensor,
             *, head_to_kv: torch.Tensor, tokens: int, budget: int,
             current_keys: torch.Tensor | None = None, current_values: torch.Tensor | None = None,
             seq_len: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
             flags: int = 0):
    """score -> select -> sparse_attention for one layer; returns (out, indices)."""
    scores = score(queries, packed, head_to_kv=head_to_kv, tokens=tokens, flags=flags,
                   seq_len=seq_len)
    rows_per_seq = int(queries.shape[1])
    indices = select(scores.view(-1, scores.shape[-1]), budget=budget, tokens=tokens,
                     seq_len=seq_len, rows_per_seq=rows_per_seq)
    out = sparse_attention(queries, key_cache, value_cache, indices, budget=budget,
                           tokens=tokens, current_keys=current_keys,
                           current_values=current_values, seq_len=seq_len, workspace=workspace)
    return out, indices


# ---- decoder plumbing (fused elementwise steps of a Llama decode step) --------
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: torch.Tensor) -> torch.Tensor:
    """out = weight * round(x * rsqrt(mean(x^2) + eps)) over the last dimension (LlamaRMSNorm)."""
    extension().rmsnorm(x, weight, float(eps), out)
    return out


def rope_qkv(qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, positions: torch.Tensor, *,
             q_heads: int, kv_heads: int, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
    """Split a fused [q | k | v] row per sequence, rotate q and k at positions[b]."""
    extension().rope_qkv(qkv, cos, sin, positions, int(q_heads), int(kv_heads), q, k, v)


def gemv(x: torch.Tensor, weight: torch.Tensor, out: torch.Tensor,
         residual: torch.Tensor | None = None) -> torch.Tensor:
    """out = residual + x @ weight.T for one activation row (fp32 accumulation)."""
    extension().gemv(x, weight, residual, out)
    return out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out = round(silu(gate)) * up for gate_up = [gate | up] (LlamaMLP)."""
    extension().silu_mul(gate_up, out)
    return out
