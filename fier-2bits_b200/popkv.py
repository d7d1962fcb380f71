"""Pop-KV decode-time retrieval on B200: host-side mirror of the reference ``popkv.py``.

Kept from the reference surface (kw78999/FIER-2bits popkv.py):
  METHODS, RetrievalConfig                 popkv.py:17-34
  PopKVCache, build_popkv_cache, append_popkv   popkv.py:58-64, 255-280
  StaticKVCache                            popkv.py:73-78
  popkv_attention                          one sparse layer of LlamaSparseDecoder.decode
                                           (popkv.py:585-611: score -> top-k -> gather -> SDPA)
  dense_attention                          the `full` path (popkv.py:542-551)
New for multi-layer, multi-step and multi-GPU use:
  RetrievalStack   L attention layers with static caches, device-resident sequence
                   lengths, one CUDA graph per decode step and optional KV-head
                   sharding across ranks with an all-gather of the outputs.

All compute goes through ``popkv_cuda`` (native sm_100a kernels); nothing here
computes on the CPU.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

import popkv_cuda as pk

METHODS = ("full", "quest", "fier", "popkv")


@dataclass(frozen=True)
class RetrievalConfig:
    budget: int = 4096
    group_size: int = 32
    quest_page_size: int = 16
    full_layers: tuple[int, ...] = (0, 1)

    def validate(self) -> None:
        if self.budget <= 1:
            raise ValueError("budget must reserve at least one retrieved and one current token")
        if self.group_size != 32:
            raise ValueError("the released Pop-KV/FIER kernels use group_size=32")
        if self.quest_page_size <= 0:
            raise ValueError("quest_page_size must be positive")


@dataclass
class StaticKVCache:
    key_storage: list[torch.Tensor]
    value_storage: list[torch.Tensor]
    length: int
    capacity: int


@dataclass
class PopKVCache:
    """Packed key cache of one layer (reference popkv.py:58-64).

    ``open_keys`` [KVH, 32, D] holds the keys of the open (unsealed) group, so an
    append re-packs the group in place without concatenating tensors.
    """
    group_size: int
    token_count: int
    sealed_tokens: int
    packed: tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]
    open_keys: torch.Tensor = field(repr=False)

    @property
    def active_keys(self) -> torch.Tensor:
        return self.open_keys[:, : self.token_count - self.sealed_tokens]

    @property
    def capacity(self) -> int:
        return int(self.packed[0].shape[1])


def build_popkv_cache(keys: torch.Tensor, *, group_size: int, reserve_tokens: int) -> PopKVCache:
    """Pack a prefix keys [KVH, T, D] with room for ``reserve_tokens`` appends."""
    if group_size != 32:
        raise ValueError("Pop-KV release kernel requires group_size=32")
    tokens = int(keys.shape[1])
    capacity = math.ceil((tokens + reserve_tokens) / group_size) * group_size
    packed = pk.pack_keys(keys.contiguous(), token_capacity=capacity)
    sealed = (tokens // group_size) * group_size
    open_keys = torch.empty((keys.shape[0], group_size, keys.shape[2]), device=keys.device,
                            dtype=keys.dtype)
    open_keys[:, : tokens - sealed].copy_(keys[:, sealed:])
    return PopKVCache(group_size, tokens, sealed, packed, open_keys)


def append_popkv(cache: PopKVCache, keys: torch.Tensor) -> None:
    """Append one token's keys [KVH, 1, D] and re-pack the open group (popkv.py:270-280)."""
    n_open = cache.token_count - cache.sealed_tokens
    if cache.sealed_tokens + n_open + 1 > cache.capacity:
        raise RuntimeError("Pop-KV cache reserve exhausted")
    cache.open_keys[:, n_open : n_open + 1].copy_(keys.detach())
    pk.pack_keys_into(cache.open_keys[:, : n_open + 1].contiguous(), cache.packed,
                      token_offset=cache.sealed_tokens)
    cache.token_count += 1
    if n_open + 1 == cache.group_size:
        cache.sealed_tokens += cache.group_size


def popkv_attention(queries: torch.Tensor, cache: PopKVCache, prefix_keys: torch.Tensor,
                    prefix_values: torch.Tensor, current_keys: torch.Tensor,
                    current_values: torch.Tensor, *, head_to_kv: torch.Tensor, budget: int,
                    workspace: torch.Tensor | None = None):
    """One sparse layer of the decode step (popkv.py:587-611).

    queries [QH, D]; prefix caches [KVH, >= L, D] (a static-cache view is fine);
    current k/v [KVH, D]; scores cover the L packed prefix tokens and the newest
    token (index L) is always attended.  Returns (output [QH, D], indices int32
    [QH, budget]).
    """
    L = cache.token_count
    q = queries.reshape(1, queries.shape[0], queries.shape[-1]).contiguous()
    scores = pk.score(q, cache.packed, head_to_kv=head_to_kv, tokens=L)
    indices = pk.select(scores.view(-1, L), budget=budget)
    out = pk.sparse_attention(q, prefix_keys.contiguous(), prefix_values.contiguous(), indices,
                              budget=budget, tokens=L,
                              current_keys=current_keys.reshape(1, *current_keys.shape).contiguous(),
                              current_values=current_values.reshape(1, *current_values.shape).contiguous(),
                              workspace=workspace)
    return out[0], indices


def dense_attention(queries: torch.Tensor, prefix_keys: torch.Tensor, prefix_values: torch.Tensor,
                    current_keys: torch.Tensor, current_values: torch.Tensor,
                    workspace: torch.Tensor | None = None) -> torch.Tensor:
    """The `full` method's attention over all L prefix tokens plus the current one."""
    L = int(prefix_keys.shape[1])
    q = queries.reshape(1, queries.shape[0], queries.shape[-1]).contiguous()
    out = pk.sparse_attention(q, prefix_keys.contiguous(), prefix_values.contiguous(), None,
                              budget=2, tokens=L,
                              current_keys=current_keys.reshape(1, *current_keys.shape).contiguous(),
                              current_values=current_values.reshape(1, *current_values.shape).contiguous(),
                              workspace=workspace)
    return out[0]


def shard_heads(rank: int, world: int, kv_heads: int, q_heads: int):
    """KV-head sharding: rank r owns KV heads [r*KVH/W, (r+1)*KVH/W) and their query heads."""
    if kv_heads % world or q_heads % kv_heads:
        raise ValueError("kv_heads must divide by the world size and q_heads by kv_heads")
    kv_local = kv_heads // world
    group = q_heads // kv_heads
    kv0 = rank * kv_local
    return (kv0, kv0 + kv_local), (kv0 * group, (kv0 + kv_local) * group)


def gather_head_shards(shards: torch.Tensor, batch: int) -> torch.Tensor:
    """[W*B, QH/W, D] rank-major all-gather result -> [B, QH, D] in head order."""
    world = shards.shape[0] // batch
    return shards.view(world, batch, shards.shape[1], shards.shape[2]).transpose(0, 1).reshape(
        batch, world * shards.shape[1], shards.shape[2])


class RetrievalStack:
    """``layers`` Pop-KV attention layers over per-sequence static caches.

    Per layer it owns a bf16 K/V cache [B, KVH, kv_capacity, D], the packed cache
    [B, KVH, capacity, W], score/index buffers and an attention workspace; all
    layers share one device array ``seq_len`` [B] (int32).  ``step`` runs, for every
    layer: score (prefix) -> select -> sparse attention (with the current k/v) ->
    append (write k/v, re-pack the open group), then advances ``seq_len`` -- the
    reference's decode + append_kv + append_retrieval_caches order
    (popkv.py:510-627, run_pg19.py:136-143).  ``capture`` records one decode step as
    a CUDA graph over static input/output buffers.

    With ``process_group`` (NCCL) of size W the stack holds KV heads
    [r*KVH/W, (r+1)*KVH/W) of every sequence and all-gathers each layer's
    attention output over the group: inside the attention's combine kernel over
    NVLink peer memory, or with POPKV_GATHER=nccl by an NCCL all-gather after it
    (``gathered`` either way).
    """

    def __init__(self, *, layers: int, batch: int, kv_heads: int, q_heads: int, head_dim: int,
                 max_tokens: int, budget: int, dtype=torch.bfloat16, device=None,
                 process_group=None):
        self.device = torch.device(device or "cuda")
        self.layers, self.batch, self.head_dim, self.budget = layers, batch, head_dim, budget
        self.dtype = dtype
        self.group = process_group
        if process_group is not None:
            import torch.distributed as dist
            self.world, self.rank = dist.get_world_size(process_group), dist.get_rank(process_group)
        else:
            self.world, self.rank = 1, 0
        (kv0, kv1), (q0, q1) = shard_heads(self.rank, self.world, kv_heads, q_heads)
        self.kv_heads_total, self.q_heads_total = kv_heads, q_heads
        self.kv_heads, self.q_heads = kv1 - kv0, q1 - q0
        self.kv_range, self.q_range = (kv0, kv1), (q0, q1)
        self.max_tokens = int(max_tokens)
        self.kv_capacity = self.max_tokens + 1
        self.capacity = math.ceil((self.max_tokens + 1) / 32) * 32
        words = (head_dim + 31) // 32
        dev = self.device
        B, H, QH = batch, self.kv_heads, self.q_heads
        self.key_cache = [torch.zeros(B, H, self.kv_capacity, head_dim, dtype=dtype, device=dev) for _ in range(layers)]
        self.value_cache = [torch.zeros(B, H, self.kv_capacity, head_dim, dtype=dtype, device=dev) for _ in range(layers)]
        self.packed = [(torch.zeros(B, H, self.capacity, words, dtype=torch.int32, device=dev),
                        torch.zeros(B, H, self.capacity, words, dtype=torch.int32, device=dev),
                        torch.zeros(B, H, self.capacity, words, dtype=torch.float16, device=dev),
                        torch.zeros(B, H, self.capacity, words, dtype=torch.float16, device=dev))
                       for _ in range(layers)]
        self.head_to_kv = (torch.arange(QH, device=dev) // (QH // H)).to(torch.int64)
        self.scores = torch.empty(B, QH, self.capacity, dtype=torch.float32, device=dev)
        self.score_hist = pk.new_select_workspace(B * QH, self.max_tokens, dev)
        self.indices = [torch.empty(B * QH, budget, dtype=torch.int32, device=dev) for _ in range(layers)]
        self.workspace = [pk.new_workspace(B, QH, H, head_dim, self.max_tokens, dev) for _ in range(layers)]
        self.seq_len = torch.zeros(B, dtype=torch.int32, device=dev)
        self.length = 0  # host mirror of seq_len (all sequences advance together)
        # Static step buffers (graph inputs / outputs).
        self.q_in = torch.zeros(layers, B, QH, head_dim, dtype=dtype, device=dev)
        self.k_in = torch.zeros(layers, B, H, head_dim, dtype=dtype, device=dev)
        self.v_in = torch.zeros(layers, B, H, head_dim, dtype=dtype, device=dev)
        self.out = torch.zeros(layers, B, QH, head_dim, dtype=dtype, device=dev)
        # world > 1: the attention combine all-gathers each layer's output over NVLink
        # peer memory (symmetric buffers); POPKV_GATHER=nccl selects an NCCL
        # all-gather after the attention instead.
        self.peer = None
        self.gathered = None
        if self.world > 1:
            import os
            if os.environ.get("POPKV_GATHER", "peer") == "nccl":
                self.gathered = torch.zeros(layers, self.world * B, QH, head_dim, dtype=dtype, device=dev)
            else:
                self.peer = pk.PeerGather(layers, B * QH, head_dim, dtype, group=process_group)
                self.gathered = self.peer.gathered.view(layers, self.world * B, QH, head_dim)
        self.graph = None
        # The append of a layer only has to follow that layer's score, so it runs on a
        # side stream in parallel with select and attention; steps join it at the end.
        self.side = torch.cuda.Stream(device=dev)

    # ------------------------------------------------------------------ setup
    def prefill(self, layer: int, keys: torch.Tensor, values: torch.Tensor) -> None:
        """keys/values [B, KVH_local, T, D] (this rank's heads); packs the prefix."""
        T = int(keys.shape[2])
        if T > self.max_tokens:
            raise RuntimeError("prefix longer than the stack's max_tokens")
        self.key_cache[layer][:, :, :T].copy_(keys)
        self.value_cache[layer][:, :, :T].copy_(values)
        heads = keys.reshape(-1, T, self.head_dim).contiguous()
        packed = tuple(p.view(-1, self.capacity, p.shape[-1]) for p in self.packed[layer])
        pk.pack_keys_into(heads, packed, token_offset=0)

    def set_length(self, length: int) -> None:
        self.length = int(length)
        self.seq_len.fill_(self.length)

    # ------------------------------------------------------------------- step
    def _layer(self, i: int) -> None:
        tokens = self.max_tokens
        pk.score(self.q_in[i], self.packed[i], head_to_kv=self.head_to_kv, tokens=tokens,
                 seq_len=self.seq_len, out=self.scores, hist=self.score_hist)
        self.side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.side):
            pk.append_keys(self.key_cache[i], self.value_cache[i], self.k_in[i], self.v_in[i],
                           self.packed[i], position=0, seq_len=self.seq_len,
                           kv_heads_per_seq=self.kv_heads)
        sizes = (self.batch, self.q_heads, self.kv_heads, self.head_dim, tokens, 0)
        pk.select(self.scores.view(-1, self.capacity), budget=self.budget, tokens=tokens,
                  seq_len=self.seq_len, rows_per_seq=self.q_heads, out=self.indices[i],
                  attn_workspace=self.workspace[i], attn_sizes=sizes, hist=self.score_hist)
        pk.sparse_attention_premasked(self.q_in[i], self.key_cache[i], self.value_cache[i],
                                      tokens=tokens, current_keys=self.k_in[i],
                                      current_values=self.v_in[i], seq_len=self.seq_len,
                                      workspace=self.workspace[i], out=self.out[i],
                                      gather=self.peer, layer=i)
        if self.world > 1 and self.peer is None:
            import torch.distributed as dist
            dist.all_gather_into_tensor(self.gathered[i], self.out[i], group=self.group)

    def _step_launches(self) -> None:
        for i in range(self.layers):
            self._layer(i)
        torch.cuda.current_stream().wait_stream(self.side)
        pk.advance(self.seq_len, 1)

    def step(self, q=None, k=None, v=None) -> torch.Tensor:
        """One decode step over all layers. q [layers, B, QH_l, D], k/v [layers, B, KVH_l, D]."""
        if self.length + 1 > self.max_tokens:
            raise RuntimeError("Pop-KV cache reserve exhausted")
        if q is not None:
            self.q_in.copy_(q, non_blocking=True)
            self.k_in.copy_(k, non_blocking=True)
            self.v_in.copy_(v, non_blocking=True)
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step_launches()
        self.length += 1
        return self.out if self.world == 1 else self.gathered

    def capture(self) -> None:
        """Record one decode step as a CUDA graph (run once eagerly first to warm up)."""
        self.graph = None
        g = torch.cuda.CUDAGraph()
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            with torch.cuda.graph(g, stream=stream):
                self._step_launches()
        torch.cuda.current_stream().wait_stream(stream)
        # Capturing enqueued nothing: the graph is replayed by step().
        self.graph = g

    def peer_errors(self) -> int:
        """Peer all-gather waits that ran out (0 on a healthy run)."""
        return 0 if self.peer is None else self.peer.errors()

    def launches_per_step(self) -> int:
        # score, select, attention + combine, append per layer, + advance.
        return self.layers * 5 + 1
