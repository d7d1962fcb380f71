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
import os
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


# ---- Quest and FIER (comparison methods of the reference, plain torch) ------

@dataclass
class QuestCache:
    """Per-page channel bounds of one layer's keys (reference popkv.py:37-44)."""
    page_size: int
    token_count: int
    sealed_pages: int
    page_min: torch.Tensor
    page_max: torch.Tensor
    active_keys: torch.Tensor


def _append_current(indices: torch.Tensor, num_tokens: int) -> torch.Tensor:
    """Append the newest token (index num_tokens - 1) to every row (popkv.py:141-145)."""
    newest = indices.new_full((*indices.shape[:-1], 1), num_tokens - 1, dtype=torch.long)
    return torch.cat([indices.long(), newest], dim=-1)


def build_quest_cache(keys: torch.Tensor, *, page_size: int, reserve_tokens: int) -> QuestCache:
    """Quest page bounds of keys [KVH, T, D]; the open page's keys stay raw (popkv.py:150-164)."""
    kvh, tokens, dim = (int(x) for x in keys.shape)
    sealed = tokens // page_size
    pages_cap = math.ceil((tokens + reserve_tokens + 1) / page_size)
    page_min = torch.empty((kvh, pages_cap, dim), device=keys.device, dtype=torch.float32)
    page_max = torch.empty_like(page_min)
    if sealed:
        paged = keys[:, : sealed * page_size].float().view(kvh, sealed, page_size, dim)
        page_min[:, :sealed] = paged.amin(dim=2)
        page_max[:, :sealed] = paged.amax(dim=2)
    return QuestCache(page_size, tokens, sealed, page_min, page_max,
                      keys[:, sealed * page_size:].detach().clone().contiguous())


def quest_scores(queries: torch.Tensor, cache: QuestCache, current_keys: torch.Tensor,
                 head_to_kv: torch.Tensor) -> torch.Tensor:
    """Upper bound of q.k per page, the open page including the current key (popkv.py:167-178).

    queries [QH, D], current_keys [KVH, D] -> fp32 [QH, pages].  Like the reference,
    it writes the open page's bounds into the cache.
    """
    open_keys = torch.cat([cache.active_keys, current_keys[:, None].detach()], dim=1).float()
    page = cache.sealed_pages
    cache.page_min[:, page] = open_keys.amin(dim=1)
    cache.page_max[:, page] = open_keys.amax(dim=1)
    lo = cache.page_min[:, : page + 1].index_select(0, head_to_kv)
    hi = cache.page_max[:, : page + 1].index_select(0, head_to_kv)
    q = queries.float()[:, None]
    return torch.maximum(q * lo, q * hi).sum(dim=-1)


def quest_indices(scores: torch.Tensor, *, num_tokens: int, page_size: int, budget: int):
    """Token indices of the top pages, the newest token forced in (popkv.py:181-194).

    Returns (indices int64 [QH, pages*page_size], valid bool of the same shape).
    """
    n_pages = min(int(scores.shape[-1]), max(1, math.ceil(budget / page_size)))
    pages = torch.topk(scores, k=n_pages, dim=-1, sorted=False).indices
    tokens = (pages[:, :, None] * page_size + torch.arange(page_size, device=scores.device)).flatten(1)
    valid = tokens < num_tokens
    newest = num_tokens - 1
    present = ((tokens == newest) & valid).any(dim=-1)
    tokens[:, -1] = torch.where(present, tokens[:, -1], tokens.new_tensor(newest))
    valid[:, -1] = torch.where(present, valid[:, -1], valid.new_tensor(True))
    return tokens, valid


def append_quest(cache: QuestCache, keys: torch.Tensor) -> None:
    """Append keys [KVH, n, D]; a page that fills up is sealed (popkv.py:197-207)."""
    cache.active_keys = torch.cat([cache.active_keys, keys.detach()], dim=1).contiguous()
    cache.token_count += int(keys.shape[1])
    if int(cache.active_keys.shape[1]) == cache.page_size:
        page = cache.sealed_pages
        full = cache.active_keys.float()
        cache.page_min[:, page] = full.amin(dim=1)
        cache.page_max[:, page] = full.amax(dim=1)
        cache.sealed_pages += 1
        cache.active_keys = cache.active_keys[:, :0].contiguous()


@dataclass
class FIERCache:
    """FIER 1-bit packed keys with per-group channel extrema (reference popkv.py:47-55)."""
    group_size: int
    token_count: int
    sealed_tokens: int
    packed: torch.Tensor
    group_min: torch.Tensor
    group_max: torch.Tensor
    active_keys: torch.Tensor


def build_fier_cache(keys: torch.Tensor, *, group_size: int, reserve_tokens: int) -> FIERCache:
    """Pack keys [KVH, T, D] into storage with room for the reserve (popkv.py:212-235)."""
    import fier_torch
    packed, mins, maxs = fier_torch.pack_keys(keys.contiguous(), group_size=group_size)
    kvh, tokens, dim = (int(x) for x in keys.shape)
    capacity = math.ceil((tokens + reserve_tokens) / group_size) * group_size
    words = torch.empty((kvh, dim, math.ceil(capacity / 32)), device=keys.device, dtype=packed.dtype)
    lo = torch.empty((kvh, math.ceil(capacity / group_size), dim), device=keys.device, dtype=mins.dtype)
    hi = torch.empty_like(lo)
    words[:, :, : packed.shape[2]] = packed
    lo[:, : mins.shape[1]] = mins
    hi[:, : maxs.shape[1]] = maxs
    sealed = (tokens // group_size) * group_size
    return FIERCache(group_size, tokens, sealed, words, lo, hi,
                     keys[:, sealed:].detach().clone().contiguous())


def stage_fier(cache: FIERCache, current_keys: torch.Tensor) -> None:
    """Re-pack the open group with the current keys [KVH, 1, D] (popkv.py:238-247)."""
    import fier_torch
    open_keys = torch.cat([cache.active_keys, current_keys.detach()], dim=1).contiguous()
    packed, mins, maxs = fier_torch.pack_keys(open_keys, group_size=cache.group_size)
    w0 = cache.sealed_tokens // 32
    g0 = cache.sealed_tokens // cache.group_size
    cache.packed[:, :, w0 : w0 + packed.shape[2]] = packed
    cache.group_min[:, g0 : g0 + mins.shape[1]] = mins
    cache.group_max[:, g0 : g0 + maxs.shape[1]] = maxs


def append_fier(cache: FIERCache, keys: torch.Tensor) -> None:
    """Record appended keys [KVH, n, D]; a full group is sealed (popkv.py:250-255)."""
    cache.active_keys = torch.cat([cache.active_keys, keys.detach()], dim=1).contiguous()
    cache.token_count += int(keys.shape[1])
    if int(cache.active_keys.shape[1]) == cache.group_size:
        cache.sealed_tokens += cache.group_size
        cache.active_keys = cache.active_keys[:, :0].contiguous()


def fier_scores(queries: torch.Tensor, cache: FIERCache, current_keys: torch.Tensor,
                head_to_kv: torch.Tensor, *, num_tokens: int) -> torch.Tensor:
    """stage_fier + FIER score of queries [QH, D] over num_tokens tokens (popkv.py:575-581)."""
    import fier_torch
    stage_fier(cache, current_keys)
    return fier_torch.score_packed_batched(queries[None], cache.packed, cache.group_min,
                                           cache.group_max, head_to_kv, tokens=num_tokens,
                                           group_size=cache.group_size)


def gather_selected_kv(prefix_keys, prefix_values, current_keys, current_values, indices,
                       head_to_kv):
    """Materialised gather of the selected rows (popkv.py:341-357), for the torch methods.

    prefix [KVH, L, D], current [KVH, D], indices [QH, n] -> keys, values [QH, n, D];
    index L selects the current row.
    """
    L = int(prefix_keys.shape[1])
    clamped = indices.clamp_max(L - 1)
    heads = head_to_kv[:, None].expand_as(clamped)
    is_current = indices.eq(L).unsqueeze(-1)
    keys = torch.where(is_current, current_keys.index_select(0, head_to_kv)[:, None],
                       prefix_keys[heads, clamped])
    values = torch.where(is_current, current_values.index_select(0, head_to_kv)[:, None],
                         prefix_values[heads, clamped])
    return keys, values


def selected_attention(queries, keys, values, valid_mask=None):
    """SDPA of queries [QH, D] over their own rows [QH, n, D] (popkv.py:360-368)."""
    mask = None if valid_mask is None else valid_mask[None, :, None]
    return torch.nn.functional.scaled_dot_product_attention(
        queries[None, :, None], keys[None], values[None], attn_mask=mask, dropout_p=0.0,
        is_causal=False)[0, :, 0]


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
                 process_group=None, gather_wait: str | None = None,
                 dense_layers: tuple[int, ...] = (), fused_select: bool | None = None):
        self.device = torch.device(device or "cuda")
        # Score and select in one kernel (default; POPKV_FUSED_SELECT=0 or
        # fused_select=False keeps the scorer and the select as two kernels).
        if fused_select is None:
            fused_select = os.environ.get("POPKV_FUSED_SELECT", "1") != "0"
        self.fused_select = bool(fused_select)
        # Layers attended densely (the reference's full_layers, popkv.py:542-551):
        # no score/select, attention over every cached token plus the current one.
        self.dense_layers = frozenset(int(i) for i in dense_layers)
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
        # peer memory (symmetric buffers, two of them used by alternate steps);
        # POPKV_GATHER=nccl selects an NCCL all-gather after the attention instead.
        # gather_wait "step" (default): one wait for all layers at the end of the step,
        # so no layer waits for the slowest rank; "layer": every layer's combine waits
        # for its own rows (what a decoder whose next layer reads them needs).
        self.peer = None
        self._gathered = None
        self.gather_wait = gather_wait or os.environ.get("POPKV_GATHER_WAIT", "step")
        if self.gather_wait not in ("step", "layer"):
            raise ValueError("gather_wait is 'step' or 'layer'")
        if self.world > 1:
            if os.environ.get("POPKV_GATHER", "peer") == "nccl":
                g = torch.zeros(layers, self.world * B, QH, head_dim, dtype=dtype, device=dev)
                self._gathered = (g, g)
            else:
                self.peer = pk.PeerGather(layers, B * QH, head_dim, dtype, group=process_group)
                g = self.peer.gathered.view(2, layers, self.world * B, QH, head_dim)
                self._gathered = (g[0], g[1])
        self.steps_done = 0  # parity of the next step picks its gathered buffer
        self.graphs = None
        # The append of a layer only has to follow that layer's score, so it runs on a
        # side stream in parallel with select and attention; steps join it at the end.
        self.side = torch.cuda.Stream(device=dev)
        self.push_stream = torch.cuda.Stream(device=dev)

    @property
    def gathered(self):
        """All-gathered outputs [layers, world*B, QH_l, D] of the last step (world > 1).

        With the peer all-gather the buffer alternates between steps: the rows of a
        step stay valid until the step after next is queued.
        """
        if self._gathered is None:
            return None
        return self._gathered[(self.steps_done - 1) % 2]

    @property
    def graph(self):
        return self.graphs

    @graph.setter
    def graph(self, value):
        self.graphs = value

    # ------------------------------------------------------------------ setup
    def prefill(self, layer: int, keys: torch.Tensor, values: torch.Tensor,
                sequence: int | None = None) -> None:
        """Store and pack a prefix of this rank's heads.

        keys/values [B, KVH_local, T, D], or [KVH_local, T, D] for one ``sequence``
        (long contexts are prefilled a sequence at a time).
        """
        T = int(keys.shape[-2])
        if T > self.max_tokens:
            raise RuntimeError("prefix longer than the stack's max_tokens")
        if sequence is None:
            kc, vc, packed = self.key_cache[layer], self.value_cache[layer], self.packed[layer]
        else:
            kc, vc = self.key_cache[layer][sequence], self.value_cache[layer][sequence]
            packed = tuple(p[sequence] for p in self.packed[layer])
        kc[..., :T, :].copy_(keys)
        vc[..., :T, :].copy_(values)
        heads = keys.reshape(-1, T, self.head_dim).contiguous()
        packed = tuple(p.reshape(-1, self.capacity, p.shape[-1]) for p in packed)
        pk.pack_keys_into(heads, packed, token_offset=0)

    def set_length(self, length: int) -> None:
        self.length = int(length)
        self.seq_len.fill_(self.length)

    # ------------------------------------------------------------------- step
    def _layer(self, i: int, parity: int) -> None:
        tokens = self.max_tokens
        if i in self.dense_layers:
            self.side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.side):
                pk.append_keys(self.key_cache[i], self.value_cache[i], self.k_in[i], self.v_in[i],
                               self.packed[i], position=0, seq_len=self.seq_len,
                               kv_heads_per_seq=self.kv_heads)
            pk.sparse_attention(self.q_in[i], self.key_cache[i], self.value_cache[i], None,
                                budget=2, tokens=tokens, current_keys=self.k_in[i],
                                current_values=self.v_in[i], seq_len=self.seq_len,
                                workspace=self.workspace[i], out=self.out[i])
            if self.world > 1:
                raise RuntimeError("dense layers are not sharded")
            return
        sizes = (self.batch, self.q_heads, self.kv_heads, self.head_dim, tokens, 0)
        # Score + select in one launch (the score buffer and histogram workspace serve
        # the two-kernel form, for sizes the fused kernel does not take).
        pk.score_select(self.q_in[i], self.packed[i], head_to_kv=self.head_to_kv,
                        budget=self.budget, tokens=tokens, seq_len=self.seq_len,
                        out=self.indices[i], attn_workspace=self.workspace[i], attn_sizes=sizes,
                        scores=self.scores, hist=self.score_hist,
                        flags=0 if self.fused_select else pk.UNFUSED_SELECT)
        self.side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self.side):
            pk.append_keys(self.key_cache[i], self.value_cache[i], self.k_in[i], self.v_in[i],
                           self.packed[i], position=0, seq_len=self.seq_len,
                           kv_heads_per_seq=self.kv_heads)
        push = self.peer is not None and self.gather_wait == "step"
        pk.sparse_attention_premasked(self.q_in[i], self.key_cache[i], self.value_cache[i],
                                      tokens=tokens, current_keys=self.k_in[i],
                                      current_values=self.v_in[i], seq_len=self.seq_len,
                                      workspace=self.workspace[i], out=self.out[i],
                                      gather=None if push else self.peer, layer=i, parity=parity)
        if push:
            # The NVLink all-gather of this layer runs on its own stream: the next
            # layer's kernels do not wait for it; the step's end waits for all layers.
            self.push_stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(self.push_stream):
                self.peer.push(self.out[i].view(-1, self.head_dim), i, parity)
        if self.world > 1 and self.peer is None:
            import torch.distributed as dist
            dist.all_gather_into_tensor(self._gathered[parity][i], self.out[i], group=self.group)

    def _step_launches(self, parity: int) -> None:
        for i in range(self.layers):
            self._layer(i, parity)
        if self.peer is not None and self.gather_wait == "step":
            torch.cuda.current_stream().wait_stream(self.push_stream)
            self.peer.wait()
        torch.cuda.current_stream().wait_stream(self.side)
        pk.advance(self.seq_len, 1)

    def step(self, q=None, k=None, v=None, *, check: bool = False) -> torch.Tensor:
        """One decode step over all layers. q [layers, B, QH_l, D], k/v [layers, B, KVH_l, D].

        Returns ``out`` [layers, B, QH_l, D] (one rank) or the all-gathered outputs
        [layers, world*B, QH_l, D].  With ``check`` the call synchronises and raises
        RuntimeError if a peer all-gather wait ran out (the gathered rows are then
        incomplete); without it, poll ``peer_errors()``.
        """
        if self.length + 1 > self.max_tokens:
            raise RuntimeError("Pop-KV cache reserve exhausted")
        if q is not None:
            self.q_in.copy_(q, non_blocking=True)
            self.k_in.copy_(k, non_blocking=True)
            self.v_in.copy_(v, non_blocking=True)
        parity = self.steps_done % 2
        if self.graphs is not None:
            self.graphs[parity].replay()
        else:
            self._step_launches(parity)
        self.length += 1
        self.steps_done += 1
        if check and self.peer_errors():
            raise RuntimeError(f"{self.peer_errors()} peer all-gather waits ran out: "
                               "the gathered outputs are incomplete")
        return self.out if self.world == 1 else self.gathered

    def capture(self) -> None:
        """Record the decode step as CUDA graphs (run once eagerly first to warm up).

        Two graphs, one per gathered buffer, replayed by alternate steps.
        """
        self.graphs = None
        graphs = []
        for parity in (0, 1):
            g = torch.cuda.CUDAGraph()
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                with torch.cuda.graph(g, stream=stream):
                    self._step_launches(parity)
            torch.cuda.current_stream().wait_stream(stream)
            graphs.append(g)
        # Capturing enqueued nothing: the graphs are replayed by step().
        self.graphs = graphs

    def peer_errors(self) -> int:
        """Peer all-gather waits that ran out (0 on a healthy run)."""
        return 0 if self.peer is None else self.peer.errors()

    def launches_per_step(self) -> int:
        # score, select, attention + combine, append per layer, + advance
        # (+ the deferred peer wait).
        sparse = self.layers - len(self.dense_layers)
        step_push = self.peer is not None and self.gather_wait == "step"
        return sparse * 5 + (self.layers - sparse) * 3 + 1 + \
            ((self.layers + 1) if step_push else 0)
