"""Llama decoding with the four retrieval methods of the reference (full/quest/fier/popkv).

Two front ends over the same model (a transformers ``LlamaForCausalLM``):

``LlamaSparseDecoder``
    The reference's decoder surface (kw78999/FIER-2bits popkv.py:411-627):
    ``build_prefix_cache``, ``build_retrieval_caches``, ``append_retrieval_caches``,
    ``build_static_kv_cache``, ``append_kv`` and ``decode(cache, token, method=...)``
    returning ``(logits, DecodeDiagnostics)``.  One token per call, layer by layer,
    in the reference's order: the dense ``full_layers`` and the ``full`` method use
    SDPA over every cached token, ``quest``/``fier`` their plain-torch scorers, and
    ``popkv`` the sm_100a kernels (pack, popcount score, exact top-k, fused gather +
    attention).  Two harness faults of the reference are fixed here: transformers 5
    caches (``_layer_cache``, popkv.py:401-409) and the static cache's token-axis
    slice (popkv.py:483).

``GraphedDecoder``
    Greedy decoding for throughput: the whole token step -- embedding, 32 layers
    (fused QKV projection, RoPE, retrieval on the kernels, o_proj, MLP; every weight
    product a one-row GEMV kernel, popkv_gemv), final norm,
    lm_head and the argmax that feeds the next step -- is one CUDA graph over
    device-resident state (token id, sequence length, K/V caches, packed keys), so
    a step costs one graph launch.  Retrieval and the static-cache append run through
    ``popkv.RetrievalStack``; the reference's ``full_layers`` attend densely.
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import Any, Sequence

import torch
import torch.nn.functional as F

import popkv
from popkv import (METHODS, FIERCache, PopKVCache, QuestCache, RetrievalConfig, StaticKVCache)


@dataclass
class RetrievalCaches:
    method: str
    layers: dict


@dataclass
class DecodeDiagnostics:
    """Per-call stage times and selection counts (popkv.py:82-94)."""
    selected_tokens: int = 0
    available_tokens: int = 0
    sparse_head_calls: int = 0
    candidate_search_ms: float = 0.0
    candidate_score_ms: float = 0.0
    candidate_topk_ms: float = 0.0
    selected_gather_ms: float = 0.0
    selected_attention_ms: float = 0.0

    @property
    def candidate_ratio(self) -> float:
        return 1.0 if self.available_tokens == 0 else self.selected_tokens / self.available_tokens


def _timed(operation, device: torch.device, events: list):
    """Run and time one stage: CUDA events on a GPU, wall clock on a CPU (popkv.py:371-378)."""
    if device.type == "cuda":
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        result = operation()
        end.record()
        events.append((start, end, device))
        return result, 0.0
    started = time.perf_counter()
    result = operation()
    return result, (time.perf_counter() - started) * 1000


def _finish(events: Sequence) -> float:
    if not events:
        return 0.0
    for device in {x[2] for x in events}:
        torch.cuda.synchronize(device)
    return sum(float(start.elapsed_time(end)) for start, end, _ in events)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    first, second = x.chunk(2, dim=-1)
    return torch.cat((-second, first), dim=-1)


def _apply_rope(q, k, cos, sin):
    """Rotate-half RoPE of q/k [B, heads, T, D] with cos/sin [B, T, D] (popkv.py:393-398)."""
    if cos.ndim == 2:
        cos, sin = cos.unsqueeze(0), sin.unsqueeze(0)
    cos, sin = cos.unsqueeze(1), sin.unsqueeze(1)
    return q * cos + _rotate_half(q) * sin, k * cos + _rotate_half(k) * sin


def _layer_cache(cache: Any, layer: int):
    """(keys, values) [1, KVH, T, D] of one layer of a static or transformers cache."""
    if isinstance(cache, StaticKVCache):
        return (cache.key_storage[layer][..., : cache.length, :],
                cache.value_storage[layer][..., : cache.length, :])
    if hasattr(cache, "layers"):  # transformers >= 5 DynamicCache
        entry = cache.layers[layer]
        return entry.keys, entry.values
    if hasattr(cache, "key_cache") and hasattr(cache, "value_cache"):
        return cache.key_cache[layer], cache.value_cache[layer]
    try:
        return cache[layer][:2]
    except (TypeError, IndexError, KeyError) as exc:
        raise TypeError(f"unsupported Transformers cache: {type(cache).__name__}") from exc


class LlamaSparseDecoder:
    """One-token Llama decoder exposing FullAttention, Quest, FIER and Pop-KV (popkv.py:411)."""

    def __init__(self, model: Any, retrieval: RetrievalConfig = RetrievalConfig()) -> None:
        retrieval.validate()
        self.model = model
        self.backbone = getattr(model, "model", None)
        if self.backbone is None:
            raise TypeError("expected a LlamaForCausalLM-compatible model")
        self.layers = self.backbone.layers
        self.retrieval = retrieval
        cfg = model.config
        self.num_heads = int(cfg.num_attention_heads)
        self.num_kv_heads = int(getattr(cfg, "num_key_value_heads", self.num_heads))
        self.kv_group_size = self.num_heads // self.num_kv_heads
        self.head_dim = int(getattr(cfg, "head_dim", None) or cfg.hidden_size // self.num_heads)
        self.head_to_kv = (torch.arange(self.num_heads, device=self.device, dtype=torch.long)
                           // self.kv_group_size)

    @property
    def device(self) -> torch.device:
        return self.backbone.embed_tokens.weight.device

    @torch.inference_mode()
    def build_prefix_cache(self, prefix_ids: torch.Tensor):
        ids = prefix_ids.to(self.device).view(1, -1)
        return self.backbone(input_ids=ids, attention_mask=torch.ones_like(ids), use_cache=True,
                             output_hidden_states=False, return_dict=True).past_key_values

    @torch.inference_mode()
    def build_retrieval_caches(self, prefix_cache: Any, *, method: str,
                               reserve_tokens: int = 2048) -> RetrievalCaches:
        if method not in {"quest", "fier", "popkv"}:
            raise ValueError("retrieval caches are only used by sparse methods")
        layers = {}
        for layer in range(len(self.layers)):
            keys, _ = _layer_cache(prefix_cache, layer)
            keys = keys[0].to(self.device)
            if method == "quest":
                layers[layer] = popkv.build_quest_cache(
                    keys, page_size=self.retrieval.quest_page_size, reserve_tokens=reserve_tokens)
            elif method == "fier":
                layers[layer] = popkv.build_fier_cache(
                    keys, group_size=self.retrieval.group_size, reserve_tokens=reserve_tokens)
            else:
                layers[layer] = popkv.build_popkv_cache(
                    keys, group_size=self.retrieval.group_size, reserve_tokens=reserve_tokens)
        return RetrievalCaches(method, layers)

    @torch.inference_mode()
    def append_retrieval_caches(self, caches: RetrievalCaches, new_keys: Sequence[torch.Tensor]) -> None:
        for layer, keys in enumerate(new_keys):
            cache = caches.layers[layer]
            if isinstance(cache, QuestCache):
                popkv.append_quest(cache, keys[0])
            elif isinstance(cache, FIERCache):
                popkv.append_fier(cache, keys[0])
            elif isinstance(cache, PopKVCache):
                popkv.append_popkv(cache, keys[0])
            else:
                raise TypeError("unknown retrieval cache")

    @torch.inference_mode()
    def build_static_kv_cache(self, prefix_cache: Any, *, reserve_tokens: int) -> StaticKVCache:
        first, _ = _layer_cache(prefix_cache, 0)
        length = int(first.shape[-2])
        capacity = length + reserve_tokens
        keys_out, values_out = [], []
        for layer in range(len(self.layers)):
            keys, values = _layer_cache(prefix_cache, layer)
            key_store = torch.empty((*keys.shape[:-2], capacity, keys.shape[-1]), device=keys.device,
                                    dtype=keys.dtype)
            value_store = torch.empty_like(key_store)
            key_store[..., :length, :].copy_(keys)
            value_store[..., :length, :].copy_(values)
            keys_out.append(key_store)
            values_out.append(value_store)
        return StaticKVCache(keys_out, values_out, length, capacity)

    @torch.inference_mode()
    def append_kv(self, cache: StaticKVCache, new_keys, new_values) -> None:
        if cache.length >= cache.capacity:
            raise RuntimeError("static KV cache capacity exhausted")
        position = cache.length
        for layer, (keys, values) in enumerate(zip(new_keys, new_values)):
            cache.key_storage[layer][..., position:position + 1, :].copy_(keys)
            cache.value_storage[layer][..., position:position + 1, :].copy_(values)
        cache.length += 1

    def _position_embeddings(self, hidden: torch.Tensor, positions: torch.Tensor):
        return self.backbone.rotary_emb(hidden, positions)

    @torch.inference_mode()
    def decode(self, cache: StaticKVCache, token_id, *, method: str,
               retrieval_caches: RetrievalCaches | None = None, return_new_kv: bool = False):
        if method not in METHODS:
            raise ValueError(f"method must be one of {METHODS}")
        if method != "full" and retrieval_caches is None:
            raise ValueError(f"{method} requires build_retrieval_caches()")
        prefix_length = cache.length
        token = torch.as_tensor(token_id, device=self.device, dtype=torch.long).view(1, 1)
        hidden = self.backbone.embed_tokens(token)
        positions = torch.tensor([[prefix_length]], device=self.device)
        cos, sin = self._position_embeddings(hidden, positions)
        diag = DecodeDiagnostics()
        score_events, topk_events, gather_events, attention_events = [], [], [], []
        new_keys, new_values = [], []
        H, KVH, D = self.num_heads, self.num_kv_heads, self.head_dim
        for layer_idx, layer in enumerate(self.layers):
            attention = layer.self_attn
            residual = hidden
            normalized = layer.input_layernorm(hidden)
            q = attention.q_proj(normalized).view(1, 1, H, D).transpose(1, 2)
            k = attention.k_proj(normalized).view(1, 1, KVH, D).transpose(1, 2)
            v = attention.v_proj(normalized).view(1, 1, KVH, D).transpose(1, 2)
            q, k = _apply_rope(q, k, cos.to(q.device), sin.to(q.device))
            prefix_k, prefix_v = _layer_cache(cache, layer_idx)
            if return_new_kv:
                new_keys.append(k.detach())
                new_values.append(v.detach())
            force_full = method == "full" or layer_idx in self.retrieval.full_layers
            if force_full:
                def gather_full():
                    return torch.cat([prefix_k, k], 2), torch.cat([prefix_v, v], 2)
                (all_k, all_v), ms = _timed(gather_full, q.device, gather_events)
                diag.selected_gather_ms += ms

                def attend_full():
                    grouped = q[0].view(KVH, self.kv_group_size, 1, D)
                    return F.scaled_dot_product_attention(
                        grouped, all_k[0, :, None], all_v[0, :, None], dropout_p=0.0,
                        is_causal=False).reshape(H, D)
                output, ms = _timed(attend_full, q.device, attention_events)
                diag.selected_attention_ms += ms
            else:
                num_tokens = prefix_length + 1
                sparse = retrieval_caches.layers[layer_idx]
                valid = None
                if method == "popkv":
                    output, ms_parts = self._popkv_layer(q, k, v, sparse, cache, layer_idx,
                                                         score_events, topk_events, attention_events)
                    diag.selected_tokens += min(self.retrieval.budget, num_tokens) * H
                else:
                    if method == "quest":
                        scores, ms = _timed(lambda: popkv.quest_scores(q[0, :, 0], sparse, k[0, :, 0],
                                                                       self.head_to_kv),
                                            q.device, score_events)
                        diag.candidate_score_ms += ms
                        (indices, valid), ms = _timed(
                            lambda: popkv.quest_indices(scores, num_tokens=num_tokens,
                                                        page_size=self.retrieval.quest_page_size,
                                                        budget=self.retrieval.budget),
                            q.device, topk_events)
                        diag.candidate_topk_ms += ms
                    else:
                        scores, ms = _timed(lambda: popkv.fier_scores(q[0, :, 0], sparse, k[0],
                                                                      self.head_to_kv,
                                                                      num_tokens=num_tokens),
                                            q.device, score_events)
                        diag.candidate_score_ms += ms

                        def topk_fier():
                            selected = torch.topk(scores[..., :prefix_length],
                                                  k=min(self.retrieval.budget - 1, prefix_length),
                                                  dim=-1, sorted=False).indices[0]
                            return popkv._append_current(selected, num_tokens)
                        indices, ms = _timed(topk_fier, q.device, topk_events)
                        diag.candidate_topk_ms += ms
                    diag.selected_tokens += int(indices.numel())

                    def gather_sparse():
                        return popkv.gather_selected_kv(prefix_k[0], prefix_v[0], k[0, :, 0],
                                                        v[0, :, 0], indices, self.head_to_kv)
                    (sel_k, sel_v), ms = _timed(gather_sparse, q.device, gather_events)
                    diag.selected_gather_ms += ms
                    output, ms = _timed(lambda: popkv.selected_attention(q[0, :, 0], sel_k, sel_v, valid),
                                        q.device, attention_events)
                    diag.selected_attention_ms += ms
                diag.available_tokens += num_tokens * H
                diag.sparse_head_calls += H
            output = output.reshape(1, 1, -1).to(normalized.dtype)
            hidden = residual + attention.o_proj(output)
            residual = hidden
            hidden = residual + layer.mlp(layer.post_attention_layernorm(hidden))
        hidden = self.backbone.norm(hidden)
        logits = self.model.lm_head(hidden).float()[0, -1]
        diag.candidate_score_ms += _finish(score_events)
        diag.candidate_topk_ms += _finish(topk_events)
        diag.candidate_search_ms = diag.candidate_score_ms + diag.candidate_topk_ms
        diag.selected_gather_ms += _finish(gather_events)
        diag.selected_attention_ms += _finish(attention_events)
        if return_new_kv:
            return logits, diag, new_keys, new_values
        return logits, diag

    def _popkv_layer(self, q, k, v, sparse: PopKVCache, cache: StaticKVCache, layer_idx: int,
                     score_events, topk_events, attention_events):
        """Score -> exact top-k -> fused gather + attention on the kernels (popkv.py:587-611).

        The gather is fused into the attention kernel, so its time is part of the
        attention stage.
        """
        import popkv_cuda as pk
        L = sparse.token_count
        queries = q[0, :, 0].unsqueeze(0).contiguous()
        scores, _ = _timed(lambda: pk.score(queries, sparse.packed, head_to_kv=self.head_to_kv,
                                            tokens=L), q.device, score_events)
        indices, _ = _timed(lambda: pk.select(scores.view(-1, L), budget=self.retrieval.budget),
                            q.device, topk_events)
        store_k = cache.key_storage[layer_idx][0]
        store_v = cache.value_storage[layer_idx][0]
        out, _ = _timed(lambda: pk.sparse_attention(
            queries, store_k, store_v, indices, budget=self.retrieval.budget, tokens=L,
            current_keys=k[0, :, 0].unsqueeze(0).contiguous(),
            current_values=v[0, :, 0].unsqueeze(0).contiguous()), q.device, attention_events)
        return out[0], None


class GraphedDecoder:
    """Greedy decoding with one CUDA graph per token (popkv or full retrieval).

    model: a bf16 ``LlamaForCausalLM`` on a CUDA device.  ``prefill(ids)`` runs the
    backbone over the prompt, fills the static caches and packs every layer's keys;
    ``step()`` decodes one token (the argmax of the previous logits) and returns the
    device tensor holding it; ``generate(n)`` runs n steps and copies the tokens to
    the host once.
    """

    def __init__(self, model: Any, retrieval: RetrievalConfig = RetrievalConfig(), *,
                 max_tokens: int, method: str = "popkv") -> None:
        if method not in ("popkv", "full"):
            raise ValueError("the graphed decoder runs the popkv and full methods")
        retrieval.validate()
        self.model, self.method, self.retrieval = model, method, retrieval
        self.backbone = model.model
        cfg = model.config
        self.H = int(cfg.num_attention_heads)
        self.KVH = int(getattr(cfg, "num_key_value_heads", self.H))
        self.D = int(getattr(cfg, "head_dim", None) or cfg.hidden_size // self.H)
        self.hidden_size = int(cfg.hidden_size)
        self.device = self.backbone.embed_tokens.weight.device
        self.dtype = self.backbone.embed_tokens.weight.dtype
        n_layers = len(self.backbone.layers)
        dense = tuple(range(n_layers)) if method == "full" else tuple(
            i for i in retrieval.full_layers if i < n_layers)
        self.stack = popkv.RetrievalStack(layers=n_layers, batch=1, kv_heads=self.KVH,
                                          q_heads=self.H, head_dim=self.D, max_tokens=max_tokens,
                                          budget=retrieval.budget, dtype=self.dtype,
                                          device=self.device, dense_layers=dense)
        # Fused projection weights: [q; k; v] and [gate; up] (one GEMV each).
        self.w_qkv, self.w_gate_up = [], []
        for layer in self.backbone.layers:
            at, mlp = layer.self_attn, layer.mlp
            self.w_qkv.append(torch.cat([at.q_proj.weight, at.k_proj.weight, at.v_proj.weight], 0))
            self.w_gate_up.append(torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight], 0))
        self.ffn = int(self.backbone.layers[0].mlp.gate_proj.weight.shape[0])
        # RoPE tables at every position the stack can hold (the model's own rotary).
        pos = torch.arange(max_tokens + 1, device=self.device)[None]
        probe = torch.zeros(1, 1, self.hidden_size, device=self.device, dtype=self.dtype)
        cos, sin = self.backbone.rotary_emb(probe, pos)
        self.cos, self.sin = cos[0].contiguous(), sin[0].contiguous()  # [P, D]
        self.eps = float(cfg.rms_norm_eps)
        hs, dt, dev = self.hidden_size, self.dtype, self.device
        # Static activations of the graphed step.
        self.h = torch.zeros(1, hs, dtype=dt, device=dev)
        self.h2 = torch.zeros(1, hs, dtype=dt, device=dev)
        self.x = torch.zeros(1, hs, dtype=dt, device=dev)
        self.qkv = torch.zeros(1, (self.H + 2 * self.KVH) * self.D, dtype=dt, device=dev)
        self.gu = torch.zeros(1, 2 * self.ffn, dtype=dt, device=dev)
        self.act = torch.zeros(1, self.ffn, dtype=dt, device=dev)
        self.logits_lp = torch.zeros(1, int(cfg.vocab_size), dtype=dt, device=dev)
        self.token = torch.zeros(1, dtype=torch.long, device=self.device)
        self.logits = torch.zeros(1, int(cfg.vocab_size), dtype=torch.float32, device=self.device)
        self.graph = None

    # ------------------------------------------------------------- prefill
    @torch.inference_mode()
    def prefill(self, ids: torch.Tensor) -> None:
        """Run the prompt through the backbone; fill and pack every layer's caches."""
        ids = ids.to(self.device).view(1, -1)
        T = int(ids.shape[1])
        out = self.backbone(input_ids=ids, use_cache=True, return_dict=True)
        cache = out.past_key_values
        for i in range(len(self.backbone.layers)):
            k, v = _layer_cache(cache, i)
            self.stack.prefill(i, k.to(self.dtype), v.to(self.dtype))
        del cache
        last = self.backbone.norm(out.last_hidden_state[:, -1])
        self.logits.copy_(self.model.lm_head(last).float())
        torch.argmax(self.logits, dim=-1, out=self.token)
        self.stack.set_length(T)

    # ---------------------------------------------------------------- step
    def _step_body(self) -> None:
        import popkv_cuda as pk
        st = self.stack
        H, KVH, D, hs = self.H, self.KVH, self.D, self.hidden_size
        h = self.h
        torch.index_select(self.backbone.embed_tokens.weight, 0, self.token, out=h)
        for i, layer in enumerate(self.backbone.layers):
            pk.rmsnorm(h, layer.input_layernorm.weight, self.eps, self.x)
            pk.gemv(self.x, self.w_qkv[i], self.qkv)
            pk.rope_qkv(self.qkv, self.cos, self.sin, st.seq_len, q_heads=H, kv_heads=KVH,
                        q=st.q_in[i], k=st.k_in[i], v=st.v_in[i])
            st._layer(i, 0)
            pk.gemv(st.out[i], layer.self_attn.o_proj.weight, self.h2, residual=h)
            pk.rmsnorm(self.h2, layer.post_attention_layernorm.weight, self.eps, self.x)
            pk.gemv(self.x, self.w_gate_up[i], self.gu)
            pk.silu_mul(self.gu, self.act)
            pk.gemv(self.act, layer.mlp.down_proj.weight, h, residual=self.h2)
        pk.rmsnorm(h, self.backbone.norm.weight, self.eps, self.x)
        pk.gemv(self.x, self.model.lm_head.weight, self.logits_lp)
        self.logits.copy_(self.logits_lp)
        torch.argmax(self.logits, dim=-1, out=self.token)
        torch.cuda.current_stream().wait_stream(st.side)
        pk.advance(st.seq_len, 1)

    @torch.inference_mode()
    def capture(self) -> None:
        """Warm up once eagerly, then record the step as a CUDA graph."""
        self.graph = None
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._step_body()
        torch.cuda.current_stream().wait_stream(s)
        self.graph = g

    @torch.inference_mode()
    def step(self) -> torch.Tensor:
        if self.stack.length + 1 > self.stack.max_tokens:
            raise RuntimeError("static KV cache capacity exhausted")
        if self.graph is None:
            self._step_body()
        else:
            self.graph.replay()
        self.stack.length += 1
        return self.token

    @torch.inference_mode()
    def generate(self, steps: int) -> torch.Tensor:
        """Decode ``steps`` tokens greedily; returns them on the host."""
        out = torch.empty(steps, dtype=torch.long, device=self.device)
        for s in range(steps):
            out[s: s + 1].copy_(self.step())
        return out.cpu()
