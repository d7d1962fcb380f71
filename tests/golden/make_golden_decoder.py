"""Golden fixtures for the Llama decoder: the reference's own LlamaSparseDecoder on CPU.

Usage:  TRITON_INTERPRET=1 python tests/golden/make_golden_decoder.py <path-to-reference-checkout>

Builds a tiny random-init LlamaForCausalLM (fp32, seeded), runs the reference's
``LlamaSparseDecoder`` (popkv.py:411-627) the way its PG19 runner does
(run_pg19.py:120-143: prefix cache -> retrieval caches -> static cache -> decode,
append_kv, append_retrieval_caches per step) for the methods that run on a CPU --
``full``, ``quest`` and ``fier`` (FIER's Triton kernels under Triton's CPU
interpreter) -- and stores the model weights, token ids and per-step logits.
Pop-KV itself needs the reference's CUDA extension and is checked on the GPU
against the same decoder with the Pop-KV kernels.

Two harness bugs of the reference are shimmed here (the reference checkout is not
modified): ``_layer_cache`` does not know transformers 5's DynamicCache
(popkv.py:401-409), and ``build_static_kv_cache`` slices the head-dim axis
instead of the token axis (popkv.py:483).
"""
from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

CONFIG = dict(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=4,
              num_attention_heads=4, num_key_value_heads=2, head_dim=16, rms_norm_eps=1e-5,
              rope_theta=500000.0, max_position_embeddings=512, tie_word_embeddings=False,
              attention_bias=False, mlp_bias=False)
PREFIX, STEPS, BUDGET, PAGE = 70, 4, 24, 8


def tiny_model():
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(**CONFIG)
    cfg._attn_implementation = "sdpa"
    model = LlamaForCausalLM(cfg).float().eval()
    return model


def patch_reference(ref):
    original = ref._layer_cache

    def layer_cache(cache, layer):
        if hasattr(cache, "layers") and not isinstance(cache, ref.StaticKVCache):
            return cache.layers[layer].keys, cache.layers[layer].values
        return original(cache, layer)

    def build_static_kv_cache(self, prefix_cache, *, reserve_tokens):
        first, _ = ref._layer_cache(prefix_cache, 0)
        length, capacity = int(first.shape[-2]), int(first.shape[-2]) + reserve_tokens
        keys_out, values_out = [], []
        for layer in range(len(self.layers)):
            keys, values = ref._layer_cache(prefix_cache, layer)
            ks = torch.empty((*keys.shape[:-2], capacity, keys.shape[-1]), dtype=keys.dtype)
            vs = torch.empty_like(ks)
            ks[..., :length, :].copy_(keys)
            vs[..., :length, :].copy_(values)
            keys_out.append(ks)
            values_out.append(vs)
        return ref.StaticKVCache(keys_out, values_out, length, capacity)

    ref._layer_cache = layer_cache
    ref.LlamaSparseDecoder.build_static_kv_cache = build_static_kv_cache


def patch_fier_for_cpu():
    """Let FIER's Triton kernels run under the CPU interpreter: its host wrappers
    insist on CUDA tensors (fier_triton.py:141, 170, 211, 239); the kernels do not."""
    import contextlib
    import math

    import fier_triton as F
    torch.cuda.device = lambda device: contextlib.nullcontext()
    F._validate_keys = lambda keys, group_size: None

    def score_packed_batched(queries, packed, mins, maxs, head_to_kv, *, tokens, group_size):
        batch, q_heads, head_dim = (int(v) for v in queries.shape)
        scores = torch.empty((batch, q_heads, tokens), dtype=torch.float32)
        F._score_kernel[(math.ceil(tokens / 32), batch * q_heads)](
            queries.contiguous(), packed, mins, maxs, head_to_kv.to(torch.int64).contiguous(),
            scores, tokens=tokens, q_heads=q_heads, head_dim=head_dim,
            num_groups=int(mins.shape[1]), words=int(packed.shape[2]), group_size=group_size,
            BLOCK_D=1 << (head_dim - 1).bit_length(), BLOCK_T=32)
        return scores

    F.score_packed_batched = score_packed_batched


def main(reference: str) -> None:
    if os.environ.get("TRITON_INTERPRET") != "1":
        raise SystemExit("run with TRITON_INTERPRET=1 (FIER's Triton kernels run on the CPU)")
    sys.path.insert(0, reference)
    import popkv as ref
    patch_reference(ref)
    patch_fier_for_cpu()
    model = tiny_model()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, CONFIG["vocab_size"], (PREFIX + STEPS,), generator=g)
    out = {f"weights/{k}": v.detach().numpy() for k, v in model.state_dict().items()}
    out["ids"] = ids.numpy()
    out["meta"] = np.array([PREFIX, STEPS, BUDGET, PAGE])
    cfg = ref.RetrievalConfig(budget=BUDGET, group_size=32, quest_page_size=PAGE, full_layers=(0, 1))
    decoder = ref.LlamaSparseDecoder(model, cfg)
    prefix_ids, current = ids[:PREFIX], ids[PREFIX:]
    with torch.inference_mode():
        # HF's own logits for the whole sequence: the dense decode must agree.
        out["hf_logits"] = model(ids[None]).logits[0, PREFIX:].float().numpy()
        for method in ("full", "quest", "fier"):
            prefix = decoder.build_prefix_cache(prefix_ids)
            caches = None if method == "full" else decoder.build_retrieval_caches(
                prefix, method=method, reserve_tokens=STEPS + 1)
            kv = decoder.build_static_kv_cache(prefix, reserve_tokens=STEPS + 1)
            logits_all = []
            for step in range(STEPS):
                logits, diag, nk, nv = decoder.decode(kv, current[step], method=method,
                                                      retrieval_caches=caches, return_new_kv=True)
                decoder.append_kv(kv, nk, nv)
                if caches is not None:
                    decoder.append_retrieval_caches(caches, nk)
                logits_all.append(logits.numpy())
            out[f"{method}/logits"] = np.stack(logits_all)
    np.savez_compressed(HERE / "reference_decoder.npz", **out)
    print("wrote", HERE / "reference_decoder.npz", len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else str(Path.home() / "reference"))
