"""LlamaSparseDecoder (full / quest / fier) against the reference's own decoder.

tests/golden/reference_decoder.npz was made by tests/golden/make_golden_decoder.py:
a tiny random Llama run through the reference's LlamaSparseDecoder on the CPU
(popkv.py:411-627) for several decode steps, appending to the static and retrieval
caches after each step as its PG19 runner does (run_pg19.py:136-143).
"""
from pathlib import Path

import numpy as np
import pytest
import torch

import popkv
from decoder import LlamaSparseDecoder

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_decoder.npz"


@pytest.fixture(scope="module")
def ref():
    return np.load(GOLDEN)


def tiny_model(ref):
    import sys
    sys.path.insert(0, str(GOLDEN.parent))
    from make_golden_decoder import CONFIG
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(**CONFIG)
    cfg._attn_implementation = "sdpa"
    model = LlamaForCausalLM(cfg).float().eval()
    state = {k[len("weights/"):]: torch.from_numpy(ref[k]) for k in ref.files if k.startswith("weights/")}
    model.load_state_dict(state)
    return model


@pytest.mark.parametrize("method", ["full", "quest", "fier"])
def test_decoder_matches_reference_decoder(ref, method):
    model = tiny_model(ref)
    prefix, steps, budget, page = (int(x) for x in ref["meta"])
    ids = torch.from_numpy(ref["ids"])
    cfg = popkv.RetrievalConfig(budget=budget, group_size=32, quest_page_size=page, full_layers=(0, 1))
    dec = LlamaSparseDecoder(model, cfg)
    prefix_cache = dec.build_prefix_cache(ids[:prefix])
    caches = None if method == "full" else dec.build_retrieval_caches(
        prefix_cache, method=method, reserve_tokens=steps + 1)
    kv = dec.build_static_kv_cache(prefix_cache, reserve_tokens=steps + 1)
    want = ref[f"{method}/logits"]
    for s in range(steps):
        logits, diag, nk, nv = dec.decode(kv, ids[prefix + s], method=method, retrieval_caches=caches,
                                          return_new_kv=True)
        dec.append_kv(kv, nk, nv)
        if caches is not None:
            dec.append_retrieval_caches(caches, nk)
        np.testing.assert_allclose(logits.numpy(), want[s], rtol=0, atol=2e-5)
        if method != "full":
            assert 0 < diag.candidate_ratio <= 1


def test_full_decode_matches_transformers_forward(ref):
    model = tiny_model(ref)
    prefix, steps, _, _ = (int(x) for x in ref["meta"])
    ids = torch.from_numpy(ref["ids"])
    dec = LlamaSparseDecoder(model, popkv.RetrievalConfig(budget=8, full_layers=(0, 1)))
    kv = dec.build_static_kv_cache(dec.build_prefix_cache(ids[:prefix]), reserve_tokens=steps + 1)
    for s in range(steps):
        logits, _, nk, nv = dec.decode(kv, ids[prefix + s], method="full", return_new_kv=True)
        dec.append_kv(kv, nk, nv)
        np.testing.assert_allclose(logits.numpy(), ref["hf_logits"][s], rtol=0, atol=2e-5)


def test_decoder_rejects_unknown_methods(ref):
    dec = LlamaSparseDecoder(tiny_model(ref), popkv.RetrievalConfig(budget=8))
    with pytest.raises(ValueError):
        dec.decode(None, 0, method="dense")
    with pytest.raises(ValueError):
        dec.decode(None, 0, method="quest")
