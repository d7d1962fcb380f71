"""Llama decoding on the GPU: the Pop-KV decoder paths against dense attention and
against transformers' own forward pass (tiny random bf16 Llama, head_dim 64)."""
import pytest
import torch

import popkv
from decoder import GraphedDecoder, LlamaSparseDecoder

pytestmark = pytest.mark.gpu

CONFIG = dict(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
              num_attention_heads=4, num_key_value_heads=2, head_dim=64, rms_norm_eps=1e-5,
              rope_theta=500000.0, max_position_embeddings=2048, tie_word_embeddings=False)
PREFIX = 300


def tiny_model():
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(**CONFIG)
    cfg._attn_implementation = "sdpa"
    with torch.device("cuda"):
        model = LlamaForCausalLM(cfg)
    for p in model.parameters():  # larger weights: attention that is not uniform
        p.data.mul_(4.0)
    return model.to(torch.bfloat16).eval()


def ids(n, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, CONFIG["vocab_size"], (n,), generator=g)


def _close(a, b, tol):
    scale = float(b.abs().max())
    assert float((a - b).abs().max()) <= tol * scale, (float((a - b).abs().max()), scale)


def test_popkv_with_budget_covering_the_context_equals_full():
    model = tiny_model()
    tok = ids(PREFIX + 3)
    out = {}
    for method in ("full", "popkv"):
        dec = LlamaSparseDecoder(model, popkv.RetrievalConfig(budget=PREFIX + 8, full_layers=(0,)))
        pc = dec.build_prefix_cache(tok[:PREFIX])
        caches = None if method == "full" else dec.build_retrieval_caches(pc, method=method, reserve_tokens=4)
        kv = dec.build_static_kv_cache(pc, reserve_tokens=4)
        logits = []
        for s in range(3):
            lg, diag, nk, nv = dec.decode(kv, tok[PREFIX + s], method=method, retrieval_caches=caches,
                                          return_new_kv=True)
            dec.append_kv(kv, nk, nv)
            if caches is not None:
                dec.append_retrieval_caches(caches, nk)
            logits.append(lg)
        out[method] = torch.stack(logits)
    _close(out["popkv"], out["full"], 2e-2)


def test_graphed_full_decoder_matches_transformers_forward():
    model = tiny_model()
    tok = ids(PREFIX)
    dec = GraphedDecoder(model, popkv.RetrievalConfig(budget=64), max_tokens=PREFIX + 8, method="full")
    dec.prefill(tok)
    dec.capture()
    seq = tok.tolist()
    for s in range(4):
        consumed = int(dec.token.item())
        dec.step()
        seq.append(consumed)
        with torch.inference_mode():
            want = model(torch.tensor([seq], device="cuda")).logits[0, -1].float()
        _close(dec.logits[0], want, 3e-2)


def test_graphed_popkv_decoder_matches_eager_popkv_decoder():
    model = tiny_model()
    tok = ids(PREFIX, seed=2)
    cfg = popkv.RetrievalConfig(budget=64, full_layers=(0, 1))
    graphed = GraphedDecoder(model, cfg, max_tokens=PREFIX + 8, method="popkv")
    graphed.prefill(tok)
    graphed.capture()
    eager = LlamaSparseDecoder(model, cfg)
    pc = eager.build_prefix_cache(tok)
    caches = eager.build_retrieval_caches(pc, method="popkv", reserve_tokens=8)
    kv = eager.build_static_kv_cache(pc, reserve_tokens=8)
    for s in range(4):
        consumed = int(graphed.token.item())
        graphed.step()
        lg, diag, nk, nv = eager.decode(kv, consumed, method="popkv", retrieval_caches=caches,
                                        return_new_kv=True)
        eager.append_kv(kv, nk, nv)
        eager.append_retrieval_caches(caches, nk)
        _close(graphed.logits[0], lg, 3e-2)
        assert diag.candidate_ratio < 1.0
    tokens = graphed.generate(3)
    assert tokens.shape == (3,) and graphed.stack.length == PREFIX + 7


def test_fused_decoder_steps_match_transformers_modules():
    """rmsnorm / rope_qkv / silu_mul against LlamaRMSNorm, apply_rotary_pos_emb and
    LlamaMLP's act_fn(gate) * up, in bf16."""
    import popkv_cuda as pk
    from transformers.models.llama import modeling_llama as m
    model = tiny_model()
    layer = model.model.layers[0]
    g = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.randn(3, CONFIG["hidden_size"], device="cuda", generator=g) * 2).bfloat16()
    out = torch.empty_like(x)
    pk.rmsnorm(x, layer.input_layernorm.weight, CONFIG["rms_norm_eps"], out)
    want = layer.input_layernorm(x)
    assert float((out.float() - want.float()).abs().max()) <= 2 ** -6 * float(want.abs().max())
    H, KVH, D = 4, 2, 64
    qkv = torch.randn(2, (H + 2 * KVH) * D, device="cuda", generator=g).bfloat16()
    pos = torch.tensor([5, 1000], dtype=torch.int32, device="cuda")
    cos, sin = model.model.rotary_emb(x[:1, None], torch.arange(2048, device="cuda")[None])
    cos, sin = cos[0].contiguous(), sin[0].contiguous()
    q = torch.empty(2, H, D, dtype=torch.bfloat16, device="cuda")
    k = torch.empty(2, KVH, D, dtype=torch.bfloat16, device="cuda")
    v = torch.empty_like(k)
    pk.rope_qkv(qkv, cos, sin, pos, q_heads=H, kv_heads=KVH, q=q, k=k, v=v)
    qr = qkv[:, : H * D].view(2, H, 1, D).transpose(1, 2).transpose(1, 2)
    kr = qkv[:, H * D: (H + KVH) * D].view(2, KVH, 1, D)
    c, s = cos[pos.long()][:, None], sin[pos.long()][:, None]
    wq, wk = m.apply_rotary_pos_emb(qr, kr, c, s)
    torch.testing.assert_close(q, wq[:, :, 0], rtol=0, atol=0)
    torch.testing.assert_close(k, wk[:, :, 0], rtol=0, atol=0)
    torch.testing.assert_close(v, qkv[:, (H + KVH) * D:].view(2, KVH, D), rtol=0, atol=0)
    gu = torch.randn(3, 2 * 512, device="cuda", generator=g).bfloat16()
    act = torch.empty(3, 512, dtype=torch.bfloat16, device="cuda")
    pk.silu_mul(gu, act)
    want = torch.nn.functional.silu(gu[:, :512]) * gu[:, 512:]
    assert float((act.float() - want.float()).abs().max()) <= 2 ** -7 * float(want.abs().max())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,k,res", [(6144, 4096, False), (4096, 4096, True), (4096, 14336, True),
                                     (1000, 72, False), (3, 8, True), (128256, 4096, False)])
def test_gemv_matches_fp32_matmul(dtype, n, k, res):
    """popkv_gemv (the decoder's weight products) against an fp32 matmul of the same
    16-bit inputs: the product rounded once, then the residual added and rounded."""
    import popkv_cuda as pk
    g = torch.Generator().manual_seed(n + k)
    x = torch.randn(k, generator=g).to(dtype).cuda()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(dtype).cuda()
    r = torch.randn(n, generator=g).to(dtype).cuda() if res else None
    out = torch.empty(n, dtype=dtype, device="cuda")
    pk.gemv(x, w, out, residual=r)
    want = (w.float() @ x.float()).to(dtype).float() + (r.float() if res else 0.0)
    err = (out.float() - want).abs()
    tol = 2 ** -7 * want.abs() + 1e-3
    assert bool((err <= tol).all()), float((err - tol).max())
