"""End-to-end retrieval step (configs[0]/[1] shapes) and the multi-layer stack."""
import numpy as np
import pytest
import torch

import popkv
import popkv_cuda as pk
import popkv_oracle as O
import reconstruction as R
from synthetic import SyntheticLayer

pytestmark = pytest.mark.gpu
DEV = "cuda"


def test_configs0_step_matches_oracle_and_reference_path():
    """fp32, 32/8 heads, D=128, L=4096, budget 1024, outliers + RoPE, seed 0."""
    L, budget = 4096, 1024
    layer = SyntheticLayer(kv_heads=8, q_heads=32, head_dim=128, seed=0)
    k, v = layer.keys_values(L + 1)
    k, v = k[0], v[0]
    q = layer.queries(L)
    h2k = torch.arange(32) // 4
    cache = popkv.build_popkv_cache(k[:, :L].contiguous().to(DEV), group_size=32, reserve_tokens=16)
    out, idx = popkv.popkv_attention(q[0].to(DEV), cache, k[:, :L].contiguous().to(DEV),
                                     v[:, :L].contiguous().to(DEV), k[:, L].contiguous().to(DEV),
                                     v[:, L].contiguous().to(DEV), head_to_kv=h2k.to(DEV),
                                     budget=budget)
    # Oracle with the kernels' own arithmetic: identical selection, exact attention.
    ref_scores = O.score(q.numpy(), O.pack_keys(k[:, :L].numpy()), head_to_kv=h2k.numpy(), tokens=L)
    ref_idx = O.select(ref_scores.reshape(32, L), budget=budget)
    np.testing.assert_array_equal(idx.cpu().numpy(), ref_idx)
    ref_out = O.attention(q.numpy(), k.numpy(), v.numpy(), head_to_kv=h2k.numpy(), lengths=[L],
                          indices=ref_idx)
    np.testing.assert_allclose(out.cpu().numpy(), ref_out[0], atol=1e-4, rtol=1e-4)
    # The reference's readable CPU path: same attention up to its fp32 representatives.
    ref_out2, ref_scores2, ref_idx2 = R.decode_step(q[0], k[:, :L], v[:, :L], k[:, L], v[:, L],
                                                    head_to_kv=h2k, budget=budget)
    overlap = np.mean([len(set(a[:-1]) & set(b[:-1].tolist())) / (budget - 1)
                       for a, b in zip(ref_idx, ref_idx2.numpy())])
    assert overlap > 0.99
    assert np.abs(out.cpu().numpy() - ref_out2.numpy()).max() < 0.05


def test_stack_graph_replay_matches_eager_and_oracle():
    layers, B, KVH, QH, D, L0, budget = 2, 2, 2, 8, 128, 1000, 128
    steps = 40
    syn = SyntheticLayer(kv_heads=KVH, q_heads=QH, head_dim=D, seed=1, batch=B)
    k_all, v_all = syn.keys_values(L0 + steps)
    k_all, v_all = k_all.bfloat16(), v_all.bfloat16()
    qs = torch.stack([syn.queries(L0 + s) for s in range(steps)]).bfloat16()

    def make():
        st = popkv.RetrievalStack(layers=layers, batch=B, kv_heads=KVH, q_heads=QH, head_dim=D,
                                  max_tokens=L0 + steps, budget=budget, device=DEV)
        for i in range(layers):
            st.prefill(i, k_all[:, :, :L0].to(DEV), v_all[:, :, :L0].to(DEV))
        st.set_length(L0)
        return st

    eager, graphed = make(), make()
    graphed.step(qs[0].expand(layers, *qs[0].shape).to(DEV), k_all[:, :, L0].expand(layers, B, KVH, D).to(DEV),
                 v_all[:, :, L0].expand(layers, B, KVH, D).to(DEV))
    eager.step(qs[0].expand(layers, *qs[0].shape).to(DEV), k_all[:, :, L0].expand(layers, B, KVH, D).to(DEV),
               v_all[:, :, L0].expand(layers, B, KVH, D).to(DEV))
    graphed.capture()
    for s in range(1, steps):
        args = (qs[s].expand(layers, *qs[s].shape).to(DEV),
                k_all[:, :, L0 + s].expand(layers, B, KVH, D).to(DEV),
                v_all[:, :, L0 + s].expand(layers, B, KVH, D).to(DEV))
        a = eager.step(*args).clone()
        b = graphed.step(*args).clone()
        torch.testing.assert_close(a, b, rtol=0, atol=0)
    torch.cuda.synchronize()
    L = L0 + steps - 1
    assert eager.seq_len.tolist() == [L + 1] * B
    # Last step against the oracle: packed state and output of layer 0.
    packed_ref = O.pack_keys(k_all[:, :, :L].reshape(B * KVH, L, D).float().numpy(),
                             capacity=eager.capacity)
    got = [t.view(B * KVH, eager.capacity, -1).cpu() for t in eager.packed[0]]
    np.testing.assert_array_equal(got[0].numpy()[:, :L], packed_ref[0][:, :L])
    q = qs[steps - 1].float().numpy()
    sc = O.score(q, packed_ref, head_to_kv=np.arange(QH) // (QH // KVH), lengths=[L] * B,
                 cache_per_batch=True, kv_heads=KVH, tokens=L)
    idx = O.select(sc.reshape(B * QH, L), budget=budget)
    ref = O.attention(q, k_all.reshape(B * KVH, -1, D).float().numpy(),
                      v_all.reshape(B * KVH, -1, D).float().numpy(),
                      head_to_kv=np.arange(QH) // (QH // KVH), lengths=[L] * B, indices=idx,
                      cache_per_batch=True, kv_heads=KVH)
    np.testing.assert_allclose(b[0].float().cpu().numpy(), ref, atol=2e-2)
