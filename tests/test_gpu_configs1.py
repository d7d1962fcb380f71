"""The benchmarked configuration itself, checked against the oracle.

BASELINE configs[1] as bench.py builds it: RetrievalStack with one sequence,
32 query / 8 KV heads, head_dim 128, bf16 caches, 32768 prefix tokens, budget
4096, the scorer's histogram feeding the clustered select (4 CTAs per row at 32
rows) and the premasked attention, one eager step, graph capture, then graph
replays.  After the last step every layer's index lists must equal the oracle's
select over the oracle's scores bit for bit (ties to the lowest index), the
packed cache must equal the oracle's packing of the cached keys (the appends
included), and the attention output must be within 2e-2 of the fp64 oracle
(reference popkv.py:585-611)."""
import numpy as np
import pytest
import torch

import popkv
import popkv_oracle as O
from synthetic import SyntheticLayer

pytestmark = pytest.mark.gpu

KVH, QH, D, L0, BUDGET = 8, 32, 128, 32768, 4096


@pytest.mark.parametrize("fused", [True, False])
def test_configs1_stack_matches_oracle(fused):
    layers, steps = 2, 3
    dev = torch.device("cuda")
    stack = popkv.RetrievalStack(layers=layers, batch=1, kv_heads=KVH, q_heads=QH, head_dim=D,
                                 max_tokens=L0 + 16, budget=BUDGET, dtype=torch.bfloat16, device=dev,
                                 fused_select=fused)
    gens = []
    for i in range(layers):
        syn = SyntheticLayer(kv_heads=KVH, q_heads=QH, head_dim=D, seed=1000 + i, device=dev)
        k, v = syn.keys_values(L0)
        stack.prefill(i, k.bfloat16(), v.bfloat16())
        gens.append(syn)
    stack.set_length(L0)

    def inputs(s):
        q = torch.stack([g.queries(L0 + s).bfloat16() for g in gens])
        kv = [g.keys_values(1, start=L0 + s) for g in gens]
        k = torch.stack([x[0][:, :, 0].bfloat16() for x in kv])
        v = torch.stack([x[1][:, :, 0].bfloat16() for x in kv])
        return q, k, v

    stack.step(*inputs(0))
    stack.capture()
    for s in range(1, steps):
        stack.step(*inputs(s))
    torch.cuda.synchronize()

    L = L0 + steps - 1  # prefix length seen by the last step; token L was its current row
    h2k = np.arange(QH) // (QH // KVH)
    for i in range(layers):
        kc = stack.key_cache[i][0, :, : L + 1].float().cpu().numpy()
        vc = stack.value_cache[i][0, :, : L + 1].float().cpu().numpy()
        np.testing.assert_array_equal(kc[:, L], stack.k_in[i][0].float().cpu().numpy())
        packed_ref = O.pack_keys(kc, capacity=stack.capacity)
        got = [t[0].cpu() for t in stack.packed[i]]
        np.testing.assert_array_equal(got[0].numpy()[:, : L + 1], packed_ref[0][:, : L + 1])
        np.testing.assert_array_equal(got[1].numpy()[:, : L + 1], packed_ref[1][:, : L + 1])
        np.testing.assert_array_equal(got[2].view(torch.int16).numpy().view(np.uint16)[:, : L + 1],
                                      packed_ref[2][:, : L + 1])
        np.testing.assert_array_equal(got[3].view(torch.int16).numpy().view(np.uint16)[:, : L + 1],
                                      packed_ref[3][:, : L + 1])
        # The last step scored the prefix 0..L-1 with the then-current packing.
        packed_last = O.pack_keys(kc[:, :L], capacity=stack.capacity)
        q = stack.q_in[i].float().cpu().numpy()
        sc = O.score(q, packed_last, head_to_kv=h2k, tokens=L)
        idx_ref = O.select(sc.reshape(QH, L), budget=BUDGET)
        idx = stack.indices[i].cpu().numpy()
        np.testing.assert_array_equal(idx, idx_ref)
        out_ref = O.attention(q, kc, vc, head_to_kv=h2k, lengths=[L], indices=idx_ref)
        np.testing.assert_allclose(stack.out[i].float().cpu().numpy(), out_ref, atol=2e-2, rtol=0)
