"""(c)+(d) query pack + popcount scorer: bit-exact against the oracle (IEEE mode),
within the reference test's tolerance of the reference's readable scores."""
import numpy as np
import pytest
import torch

import popkv_cuda as pk
import popkv_oracle as O
from conftest import synthetic_keys

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("qdtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("kvh,qh,tokens,dim", [(2, 8, 37, 64), (8, 32, 1000, 128), (1, 4, 1, 128),
                                               (2, 8, 513, 96), (3, 6, 300, 256), (2, 16, 77, 80)])
def test_score_bit_exact(qdtype, kvh, qh, tokens, dim):
    k = synthetic_keys(kvh, tokens, dim, seed=tokens, dtype=torch.bfloat16)
    q = synthetic_keys(1, qh, dim, seed=tokens + 1, dtype=qdtype)
    h2k = torch.arange(qh) // (qh // kvh)
    packed = pk.pack_keys(k.to(DEV), token_capacity=tokens + 16)
    got = pk.score(q.to(DEV), packed, head_to_kv=h2k.to(DEV), tokens=tokens).cpu().numpy()
    ref = O.score(q.float().numpy(), O.pack_keys(k.float().numpy(), capacity=tokens + 16),
                  head_to_kv=h2k.numpy(), tokens=tokens)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("kvh,qh,tokens,dim", [(4, 4, 2000, 128), (2, 6, 1500, 64), (8, 32, 2500, 128),
                                               (2, 16, 1100, 128), (1, 12, 3000, 128), (2, 32, 700, 128),
                                               (3, 12, 1024, 256), (2, 8, 4096, 96)])
def test_score_aligned_capacity_head_groups_bit_exact(kvh, qh, tokens, dim):
    """Bit-exact for 1 to 16 query heads per KV head and ragged last tiles; the
    histograms add up to the row length (and are skipped above 8 heads per KV head)."""
    k = synthetic_keys(kvh, tokens, dim, seed=tokens + dim, dtype=torch.bfloat16)
    q = synthetic_keys(1, qh, dim, seed=tokens + 2, dtype=torch.bfloat16)
    h2k = torch.arange(qh) // (qh // kvh)
    cap = (tokens + 63) // 64 * 64
    packed = pk.pack_keys(k.to(DEV), token_capacity=cap)
    hist = pk.new_select_workspace(qh, tokens, DEV)
    got = pk.score(q.to(DEV), packed, head_to_kv=h2k.to(DEV), tokens=tokens, hist=hist)
    ref = O.score(q.float().numpy(), O.pack_keys(k.float().numpy(), capacity=cap),
                  head_to_kv=h2k.numpy(), tokens=tokens)
    np.testing.assert_array_equal(got.cpu().numpy(), ref)
    counts = hist[: qh * 2048 * 4].view(torch.int32).view(qh, 2048).sum(1).cpu()
    per_kv = qh // kvh
    if per_kv <= 8:
        assert (counts == tokens).all()
    else:  # histogram skipped for KV heads with more than 8 query heads
        assert (counts == 0).all()


def test_score_reference_tolerance(golden):
    """The reference test's own case (tests/test_popkv.py:45-54) against its readable scores."""
    keys, queries = golden["ref_test_shape/keys"], golden["ref_test_shape/queries"]
    mapping, expected = golden["ref_test_shape/head_to_kv"], golden["ref_test_shape/scores"]
    packed = pk.pack_keys(torch.from_numpy(keys).bfloat16().to(DEV))
    got = pk.score(torch.from_numpy(queries).bfloat16().to(DEV), packed,
                   head_to_kv=torch.from_numpy(mapping).to(DEV), tokens=keys.shape[1])
    torch.testing.assert_close(got.cpu(), torch.from_numpy(expected), atol=0.12, rtol=0.02)


def test_score_nonstandard_head_mapping_and_batch():
    k = synthetic_keys(4, 200, 128, seed=1, dtype=torch.bfloat16)
    q = synthetic_keys(3, 8, 128, seed=2, dtype=torch.bfloat16)
    h2k = torch.tensor([3, 0, 0, 2, 1, 3, 2, 0])
    packed = pk.pack_keys(k.to(DEV))
    got = pk.score(q.to(DEV), packed, head_to_kv=h2k.to(DEV), tokens=200).cpu().numpy()
    ref = O.score(q.float().numpy(), O.pack_keys(k.float().numpy()), head_to_kv=h2k.numpy(), tokens=200)
    np.testing.assert_array_equal(got, ref)


def test_score_per_batch_caches_and_device_lengths():
    B, H, QH, D, cap = 3, 2, 8, 128, 160
    k = synthetic_keys(B * H, cap, D, seed=11, dtype=torch.bfloat16)
    q = synthetic_keys(B, QH, D, seed=12, dtype=torch.bfloat16)
    packed = pk.pack_keys(k.to(DEV), token_capacity=cap)
    packed4 = tuple(t.view(B, H, cap, -1) for t in packed)
    lens = [160, 33, 100]
    h2k = torch.arange(QH) // (QH // H)
    out = torch.full((B, QH, cap), -7.0, device=DEV)
    pk.score(q.to(DEV), packed4, head_to_kv=h2k.to(DEV), tokens=cap,
             seq_len=torch.tensor(lens, dtype=torch.int32, device=DEV), out=out)
    got = out.cpu().numpy()
    ref = O.score(q.float().numpy(), O.pack_keys(k.float().numpy(), capacity=cap),
                  head_to_kv=h2k.numpy(), lengths=lens, cache_per_batch=True, kv_heads=H,
                  tokens=cap)
    for b, L in enumerate(lens):
        np.testing.assert_array_equal(got[b, :, :L], ref[b, :, :L])
        assert (got[b, :, L:] == -7.0).all()


def test_score_full_size_llama_layer():
    L = 32768
    k = synthetic_keys(8, L, 128, seed=0, dtype=torch.bfloat16)
    q = synthetic_keys(1, 32, 128, seed=1, dtype=torch.bfloat16)
    h2k = torch.arange(32) // 4
    packed = pk.pack_keys(k.to(DEV), token_capacity=L + 2048)
    got = pk.score(q.to(DEV), packed, head_to_kv=h2k.to(DEV), tokens=L).cpu().numpy()
    ref = O.score(q.float().numpy(), O.pack_keys(k.float().numpy(), capacity=L + 2048),
                  head_to_kv=h2k.numpy(), tokens=L)
    np.testing.assert_array_equal(got, ref)


def test_score_errors():
    packed = pk.pack_keys(torch.zeros(2, 32, 64, device=DEV))
    q = torch.zeros(1, 4, 64, device=DEV)
    with pytest.raises(RuntimeError, match="token count"):
        pk.score(q, packed, head_to_kv=torch.zeros(4, dtype=torch.long, device=DEV), tokens=33)
    with pytest.raises(ValueError):
        pk.score(q[0], packed, head_to_kv=torch.zeros(4, dtype=torch.long, device=DEV), tokens=3)
