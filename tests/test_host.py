"""Host-side logic that needs no GPU: configuration, sharding, the Python surface's
argument checks and the loud failure without a GPU."""
import pytest
import torch

import popkv
import popkv_cuda
import _native


def test_public_methods_are_the_reference_methods():
    assert popkv.METHODS == ("full", "quest", "fier", "popkv")


def test_release_configuration_is_explicit():
    popkv.RetrievalConfig().validate()
    with pytest.raises(ValueError):
        popkv.RetrievalConfig(group_size=64).validate()
    with pytest.raises(ValueError):
        popkv.RetrievalConfig(budget=1).validate()


def test_entry_points_reject_cpu_and_noncontiguous_inputs():
    with pytest.raises(ValueError):
        popkv_cuda.pack_keys(torch.zeros(2, 8, 64))
    with pytest.raises(ValueError):
        popkv_cuda.pack_keys_into(torch.zeros(2, 8, 64), (None,) * 4, token_offset=0)
    with pytest.raises(ValueError):
        popkv_cuda.score(torch.zeros(1, 8, 64), (None,) * 4, head_to_kv=torch.zeros(8), tokens=8)
    with pytest.raises(ValueError):
        popkv_cuda.pack_keys(torch.zeros(2, 8))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU failure")
def test_extension_raises_without_gpu():
    with pytest.raises(RuntimeError, match="requires an NVIDIA GPU"):
        _native.extension()


def test_shard_heads_partitions_kv_and_query_heads():
    seen_kv, seen_q = [], []
    for r in range(4):
        (k0, k1), (q0, q1) = popkv.shard_heads(r, 4, 8, 32)
        seen_kv += list(range(k0, k1))
        seen_q += list(range(q0, q1))
        assert all(q // 4 in range(k0, k1) for q in range(q0, q1))
    assert seen_kv == list(range(8)) and seen_q == list(range(32))
    with pytest.raises(ValueError):
        popkv.shard_heads(0, 3, 8, 32)


def test_gather_head_shards_restores_head_order():
    B, W, QHl, D = 3, 2, 4, 5
    full = torch.arange(B * W * QHl * D, dtype=torch.float32).view(B, W * QHl, D)
    shards = torch.cat([full[:, r * QHl:(r + 1) * QHl] for r in range(W)], dim=0)
    torch.testing.assert_close(popkv.gather_head_shards(shards, B), full)
