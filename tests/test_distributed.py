"""KV-head sharding across ranks with an all-gather of the outputs (gloo, world size 2).

Each rank attends with its shard of KV heads (the CPU oracle stands in for the
kernels, which need a GPU); the all-gathered, re-ordered outputs must equal the
unsharded attention.
"""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import popkv
import popkv_oracle as O


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(0)
    B, KVH, QH, D, L, budget = 2, 4, 16, 64, 80, 24
    q = rng.standard_normal((B, QH, D)).astype(np.float32)
    kc = rng.standard_normal((B, KVH, L + 1, D)).astype(np.float32)
    vc = rng.standard_normal((B, KVH, L + 1, D)).astype(np.float32)
    scores = rng.standard_normal((B * QH, L)).astype(np.float32)
    idx = O.select(scores, budget=budget)
    return B, KVH, QH, D, L, budget, q, kc, vc, idx


def _worker(rank, world, port, result):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    B, KVH, QH, D, L, budget, q, kc, vc, idx = _inputs()
    (k0, k1), (q0, q1) = popkv.shard_heads(rank, world, KVH, QH)
    G = QH // KVH
    idx_local = idx.reshape(B, QH, budget)[:, q0:q1].reshape(-1, budget)
    out = O.attention(q[:, q0:q1], kc[:, k0:k1].reshape(-1, L + 1, D), vc[:, k0:k1].reshape(-1, L + 1, D),
                      head_to_kv=np.arange(q1 - q0) // G, lengths=[L] * B, indices=idx_local,
                      cache_per_batch=True, kv_heads=k1 - k0)
    local = torch.from_numpy(out).reshape(B, q1 - q0, D)
    gathered = torch.empty(world * B, q1 - q0, D)
    dist.all_gather_into_tensor(gathered, local)
    if rank == 0:
        result.put(popkv.gather_head_shards(gathered, B).numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_head_sharded_attention_all_gather_matches_unsharded():
    B, KVH, QH, D, L, budget, q, kc, vc, idx = _inputs()
    full = O.attention(q, kc.reshape(-1, L + 1, D), vc.reshape(-1, L + 1, D),
                       head_to_kv=np.arange(QH) // (QH // KVH), lengths=[L] * B, indices=idx,
                       cache_per_batch=True, kv_heads=KVH)
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    got = result.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    np.testing.assert_allclose(got, full, rtol=1e-6, atol=1e-6)
