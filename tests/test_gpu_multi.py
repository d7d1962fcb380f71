"""Multi-GPU decode step (one process per GPU): the output all-gather fused into the
attention combine (NVLink peer stores + arrival words) equals an NCCL all-gather of
the same outputs, eagerly and under CUDA-graph replay.  Needs 2 GPUs; skipped otherwise."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int) -> None:
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        import popkv
        layers, B, KVH, QH, D, T, budget = 2, 2, 4, 16, 128, 700, 64
        os.environ["POPKV_GATHER"] = "peer"
        stack = popkv.RetrievalStack(layers=layers, batch=B, kv_heads=KVH, q_heads=QH, head_dim=D,
                                     max_tokens=T + 8, budget=budget, process_group=dist.group.WORLD)
        assert stack.peer is not None
        g = torch.Generator(device="cuda").manual_seed(100 + rank)
        for i in range(layers):
            k = torch.randn(B, stack.kv_heads, T, D, device="cuda", generator=g, dtype=torch.float32)
            v = torch.randn(B, stack.kv_heads, T, D, device="cuda", generator=g, dtype=torch.float32)
            stack.prefill(i, k.bfloat16(), v.bfloat16())
        stack.set_length(T)

        def inputs():
            q = torch.randn(layers, B, stack.q_heads, D, device="cuda", generator=g).bfloat16()
            kk = torch.randn(layers, B, stack.kv_heads, D, device="cuda", generator=g).bfloat16()
            vv = torch.randn(layers, B, stack.kv_heads, D, device="cuda", generator=g).bfloat16()
            return q, kk, vv

        for step in range(4):
            if step == 2:
                stack.capture()
            got = stack.step(*inputs()).clone()
            torch.cuda.synchronize()
            ref = torch.empty_like(got)
            for i in range(layers):
                dist.all_gather_into_tensor(ref[i], stack.out[i], group=dist.group.WORLD)
            torch.cuda.synchronize()
            assert torch.equal(got, ref), f"rank {rank} step {step}: peer all-gather differs"
        assert stack.peer_errors() == 0
        stack.graph = None
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_peer_allgather_matches_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)
