"""Multi-GPU decode step (one process per GPU): the output all-gather fused into the
attention combine (NVLink peer stores + arrival words) equals an NCCL all-gather of
the same outputs -- eagerly and under CUDA-graph replay, with the per-layer and the
per-step (deferred) wait, and over back-to-back graph replays with no host barrier
between steps while one rank lags behind (the cross-step reuse of the gathered
buffers).  Needs 2 GPUs; skipped otherwise."""
import os
import socket
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _make_stack(rank, layers, B, KVH, QH, D, T, budget, gather_wait, steps_reserve=32):
    import torch.distributed as dist

    import popkv
    stack = popkv.RetrievalStack(layers=layers, batch=B, kv_heads=KVH, q_heads=QH, head_dim=D,
                                 max_tokens=T + steps_reserve, budget=budget,
                                 process_group=dist.group.WORLD, gather_wait=gather_wait)
    assert stack.peer is not None
    g = torch.Generator(device="cuda").manual_seed(100 + rank)
    for i in range(layers):
        k = torch.randn(B, stack.kv_heads, T, D, device="cuda", generator=g, dtype=torch.float32)
        v = torch.randn(B, stack.kv_heads, T, D, device="cuda", generator=g, dtype=torch.float32)
        stack.prefill(i, k.bfloat16(), v.bfloat16())
    stack.set_length(T)
    return stack, g


def _inputs(stack, layers, B, D, g):
    q = torch.randn(layers, B, stack.q_heads, D, device="cuda", generator=g).bfloat16()
    kk = torch.randn(layers, B, stack.kv_heads, D, device="cuda", generator=g).bfloat16()
    vv = torch.randn(layers, B, stack.kv_heads, D, device="cuda", generator=g).bfloat16()
    return q, kk, vv


def _rank_main(rank: int, world: int, port: int) -> None:
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["POPKV_GATHER"] = "peer"
    torch.cuda.set_device(rank)
    from datetime import timedelta
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        layers, B, KVH, QH, D, T, budget = 2, 2, 4, 16, 128, 700, 64
        # 1. Eager then graph-replayed steps, host-synchronised, both wait modes.
        for mode in ("layer", "step"):
            stack, g = _make_stack(rank, layers, B, KVH, QH, D, T, budget, mode)
            for step in range(5):
                if step == 2:
                    stack.capture()
                got = stack.step(*_inputs(stack, layers, B, D, g), check=True).clone()
                torch.cuda.synchronize()
                ref = torch.empty_like(got)
                for i in range(layers):
                    dist.all_gather_into_tensor(ref[i], stack.out[i], group=dist.group.WORLD)
                torch.cuda.synchronize()
                assert torch.equal(got, ref), f"rank {rank} {mode} step {step}: peer all-gather differs"
            assert stack.peer_errors() == 0
            stack.graph = None
            dist.barrier()
            del stack

        # 2. Back-to-back replays with no host barrier between steps; rank 1 lags on
        #    the host before some steps, so rank 0 runs ahead into the next step.
        #    Every step's own outputs and gathered rows are copied to pinned host
        #    memory on the stream (the consumer of the step), then compared at the end.
        for mode in ("step", "layer"):
            stack, g = _make_stack(rank, layers, B, KVH, QH, D, T, budget, mode)
            steps = 10
            ins = [_inputs(stack, layers, B, D, g) for _ in range(steps)]
            stack.step(*ins[0])
            stack.capture()
            torch.cuda.synchronize()
            dist.barrier()
            outs = [torch.empty(stack.out.shape, dtype=stack.out.dtype).pin_memory() for _ in range(steps)]
            gath = [torch.empty(stack.gathered.shape, dtype=stack.out.dtype).pin_memory() for _ in range(steps)]
            for s in range(1, steps):
                if rank == 1 and s % 3 == 1:
                    time.sleep(0.05)
                res = stack.step(*ins[s])
                gath[s].copy_(res, non_blocking=True)
                outs[s].copy_(stack.out, non_blocking=True)
            torch.cuda.synchronize()
            assert stack.peer_errors() == 0
            for s in range(1, steps):
                mine = outs[s].cuda()
                ref = torch.empty(gath[s].shape, dtype=mine.dtype, device="cuda")
                for i in range(layers):
                    dist.all_gather_into_tensor(ref[i], mine[i], group=dist.group.WORLD)
                torch.cuda.synchronize()
                assert torch.equal(gath[s], ref.cpu()), f"rank {rank} {mode} replay {s}: gathered rows differ"
            stack.graph = None
            dist.barrier()
            del stack
    finally:
        dist.destroy_process_group()


def test_peer_allgather_matches_nccl():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)
