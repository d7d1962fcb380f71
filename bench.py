"""Pop-KV decode-time retrieval benchmark (B200).

Workload: Llama-3.1-8B attention shapes -- 32 query / 8 KV
heads, head_dim 128, bf16 K/V cache at 32768 tokens, group 32, budget 4096 --
over 32 layer copies (so every step touches far more than the 126 MB L2), each
decode step appending one token per layer (open-group re-pack) and scoring a
fresh synthetic query.  One step = score -> select -> fused gather+attention ->
append for all 32 layers, replayed as one CUDA graph.

Multi-GPU (torchrun, one rank per GPU): weak scaling by KV head -- the job holds
N sequences, rank r owns KV heads [r*8/N, (r+1)*8/N) of all of them (so per-GPU
bytes stay those of one 8-head sequence) and all-gathers every layer's attention
output over NCCL.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  --impl reference times the reference's own CPU
path (the readable reconstruction scorer + torch.topk + gather + SDPA, restated
in oracle/reconstruction.py) on the host cores, one layer-step per step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for p in (ROOT / "fier-2bits_b200", ROOT / "oracle"):
    sys.path.insert(0, str(p))

import torch  # noqa: E402

METRIC = "retrieval ms/decode-step per layer (score+topk+gather+attn) and HBM GB/s vs peak"
KVH, QH, D = 8, 32, 128
PACKED_BYTES = 48  # per token per KV head at D = 128
WORKLOADS = {
    1: "configs[1]: Llama-3.1-8B attention layer, 32 q / 8 kv heads, head_dim 128, bf16 cache, "
       "group 32, one append per step",
    3: "configs[3]: batched long-context attention-only stack, 16 sequences x 131072 tokens, "
       "32 q / 8 kv heads, head_dim 128, bf16 cache, budget 4096, one append per step, "
       "KV heads sharded over the GPUs",
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--context", type=int, default=32768)
    ap.add_argument("--budget", type=int, default=4096)
    ap.add_argument("--cpu-sample-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, choices=(1, 2, 3), default=1,
                    help="1: configs[1] (default, weak scaling by sequence); "
                         "2: configs[2] (32-layer Llama-3.1-8B-shaped decoder, 32K prefill, greedy decode); "
                         "3: configs[3] (16 sequences x 128K tokens, strong scaling by KV head)")
    return ap.parse_args()


def measured_peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling (every 100 ms) filtered to the timed window afterwards."""
    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.lines = index, None, []
        self.window = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        import datetime as dt
        rows = []
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                ts = dt.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(f[1]), float(f[2]), [n for n, v in zip(self.NAMES, f[5:9])
                                                            if v.lower() == "active"]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        t0, t1 = self.window or (rows[0][0], rows[-1][0])
        inside = [r for r in rows if t0 - 0.05 <= r[0] <= t1 + 0.05]
        picked = inside or [min(rows, key=lambda r: abs(r[0] - (t0 + t1) / 2))]
        reasons = sorted({n for r in picked for n in r[3]})
        return {"sm_mhz": statistics.median(r[1] for r in picked), "sm_max_mhz": picked[-1][2],
                "reasons": reasons, "samples_in_window": len(inside),
                "window_s": round(t1 - t0, 3)}


# --------------------------------------------------------------- CPU paths
def cpu_layer_step(L: int, budget: int, seed: int):
    """Inputs for one layer-step of the reference CPU path (fp32, configs[1] shapes)."""
    from synthetic import SyntheticLayer
    syn = SyntheticLayer(kv_heads=KVH, q_heads=QH, head_dim=D, seed=seed)
    k, v = syn.keys_values(L + 1)
    k, v = k[0].bfloat16().float(), v[0].bfloat16().float()
    q = syn.queries(L)[0].bfloat16().float()
    return q, k, v


def time_cpu_reference(L: int, budget: int, steps: int, warmup: int):
    """ms per layer-step of the reference's readable CPU path on all host threads."""
    import reconstruction as R
    torch.set_num_threads(os.cpu_count() or 1)
    q, k, v = cpu_layer_step(L, budget, seed=123)
    h2k = torch.arange(QH) // (QH // KVH)
    prefix_k, prefix_v = k[:, :L].contiguous(), v[:, :L].contiguous()
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        R.decode_step(q, prefix_k, prefix_v, k[:, L], v[:, L], head_to_kv=h2k, budget=budget)
        if i >= warmup:
            times.append((time.perf_counter() - t0) * 1e3)
    return sum(times) / len(times), torch.get_num_threads()


# -------------------------------------------------------------- GPU run
def algorithmic_bytes(L, budget, B, kvh, qh, union_rows):
    score = B * kvh * L * PACKED_BYTES + B * qh * D * 2 + B * qh * L * 4
    select = B * qh * L * 4 + B * qh * budget * 4
    attn = 2 * D * 2 * union_rows + B * qh * budget * 4 + 2 * B * qh * D * 2
    append = B * kvh * (32 * D * 2 + 32 * PACKED_BYTES)  # worst case: a full open group
    # Fused score + select: the packed rows and queries in, the selections out; the
    # fp32 score round trip of the two-kernel form is gone.
    score_select = B * kvh * L * PACKED_BYTES + B * qh * D * 2 + B * qh * budget * 4
    return {"score": score, "select": select, "attention": attn, "append": append,
            "score_select": score_select}


def layer_bytes(B, kvh_local, kv_cap):
    """Device bytes one RetrievalStack layer holds: bf16 K and V caches + packed keys."""
    cap = (kv_cap + 31) // 32 * 32
    return 2 * B * kvh_local * kv_cap * D * 2 + B * kvh_local * cap * PACKED_BYTES


def run_ours(args):
    import torch.distributed as dist

    import popkv
    import popkv_cuda as pk
    from synthetic import SyntheticLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(minutes=5))
        group = dist.group.WORLD
    layers, L0, budget = args.layers, args.context, args.budget
    total_steps = min(args.warmup + args.steps + 2, 64)  # distinct per-step inputs, reused cyclically
    reserve = args.warmup + 2 * args.steps + 4
    if args.config == 3:
        # 16 sequences x 131072 tokens, KV heads sharded over the ranks
        # (total work fixed); as many of the 32 layers as this GPU's HBM holds.
        B = 16
        if args.context == 32768:
            L0 = 131072
        per_layer = layer_bytes(B, KVH // world, L0 + reserve + 1)
        free = torch.cuda.mem_get_info(dev)[0] - (6 << 30)
        layers = max(1, min(32 if args.layers == 32 else args.layers, int(free // per_layer)))
    else:
        B = world  # weak scaling: one sequence per GPU, sharded by KV head
    stack = popkv.RetrievalStack(layers=layers, batch=B, kv_heads=KVH, q_heads=QH, head_dim=D,
                                 max_tokens=L0 + reserve, budget=budget,
                                 dtype=torch.bfloat16, device=dev, process_group=group)
    (k0, k1), (q0, q1) = stack.kv_range, stack.q_range
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)  # 2x L2
    # One untimed pack first: the kernel's module load and launch set-up stay out of
    # the timed prefill packs.
    warm = torch.zeros(k1 - k0, 64, D, dtype=torch.bfloat16, device=dev)
    pk.pack_keys(warm, token_capacity=64)
    torch.cuda.synchronize()
    del warm
    pack_ms = 0.0
    gens = []
    for i in range(layers):
        syn = SyntheticLayer(kv_heads=KVH, q_heads=QH, head_dim=D, seed=1000 + i, batch=B, device=dev)
        for b in range(B):
            # Prefill a sequence at a time (same outlier channels as the layer's queries).
            one = SyntheticLayer(kv_heads=KVH, q_heads=QH, head_dim=D, seed=1000 + i, device=dev)
            one.gen.manual_seed(7919 * (i + 1) + b)
            k, v = one.keys_values(L0)
            kb, vb = k[0, k0:k1].bfloat16().contiguous(), v[0, k0:k1].bfloat16()
            del k, v
            # The prefill pack of this sequence's heads, timed cold (L2 flushed).
            packed_b = tuple(p[b].reshape(-1, stack.capacity, p.shape[-1]) for p in stack.packed[i])
            flush.fill_(i & 0xff)
            a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda._sleep(400000)  # keep the GPU busy while the host queues the pack
            a.record()
            pk.pack_keys_into(kb, packed_b, token_offset=0)
            z.record()
            stack.prefill(i, kb, vb, sequence=b)
            torch.cuda.synchronize()
            pack_ms += a.elapsed_time(z)
            del kb, vb
        gens.append(syn)
    pack_ms /= layers
    del flush
    stack.set_length(L0)
    # Per-step inputs, generated up front (device pool for the kernel-only timing).
    qs, ks, vs = [], [], []
    for s in range(total_steps):
        q_l, k_l, v_l = [], [], []
        for i in range(layers):
            syn = gens[i]
            q_l.append(syn.queries(L0 + s)[:, q0:q1].bfloat16())
            kn, vn = syn.keys_values(1, start=L0 + s)
            k_l.append(kn[:, k0:k1, 0].bfloat16())
            v_l.append(vn[:, k0:k1, 0].bfloat16())
        qs.append(torch.stack(q_l)); ks.append(torch.stack(k_l)); vs.append(torch.stack(v_l))
    torch.cuda.synchronize()

    clocks = ClockSampler(local).start()
    # Warm-up (eager first step, then graph capture, then graph replays).
    stack.step(qs[0], ks[0], vs[0])
    stack.capture()
    step_idx = 1
    for _ in range(max(args.warmup - 1, 0)):
        j = step_idx % total_steps
        stack.step(qs[j], ks[j], vs[j]); step_idx += 1
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- timed region: K graph-replayed decode steps, inputs resident in HBM.
    stream = torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(); torch.cuda.synchronize()
    w0 = time.time()
    start.record(stream)
    for s in range(args.steps):
        j = step_idx + s
        stack.step(qs[j % total_steps], ks[j % total_steps], vs[j % total_steps])
    end.record(stream)
    torch.cuda.synchronize()
    clocks.window = (w0, time.time())
    time.sleep(0.3)
    clocks.stop()
    barrier()
    elapsed = torch.tensor([start.elapsed_time(end)], device=dev)
    gather_check = None
    if world > 1:
        # The last timed step's all-gathered outputs against an NCCL all-gather of
        # every rank's own outputs of that step: bit for bit.
        ref = torch.empty_like(stack.gathered)
        for i in range(layers):
            dist.all_gather_into_tensor(ref[i], stack.out[i], group=group)
        bad = torch.tensor([int((ref != stack.gathered).any(dim=-1).sum())], device=dev)
        dist.all_reduce(bad)
        gather_check = "ok" if int(bad) == 0 else f"{int(bad)} rows differ"
    if world > 1:
        dist.all_reduce(elapsed, op=dist.ReduceOp.MAX)
    ms_step = float(elapsed) / args.steps
    ms_layer = ms_step / layers

    # ---- per-stage timing (idempotent re-runs of each stage over all layers, no advance).
    stage_ms = {}
    reps = 20
    tokens = stack.max_tokens

    sizes = (B, stack.q_heads, stack.kv_heads, D, tokens, 0)

    def run_stage(name, i):
        parts = name.split("+")
        if "scoresel" in parts:
            pk.score_select(stack.q_in[i], stack.packed[i], head_to_kv=stack.head_to_kv,
                            budget=budget, tokens=tokens, seq_len=stack.seq_len,
                            out=stack.indices[i], attn_workspace=stack.workspace[i],
                            attn_sizes=sizes, scores=stack.scores, hist=stack.score_hist)
        if "score" in parts:
            pk.score(stack.q_in[i], stack.packed[i], head_to_kv=stack.head_to_kv, tokens=tokens,
                     seq_len=stack.seq_len, out=stack.scores, hist=stack.score_hist)
        if "select" in parts:
            pk.select(stack.scores.view(-1, stack.capacity), budget=budget, tokens=tokens,
                      seq_len=stack.seq_len, rows_per_seq=stack.q_heads, out=stack.indices[i],
                      attn_workspace=stack.workspace[i], attn_sizes=sizes, hist=stack.score_hist)
        if "attention" in parts:  # consumes (and clears) the masks select wrote
            pk.sparse_attention_premasked(stack.q_in[i], stack.key_cache[i], stack.value_cache[i],
                                          tokens=tokens, current_keys=stack.k_in[i],
                                          current_values=stack.v_in[i], seq_len=stack.seq_len,
                                          workspace=stack.workspace[i], out=stack.out[i])
        if "append" in parts:
            pk.append_keys(stack.key_cache[i], stack.value_cache[i], stack.k_in[i], stack.v_in[i],
                           stack.packed[i], position=0, seq_len=stack.seq_len,
                           kv_heads_per_seq=stack.kv_heads)

    def stage_graph(name):
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                for i in range(layers):
                    run_stage(name, i)
        stream.wait_stream(side)
        return g

    # Each select needs the histogram its score just built, and each attention the
    # masks its select just wrote: time the prefixes of the layer pipeline and take
    # differences.
    timed = {}
    names = ["score+select+attention", "score", "score+select", "append"]
    if stack.fused_select:
        names = ["scoresel+attention", "scoresel"] + names
    for name in names:
        for i in range(layers):
            run_stage(name, i)  # eager warm-up of this stage
        if name == "score":
            torch.cuda.synchronize()
        g = stage_graph(name)
        g.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            g.replay()
        b.record(stream)
        torch.cuda.synchronize()
        timed[name] = a.elapsed_time(b) / (reps * layers)
        if name == "score":  # histograms accumulated without a select: start clean
            stack.score_hist.zero_()
        del g
    stage_ms["score"] = timed["score"]
    stage_ms["select"] = timed["score+select"] - timed["score"]
    stage_ms["attention"] = timed["score+select+attention"] - timed["score+select"]
    stage_ms["append"] = timed["append"]
    if stack.fused_select:  # the decode step runs the fused kernel
        stage_ms["score_select"] = timed["scoresel"]
        stage_ms["attention"] = timed["scoresel+attention"] - timed["scoresel"]
    # The score+select replays left masks set: clear them with one attention pass.
    for i in range(layers):
        run_stage("attention", i)
    torch.cuda.synchronize()

    # Union of selections per (sequence, KV head) -> attention's algorithmic bytes.
    L_now = stack.length
    union_rows = 0
    G = stack.q_heads // stack.kv_heads
    for i in range(layers):
        # Rows of one (sequence, KV head) group are contiguous: sort each group's
        # selections and count distinct non-negative indices.
        idx = stack.indices[i].view(B * stack.kv_heads, G * budget).sort(dim=1).values
        new = torch.ones_like(idx, dtype=torch.bool)
        new[:, 1:] = idx[:, 1:] != idx[:, :-1]
        union_rows += int((new & (idx >= 0)).sum())
    union_rows //= layers
    nbytes = algorithmic_bytes(L_now, budget, B, stack.kv_heads, stack.q_heads, union_rows)
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    # Prefill pack (once per prefix, not part of the decode step): keys in, packed out.
    stage_ms["pack"] = pack_ms
    nbytes["pack"] = B * stack.kv_heads * L0 * (D * 2 + PACKED_BYTES)
    stages = {n: {"ms": stage_ms[n], "bytes": nbytes[n],
                  "gbs": nbytes[n] / (stage_ms[n] * 1e-3) / 1e9,
                  "frac": nbytes[n] / (stage_ms[n] * 1e-3) / 1e9 / hbm} for n in stage_ms}
    stages["pack"]["note"] = "one-time prefill pack per layer (all sequences), L2 flushed, not in value"
    in_step = ("score_select", "attention") if stack.fused_select else ("score", "select", "attention")
    if stack.fused_select:
        for n in ("score", "select"):
            stages[n]["note"] = "two-kernel form, not in the decode step (the fused score_select runs)"
    dominant = max(in_step, key=lambda n: stage_ms[n])
    traffic = None  # DRAM bytes per launch from the committed ncu summary of this workload
    try:
        for ln in (ROOT / "profiles" / "roofline_traffic_configs1.txt").read_text().splitlines():
            name, val = ln.split()[:2]
            if name.startswith(dominant) and L0 == 32768 and world == 1 and args.config == 1:
                traffic = float(val)
    except Exception:
        traffic = None
    step_bytes = sum(nbytes[n] for n in in_step + ("append",))

    # ---- e2e: public API with pinned host inputs and outputs, copies inside the region.
    host_q = [qs[s].cpu().pin_memory() for s in range(total_steps)]
    host_k = [ks[s].cpu().pin_memory() for s in range(total_steps)]
    host_v = [vs[s].cpu().pin_memory() for s in range(total_steps)]
    out_shape = (stack.gathered if world > 1 else stack.out).shape
    host_out = torch.empty(out_shape, dtype=torch.bfloat16).pin_memory()
    # Reset lengths so the e2e steps stay inside the reserve.
    stack.set_length(L0)
    torch.cuda.synchronize(); barrier()
    t0 = time.perf_counter()
    for s in range(args.steps):
        j = s % total_steps
        res = stack.step(host_q[j].to(dev, non_blocking=True), host_k[j].to(dev, non_blocking=True),
                         host_v[j].to(dev, non_blocking=True))
        host_out.copy_(res, non_blocking=True)
    torch.cuda.synchronize()
    e2e_ms = torch.tensor([(time.perf_counter() - t0) * 1e3], device=dev)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_layer = float(e2e_ms) / (args.steps * layers)
    h2d = host_q[0].nbytes + host_k[0].nbytes + host_v[0].nbytes
    d2h = host_out.nbytes

    peer_errors = stack.peer_errors() if world > 1 else 0
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_ms, cores = time_cpu_reference(L0, budget, args.cpu_sample_steps, 1)
        cpu_baseline = {"value": cpu_ms * B, "unit": "ms", "cores": cores, "kind": "port",
                        "sample": f"{args.cpu_sample_steps} layer-steps of one sequence "
                                  f"(L={L0}, budget={budget}, 8 KV / 32 q heads, fp32 upcast of "
                                  f"bf16), after 1 warm-up" + (f"; x{B} sequences" if B > 1 else "")}

    if rank == 0:
        dom = stages[dominant]
        line = {
            "metric": METRIC, "value": ms_layer, "unit": "ms", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": False, "scaling": "weak" if args.config == 1 else "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) K/V/Q, 4 outlier channels x8, RoPE 5e5)",
            "config": {"workload": WORKLOADS[args.config] + (f" ({layers} of 32 layers: what one GPU holds)"
                                                             if args.config == 3 and layers < 32 else ""),
                       "context": L0, "budget": budget, "layers_per_step": layers,
                       "sequences": B, "parallelism": (f"kv-head shards x{world}, " + ("output all-gather fused into the attention combine (NVLink peer stores)"
                                                                       if stack.peer is not None else "NCCL all-gather per layer"))
                                      if world > 1 else "none",
                       "l2": f"inputs larger than L2 ({layers} layers rotate through "
                             f"{layers * layer_bytes(B, stack.kv_heads, stack.kv_capacity) / 1e9:.1f} GB per GPU)",
                       "graph": "one CUDA graph per decode step"},
            "hbm_gbs_step": step_bytes / (ms_layer * 1e-3) / 1e9,
            "stages": stages,
            "roofline": {"kernel": dominant, "bound": "hbm", "achieved": dom["gbs"],
                         "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s", "frac": dom["frac"],
                         "traffic": traffic, "algorithmic_bytes": dom["bytes"],
                         "union_rows_per_layer": union_rows},
            # The fused score + select is bound by the POPC pipe, not by HBM: 24
            # popcounts per token·query head (5 per head·word + 1 per token·word).
            "popc_roofline": {
                "kernel": "score_select",
                "achieved": B * stack.q_heads * L_now * 24 / (stage_ms.get("score_select", float("nan")) * 1e-3) / 1e9,
                "peak": 16 * torch.cuda.get_device_properties(dev).multi_processor_count
                        * float(clocks.summary().get("sm_max_mhz") or 1965.0) / 1e3,
                "unit": "Gpopc/s", "peak_note": "16 POPC per clock per SM at the max SM clock"}
            if stack.fused_select else None,
            "clocks": clocks.summary(),
            "e2e": {"value": e2e_layer, "unit": "ms", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": stack.launches_per_step() * args.steps,
            "cpu_baseline": cpu_baseline,
        }
        if line.get("popc_roofline"):
            pr = line["popc_roofline"]
            pr["frac"] = pr["achieved"] / pr["peak"]
        if world > 1:
            line["gather_check"] = gather_check
            line["config"]["gather_wait"] = stack.gather_wait if stack.peer is not None else "nccl"
        if world > 1 and peer_errors:
            line["error"] = f"{peer_errors} peer all-gather waits ran out"
        print(json.dumps(line), flush=True)
    if world > 1:
        # Tearing NCCL down while captured graphs still reference its communicator can
        # block; every rank has finished its collectives, so drop the graphs and leave.
        stack.graph = None
        torch.cuda.synchronize()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(0)


def run_decoder(args):
    """random-init Llama-3.1-8B-shaped decoder, prefill + greedy decode.

    One step = one token through all 32 layers (Pop-KV retrieval at the given budget
    in layers 2..31, dense attention in layers 0 and 1, as the reference's
    full_layers default), replayed as one CUDA graph.  The `full` method (dense
    attention in every layer) is timed the same way for comparison.
    """
    from transformers import LlamaConfig, LlamaForCausalLM

    import popkv
    from decoder import GraphedDecoder

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        raise SystemExit("--config 2 runs on one GPU")
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L0, budget = args.context, args.budget
    cfg = LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                      num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, rms_norm_eps=1e-5, rope_theta=500000.0,
                      max_position_embeddings=L0 + args.steps + args.warmup + 64,
                      tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    with torch.device(dev):
        model = LlamaForCausalLM(cfg).to(torch.bfloat16).eval()
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (L0,), generator=g)
    peaks, peak_kind = measured_peaks()
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    results = {}
    clocks = None
    for method in ("popkv", "full"):
        dec = GraphedDecoder(model, popkv.RetrievalConfig(budget=budget),
                             max_tokens=L0 + args.warmup + 2 * args.steps + 8, method=method)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        dec.prefill(prompt)
        torch.cuda.synchronize()
        prefill_s = time.perf_counter() - t0
        dec.step()  # eager warm-up
        dec.capture()
        for _ in range(args.warmup - 1):
            dec.step()
        torch.cuda.synchronize()
        if method == "popkv":
            clocks = ClockSampler(0).start()
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        w0 = time.time()
        a.record()
        for _ in range(args.steps):
            dec.step()
        z.record()
        torch.cuda.synchronize()
        if method == "popkv":
            clocks.window = (w0, time.time())
            time.sleep(0.3)
            clocks.stop()
        ms_token = a.elapsed_time(z) / args.steps
        # End to end through the public API: each step's token read back to the host.
        host = torch.empty(1, dtype=torch.long).pin_memory()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            host.copy_(dec.step(), non_blocking=True)
        torch.cuda.synchronize()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
        entry = {"ms_per_token": ms_token, "e2e_ms_per_token": e2e_ms, "prefill_s": prefill_s}
        if method == "popkv":
            entry["stages"] = decoder_stage_times(dec, budget, hbm)
        results[method] = entry
        del dec
        torch.cuda.empty_cache()
    weights = sum(p.numel() * p.element_size() for p in model.parameters())
    pop = results["popkv"]
    line = {
        "metric": "decode ms/token end to end (configs[2]: 32-layer Llama-3.1-8B-shaped decoder)",
        "value": pop["ms_per_token"], "unit": "ms", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": pop["ms_per_token"], "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init weights, uniform random prompt ids)",
        "config": {"workload": "configs[2]: random-init Llama-3.1-8B shapes (hidden 4096, 32 layers, "
                               "32/8 heads, FFN 14336, vocab 128256), bf16, prefill then greedy "
                               "decode, Pop-KV in layers 2-31, dense layers 0-1",
                   "context": L0, "budget": budget, "graph": "one CUDA graph per token",
                   "l2": "every token reads ~16 GB of weights (far beyond L2)"},
        "methods": results,
        "weight_bytes": weights,
        "weights_hbm_gbs": weights / (pop["ms_per_token"] * 1e-3) / 1e9,
        "clocks": clocks.summary() if clocks else None,
        "e2e": {"value": pop["e2e_ms_per_token"], "unit": "ms", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 8},
        "cpu_baseline": None,
    }
    print(json.dumps(line), flush=True)


def decoder_stage_times(dec, budget, hbm, reps=10):
    """Per-stage device time of the retrieval path over the decoder's sparse layers."""
    import popkv_cuda as pk
    st = dec.stack
    sparse = [i for i in range(st.layers) if i not in st.dense_layers]
    tokens = st.max_tokens
    sizes = (1, st.q_heads, st.kv_heads, st.head_dim, tokens, 0)

    def run(name):
        for i in sparse:
            if "fused" in name:
                pk.score_select(st.q_in[i], st.packed[i], head_to_kv=st.head_to_kv, budget=budget,
                                tokens=tokens, seq_len=st.seq_len, out=st.indices[i],
                                attn_workspace=st.workspace[i], attn_sizes=sizes,
                                scores=st.scores, hist=st.score_hist)
            if "score" in name:
                pk.score(st.q_in[i], st.packed[i], head_to_kv=st.head_to_kv, tokens=tokens,
                         seq_len=st.seq_len, out=st.scores, hist=st.score_hist)
            if "select" in name:
                pk.select(st.scores.view(-1, st.capacity), budget=budget, tokens=tokens,
                          seq_len=st.seq_len, rows_per_seq=st.q_heads, out=st.indices[i],
                          attn_workspace=st.workspace[i], attn_sizes=sizes, hist=st.score_hist)
            if "attention" in name:
                pk.sparse_attention_premasked(st.q_in[i], st.key_cache[i], st.value_cache[i],
                                              tokens=tokens, current_keys=st.k_in[i],
                                              current_values=st.v_in[i], seq_len=st.seq_len,
                                              workspace=st.workspace[i], out=st.out[i])

    timed = {}
    for name in ("score", "score+select", "score+select+attention", "fused", "fused+attention"):
        run(name)
        torch.cuda.synchronize()
        st.score_hist.zero_()
        a, z = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            run(name)
        z.record()
        torch.cuda.synchronize()
        st.score_hist.zero_()  # a score-only pass leaves its histograms behind
        timed[name] = a.elapsed_time(z) / (reps * len(sparse))
    run("attention")  # clears the masks the score+select runs left
    torch.cuda.synchronize()
    return {"score_ms": timed["score"], "topk_ms": timed["score+select"] - timed["score"],
            "gather_attention_ms": timed["score+select+attention"] - timed["score+select"],
            "score_topk_fused_ms": timed["fused"],
            "gather_attention_after_fused_ms": timed["fused+attention"] - timed["fused"],
            "per": f"sparse layer ({len(sparse)} per token); gather is fused into attention; "
                   "the decode step runs the fused score+topk kernel (score_topk_fused_ms), "
                   "score_ms/topk_ms are the two-kernel form of the same stage"}


def run_reference(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    L, budget = args.context, args.budget
    ms, cores = time_cpu_reference(L, budget, args.steps, args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": ms, "unit": "ms", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,1) K/V/Q, 4 outlier channels x8, RoPE 5e5)",
        "config": {"workload": "configs[1] shapes, one layer-step per step on the host CPU "
                               "(reference readable reconstruction + torch.topk + gather + SDPA)",
                   "context": L, "budget": budget},
        "cpu_baseline": {"value": ms, "unit": "ms", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} layer-steps (L={L}, budget={budget})"},
        "e2e": {"value": ms, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.config == 2:
        run_decoder(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
