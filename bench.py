"""Benchmark of the paged decode step (KV write + paged decode attention) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 2|3|4] [--layers L] [--variant auto|sched|stream|mma|fma]

One *step* is one pass of the hot path over one batch: the KV write of the
batch's new tokens (one per sequence) into one layer's pool, then the paged
decode of every sequence against that layer.  Steps rotate over L layers
(independent K/V pools; default 24, the layer count of the Qwen2-0.5B model
config 2 is shaped after: 24 x 164 MB), so each step streams a pool that is not
in the 126 MB L2: "inputs larger than L2".  A model step is L layer-steps: it
starts with the decode schedule (one per model step; kv_len and the block
tables are those of every layer) and, with N GPUs, ends with the all-gather of
the outputs.

Workload (default): config 2 — 256 sequences per GPU, context lengths
U[128, 2048], 14 query / 2 KV heads, head_dim 64, block 16, bf16, seeded
synthetic data (no dataset exists for this path).  N GPUs run one process each
(torchrun); each rank owns its own 256 sequences and pool (sequence sharding,
weak scaling); the NCCL all-gather of the outputs is the only collective.

Timing: W warm-up layer-steps, then a timed region of exactly K layer-steps
(CUDA graphs of model steps), repeated R >= 20 times (enough for ~1.5 s of
load, so the clock sampler sees it); the median repeat, max over ranks.

Printed (rank 0, one JSON line):
  value       aggregate algorithmic HBM GB/s of the step (algorithmic bytes
              of the write + decode: K/V read once per KV head, q read,
              output written, block-table entries and context lengths read;
              workloads.PagedDecodeSpec) over the step time;
  e2e         the same metric through the public backend API with the step's
              query and new K/V copied from pinned host memory each layer-step,
              the step's metadata once per model step, and the output copied
              back (side stream, double-buffered, as in a serving loop);
  roofline    the decode kernel alone: algorithmic bytes per launch / launch
              time from a CUDA graph of L back-to-back decodes, against
              MEASURED_PEAKS.json hbm_gbs;
  cpu_baseline  the CPU port of the reference's path (oracle/, C/OpenMP) on this
              host's cores, and the reference's own Python functions from
              baseline/_ref beside it, rank 0 at N=1.

``--impl reference`` times the CPU side alone on the same workload (rank 0;
other ranks exit 0) and prints the same line with "impl": "reference".
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402

METRIC = "paged decode attn HBM GB/s (% of peak) + decode tok/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=240)
    p.add_argument("--warmup", type=int, default=24)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, default=2, choices=[2, 3, 4])
    p.add_argument("--layers", type=int, default=24)
    p.add_argument("--variant", default="auto", choices=["auto", "sched", "stream", "mma", "fma"])
    p.add_argument("--partition-tokens", type=int, default=0)
    p.add_argument("--e2e-steps", type=int, default=1200)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-config4", action="store_true", help="skip the config-4 strong-scaling sub-object")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--requests", type=int, default=256, help="--op engine: requests per replica")
    p.add_argument("--shard-of", type=int, default=1,
                   help="--op profile / trace: run rank 0's shard of an N-GPU run of --config (config 4: "
                        "its snake-assigned quarter at 4, a capture-sized case)")
    p.add_argument("--trace-out", default="", help="--op trace: also save the raw stamps (.npz) here")
    p.add_argument("--op", choices=["step", "gather", "rope_write", "metadata", "sweep", "engine", "profile",
                                    "variants", "trace"],
                   default="step",
                   help="step: the decode step (the headline); sweep: decode time per launch of every "
                        "kernel over batch x context (the plan's crossover table); variants: decode time per "
                        "launch of every kernel at configs 2, 3 and 4; engine: continuous-batching "
                        "serving in the reference's own engine (config 5, bounded: --requests per replica; "
                        "--impl reference runs the reference's GPU backend); profile: a few KV writes and "
                        "decodes of --variant on --config over --layers pools, untimed (the case ncu captures); "
                        "trace: the per-warp timeline of the stream decode (the trace build of the library, "
                        "min(--layers, 8) KV writes + scheduled decodes in one CUDA graph); "
                        "gather: the prefill prefix gather "
                        "(mvb_paged_gather) of every config-2 context; rope_write: the fused RoPE + "
                        "KV write (mvb_rope_kv_cache_write) of an 8192-token prefill chunk; metadata: "
                        "the per-step attention metadata of a config-2 decode step (StepMetadataBuilder)")
    return p.parse_args()


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def workload_desc(config: int) -> str:
    return {
        2: "config2: paged decode + KV write, 256 seqs/GPU, ctx U[128,2048], 14q/2kv/d64, block 16, bf16",
        3: "config3: split-K paged decode + KV write, 32 seqs/GPU, ctx 32768, 14q/2kv/d64, block 16, bf16",
        4: "config4: paged decode + KV write, 32q/8kv/d128, ctx lognormal(7,0.8) in [16,8192], block 16, bf16",
    }[config]


def rank_spec(config: int, rank: int, world: int, seed: int):
    from mini_vllm_b200 import workloads as W

    if config == 4:
        # global batch 1024 sharded by sequence (token-balanced snake assignment)
        from mini_vllm_b200 import sharding

        ctx = W.context_lengths(4, seed=seed)
        owned = sharding.snake_assignment(ctx, world)[rank]
        c = W.CONFIGS[4]
        spec = W.build_spec("config4", ctx[owned], c["num_heads"], c["num_kv_heads"], c["head_dim"],
                            c["block_size"], seed=seed + 101 * rank)
        return spec, owned
    spec = W.make_spec(config, seed=seed + 101 * rank)
    owned = np.arange(spec.num_seqs, dtype=np.int64) + rank * spec.num_seqs
    return spec, owned


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.gpu = gpu_id
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU side: the oracle port of the reference's CPU path
# ---------------------------------------------------------------------------
def host_threads() -> int:
    """Host cores this process may use (torchrun sets OMP_NUM_THREADS=1 per rank;
    the CPU baseline asks OpenMP for every core explicitly)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_port_run(spec, tensors_np, steps: int, budget_s: float):
    """Time write + decode of the oracle on the host cores; returns (s/step, threads, reps)."""
    import oracle

    threads = host_threads()
    kc, vc = tensors_np["key_cache"].copy(), tensors_np["value_cache"].copy()
    times = []
    t_end = time.perf_counter() + budget_s
    for i in range(steps):
        t0 = time.perf_counter()
        oracle.cache_write(tensors_np["new_key"], tensors_np["new_value"], kc, vc, spec.slot_mapping,
                           spec.block_size, "bf16")
        oracle.decode(tensors_np["query"], kc, vc, spec.block_tables, spec.context_lens, spec.block_size,
                      "bf16", threads=threads)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end and i >= 2:
            break
    return statistics.median(times), threads, len(times)


def reference_cpu_run(spec, host, budget_s: float):
    """The reference's own CPU path for the step — AttentionBackendRef.write_kv_cache
    (cache_write.write_to_paged_cache) + AttentionBackendRef.decode_attention
    (paged_attention_ref.py:81-161) — imported from baseline/_ref, on this
    host's cores (bf16 CPU tensors, torch threads = host threads).  Returns
    (s/step, threads, reps) or None when the reference is not installed."""
    try:
        from mini_vllm_b200 import reference_engine as RE

        RE.import_reference()
        import torch
        from mini_vllm.attention.paged_attention_ref import AttentionBackendRef
        from mini_vllm.model_runner.base import AttentionGroup, AttentionMetadata, ModelConfig
    except Exception:
        return None
    threads = host_threads()
    torch.set_num_threads(threads)
    cfg = ModelConfig(num_heads=spec.num_heads, num_kv_heads=spec.num_kv_heads, head_dim=spec.head_dim)
    be = AttentionBackendRef(cfg)
    pool = be.allocate_pool(1, spec.num_blocks, spec.block_size, spec.num_kv_heads, spec.head_dim,
                            torch.bfloat16, torch.device("cpu"))

    def t(x):
        return torch.from_numpy(x.view(np.int16).copy()).view(torch.bfloat16)

    kc0, vc0 = t(host["key_cache"]), t(host["value_cache"])
    q, nk, nv = t(host["query"]), t(host["new_key"]), t(host["new_value"])
    slots = torch.from_numpy(spec.slot_mapping.astype(np.int64))
    group = AttentionGroup(seq_indices=list(range(spec.num_seqs)), attention_type="decode_gpu",
                           cached_len_before=torch.from_numpy(spec.context_lens.astype(np.int64) - 1),
                           query_len=torch.ones(spec.num_seqs, dtype=torch.int64),
                           kv_len_after=torch.from_numpy(spec.context_lens.astype(np.int64)))
    meta = AttentionMetadata(groups=[group], decode_block_tables=torch.from_numpy(spec.block_tables),
                             block_size=spec.block_size, num_kv_heads=spec.num_kv_heads, head_dim=spec.head_dim)
    times = []
    t_end = time.perf_counter() + budget_s
    while True:
        pool.key_caches[0].copy_(kc0)
        pool.value_caches[0].copy_(vc0)
        t0 = time.perf_counter()
        be.write_kv_cache(0, nk, nv, slots)
        be.decode_attention(0, q, meta, pool)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(times) >= 20:
            break
    return statistics.median(times), threads, len(times)


def config_dict(args, spec, world: int, L: int) -> dict:
    """The workload description both arms print (same keys and values)."""
    nb = 2 * spec.num_blocks * spec.num_kv_heads * spec.block_size * spec.head_dim * 2
    gb = 1024 if args.config == 4 else spec.num_seqs * world
    return {"workload": workload_desc(args.config), "global_batch": gb, "seqs_per_gpu": spec.num_seqs,
            "layers_rotated": L, "l2": f"inputs larger than L2: {L} layer pools of {nb / 1e6:.0f} MB rotated",
            "parallelism": f"sequence-sharded x{world}" + (" + NCCL all-gather of outputs" if world > 1 else ""),
            "timing": "median of repeated timed regions of exactly --steps layer-steps (CUDA graphs of L "
                      "layer-steps + the remainder, one decode schedule per model step), CUDA events"}


def reference_arm(args, rank, world):
    """The reference arm: the reference's CPU algorithm for the path, timed on
    this host's cores.  The reference is pure Python (torch and Triton), so
    nothing of it compiles into a CPU library here; the arm times the C/OpenMP
    port of its write + decode (oracle/, every host thread) and, beside it, the
    reference's own Python functions from baseline/_ref when installed."""
    if rank != 0:
        return
    from mini_vllm_b200 import workloads as W

    spec, _ = rank_spec(args.config, 0, 1, args.seed)
    t = W.numpy_tensors(spec, "bf16")
    for _ in range(max(1, min(args.warmup, 3))):
        cpu_port_run(spec, t, 1, 0.0)
    steps = max(1, min(args.steps, 50))
    sec, threads, reps = cpu_port_run(spec, t, steps, budget_s=60.0)
    nbytes = spec.decode_bytes(2) + spec.write_bytes(2)
    gbs = nbytes / sec / 1e9
    cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
           "sample": f"full {spec.name} step (write {spec.num_seqs} tokens + decode {spec.num_seqs} seqs), "
                     f"median of {reps}"}
    ref = reference_cpu_run(spec, t, budget_s=30.0)
    if ref is not None:
        rsec, rthreads, rrep = ref
        cpu["reference_cpu"] = {
            "value": round(nbytes / rsec / 1e9, 4), "unit": "GB/s", "cores": rthreads, "kind": "reference",
            "ms_per_step": round(rsec * 1e3, 2),
            "sample": f"the reference's own AttentionBackendRef.write_kv_cache + decode_attention (baseline/_ref, "
                      f"bf16 CPU tensors) on the full {spec.name} step, median of {rrep}"}
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": reps, "warmup": min(args.warmup, 3), "ms_per_step": round(sec * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": config_dict(args, spec, world, args.layers),
        "decode_tok_s": round(spec.num_seqs / sec, 1),
        "cpu_baseline": cpu,
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import mini_vllm_b200 as M
    from mini_vllm_b200 import sharding
    from mini_vllm_b200 import workloads as W

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    spec, owned = rank_spec(args.config, rank, world, args.seed)
    L = args.layers
    K, Wm = args.steps, args.warmup
    t = W.torch_tensors(spec, torch.bfloat16, dev, num_layers=L)
    kcs, vcs = t["key_caches"], t["value_caches"]
    q, nk, nv = t["query"], t["new_key"], t["new_value"]
    bt, kvl, slots = t["block_tables"], t["kv_len"], t["slot_mapping"]
    out = torch.empty_like(q)
    pt = args.partition_tokens or None
    gather = None
    if world > 1:
        counts = [None] * world
        dist.all_gather_object(counts, owned.tolist())
        owned_all = [np.asarray(c, dtype=np.int64) for c in counts]
        gather = sharding.OutputGather(owned_all, spec.num_heads, spec.head_dim, torch.bfloat16, dev)
        out = gather.send_view(spec.num_seqs)  # the decode writes where the all-gather sends from

    plan = M.decode_plan(spec.num_seqs, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
                         spec.num_blocks, spec.max_blocks, torch.bfloat16, args.variant, pt,
                         kcs[0].data_ptr())
    scheduled = plan["variant"] in ("sched", "stream")  # kernels with a per-step set-up
    sched = None

    def begin_model_step():
        # kv_len and the block tables are those of every layer of the step: one
        # schedule serves the step's L layer-steps
        nonlocal sched
        if scheduled:
            sched = M.build_decode_schedule(kvl, bt, spec.num_heads, spec.num_kv_heads, spec.head_dim,
                                            spec.block_size, spec.num_blocks, torch.bfloat16,
                                            schedule=sched, strict=False, variant=plan["variant"])

    def step(layer):
        M.paged_cache_write(nk, nv, kcs[layer], vcs[layer], slots, spec.block_size, strict=False,
                            check_duplicates=False)
        M.paged_decode_attention(q, kcs[layer], vcs[layer], bt, kvl, spec.block_size, out=out,
                                 variant=args.variant, partition_tokens=pt, strict=False, after_write=True,
                                 schedule=sched)

    def model_step(n):  # one model step of n layer-steps (n <= L)
        begin_model_step()
        for layer in range(n):
            step(layer)
        if gather is not None:
            gather(out)

    # launches per layer-step of this repository's kernels: write + decode
    # (+ the stream kernel's fixup / split-K reduction); the schedule once per model step
    per_layer = 1 + plan["launches"] - (1 if plan["variant"] == "sched" else 0)

    # correctness gate before timing: one strict step through the public API
    M.paged_cache_write(nk, nv, kcs[0], vcs[0], slots, spec.block_size)
    M.paged_decode_attention(q, kcs[0], vcs[0], bt, kvl, spec.block_size, out=out, variant=args.variant,
                             partition_tokens=pt)
    torch.cuda.synchronize()

    # ---- warm-up: exactly W layer-steps, eager, on the capture stream ----
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for i in range(Wm):
            if i % L == 0:
                begin_model_step()
            step(i % L)
            if gather is not None and (i % L == L - 1 or i == Wm - 1):
                gather(out)
        if Wm == 0:
            model_step(L)
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize()

    # ---- the timed region: exactly K layer-steps = K // L model steps of L
    # layer-steps (one CUDA graph) + one model step of the remaining K % L ----
    g_full = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_full):
        model_step(L)
    rem = K % L
    g_rem = None
    if rem:
        g_rem = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_rem):
            model_step(rem)

    def timed_region():
        for _ in range(K // L):
            g_full.replay()
        if g_rem is not None:
            g_rem.replay()

    esz = 2
    step_bytes_rank = spec.decode_bytes(esz) + spec.write_bytes(esz)
    # repeats: >= 20, and enough for ~1.5 s of load so the clock sampler sees it
    est = K * step_bytes_rank / 5e12
    R = int(min(5000, max(20, math.ceil(1.5 / max(est, 1e-6)))))
    if world > 1:
        # the same number of replays on every rank: each replay runs the graph's
        # NCCL all-gathers, so a rank that replays more waits for a peer forever
        rt = torch.tensor([R], device=dev, dtype=torch.int64)
        dist.all_reduce(rt, op=dist.ReduceOp.MAX)
        R = int(rt.item())
    timed_region()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(R)]
    with ClockSampler(physical_gpu(local_rank)) as clocks:
        for a, b in evs:
            a.record()
            timed_region()
            b.record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    reps_s = sorted(a.elapsed_time(b) / 1e3 for a, b in evs)
    elapsed = statistics.median(reps_s)
    if world > 1:
        tt = torch.tensor([elapsed], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        elapsed = float(tt.item())
    sec_per_step = elapsed / K
    tot = torch.tensor([step_bytes_rank, spec.num_seqs], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(tot)
    step_bytes_all, seqs_all = float(tot[0]), float(tot[1])
    value_gbs = step_bytes_all / sec_per_step / 1e9
    M.check_device_errors(dev)

    # ---- roofline: the decode kernel alone — a CUDA graph of L back-to-back
    # decodes (rotating layers; schedule ready), time / launches ----
    def graph_of(fn):
        s2 = torch.cuda.Stream(device=dev)
        s2.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s2):
            fn()
        torch.cuda.current_stream(dev).wait_stream(s2)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    def decodes():
        for layer in range(L):
            M.paged_decode_attention(q, kcs[layer], vcs[layer], bt, kvl, spec.block_size, out=out,
                                     variant=args.variant, partition_tokens=pt, strict=False, schedule=sched)

    def schedules():
        for _ in range(L):
            begin_model_step()

    def writes():
        for layer in range(L):
            M.paged_cache_write(nk, nv, kcs[layer], vcs[layer], slots, spec.block_size, strict=False,
                                check_duplicates=False)

    def per_launch_us(g, n_per_replay, target_s=0.5):
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        one = e0.elapsed_time(e1) / 1e3
        n = int(min(2000, max(5, target_s / max(one, 1e-7))))
        samples = []
        for _ in range(n):
            e0.record()
            g.replay()
            e1.record()
            e1.synchronize()
            samples.append(e0.elapsed_time(e1) / 1e3 / n_per_replay)
        return statistics.median(samples) * 1e6, np.percentile(samples, 10) * 1e6, np.percentile(samples, 90) * 1e6

    g_dec = graph_of(decodes)
    dec_us, dec_p10, dec_p90 = per_launch_us(g_dec, L)
    sched_us = per_launch_us(graph_of(schedules), L)[0] if scheduled else None
    write_us = per_launch_us(graph_of(writes), L)[0]
    peak, peak_kind = peaks()
    dec_bytes = spec.decode_bytes(esz)
    achieved = dec_bytes / (dec_us * 1e-6) / 1e9
    traffic = read_traffic(args.config)
    M.check_device_errors(dev)

    # ---- e2e: the public backend API with host buffers.  Per layer-step the
    # step's query and new K/V rows go host -> device and the output comes back;
    # per model step (every L layer-steps) the step's metadata (slot mapping,
    # block tables, kv_len) goes host -> device once, as an engine builds it
    # once per step.  Copies run on a side stream, double-buffered, and overlap
    # the neighbouring steps' attention as in a serving loop. ----
    backend = M.AttentionBackendB200(M.ModelConfig(num_heads=spec.num_heads, num_kv_heads=spec.num_kv_heads,
                                                   head_dim=spec.head_dim), strict=False,
                                     decode_variant=args.variant, partition_tokens=pt, overlap_after_write=True)
    pool = M.KVCachePool(kcs, vcs, spec.num_blocks, spec.block_size, L, spec.num_kv_heads, spec.head_dim,
                         dev, torch.bfloat16)
    backend._pool = pool
    backend._block_size = spec.block_size
    kvl32 = torch.from_numpy(spec.context_lens.astype(np.int32)).to(dev)

    def staged(parts):
        offs, total = {}, 0
        for name, ten in parts:
            offs[name] = total
            total += (ten.numel() * ten.element_size() + 255) // 256 * 256
        host = torch.empty(total, dtype=torch.uint8).pin_memory()
        for name, ten in parts:
            nbytes = ten.numel() * ten.element_size()
            host[offs[name]:offs[name] + nbytes].copy_(ten.detach().cpu().contiguous().view(-1).view(torch.uint8))
        slots_ = []
        for _ in range(2):
            buf = torch.empty(total, dtype=torch.uint8, device=dev)
            views = {name: buf[offs[name]:offs[name] + ten.numel() * ten.element_size()].view(ten.dtype).view(ten.shape)
                     for name, ten in parts}
            slots_.append({"buf": buf, "views": views, "ready": torch.cuda.Event(), "done": torch.cuda.Event()})
        return host, total, slots_

    layer_host, layer_bytes, layer_slots = staged([("q", q), ("nk", nk), ("nv", nv)])
    meta_host, meta_bytes, meta_slots = staged([("slots", slots), ("bt", bt), ("kvl", kvl32)])
    outs_host = [torch.empty(q.shape, dtype=q.dtype).pin_memory() for _ in range(2)]
    outs_dev = [torch.empty_like(q) for _ in range(2)]  # the decode writes its output here (out=)
    out_copied = [torch.cuda.Event(), torch.cuda.Event()]
    d2h = outs_host[0].numel() * outs_host[0].element_size()
    compute = torch.cuda.current_stream(dev)
    side = torch.cuda.Stream(dev)      # host -> device copies
    side_d2h = torch.cuda.Stream(dev)  # device -> host copies (the link is full duplex)
    # the loop's copies use fixed buffers: each is checked once (staging.CopyPlan)
    layer_plans = [M.staging.CopyPlan(ls["buf"], layer_host, side, wait=ls["done"], record=ls["ready"])
                   for ls in layer_slots]
    meta_plans = [M.staging.CopyPlan(ms["buf"], meta_host, side, wait=ms["done"], record=ms["ready"])
                  for ms in meta_slots]
    out_plans = [M.staging.CopyPlan(outs_host[p], outs_dev[p], side_d2h, wait=layer_slots[p]["done"],
                                    record=out_copied[p]) for p in range(2)]
    pending = []    # (step index, output) whose D2H is not issued yet
    releasing = []  # (event, output) freed once compute waited for the D2H
    meta_obj = [None]

    def e2e_step(i):
        layer, m = i % L, i // L
        ls, ms = layer_slots[i & 1], meta_slots[m & 1]
        waits = []
        if layer == 0:  # this model step's metadata, once
            meta_plans[m & 1].run()
            v = ms["views"]
            group = M.AttentionGroup(seq_indices=list(range(spec.num_seqs)), attention_type="decode_gpu",
                                     cached_len_before=None, query_len=None, kv_len_after=v["kvl"])
            meta_obj[0] = M.AttentionMetadata(groups=[group], decode_block_tables=v["bt"],
                                              block_size=spec.block_size, num_kv_heads=spec.num_kv_heads,
                                              head_dim=spec.head_dim)
            waits.append(ms["ready"])
        layer_plans[i & 1].run()
        waits.append(ls["ready"])
        if pending:  # D2H of the previous step's output
            pi, po = pending.pop()
            out_plans[pi & 1].run()
            releasing.append((out_copied[pi & 1], po))
        if len(releasing) > 1:
            # an output is freed only after the compute stream has waited for its
            # D2H (two steps later, so the wait never stalls)
            ev, ro = releasing.pop(0)
            waits.append(ev)
            del ro
        M.staging.wait_events(compute, *waits)
        v = ls["views"]
        backend.write_kv_cache(layer, v["nk"], v["nv"], ms["views"]["slots"])
        o = backend.decode_attention(layer, v["q"], meta_obj[0], pool, out=outs_dev[i & 1])
        M.staging.record(ls["done"], compute)
        if layer == L - 1:
            M.staging.record(ms["done"], compute)
        pending.append((i, o))

    def e2e_flush():
        while pending:
            pi, po = pending.pop()
            out_plans[pi & 1].run()
            releasing.append((out_copied[pi & 1], po))
        compute.wait_stream(side)
        compute.wait_stream(side_d2h)
        releasing.clear()

    e2e_n = max(L, (args.e2e_steps // L) * L)
    for i in range(2 * L):
        e2e_step(i)
    e2e_flush()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(compute)
    side.wait_stream(compute)
    side_d2h.wait_stream(compute)
    h0 = time.perf_counter()
    for i in range(e2e_n):
        e2e_step(i)
        if gather is not None and i % L == L - 1:
            gather(out)
    e2e_flush()
    e1.record(compute)
    e2e_host_us = (time.perf_counter() - h0) / e2e_n * 1e6  # host time to issue a layer-step
    torch.cuda.synchronize()
    e2e_sec = e0.elapsed_time(e1) / 1e3 / e2e_n
    if world > 1:
        tt = torch.tensor([e2e_sec], device=dev, dtype=torch.float64)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_sec = float(tt.item())
    M.check_device_errors(dev)
    e2e_gbs = step_bytes_all / e2e_sec / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host_t = {
            "query": to_np_bf16(q), "key_cache": to_np_bf16(kcs[0]), "value_cache": to_np_bf16(vcs[0]),
            "new_key": to_np_bf16(nk), "new_value": to_np_bf16(nv),
        }
        sec, threads, nrep = cpu_port_run(spec, host_t, 20, budget_s=15.0)
        cgbs = step_bytes_rank / sec / 1e9
        cpu = {"value": round(cgbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"full {spec.name} step on one layer (write {spec.num_seqs} tokens + decode "
                         f"{spec.num_seqs} seqs), median of {nrep}",
               "decode_tok_s": round(spec.num_seqs / sec, 1)}
        ref = reference_cpu_run(spec, host_t, budget_s=15.0)
        if ref is not None:
            rsec, rthreads, rrep = ref
            cpu["reference_cpu"] = {
                "value": round(step_bytes_rank / rsec / 1e9, 4), "unit": "GB/s", "cores": rthreads,
                "kind": "reference", "ms_per_step": round(rsec * 1e3, 2),
                "sample": f"the reference's own AttentionBackendRef.write_kv_cache + decode_attention "
                          f"(baseline/_ref, bf16 CPU tensors) on the full {spec.name} step, median of {rrep}"}

    c4 = None
    if args.config == 2 and not args.no_config4:
        c4 = config4_strong(args, rank, world, dev, peak)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value_gbs, 2), "unit": "GB/s", "n_gpus": world,
            "steps": K, "warmup": Wm, "ms_per_step": round(sec_per_step * 1e3, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": config_dict(args, spec, world, L),
            "kernel": {"variant": plan["variant"], "partition_tokens": plan["partition_tokens"],
                       "num_partitions": plan["num_partitions"], "timed_repeats": R,
                       "repeat_ms_p10_p50_p90": [round(np.percentile(reps_s, x) * 1e3, 4) for x in (10, 50, 90)]},
            "pct_of_peak": round(100 * value_gbs / (peak * world), 2),
            "pct_of_8tbs": round(100 * value_gbs / (8000.0 * world), 2),
            "decode_tok_s": round(seqs_all / sec_per_step, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "traffic_source": "committed ncu summary (profiles/), one launch" if traffic else None,
                         "peak_kind": peak_kind, "kernel": f"paged decode ({plan['variant']})",
                         "bytes_per_launch": dec_bytes, "mean_launch_us": round(dec_us, 2),
                         "launch_timing": f"CUDA graph of {L} back-to-back decodes, events, median of replays",
                         "p10_us": round(dec_p10, 2), "p90_us": round(dec_p90, 2),
                         "schedule_us": round(sched_us, 2) if sched_us is not None else None,
                         "kv_write_us": round(write_us, 2)},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_gbs, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": int(layer_bytes + meta_bytes / L), "d2h_bytes_per_step": int(d2h),
                    "h2d_detail": f"{layer_bytes} B of query / new K / new V per layer-step + {meta_bytes} B of "
                                  f"metadata per model step of {L} layer-steps",
                    "ms_per_step": round(e2e_sec * 1e3, 4),
                    "copies": "H2D and D2H on two side streams, double-buffered, overlapping compute and each other; "
                              "staged with mini_vllm_b200.staging (fixed buffers as staging.CopyPlan, one "
                              "binding call per copy / wait / record); the decode writes into one of two "
                              "output buffers (out=)",
                    "host_us_per_step": round(e2e_host_us, 1),
                    "decode_tok_s": round(seqs_all / e2e_sec, 1)},
            "gpu_launches": K * per_layer + (-(-K // L) if scheduled else 0),
            "clocks": clocks.summary(),
            "config4": c4,
        }
        print(json.dumps(line), flush=True)
    del g_full, g_rem, g_dec  # release graphs holding NCCL work before the group is destroyed


def config4_strong(args, rank, world, dev, peak):
    """BASELINE config 4 as strong scaling, for the same JSON line at every N:
    the global batch of 1024 sequences (32 q / 8 KV heads, head_dim 128,
    lognormal(7, 0.8) contexts in [16, 8192], block 16, bf16) sharded by
    sequence with the token-balanced snake assignment; each rank decodes its
    shard against its own pools, and the outputs are all-gathered in global
    order (NCCL all_gather_into_tensor + index_copy_).  Timed per rank as CUDA
    graphs of L back-to-back launches (decode alone, gather alone, decode then
    gather), median of repeats, max over ranks.  The decodes read the per-step
    schedule of their kernel, built once (as once per model step) and timed on
    its own (schedule_us)."""
    import torch
    import torch.distributed as dist

    import mini_vllm_b200 as M
    from mini_vllm_b200 import sharding
    from mini_vllm_b200 import workloads as W

    L = 2  # distinct pools (each shard's K/V is several GB at small N: no L2 reuse between launches)
    INNER = 8  # repetitions of the L operations inside one timed graph
    ctx_all = W.context_lengths(4, seed=args.seed)
    owned_all = sharding.snake_assignment(ctx_all, world)
    owned = owned_all[rank]
    c = W.CONFIGS[4]
    spec = W.build_spec("config4-shard", ctx_all[owned], c["num_heads"], c["num_kv_heads"], c["head_dim"],
                        c["block_size"], seed=args.seed + 101 * rank)
    t = W.torch_tensors(spec, torch.bfloat16, dev, num_layers=L)
    q, bt, kvl = t["query"], t["block_tables"], t["kv_len"]
    kcs, vcs = t["key_caches"], t["value_caches"]
    out = torch.empty_like(q)
    gather = sharding.OutputGather(owned_all, spec.num_heads, spec.head_dim, torch.bfloat16, dev) if world > 1 else None
    if gather is not None:
        out = gather.send_view(spec.num_seqs)  # the decode writes where the all-gather sends from
    plan = M.decode_plan(spec.num_seqs, spec.num_heads, spec.num_kv_heads, spec.head_dim, 16, spec.num_blocks,
                         spec.max_blocks, torch.bfloat16, "auto")
    sched = M.build_decode_schedule(kvl, bt, spec.num_heads, spec.num_kv_heads, spec.head_dim, 16, spec.num_blocks,
                                    torch.bfloat16, strict=False)

    def decodes():
        for layer in range(L):
            M.paged_decode_attention(q, kcs[layer], vcs[layer], bt, kvl, 16, out=out, strict=False, schedule=sched)

    def schedules():
        for _ in range(L):
            M.build_decode_schedule(kvl, bt, spec.num_heads, spec.num_kv_heads, spec.head_dim, 16, spec.num_blocks,
                                    torch.bfloat16, schedule=sched, strict=False)

    def gathers():
        for _ in range(L):
            if gather is not None:
                gather(out)

    def both():
        for layer in range(L):
            M.paged_decode_attention(q, kcs[layer], vcs[layer], bt, kvl, 16, out=out, strict=False, schedule=sched)
            if gather is not None:
                gather(out)

    decodes()
    gathers()
    torch.cuda.synchronize()
    M.check_device_errors(dev)

    def time_graph(fn):
        s2 = torch.cuda.Stream(device=dev)
        s2.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s2):
            fn()
        torch.cuda.current_stream(dev).wait_stream(s2)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for _ in range(INNER):
                fn()
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        # INNER x L operations per graph and back-to-back replays between two
        # events, so neither the host's launch time nor the ranks' launch skew
        # (which a collective in the graph would wait out) is measured; every
        # rank replays the same number of times
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        samples = []
        for _ in range(7):
            e0.record()
            for _ in range(2):
                g.replay()
            e1.record()
            e1.synchronize()
            samples.append(e0.elapsed_time(e1) / 1e3 / (2 * INNER * L))
        del g
        v = statistics.median(samples)
        if world > 1:
            tt = torch.tensor([v], device=dev, dtype=torch.float64)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            v = float(tt.item())
        return v

    dec_s = time_graph(decodes)
    own_dec_s = dec_s
    do_sched = torch.tensor([1 if sched.variant is not None else 0], device=dev)
    if world > 1:  # every rank takes the same collective steps
        dist.all_reduce(do_sched, op=dist.ReduceOp.MIN)
    sched_s = time_graph(schedules) if int(do_sched.item()) else 0.0
    gat_s = time_graph(gathers) if world > 1 else 0.0
    both_s = time_graph(both) if world > 1 else dec_s
    # per-rank figures
    by = spec.decode_bytes(2)
    vals = torch.tensor([by, spec.num_seqs, spec.total_tokens], device=dev, dtype=torch.float64)
    allv = [torch.zeros_like(vals) for _ in range(world)] if world > 1 else [vals]
    if world > 1:
        dist.all_gather(allv, vals)
    toks = [float(v[2]) for v in allv]
    res = {
        "workload": "config4: global batch 1024, 32q/8kv/d128, ctx lognormal(7,0.8) in [16,8192], block 16, bf16, "
                    "snake-sharded by sequence",
        "scaling": "strong", "global_batch": int(ctx_all.size), "kernel": plan["variant"],
        "decode_us_max_rank": round(dec_s * 1e6, 2), "gather_us": round(gat_s * 1e6, 2),
        "schedule_us": round(sched_s * 1e6, 2),
        "decode_then_gather_us": round(both_s * 1e6, 2),
        "decode_tok_s_no_gather": round(ctx_all.size / dec_s, 1),
        "decode_tok_s_with_gather": round(ctx_all.size / both_s, 1),
        "aggregate_GBps_no_gather": round(sum(float(v[0]) for v in allv) / dec_s / 1e9, 1),
        "rank0_GBps": round(by / own_dec_s / 1e9, 1),
        "rank0_frac": round(by / own_dec_s / 1e9 / peak, 4),
        "tokens_per_rank_max_over_mean": round(max(toks) / (sum(toks) / len(toks)), 4),
        "seqs_per_rank": [int(v[1]) for v in allv],
        "timing": f"CUDA graphs of {INNER} x {L} launches, 2 replays back to back between events, median of 7, "
                  "max over ranks",
    }
    del t, q, bt, kvl, kcs, vcs, out, sched
    torch.cuda.empty_cache()
    return res


def physical_gpu(local_rank: int) -> str:
    """nvidia-smi id of this process's GPU (CUDA_VISIBLE_DEVICES remaps indices)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local_rank < len(ids):
            return ids[local_rank]
    return str(local_rank)


def to_np_bf16(t):
    import torch

    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def read_traffic(config: int):
    """dram bytes per decode launch from the committed ncu summary, if present."""
    path = os.path.join(REPO, "profiles", f"decode_config{config}_traffic.txt")
    if not os.path.exists(path):
        return None
    for ln in open(path):
        if ln.startswith("traffic_bytes_per_launch:"):
            return int(float(ln.split(":", 1)[1]))
    return None


def gather_op(args):
    """Secondary measurement: mvb_paged_gather reading every context of the
    config-2 batch (256 sequences, ctx U[128,2048], 14/2/64, bf16) out of the
    paged pool into contiguous [T, KH, D] K and V, i.e. the prefill prefix read
    for a whole batch.  Algorithmic bytes: K+V read and written once
    (4 * sum(ctx) * KH * D * 2 B) plus the block-table entries read.  Timed as
    K launches replayed from a CUDA graph over L rotated pools; the roofline
    line is the same launches one by one behind a torch.cuda._sleep."""
    import torch

    import mini_vllm_b200 as M
    from mini_vllm_b200 import _native
    from mini_vllm_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    spec = W.make_spec(2, seed=args.seed)
    L = args.layers
    t = W.torch_tensors(spec, torch.bfloat16, dev, num_layers=L)
    kcs, vcs, bt = t["key_caches"], t["value_caches"], t["block_tables"]
    ctx = [int(c) for c in spec.context_lens]
    total = sum(ctx)
    # correctness gate through the public API (host metadata, strict checks)
    gk, gv = M.paged_gather(kcs[0], vcs[0], bt, list(range(spec.num_seqs)), ctx, spec.block_size)
    torch.cuda.synchronize()
    offsets = np.concatenate([[0], np.cumsum(ctx)]).astype(np.int64)
    meta = torch.from_numpy(np.concatenate([np.arange(spec.num_seqs), offsets]).astype(np.int64)).to(dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    counter = torch.zeros(2, dtype=torch.int32, device=dev)  # the work counter; each launch leaves it zero
    lib = _native.lib()

    def launch(layer):
        st = lib.mvb_paged_gather(kcs[layer].data_ptr(), vcs[layer].data_ptr(), bt.data_ptr(), bt.shape[0],
                                  bt.stride(0), bt.shape[1], meta.data_ptr(), meta.data_ptr() + 8 * spec.num_seqs,
                                  gk.data_ptr(), gv.data_ptr(), spec.num_seqs, total, spec.num_kv_heads,
                                  spec.head_dim, spec.block_size, spec.num_blocks, _native.DTYPE_BF16,
                                  counter.data_ptr(), err.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
        assert st == _native.OK, _native.status_string(st)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for layer in range(L):
            launch(layer)
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for layer in range(L):
            launch(layer)
    replays, warm = max(1, args.steps // L), max(3, args.warmup // L)
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu(0)) as clocks:
        ev0.record()
        for _ in range(replays):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    sec = ev0.elapsed_time(ev1) / 1e3 / (replays * L)
    assert int(err.item()) == 0 and counter.tolist() == [0, 0]
    blocks_read = int(((spec.context_lens + spec.block_size - 1) // spec.block_size).sum())
    nbytes = 4 * total * spec.num_kv_heads * spec.head_dim * 2 + 8 * blocks_read + 16 * spec.num_seqs
    # roofline: single launches behind a sleep
    gs = []
    for layer in range(L):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            launch(layer)
        gs.append(g)
    reps = 400
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for i in range(20):
        gs[i % L].replay()
    torch.cuda.synchronize()
    torch.cuda._sleep(200_000_000)
    for i, (a, b) in enumerate(evs):
        a.record()
        gs[i % L].replay()
        b.record()
    torch.cuda.synchronize()
    mean = statistics.mean(a.elapsed_time(b) / 1e3 for a, b in evs)
    peak, peak_kind = peaks()
    # CPU baseline: the oracle's gather (the reference's gather_paged_kv restated), one sequence at a time
    import oracle

    cpu_baseline = None
    if not args.no_cpu_baseline:
        kc_np, vc_np = to_np_bf16(kcs[0]), to_np_bf16(vcs[0])
        t0 = time.perf_counter()
        n_cpu = 0
        for i in range(spec.num_seqs):
            oracle.gather(kc_np, vc_np, spec.block_tables[i], ctx[i], spec.block_size, "bf16")
            n_cpu += ctx[i]
            if time.perf_counter() - t0 > 10:
                break
        cpu_sec = time.perf_counter() - t0
        cpu_gbs = 4 * n_cpu * spec.num_kv_heads * spec.head_dim * 2 / cpu_sec / 1e9
        cpu_baseline = {"value": round(cpu_gbs, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                        "sample": f"oracle gather of {n_cpu} tokens, one sequence at a time"}
    print(json.dumps({
        "metric": "paged gather GB/s (prefill prefix read of every config-2 context)", "value": round(nbytes / sec / 1e9, 2),
        "unit": "GB/s", "n_gpus": 1, "steps": replays * L, "warmup": warm * L, "ms_per_step": round(sec * 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"gather: 256 sequences, {total} tokens, 14q/2kv/d64, block 16, bf16",
                   "layers_rotated": L, "l2": "inputs larger than L2: rotated 164 MB pools",
                   "timing": "CUDA graph of L launches, CUDA events"},
        "roofline": {"bound": "hbm", "achieved": round(nbytes / mean / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(nbytes / mean / 1e9 / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "paged_gather_tma_kernel", "bytes_per_launch": int(nbytes), "mean_launch_us": round(mean * 1e6, 2)},
        "cpu_baseline": cpu_baseline, "gpu_launches": replays * L, "clocks": clocks.summary(),
    }), flush=True)


def rope_write_op(args):
    """Secondary measurement: mvb_rope_kv_cache_write on one 8192-token prefill
    chunk of the config-2 model shape (14 q / 2 KV heads, head_dim 64, bf16):
    q, k, v are views of the fused QKV output, positions 0..8191, slots spread
    over a 164 MB pool.  Algorithmic bytes: q/k/v read, the cos and sin rows of
    each token read, the rotated q written, K and V rows written, plus the
    positions and slots.  Timed as K launches replayed from a CUDA graph over L
    rotated pools and inputs."""
    import torch

    import mini_vllm_b200 as M
    from mini_vllm_b200 import _native

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, H, KH, D, BS = 8192, 14, 2, 64, 16
    L = min(args.layers, 8)
    nb = 80000  # 164 MB per K+V pool pair at bf16
    g = torch.Generator(device=dev).manual_seed(args.seed)
    qkvs = [torch.randn(T, (H + 2 * KH) * D, generator=g, device=dev).to(torch.bfloat16) for _ in range(L)]
    kcs = [torch.empty(nb, KH, BS, D, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    vcs = [torch.empty(nb, KH, BS, D, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    cos, sin = M.rope_tables(D, 1e6, 32768, torch.bfloat16, device=dev)
    pos = torch.arange(T, device=dev)
    slots = torch.randperm(nb * BS, generator=g, device=dev)[:T]
    q_out = torch.empty(T, H, D, dtype=torch.bfloat16, device=dev)
    views = [(x[:, :H * D].view(T, H, D), x[:, H * D:(H + KH) * D].view(T, KH, D), x[:, (H + KH) * D:].view(T, KH, D))
             for x in qkvs]
    # correctness gate through the public API (strict checks)
    q, k, v = views[0]
    M.rope_cache_write(q, k, v, pos, cos, sin, kcs[0], vcs[0], slots, BS, query_out=q_out)
    torch.cuda.synchronize()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    lib = _native.lib()

    def launch(i):
        q, k, v = views[i]
        st = lib.mvb_rope_kv_cache_write(
            q.data_ptr(), q.stride(0), q.stride(1), q_out.data_ptr(), q_out.stride(0), q_out.stride(1),
            k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0), v.stride(1), pos.data_ptr(),
            cos.data_ptr(), sin.data_ptr(), cos.shape[0], kcs[i].data_ptr(), vcs[i].data_ptr(), slots.data_ptr(),
            None, T, H, KH, D, BS, nb, _native.DTYPE_BF16, None, 0, err.data_ptr(),
            torch.cuda.current_stream(dev).cuda_stream)
        assert st == _native.OK, _native.status_string(st)

    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for i in range(L):
            launch(i)
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(L):
            launch(i)
    replays, warm = max(1, args.steps // L), max(3, args.warmup // L)
    for _ in range(warm):
        graph.replay()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(physical_gpu(0)) as clocks:
        ev0.record()
        for _ in range(replays):
            graph.replay()
        ev1.record()
        torch.cuda.synchronize()
    sec = ev0.elapsed_time(ev1) / 1e3 / (replays * L)
    assert int(err.item()) == 0
    es = 2
    nbytes = T * (H + 2 * KH) * D * es + 2 * T * D * es + T * H * D * es + 2 * T * KH * D * es + 16 * T
    peak, peak_kind = peaks()
    # CPU baseline: the oracle's restatement (numpy rope + C write) on the same chunk
    import oracle

    q, k, v = views[0]
    host = {n: to_np_bf16(x) for n, x in (("q", q), ("k", k), ("v", v), ("cos", cos), ("sin", sin))}
    kc_np, vc_np = to_np_bf16(kcs[0]), to_np_bf16(vcs[0])
    pos_np, slots_np = pos.cpu().numpy(), slots.cpu().numpy()
    t0 = time.perf_counter()
    oracle.rope_numpy(host["q"], pos_np, host["cos"], host["sin"], "bf16")
    k_rot = oracle.rope_numpy(host["k"], pos_np, host["cos"], host["sin"], "bf16")
    oracle.cache_write(k_rot, host["v"], kc_np, vc_np, slots_np, BS, "bf16")
    cpu_sec = time.perf_counter() - t0
    print(json.dumps({
        "metric": "fused RoPE + KV write GB/s (8192-token prefill chunk)", "value": round(nbytes / sec / 1e9, 2),
        "unit": "GB/s", "n_gpus": 1, "steps": replays * L, "warmup": warm * L, "ms_per_step": round(sec * 1e3, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"rope_write: {T} tokens, 14q/2kv/d64, block 16, bf16, fused QKV views",
                   "layers_rotated": L, "timing": "CUDA graph of L launches, CUDA events"},
        "roofline": {"bound": "hbm", "achieved": round(nbytes / sec / 1e9, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(nbytes / sec / 1e9 / peak, 4), "traffic": None, "peak_kind": peak_kind,
                     "kernel": "rope_kv_write_kernel", "bytes_per_launch": int(nbytes)},
        "cpu_baseline": {"value": round(nbytes / cpu_sec / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
                         "sample": "oracle rope (numpy) + write (C) of the same 8192-token chunk"},
        "gpu_launches": replays * L, "clocks": clocks.summary(),
    }), flush=True)


def sweep_op(args):
    """Secondary measurement: the decode kernels over batch x context, the
    table behind the plan's kernel choice (make_plan in csrc/capi.cu).  Each
    case is the Qwen2-0.5B attention shape (14 q / 2 KV heads, head_dim 64,
    block 16, bf16) with every sequence at the same context length, timed as a
    CUDA graph of L back-to-back decodes over L distinct pools (median over
    repeats, per launch).  Kernels: "stream" (persistent stream-K + fixup),
    "sched" (scheduled persistent, its per-step schedule built once outside the
    timed graph), "mma" unsplit (one CTA per (sequence, KV head)), "mma" split
    into 512-token partitions plus the reduction, "fma" (CUDA cores, the plan's
    partitions), and "auto" (the plan's choice).  One JSON line per case."""
    import torch

    import mini_vllm_b200 as M
    from mini_vllm_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    L = min(args.layers, 8)
    batches = [1, 4, 8, 32, 64, 256]
    contexts = [128, 1024, 8192]
    for ctx in contexts:
        for nb in batches:
            spec = W.build_spec(f"sweep{nb}x{ctx}", np.full(nb, ctx, np.int64), 14, 2, 64, 16, seed=args.seed)
            t = W.torch_tensors(spec, torch.bfloat16, dev, num_layers=L)
            q, bt, kvl = t["query"], t["block_tables"], t["kv_len"]
            kcs, vcs = t["key_caches"], t["value_caches"]
            out = torch.empty_like(q)
            sched = M.build_decode_schedule(kvl, bt, 14, 2, 64, 16, spec.num_blocks, torch.bfloat16, variant="sched")
            kinds = [("stream", "stream", None, None), ("sched", "sched", None, sched),
                     ("mma_unsplit", "mma", spec.max_blocks * 16, None), ("mma_split512", "mma", 512, None),
                     ("fma", "fma", None, None), ("auto", "auto", None, None)]
            res = {"batch": nb, "ctx": ctx}
            for name, variant, pt, sc in kinds:
                def launches():
                    for layer in range(L):
                        M.paged_decode_attention(q, kcs[layer], vcs[layer], bt, kvl, 16, out=out, variant=variant,
                                                 partition_tokens=pt, strict=False, schedule=sc)
                launches()
                torch.cuda.synchronize()
                M.check_device_errors(dev)
                s2 = torch.cuda.Stream(device=dev)
                s2.wait_stream(torch.cuda.current_stream(dev))
                with torch.cuda.stream(s2):
                    launches()
                torch.cuda.current_stream(dev).wait_stream(s2)
                torch.cuda.synchronize()
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    launches()
                for _ in range(3):
                    g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                samples = []
                for _ in range(30):
                    e0.record()
                    g.replay()
                    e1.record()
                    e1.synchronize()
                    samples.append(e0.elapsed_time(e1) * 1e3 / L)
                res[name + "_us"] = round(statistics.median(samples), 2)
                del g
            plan = M.decode_plan(nb, 14, 2, 64, 16, spec.num_blocks, spec.max_blocks, torch.bfloat16, "auto")
            res["auto_plan"] = plan["variant"] + (f"/{plan['num_partitions']}p" if plan["num_partitions"] else "")
            res["kv_MB"] = round(spec.kv_bytes(2) / 1e6, 3)
            print(json.dumps(res), flush=True)
            del t, q, bt, kvl, kcs, vcs, out, sched
            torch.cuda.empty_cache()


def variants_op(args):
    """Secondary measurement: decode time per launch of each kernel at the
    benchmark configs — config 2 (256 x U[128,2048], 14/2/64), config 3 (32 x
    32768, 14/2/64) and config 4 on one GPU (global batch 1024, 32/8/128,
    lognormal contexts) — as CUDA graphs of back-to-back decodes over distinct
    pools (more than L2 each), median of 20 replays.  Kernels: the stream
    kernel (+ its fixup) building its set-up in every launch ("stream") and
    reading the per-step schedule built once outside the graph
    ("stream+schedule"), the scheduled kernel (schedule built once per model
    step, outside the graph), the one-CTA-per-(sequence, KV head) kernel with
    the plan's split-K, the CUDA-core kernel (config 2 only), and AUTO.  One
    JSON line per (config, kernel)."""
    import torch

    import mini_vllm_b200 as M
    from mini_vllm_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    peak, peak_kind = peaks()
    for config, L, kinds in ((2, 24, ("stream", "stream+schedule", "sched", "mma", "fma", "auto")),
                             (3, 4, ("stream", "stream+schedule", "sched", "mma", "auto")),
                             (4, 2, ("stream", "stream+schedule", "sched", "mma", "auto"))):
        spec, _ = rank_spec(config, 0, 1, args.seed)
        t = W.torch_tensors(spec, torch.bfloat16, dev, num_layers=L)
        q, bt, kvl = t["query"], t["block_tables"], t["kv_len"]
        kcs, vcs = t["key_caches"], t["value_caches"]
        out = torch.empty_like(q)
        sched = M.build_decode_schedule(kvl, bt, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
                                        spec.num_blocks, torch.bfloat16, variant="sched")
        ssched = M.build_decode_schedule(kvl, bt, spec.num_heads, spec.num_kv_heads, spec.head_dim,
                                         spec.block_size, spec.num_blocks, torch.bfloat16, variant="stream")
        by = spec.decode_bytes(2)
        for kind in kinds:
            variant = "stream" if kind == "stream+schedule" else kind
            sc = sched if kind == "sched" else ssched if kind == "stream+schedule" else None

            def launches():
                for layer in range(L):
                    M.paged_decode_attention(q, kcs[layer], vcs[layer], bt, kvl, spec.block_size, out=out,
                                             variant=variant, strict=False, schedule=sc)
            launches()
            torch.cuda.synchronize()
            M.check_device_errors(dev)
            s2 = torch.cuda.Stream(device=dev)
            s2.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s2):
                launches()
            torch.cuda.current_stream(dev).wait_stream(s2)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                launches()
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            samples = []
            for _ in range(20):
                e0.record()
                g.replay()
                e1.record()
                e1.synchronize()
                samples.append(e0.elapsed_time(e1) * 1e3 / L)
            us = statistics.median(samples)
            plan = M.decode_plan(spec.num_seqs, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
                                 spec.num_blocks, spec.max_blocks, torch.bfloat16, variant)
            print(json.dumps({"config": config, "kernel": kind, "plan": plan["variant"],
                              "partitions": plan["num_partitions"], "us_per_launch": round(us, 2),
                              "GBps": round(by / us / 1e3, 1), "frac": round(by / us / 1e3 / peak, 4),
                              "peak": f"{peak} GB/s ({peak_kind})", "bytes_per_launch": by, "pools": L}), flush=True)
            del g
        del t, q, bt, kvl, kcs, vcs, out, sched, ssched
        torch.cuda.empty_cache()


def profile_op(args):
    """The case an ncu capture runs: for each of --layers pools, one KV write
    and one decode of --variant (with --partition-tokens) on --config, twice
    over, untimed; the scheduled kernel's schedule is built once first.
    Captures pick the kernel with -k and skip the first round with -s."""
    import torch

    import mini_vllm_b200 as M
    from mini_vllm_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    spec, _ = rank_spec(args.config, 0, args.shard_of, args.seed)
    L = args.layers
    t = W.torch_tensors(spec, torch.bfloat16, dev, num_layers=L)
    q, nk, nv = t["query"], t["new_key"], t["new_value"]
    bt, kvl, slots = t["block_tables"], t["kv_len"], t["slot_mapping"]
    out = torch.empty_like(q)
    pt = args.partition_tokens or None
    plan = M.decode_plan(spec.num_seqs, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
                         spec.num_blocks, spec.max_blocks, torch.bfloat16, args.variant, pt)
    sched = None
    if plan["variant"] in ("sched", "stream"):
        sched = M.build_decode_schedule(kvl, bt, spec.num_heads, spec.num_kv_heads, spec.head_dim,
                                        spec.block_size, spec.num_blocks, torch.bfloat16, variant=plan["variant"])
    for _ in range(2):
        for layer in range(L):
            M.paged_cache_write(nk, nv, t["key_caches"][layer], t["value_caches"][layer], slots, spec.block_size,
                                strict=False, check_duplicates=False)
            M.paged_decode_attention(q, t["key_caches"][layer], t["value_caches"][layer], bt, kvl, spec.block_size,
                                     out=out, variant=args.variant, partition_tokens=pt, strict=False,
                                     schedule=sched)
    torch.cuda.synchronize()
    M.check_device_errors(dev)
    print(json.dumps({"op": "profile", "config": args.config, "shard_of": args.shard_of, "num_seqs": spec.num_seqs,
                      "plan": plan, "layers": L,
                      "decode_bytes": spec.decode_bytes(2), "write_bytes": spec.write_bytes(2)}), flush=True)


def trace_op(args):
    """The stream decode's per-warp timeline.  Loads the trace build of the
    library (``lib/libmvb200_trace.so``: the stream and warp-fixup kernels with
    %globaltimer stamps, built by ``build.build_trace()`` when absent) and runs
    the headline step's layer-steps (KV write, then the decode with the step's
    schedule and the set-up overlapped with the write) for min(--layers, 8)
    pools in one CUDA graph.  After warm-up replays it times one replay with
    CUDA events (the trace build's own time per layer-step), clears the stamps,
    replays once more and prints, per launch, the times in microseconds from
    the launch's first stream warp entry: warps entering, first loads issued,
    first tile landed, loop end, stream end, the median time between a warp's
    consecutive tiles (and the rate all warps' tiles make at it), and the
    fixup warps' wait and end.  Launch-level figures only: the stamps cost a
    few instructions per tile."""
    import ctypes

    import torch

    from mini_vllm_b200 import _native
    from mini_vllm_b200 import build as B

    path = B.TRACE_LIB_PATH if os.path.exists(B.TRACE_LIB_PATH) else B.build_trace()
    _native.LIB_PATH = path  # before the first call loads the library
    import mini_vllm_b200 as M
    from mini_vllm_b200 import workloads as W

    lib = _native.lib()
    lib.mvb_trace_clear.restype = ctypes.c_int
    lib.mvb_trace_read.restype = ctypes.c_int
    lib.mvb_trace_read.argtypes = [ctypes.c_void_p] * 3
    NL, NW, NF, NT = 8, 4096, 16384, 32  # the trace arrays' shapes (csrc/decode_stream.cu)

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    spec, _ = rank_spec(args.config, 0, args.shard_of, args.seed)
    L = max(1, min(args.layers, NL))
    t = W.torch_tensors(spec, torch.bfloat16, dev, num_layers=L)
    q, nk, nv = t["query"], t["new_key"], t["new_value"]
    bt, kvl, slots = t["block_tables"], t["kv_len"], t["slot_mapping"]
    out = torch.empty_like(q)
    variant = "stream"
    plan = M.decode_plan(spec.num_seqs, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
                         spec.num_blocks, spec.max_blocks, torch.bfloat16, variant)
    sched = M.build_decode_schedule(kvl, bt, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
                                    spec.num_blocks, torch.bfloat16, variant=variant)

    def layer_steps():
        for layer in range(L):
            M.paged_cache_write(nk, nv, t["key_caches"][layer], t["value_caches"][layer], slots, spec.block_size,
                                strict=False, check_duplicates=False)
            M.paged_decode_attention(q, t["key_caches"][layer], t["value_caches"][layer], bt, kvl,
                                     spec.block_size, out=out, variant=variant, strict=False, after_write=True,
                                     schedule=sched)

    layer_steps()
    torch.cuda.synchronize()
    M.check_device_errors(dev)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        layer_steps()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        layer_steps()
    for _ in range(3):
        graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    graph.replay()
    e1.record()
    torch.cuda.synchronize()
    graph_us = e0.elapsed_time(e1) * 1e3 / L
    if lib.mvb_trace_clear() != 0:
        raise RuntimeError("mvb_trace_clear failed")
    torch.cuda.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    M.check_device_errors(dev)
    ws = np.zeros((NL, NW, 5), np.uint64)
    tt = np.zeros((NL, NW, NT), np.uint64)
    fx = np.zeros((NL, NF, 3), np.uint64)
    if lib.mvb_trace_read(ws.ctypes.data, tt.ctypes.data, fx.ctypes.data) != 0:
        raise RuntimeError("mvb_trace_read failed")
    del graph
    if args.trace_out:
        np.savez_compressed(args.trace_out, warps=ws, tiles=tt, fixups=fx)

    tile_bytes = 2 * 16 * spec.head_dim * 2  # K and V of one 16-token tile of one KV head, bf16
    print(json.dumps({"op": "trace", "config": args.config, "shard_of": args.shard_of, "num_seqs": spec.num_seqs,
                      "layers": L, "plan": plan,
                      "trace_build_us_per_layer_step": round(graph_us, 2),
                      "decode_bytes": spec.decode_bytes(2), "tile_bytes": tile_bytes}), flush=True)

    def pct(x, p):
        return round(float(np.percentile(x, p)) / 1e3, 2) if len(x) else None

    prev_end = None
    for i in range(L):
        w = ws[i].astype(np.int64)
        entered = w[:, 0] > 0
        if not entered.any():
            continue
        t0 = int(w[entered, 0].min())
        worked = entered & (w[:, 4] > 0) & (w[:, 2] > 0)
        rel = w[worked] - t0
        ti = tt[i][worked].astype(np.int64)
        both = (ti[:, 1:] > 0) & (ti[:, :-1] > 0)
        gaps = (ti[:, 1:] - ti[:, :-1])[both]
        f = fx[i].astype(np.int64)
        fw = f[(f[:, 0] > 0) & (f[:, 2] > 0)] - t0
        stream_end = int(rel[:, 4].max()) if len(rel) else 0
        fix_end = int(fw[:, 2].max()) if len(fw) else stream_end
        med_gap = float(np.median(gaps)) if len(gaps) else 0.0
        row = {
            "launch": i, "stream_warps": int(entered.sum()), "warps_with_tiles": int(worked.sum()),
            "entry_p50_us": pct(w[entered, 0] - t0, 50), "entry_max_us": pct(w[entered, 0] - t0, 100),
            "first_issue_p50_us": pct(rel[:, 1], 50),
            "first_tile_us": [pct(rel[:, 2], 10), pct(rel[:, 2], 50), pct(rel[:, 2], 90)],
            "loop_end_us": [pct(rel[:, 3], 10), pct(rel[:, 3], 50), pct(rel[:, 3], 90)],
            "stream_end_max_us": round(stream_end / 1e3, 2),
            "tile_interval_p50_us": round(med_gap / 1e3, 3),
            "steady_GBps": round(int(worked.sum()) * tile_bytes / med_gap, 1) if med_gap > 0 else None,
            "fixup_warps": int(len(fw)),
            "fixup_wait_us": [pct(fw[:, 1], 0), pct(fw[:, 1], 50)] if len(fw) else None,
            "fixup_end_max_us": round(fix_end / 1e3, 2),
            "fixup_after_stream_us": round((fix_end - stream_end) / 1e3, 2),
            "start_after_previous_us": round((t0 - prev_end) / 1e3, 2) if prev_end is not None else None,
        }
        prev_end = t0 + max(fix_end, stream_end)
        print(json.dumps(row), flush=True)


def engine_op(args):
    """BASELINE config 5, bounded: continuous-batching serving in the
    reference's own engine (LLMEngine -> EngineCore -> Scheduler / BlockManager
    / ModelInputBuilder -> PagedExecutor -> QwenModelRunner, installed from
    baseline/_ref), one replica per GPU, on a random-init Qwen2-0.5B (24
    layers, hidden 896, 14/2 heads of 64, MLP 4864, vocab 151936, weights
    N(0, 0.02), written to a temporary checkpoint).  Requests: --requests per
    replica with prompt token ids uniform over the vocabulary, prompt lengths
    U[32, 1024], max_tokens U[64, 512], Poisson arrivals at 64 req/s, greedy
    sampling.  Our arm serves attention with AttentionBackendB200 (the "b200"
    branch of AttentionBackend.create); --impl reference serves it with the
    reference's own GPU backend ("triton", its default).  Metric: generated
    tokens per second of wall time from the first arrival to the last
    completion (aggregate over replicas), plus the per-step decode latency."""
    import tempfile

    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    from mini_vllm_b200 import reference_engine as RE

    try:
        RE.import_reference()
    except ImportError as e:
        if rank == 0:
            print(json.dumps({"impl": args.impl, "op": "engine", "unavailable": str(e).splitlines()[0]}))
        return
    backend = "b200" if args.impl == "ours" else "triton"
    RE.register_backend(overlap_after_write=True, strict=False)
    from mini_vllm.config import Config
    from mini_vllm.engine.engine import LLMEngine

    ckpt = tempfile.mkdtemp(prefix=f"mvb_qwen2_{rank}_")
    RE.write_random_checkpoint(ckpt, seed=1)
    vocab = RE.QWEN2_0_5B["vocab_size"]
    rng = np.random.default_rng(args.seed + 1000 * rank)
    n = args.requests
    plen = rng.integers(32, 1025, n)
    maxt = rng.integers(64, 513, n)
    arrive = np.cumsum(rng.exponential(1.0 / 64.0, n))
    prompts = [RE.prompt_text(rng.integers(0, vocab, int(k))) for k in plen]
    cfg = Config(executor_type="paged", attention_backend=backend, model_path=ckpt, device=f"cuda:{local_rank}",
                 block_size=16, num_gpu_blocks=16384, max_num_seqs=128, max_num_batched_tokens=2048,
                 max_num_prefill_tokens=2048, max_prefill_chunk_size=512, max_model_len=2048,
                 max_queue_len=1 << 20, request_timeout_s=1e9, print_step_events=False,
                 enable_prefix_caching=False)
    eng = LLMEngine(cfg)
    # warm-up: a few short requests through every path (prefill chunks, decode)
    for i in range(4):
        eng.add_request(prompts[i], max_new_tokens=8)
    eng.run_until_done()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    steps, decode_steps, decode_s = 0, 0, 0.0
    t0 = time.perf_counter()
    nxt = 0
    while True:
        now = time.perf_counter() - t0
        while nxt < n and arrive[nxt] <= now:
            eng.add_request(prompts[nxt], max_new_tokens=int(maxt[nxt]))
            nxt += 1
        q = eng.queue
        if q.num_waiting == 0 and q.num_running == 0:
            if nxt >= n:
                break
            time.sleep(max(0.0, arrive[nxt] - now))
            continue
        ts = time.perf_counter()
        res = eng.step()
        steps += 1
        if not res.scheduled_prefill_groups and res.scheduled_decode_groups:
            decode_steps += 1
            decode_s += time.perf_counter() - ts
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    outs = eng.get_outputs()
    gen = int(sum(int(m) for m in maxt))  # greedy runs every request to max_tokens (no EOS in the id vocabulary)
    stats = torch.tensor([gen, len(outs) - 4, steps], dtype=torch.float64, device=dev)  # minus the warm-up ones
    wall_t = torch.tensor([wall], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(stats)
        dist.all_reduce(wall_t, op=dist.ReduceOp.MAX)
    if rank == 0:
        tok_s = float(stats[0]) / float(wall_t[0])
        line = {"metric": "config-5 engine decode tok/s (reference engine, random-init Qwen2-0.5B)",
                "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world, "impl": args.impl,
                "attention_backend": type(eng._executor._attention_backend).__name__,
                "requests": int(stats[1]), "requests_per_replica": n, "generated_tokens": int(stats[0]),
                "wall_s": round(float(wall_t[0]), 3), "engine_steps": int(stats[2]),
                "rank0_decode_only_steps": decode_steps,
                "rank0_decode_step_ms": round(1e3 * decode_s / max(1, decode_steps), 3),
                "higher_is_better": True, "scaling": "weak", "data": "synthetic",
                "config": {"workload": "config5: reference LLMEngine, random-init Qwen2-0.5B (24 layers), "
                                       "prompts U[32,1024], max_tokens U[64,512], Poisson 64 req/s, greedy",
                           "engine": {"block_size": 16, "num_gpu_blocks": 16384, "max_num_seqs": 128,
                                      "max_num_batched_tokens": 2048, "max_prefill_chunk_size": 512},
                           "parallelism": f"{world} replicas"}}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def metadata_op(args):
    """Secondary measurement: StepMetadataBuilder.build for one config-2 decode
    step (256 sequences, ctx U[128,2048], block 16: positions, slot mapping,
    padded block tables, kv_len_after, sample indices) — host time per step
    including the upload and the launch, the device work drained at the end.
    The CPU line is the oracle's restatement of ModelInputBuilder's per-token
    loops on the same step."""
    import torch

    import mini_vllm_b200 as M
    from mini_vllm_b200 import workloads as W

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    spec = W.make_spec(2, seed=args.seed)
    decode = [([int(b) for b in row if b >= 0], int(c) - 1) for row, c in zip(spec.block_tables, spec.context_lens)]
    builder = M.StepMetadataBuilder(spec.block_size, dev)
    md = builder.build([], decode)  # correctness gate: slots equal the workload's
    assert np.array_equal(md.slot_mapping.cpu().numpy(), spec.slot_mapping)
    for _ in range(max(3, args.warmup)):
        builder.build([], decode, strict=False)
    torch.cuda.synchronize()
    n = max(10, min(args.steps, 2000))
    t0 = time.perf_counter()
    for _ in range(n):
        builder.build([], decode, strict=False)
    torch.cuda.synchronize()
    sec = (time.perf_counter() - t0) / n
    import oracle

    lists = [d[0] for d in decode]
    t0 = time.perf_counter()
    reps = 0
    while reps < 3 or time.perf_counter() - t0 < 2.0:
        oracle.step_metadata_numpy(lists, [d[1] for d in decode], [1] * len(decode), [], 0, spec.block_size)
        reps += 1
    cpu_sec = (time.perf_counter() - t0) / reps
    # the padded-table entry point (an engine that keeps its tables as arrays)
    tables = spec.block_tables
    counts = (tables >= 0).sum(axis=1)
    cached = spec.context_lens.astype(np.int64) - 1
    ones = np.ones(len(decode), dtype=np.int64)
    for _ in range(max(3, args.warmup)):
        builder.build_from_arrays(tables, counts, cached, ones, [], 0, strict=False)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n):
        builder.build_from_arrays(tables, counts, cached, ones, [], 0, strict=False)
    torch.cuda.synchronize()
    sec_arrays = (time.perf_counter() - t0) / n
    print(json.dumps({
        "metric": "per-step attention metadata build, us/step (config-2 decode step)", "value": round(sec * 1e6, 2),
        "from_arrays_us": round(sec_arrays * 1e6, 2),
        "unit": "us", "n_gpus": 1, "steps": n, "warmup": max(3, args.warmup), "higher_is_better": False,
        "vs_baseline": None, "data": "synthetic",
        "config": {"workload": "metadata: 256 decode sequences, ctx U[128,2048], block 16",
                   "blocks": int(sum(len(x) for x in lists)), "timing": "host perf_counter over K builds, one sync"},
        "cpu_baseline": {"value": round(cpu_sec * 1e6, 1), "unit": "us", "cores": 1, "kind": "port",
                         "sample": "oracle restatement of ModelInputBuilder's per-token loops, same step"},
    }), flush=True)


def main():
    args = parse_args()
    if args.op == "metadata":
        metadata_op(args)
        return
    if args.op == "gather":
        gather_op(args)
        return
    if args.op == "rope_write":
        rope_write_op(args)
        return
    if args.op == "sweep":
        sweep_op(args)
        return
    if args.op == "engine":
        engine_op(args)
        return
    if args.op == "trace":
        trace_op(args)
        return
    if args.op == "profile":
        profile_op(args)
        return
    if args.op == "variants":
        variants_op(args)
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
