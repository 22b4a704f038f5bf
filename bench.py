#!/usr/bin/env python
"""Benchmark of the paged-KV hot path on B200: BASELINE config 3.

One step = one decode step of a Qwen2.5-0.5B-shaped attention stack over 24
layers for B = 256 sequences per GPU (contexts lognormal, median 1024, sigma
0.5, clipped to [16, 8192]; fp16 KV; 16-token blocks scattered over a pool of
1.1x the blocks needed; one pool per layer).  Per layer: one
reshape_and_cache launch (append the new token) and one paged decode
attention launch.  Inputs are synthetic (seeded), weights are not involved.

Multi-GPU: one process per GPU (torchrun), sequences dealt round-robin, each
GPU owns its own pools; per-GPU work is fixed as N grows ("weak"; --strong
keeps 256 sequences in total).  The timed region is bracketed by a barrier and
a device synchronisation; the time is the max over ranks.

Prints ONE JSON line (rank 0).  --impl reference times the reference
algorithm's CPU port (the oracle, oracle/pagedkv_oracle.c) on the host cores
instead.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "llm-inference-scheduler_b200"))

METRIC = "paged decode attn KV GB/s (% of HBM peak) and decode tok/s at 1/2/4/8 B200"
UNIT = "GB/s"
WORKLOAD = ("config3: paged decode step, 24 layers x (append + decode attention, one fused call), "
            "B=256 seqs/GPU, ctx lognormal(median 1024, sigma 0.5) in [16,8192], 14q/2kv, d64, fp16 KV")
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("decode", "prefill", "e2e", "cache_ops", "decode_fp8",
                                           "migrate", "model_step"),
                    default="decode",
                    help="decode = BASELINE config 3 (headline); prefill = config 4; e2e = config 5; "
                         "cache_ops = reshape_and_cache and copy_blocks at bandwidth-sized batches; "
                         "migrate = KV block migration between rank pairs over NVLink (2+ ranks); "
                         "model_step = config 5's model step replayed from its CUDA graphs")
    ap.add_argument("--migrate-blocks", type=int, default=1024,
                    help="migrate: blocks per copy launch (x 24 layers, K and V)")
    ap.add_argument("--kv-fp8", action="store_true",
                    help="prefill: fp8 e4m3 pools (quantising append, tensor-core fp8 prefill)")
    ap.add_argument("--fp8-prefill", choices=("scratch", "in-kernel"), default="scratch",
                    help="prefill --kv-fp8: 16-bit scratch pass + tcgen05 kernel, or the tcgen05 "
                         "kernel converting e4m3 tiles itself (no scratch)")
    ap.add_argument("--append-tokens", type=int, nargs="+", default=[8192, 65536],
                    help="cache_ops: tokens appended per reshape_and_cache launch")
    ap.add_argument("--copy-pairs", type=int, default=4096, help="cache_ops: (src, dst) block pairs")
    ap.add_argument("--conversations", type=int, default=64, help="config 5: conversations")
    ap.add_argument("--rate", type=float, default=40.0, help="config 5: Poisson arrivals per second")
    ap.add_argument("--max-num-seqs", type=int, default=128)
    ap.add_argument("--no-cuda-graphs", action="store_true",
                    help="config 5: run every step eagerly instead of replaying CUDA graphs")
    ap.add_argument("--max-batched-tokens", type=int, default=2048)
    ap.add_argument("--layers", type=int, default=24)
    ap.add_argument("--batch", type=int, default=256, help="sequences per GPU (weak) or in total (--strong)")
    ap.add_argument("--strong", action="store_true")
    ap.add_argument("--per-layer-calls", action="store_true",
                    help="decode: one call per layer (decode + merge each) instead of one "
                         "multi-layer call whose layers chain")
    ap.add_argument("--e2e-steps", type=int, default=50, help="e2e: steps per timing window")
    ap.add_argument("--e2e-windows", type=int, default=5, help="e2e: timing windows (median reported)")
    ap.add_argument("--e2e-chunks", default="",
                    help="e2e: layers per chunk (comma list summing to --layers; default: "
                         "DecodeStepGraph's, one layer a chunk); each chunk's copies overlap the "
                         "other chunks' compute")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="bounded CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-steps", type=int, default=0,
                    help="only run this many steps after warm-up (for ncu launch lists); no timing")
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def traffic_from_profiles():
    """DRAM bytes per decode launch from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "paged_decode_config3.md")
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                return int(line.split(":")[1].strip().split()[0])
    except (OSError, ValueError):
        pass
    return None


# --------------------------------------------------------------- clock sampling

def smi_ids(cuda_indices) -> str:
    """nvidia-smi ids (UUIDs) of this process's CUDA devices, so the sampler
    watches the GPUs the job runs on whatever CUDA_VISIBLE_DEVICES maps."""
    import torch

    ids = []
    for i in cuda_indices:
        try:
            u = str(torch.cuda.get_device_properties(i).uuid)
            ids.append(u if u.startswith("GPU-") else "GPU-" + u)
        except Exception:  # noqa: BLE001 - fall back to the index
            ids.append(str(i))
    return ",".join(ids)


class ClockSampler:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_indices):
        self.proc = None
        self.lines = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", smi_ids(gpu_indices)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self, t0: float, t1: float):
        import datetime

        rows = []
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(f[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                rows.append((ts, float(f[2]), float(f[3]), f[6], f[7], f[8], f[9]))
            except ValueError:
                continue
        if not rows:
            return None
        inside = [r for r in rows if t0 - 0.05 <= r[0] <= t1 + 0.05] or rows
        reasons = set()
        for r in inside:
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                "sw_power_cap"), r[3:]):
                if v.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r[1] for r in inside),
                "sm_max_mhz": max(r[2] for r in inside), "reasons": sorted(reasons),
                "samples": len(inside)}


# --------------------------------------------------------------- CPU baseline (oracle port)

def cpu_sample(seconds: float, n_seqs_subset: int | None = None, max_reps: int | None = None):
    """Time the oracle (CPU port of the reference's append + gather + _attention)
    on config-3 layers of rank 0's shard.  Returns (GB/s, cores, sample text)."""
    import numpy as np

    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from pagedkv import workloads as W

    ctx = W.shard_contexts(256, 0, 1)
    if n_seqs_subset is not None:
        ctx = ctx[:: max(1, len(ctx) // n_seqs_subset)][:n_seqs_subset]
    nb = int(math.ceil(1.1 * ((ctx + 15) // 16).sum()))
    tabs = W.make_tables(ctx, nb, seed=100)
    rng = np.random.default_rng(0)
    kp = rng.standard_normal((nb, 16, 2, 64), dtype=np.float32).astype(np.float16)
    vp = rng.standard_normal((nb, 16, 2, 64), dtype=np.float32).astype(np.float16)
    B = len(ctx)
    q = rng.standard_normal((B, 14, 64), dtype=np.float32).astype(np.float16)
    kn = rng.standard_normal((B, 2, 64), dtype=np.float32).astype(np.float16)
    vn = rng.standard_normal((B, 2, 64), dtype=np.float32).astype(np.float16)
    pos = ctx - 1
    slots = tabs[np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16
    qsl = np.arange(B + 1, dtype=np.int32)
    prior = (ctx - 1).astype(np.int32)
    bytes_per = W.decode_bytes(ctx) + W.append_bytes(B)
    # every host core this process may run on (torchrun sets OMP_NUM_THREADS=1)
    threads = max(1, len(os.sched_getaffinity(0)))
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.reshape_and_cache(kp, vp, kn, vn, slots, "f16")
        oracle.paged_attention(q, kp, vp, tabs, qsl, prior, "f16", threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_reps is not None and reps >= max_reps):
            break
    gbs = bytes_per * reps / el / 1e9
    sample = (f"oracle port (C, OpenMP) of the reference's append + gather + _attention; "
              f"{reps} x one config-3 layer of {B} seqs (sum ctx {int(ctx.sum())}), {el:.1f} s")
    return gbs, threads, sample, el, reps


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # each step: one layer of a 32-sequence subset of config 3 (bounded sample)
    n_sub = 32
    total = args.warmup + args.steps
    gbs_w, cores, sample, el, reps = cpu_sample(1e9, n_seqs_subset=n_sub, max_reps=max(1, args.warmup))
    gbs, cores, sample, el, reps = cpu_sample(1e9, n_seqs_subset=n_sub, max_reps=max(1, args.steps))
    line = {
        "metric": METRIC, "value": round(gbs, 3), "unit": UNIT, "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(1e3 * el / reps, 4), "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD, "reference_step": f"1 layer, {n_sub}-sequence subset, CPU"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": round(gbs, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU arm

def gpu_local_cpus(cuda_indices) -> list:
    """Per CUDA device: the host cores the driver reports as local to it
    (NVML CPU affinity, matched by UUID), or None where it cannot say."""
    out = []
    try:
        import pynvml

        pynvml.nvmlInit()
    except Exception:  # noqa: BLE001 - no NVML: no locality information
        return [None for _ in cuda_indices]
    words = (os.cpu_count() or 64) // 64 + 1
    for uid in smi_ids(cuda_indices).split(","):
        try:
            h = pynvml.nvmlDeviceGetHandleByUUID(uid)
            mask = pynvml.nvmlDeviceGetCpuAffinity(h, words)
            out.append([64 * w + b for w, m in enumerate(mask) for b in range(64) if (int(m) >> b) & 1])
        except Exception:  # noqa: BLE001
            out.append(None)
    return out


def pin_rank_cpus(local: int, local_world: int) -> list[int]:
    """Pin this process to host cores near its GPU, disjoint from the other
    local ranks' (torchrun ranks of one node would otherwise contend for the
    same cores while they enqueue launches and copies), before any pinned
    host buffer is allocated, so those land in the GPU's NUMA node.  Returns
    the cores now allowed."""
    from pagedkv import workloads as W

    cpus = sorted(os.sched_getaffinity(0))
    mine = W.local_cpu_share(cpus, gpu_local_cpus(range(local_world)), local)
    if mine:
        os.sched_setaffinity(0, mine)
    return sorted(os.sched_getaffinity(0))


class DecodeRun:
    """One rank's config-3 decode workload on its GPU: pools of 1.1x the
    needed blocks per layer (random N(0,1) contents), scattered tables, the
    step's q / new K / new V per layer, and the bound launches of one step
    (schedule build, then one fused append + decode call per layer)."""

    def __init__(self, batch: int, strong: bool, rank: int, world: int, L: int, dev,
                 per_layer_calls: bool = False):
        import numpy as np
        import torch

        from pagedkv import BlockManager, ops
        from pagedkv import workloads as W

        self.L, self.scale, self.dt = L, 0.125, torch.float16
        dt = self.dt
        self.ctx = ctx = W.shard_contexts(batch, rank, world, strong=strong)
        self.B = B = len(ctx)
        self.nblk = nblk = (ctx + 15) // 16
        self.nb = nb = int(math.ceil(1.1 * nblk.sum()))
        self.tabs_np = W.make_tables(ctx, nb, seed=100 + rank)
        g = torch.Generator(device=dev)
        g.manual_seed(1234 + rank)
        self.mgr = mgr = BlockManager(nb, 16, L, 2, 64, device=dev, dtype=dt)
        for layer in range(L):
            mgr.k_pool[layer].normal_(generator=g)
            mgr.v_pool[layer].normal_(generator=g)
        self.q = torch.randn((L, B, 14, 64), generator=g, device=dev, dtype=dt)
        self.kn = torch.randn((L, B, 2, 64), generator=g, device=dev, dtype=dt)
        self.vn = torch.randn((L, B, 2, 64), generator=g, device=dev, dtype=dt)
        self.out = torch.empty_like(self.q)
        self.tabs = torch.from_numpy(self.tabs_np).to(dev)
        self.ctx_d = torch.from_numpy(ctx.astype(np.int32)).to(dev)
        self.err = ops.new_error_flags(dev)
        self.sched = ops.new_decode_schedule(B, self.tabs.shape[1], dev)
        self.build_sched = ops.bind_decode_schedule(self.sched, self.tabs, self.ctx_d, nb, 14, 2, 64, dt,
                                                    err=self.err)
        if per_layer_calls:
            # one pkv_paged_decode_append_attention_scheduled call per layer
            self.ws = ops.new_decode_workspace(B, 14, 64, dev)
            self.decodes = [ops.bind_paged_decode_append_attention(
                self.q[l], self.kn[l], self.vn[l], mgr.k_pool[l], mgr.v_pool[l], self.tabs, self.ctx_d,
                self.scale, self.ws, self.out[l], self.err, schedule=self.sched) for l in range(L)]
        else:
            # one pkv_paged_decode_append_attention_layers call for all layers,
            # a split-K set per layer: the layers' decode kernels chain and one
            # merge launch follows them
            self.ws = ops.new_decode_workspace(B, 14, 64, dev, layers=L)
            plan = ops.DecodeAppendLayersPlan(self.tabs, self.ctx_d, self.scale, self.ws, self.err,
                                              schedule=self.sched)
            self.decodes = [lambda: plan(self.q, self.kn, self.vn, mgr.k_cache, mgr.v_cache, self.out)]
        self.dec_bytes = W.decode_bytes(ctx)
        self.app_bytes = W.append_bytes(B)
        self.step_bytes = L * (self.dec_bytes + self.app_bytes)

    def step(self):
        """One decode step: the schedule, then the layers' fused append +
        decode and their merge (one multi-layer call, or one call per layer)."""
        self.build_sched()
        for f in self.decodes:
            f()

    def calls(self):
        """The step's calls without the schedule build (it stays valid: the
        lengths and tables do not change)."""
        for f in self.decodes:
            f()

    def timed(self, fn, steps: int, barrier) -> float:
        """Device ms per call of `fn`, `steps` calls back to back bracketed by
        a barrier and a device synchronisation on both sides."""
        import torch

        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        barrier()
        return start.elapsed_time(end) / steps


def run_ours(args):
    import numpy as np
    import torch
    import torch.distributed as dist

    from pagedkv import PagedKVCache, ops
    from pagedkv import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    local_world = int(os.environ.get("LOCAL_WORLD_SIZE", str(world)))
    all_cpus = sorted(os.sched_getaffinity(0))
    cpus = pin_rank_cpus(local, local_world)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    L = args.layers
    R = DecodeRun(args.batch, args.strong, rank, world, L, dev, per_layer_calls=args.per_layer_calls)
    B, ctx, nblk, mgr, scale, dt = R.B, R.ctx, R.nblk, R.mgr, R.scale, R.dt

    for _ in range(args.warmup):
        R.step()
    torch.cuda.synchronize()
    ops.check_flags(R.err, "bench warm-up")

    if args.profile_steps:
        for _ in range(args.profile_steps):
            R.step()
        torch.cuda.synchronize()
        if world > 1:
            dist.destroy_process_group()
        return

    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    time.sleep(0.3 if sampler else 0)
    t_wall0 = time.time()
    # (1) the step: schedule build + 24 calls, the headline value
    ms_local = R.timed(R.step, args.steps, barrier)
    # (2) the roofline: the same 24 calls without the build, so that 24 x the
    # call time is part of the step time by construction
    dec_ms_local = R.timed(R.calls, args.steps, barrier) / L
    t_wall1 = time.time()
    if sampler:
        sampler.stop()
    ops.check_flags(R.err, "bench timed region")
    ms = W.max_over_ranks(ms_local)
    dec_ms = W.max_over_ranks(dec_ms_local)
    total_bytes = W.sum_over_ranks(R.step_bytes)
    total_seqs = W.sum_over_ranks(B)
    per_rank = {"sum_ctx": [int(x) for x in W.gather_over_ranks(int(ctx.sum()))],
                "seqs": [int(x) for x in W.gather_over_ranks(B)],
                "ms_local": [round(x, 5) for x in W.gather_over_ranks(ms_local)],
                "decode_call_ms_local": [round(x, 6) for x in W.gather_over_ranks(dec_ms_local)],
                "host_cpus": [int(x) for x in W.gather_over_ranks(len(cpus))]}

    # ---- end to end through the public API: pinned host inputs in, outputs back
    kv = PagedKVCache(mgr)
    for i in range(B):
        kv.add_sequence(i, R.tabs_np[i, :nblk[i]].tolist(), int(ctx[i]) - 1)
    # the step's inputs in one pinned staging buffer, [L, B, 18, 64]: a run
    # of layers' q, k and v are views of its rows (one copy per chunk)
    hqkv = torch.empty((L, B, 18, 64), dtype=dt).pin_memory()
    hqkv[:, :, :14].copy_(R.q)
    hqkv[:, :, 14:16].copy_(R.kn)
    hqkv[:, :, 16:18].copy_(R.vn)
    dqkv = torch.empty((L, B, 18, 64), device=dev, dtype=dt)
    out = R.out
    hout = torch.empty_like(out, device="cpu").pin_memory()

    # Each step is self-contained: its inputs go host -> device in chunks of
    # layers on a copy stream, each chunk's layers run as soon as it has
    # landed (one pkv_paged_decode_append_attention_layers call per chunk),
    # and each chunk's outputs go back on a second copy stream; the step ends
    # when its last output is on the host.  The next step's copies start after
    # this step's compute (no prefetch across steps).  Small first and last
    # chunks shorten the pipeline's fill (first copy in) and drain (last copy
    # out).  Headline: pagedkv.graphs.DecodeStepGraph, which holds all of that
    # in one CUDA graph (per step: the host metadata, one copy, one replay).
    # Beside it, the same pipeline issued from Python
    # (PagedKVCache.prepare_step + forward_layers per chunk).
    from pagedkv.graphs import DecodeStepGraph

    from pagedkv.graphs import event_chunks

    sizes = [int(x) for x in args.e2e_chunks.split(",")] if args.e2e_chunks else None
    if sizes is not None and sum(sizes) != L:
        sizes = [L]
    seqs_all = [(i, 1) for i in range(B)]
    runner = DecodeStepGraph(kv, hqkv, hout, scale, chunks=sizes, max_blocks_per_seq=int(nblk.max()))
    # the Python-issued pipeline waits on copy events: event_chunks' sizes
    sizes = sizes or event_chunks(L)

    def e2e_step():
        runner.run(seqs_all)

    bounds = [sum(sizes[:i]) for i in range(len(sizes) + 1)]
    chunks = [(bounds[c], bounds[c + 1]) for c in range(len(sizes))]
    views = [(dqkv[a:b, :, :14], dqkv[a:b, :, 14:16], dqkv[a:b, :, 16:18], out[a:b]) for a, b in chunks]
    h2d_s, d2h_s = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in chunks]
    ev_out = [torch.cuda.Event() for _ in chunks]

    def e2e_step_eager():
        cur = torch.cuda.current_stream(dev)
        meta = kv.prepare_step(seqs_all)
        h2d_s.wait_stream(cur)
        with torch.cuda.stream(h2d_s):
            for c, (a, b) in enumerate(chunks):
                dqkv[a:b].copy_(hqkv[a:b], non_blocking=True)
                ev_in[c].record(h2d_s)
        for c, (a, b) in enumerate(chunks):
            cur.wait_event(ev_in[c])
            q_, k_, v_, o_ = views[c]
            kv.forward_layers(a, q_, k_, v_, meta, scale, out=o_, advance=False)
            ev_out[c].record(cur)
            d2h_s.wait_event(ev_out[c])
            with torch.cuda.stream(d2h_s):
                hout[a:b].copy_(out[a:b], non_blocking=True)
        cur.wait_stream(d2h_s)

    def time_windows(fn):
        """Host-driven steps move with host hiccups on a shared machine: time
        them in windows of steps back to back (device events), median window;
        also the host's own time per step."""
        for _ in range(10):
            fn()
        torch.cuda.synchronize()
        barrier()
        n_win = max(1, args.e2e_windows)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(n_win + 1)]
        host_s = []
        evs[0].record()
        for w in range(n_win):
            h0 = time.perf_counter()
            for _ in range(args.e2e_steps):
                fn()
            host_s.append(time.perf_counter() - h0)
            evs[w + 1].record()
        torch.cuda.synchronize()
        barrier()
        win = [evs[w].elapsed_time(evs[w + 1]) / args.e2e_steps for w in range(n_win)]
        return win, 1e3 * statistics.median(host_s) / args.e2e_steps

    win_ms, host_ms_local = time_windows(e2e_step)
    eager_win, eager_host = time_windows(e2e_step_eager)
    ops.check_flags(R.err, "bench e2e")
    n_win = len(win_ms)
    e2e_ms_local = statistics.median(win_ms)
    e2e_ms = W.max_over_ranks(e2e_ms_local)
    eager_ms = W.max_over_ranks(statistics.median(eager_win))
    per_rank["e2e_ms_local"] = [round(x, 5) for x in W.gather_over_ranks(e2e_ms_local)]
    per_rank["e2e_host_enqueue_ms_local"] = [round(x, 5) for x in W.gather_over_ranks(host_ms_local)]
    per_rank["e2e_eager_host_enqueue_ms_local"] = [round(x, 5) for x in W.gather_over_ranks(eager_host)]
    meta_bytes = 4 * (B * runner.W + 2 * B + 1) + 8 * B
    h2d = hqkv.numel() * 2 + meta_bytes
    d2h = hout.numel() * 2
    e2e_chunks, e2e_ready = [b - a for a, b in runner.bounds], runner.gated
    e2e_copies = [b - a for a, b in runner.copy_bounds]
    del kv, dqkv, hqkv, hout, runner

    # ---- the same job under strong scaling (BASELINE config 3's wording:
    # 256 sequences in total, dealt over the N GPUs), same process
    strong = None
    if not args.strong:
        if world == 1:
            strong = {"same_as_weak": True}
        else:
            S = DecodeRun(args.batch, True, rank, world, L, dev, per_layer_calls=args.per_layer_calls)
            for _ in range(args.warmup):
                S.step()
            torch.cuda.synchronize()
            s_ms_local = S.timed(S.step, args.steps, barrier)
            s_dec_local = S.timed(S.calls, args.steps, barrier) / L
            ops.check_flags(S.err, "bench strong pass")
            s_ms = W.max_over_ranks(s_ms_local)
            s_dec = W.max_over_ranks(s_dec_local)
            s_bytes = W.sum_over_ranks(S.step_bytes)
            s_seqs = W.sum_over_ranks(S.B)
            s_call_bytes = W.gather_over_ranks(S.dec_bytes + S.app_bytes)
            s_dec_list = W.gather_over_ranks(s_dec_local)
            peak_s, _ = peaks()
            strong = {
                "global_batch": int(s_seqs), "ms_per_step": round(s_ms, 4),
                "value": round(s_bytes / (s_ms * 1e-3) / 1e9, 2), "unit": UNIT,
                "decode_tok_s": round(s_seqs / (s_ms * 1e-3), 1),
                "decode_call_ms": round(s_dec, 5),
                "decode_call_frac_per_rank": [round(b / (t * 1e-3) / 1e9 / peak_s, 4)
                                              for b, t in zip(s_call_bytes, s_dec_list)],
                "per_rank": {"sum_ctx": [int(x) for x in W.gather_over_ranks(int(S.ctx.sum()))],
                             "seqs": [int(x) for x in W.gather_over_ranks(S.B)],
                             "ms_local": [round(x, 5) for x in W.gather_over_ranks(s_ms_local)],
                             "decode_call_ms_local": [round(x, 6) for x in s_dec_list]},
            }
            del S

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return

    peak, peak_kind = peaks()
    ctx0 = W.shard_contexts(args.batch, 0, world, strong=args.strong)
    call_bytes = W.decode_bytes(ctx0) + W.append_bytes(len(ctx0))
    dec_ms0 = per_rank["decode_call_ms_local"][0]
    achieved = call_bytes / (dec_ms0 * 1e-3) / 1e9
    clocks = sampler.summary(t_wall0, t_wall1) if sampler else None
    mean_ms = statistics.mean(per_rank["ms_local"])
    line = {
        "metric": METRIC,
        "value": round(total_bytes / (ms * 1e-3) / 1e9, 2),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms, 4),
        "higher_is_better": True,
        "scaling": "strong" if args.strong else "weak",
        "vs_baseline": None,
        "dtype": "f16",
        "data": "synthetic (seeded normal K/V/Q; lognormal contexts); no weights involved",
        "config": {"workload": WORKLOAD, "global_batch": int(total_seqs), "layers": L,
                   "sum_ctx_rank0": int(ctx.sum()), "pool_blocks_rank0": rank0_pool_blocks(args, world),
                   "parallelism": f"sequence-sharded x{world}, no collective on the data path",
                   "l2": "inputs larger than L2: ~155 MB of KV per layer, 24 distinct layer pools per step"},
        "decode_tok_s": round(total_seqs / (ms * 1e-3), 1),
        "hbm_frac_step": round(total_bytes / world / (ms * 1e-3) / 1e9 / peak, 4),
        "per_rank": per_rank,
        "max_over_ranks_vs_mean": round(ms / mean_ms, 4),
        "roofline": {"kernel": "paged_decode_kernel<half>", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic_from_profiles(), "bytes_per_launch": call_bytes,
                     "avg_launch_ms": round(dec_ms0, 5),
                     "timing": ("rank 0; CUDA events around --steps rounds of the 24 fused append+decode "
                                "calls back to back (the step without its schedule build), / (steps x 24); "
                                "a call is the decode kernel plus its split-K merge") if args.per_layer_calls
                               else ("rank 0; CUDA events around --steps rounds of the step's multi-layer call "
                                     "(24 chained decode kernels, then one merge launch for all layers; the "
                                     "step without its schedule build), / (steps x 24)")},
        "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": UNIT,
                "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": round(e2e_ms, 4),
                "api": "pagedkv.graphs.DecodeStepGraph.run: PagedKVCache.step_arrays into pinned staging, "
                       "one metadata copy, one CUDA-graph replay (per-chunk H2D of q|k|v then a ready word, "
                       "the decode schedule, one pkv_paged_decode_append_attention_layers call per chunk "
                       "whose kernels wait on the chunk's ready word, per-chunk D2H)",
                "chunks": e2e_chunks,
                "input_copies_layers": e2e_copies,
                "ready_words": e2e_ready,
                "timing": f"median of {n_win} windows of {args.e2e_steps} steps back to back, max over ranks",
                "windows_ms_per_step": [round(x, 4) for x in win_ms],
                "copies": f"pinned host buffers; per step: metadata, then q|k|v of {L} layers H2D in "
                          "the chunks above (one copy each) on a copy stream, outputs D2H per chunk "
                          "on a second copy stream, overlapped with the step's own compute; the step ends "
                          "when its outputs are on the host",
                "eager": {"ms_per_step": round(eager_ms, 4),
                          "value": round(total_bytes / (eager_ms * 1e-3) / 1e9, 2),
                          "api": "the same pipeline issued from Python: PagedKVCache.prepare_step + "
                                 "forward_layers per chunk (host-bound), chunks waiting on copy events",
                          "chunks": sizes},
                "host_cpus_per_rank": len(cpus),
                "host_cpus_near_gpu": "NVML CPU affinity of the rank's GPU" if cpus != all_cpus else None},
        "strong": strong,
        # per timed step: the schedule, then (decode, merge) per layer, or the
        # chained decodes and one merge launch
        "gpu_launches": ((2 * L + 1) if args.per_layer_calls else (L + 2)) * args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline and world == 1:
        os.sched_setaffinity(0, all_cpus)  # the CPU baseline runs on every core the job may use
        gbs, cores, sample, _, _ = cpu_sample(args.cpu_seconds)
        line["cpu_baseline"] = {"value": round(gbs, 3), "unit": UNIT, "cores": cores,
                                "kind": "port", "sample": sample}
    print(json.dumps(line), flush=True)


def rank0_pool_blocks(args, world: int) -> int:
    """Pool blocks of rank 0 (1.1x its needed blocks)."""
    from pagedkv import workloads as W

    ctx0 = W.shard_contexts(args.batch, 0, world, strong=args.strong)
    return int(math.ceil(1.1 * ((ctx0 + 15) // 16).sum()))


def peaks_tflops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops_sustained"]), "measured (sustained)"
    except (OSError, KeyError, ValueError):
        return 1400.0, "fallback (sustained)"


def run_prefill(args):
    """BASELINE config 4 per GPU: 16 sequences x 512-token chunks over a
    48-token shared prefix + private prior U[0, 4096]; per layer one append of
    the 8192 chunk tokens and one chunked-prefill launch (tcgen05 kernel)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from pagedkv import BlockManager, ops
    from pagedkv import workloads as W

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    L, scale, dt = args.layers, 0.125, torch.float16
    prior, chunk = W.config4_layout(seed=4 + rank)
    B, T = len(prior), int(chunk.sum())
    need = int(((prior + chunk + 15) // 16).sum())
    nb = int(need * 1.1) + 8
    tabs_np = W.prefill_tables(prior, chunk, 48, nb, seed=200 + rank)
    g = torch.Generator(device=dev)
    g.manual_seed(4321 + rank)
    fp8 = args.kv_fp8
    mgr = BlockManager(nb, 16, L, 2, 64, device=dev, dtype=torch.float8_e4m3fn if fp8 else dt)
    if fp8:  # every slot quantised from N(0,1) rows
        fill = torch.empty((nb * 16, 2, 64), device=dev, dtype=dt)
        all_slots = torch.arange(nb * 16, device=dev, dtype=torch.int64)
        for layer in range(L):
            fill.normal_(generator=g)
            ops.reshape_and_cache_fp8(fill, fill, mgr.k_pool[layer], mgr.v_pool[layer],
                                      mgr.k_scale[layer], mgr.v_scale[layer], all_slots)
        del fill
    else:
        for layer in range(L):
            mgr.k_pool[layer].normal_(generator=g)
            mgr.v_pool[layer].normal_(generator=g)
    q = torch.randn((L, T, 14, 64), generator=g, device=dev, dtype=dt)
    kn = torch.randn((L, T, 2, 64), generator=g, device=dev, dtype=dt)
    vn = torch.randn((L, T, 2, 64), generator=g, device=dev, dtype=dt)
    out = torch.empty_like(q)
    slots = []
    for i in range(B):
        pos = np.arange(prior[i], prior[i] + chunk[i])
        slots.append(tabs_np[i, pos // 16].astype(np.int64) * 16 + pos % 16)
    slots = torch.from_numpy(np.concatenate(slots)).to(dev)
    tabs = torch.from_numpy(tabs_np).to(dev)
    qsl = torch.from_numpy(np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)).to(dev)
    prior_d = torch.from_numpy(prior.astype(np.int32)).to(dev)
    err = ops.new_error_flags(dev)
    if fp8:
        # quantising append, then the tensor-core fp8 prefill: the pass that
        # writes the visible blocks into the 16-bit scratch is timed with it
        scratch = (torch.empty(ops.prefill_fp8_scratch_bytes(B, tabs.shape[1], 2, 64),
                               dtype=torch.uint8, device=dev)
                   if args.fp8_prefill == "scratch" else None)  # None: the scratch-free entry
        appends = [ops.bind_reshape_and_cache_fp8(kn[l], vn[l], mgr.k_pool[l], mgr.v_pool[l],
                                                  mgr.k_scale[l], mgr.v_scale[l], slots, err)
                   for l in range(L)]
        prefills = [ops.bind_paged_prefill_attention_fp8(q[l], mgr.k_pool[l], mgr.v_pool[l],
                                                         mgr.k_scale[l], mgr.v_scale[l], tabs, qsl,
                                                         prior_d, int(chunk.max()), scale, out[l],
                                                         scratch, err)
                    for l in range(L)]
    else:
        appends = [ops.bind_reshape_and_cache(kn[l], vn[l], mgr.k_pool[l], mgr.v_pool[l], slots, err)
                   for l in range(L)]
        prefills = [ops.bind_paged_prefill_attention(q[l], mgr.k_pool[l], mgr.v_pool[l], tabs, qsl,
                                                     prior_d, int(chunk.max()), scale, out[l], err)
                    for l in range(L)]
    flops = W.prefill_flops(prior, chunk)

    def step(ev=None):
        for layer in range(L):
            appends[layer]()
            if ev is not None:
                ev[layer][0].record()
            prefills[layer]()
            if ev is not None:
                ev[layer][1].record()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.check_flags(err, "prefill warm-up")
    if args.profile_steps:
        for _ in range(args.profile_steps):
            step()
        torch.cuda.synchronize()
        if world > 1:
            dist.destroy_process_group()
        return
    every = 10
    ev_steps = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                 for _ in range(L)] for _ in range((args.steps + every - 1) // every)]
    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    time.sleep(0.3 if sampler else 0)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    t0 = time.time()
    start.record()
    for i in range(args.steps):
        step(ev_steps[i // every] if i % every == 0 else None)
    end.record()
    torch.cuda.synchronize()
    t1 = time.time()
    barrier()
    if sampler:
        sampler.stop()
    ops.check_flags(err, "prefill timed region")
    ms = W.max_over_ranks(start.elapsed_time(end) / args.steps)
    ker = [a.elapsed_time(b) for evs in ev_steps for (a, b) in evs]
    ker_ms = W.max_over_ranks(sum(ker) / len(ker))
    total_flops = W.sum_over_ranks(L * flops)
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    peak, kind = peaks_tflops()
    achieved = flops / (ker_ms * 1e-3) / 1e12
    line = {
        "metric": "paged chunked-prefill attention TFLOP/s (config 4)" + (" over fp8 e4m3 KV" if fp8 else ""),
        "value": round(total_flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic (seeded normal Q/K/V)",
        "config": {"workload": "config4: 16 seqs x 512-token chunk over 48-token shared prefix + "
                               "private prior U[0,4096], 24 layers x (append + prefill), 14q/2kv, d64",
                   "sum_prior": int(prior.sum()), "flops_per_layer": flops, "layers": L,
                   **({"fp8_prefill": args.fp8_prefill} if fp8 else {})},
        "roofline": {"kernel": "paged_prefill_tc_kernel<half>" + (
                         (" + fp8 scratch pass" if args.fp8_prefill == "scratch"
                          else " (fp8 tiles converted in kernel)") if fp8 else ""),
                     "bound": "tensor",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "peak_kind": kind,
                     "avg_launch_ms": round(ker_ms, 5)},
        "gpu_launches": (3 if fp8 and args.fp8_prefill == "scratch" else 2) * L * args.steps,
        "clocks": sampler.summary(t0, t1) if sampler else None,
    }
    print(json.dumps(line), flush=True)


def run_e2e(args):
    """continuous-batching greedy decoding of a random-init
    Qwen2.5-0.5B-shaped model (fp16) with the paged-KV path, fed by Poisson
    arrivals of two-turn conversations: prompts of random token ids, 64-512
    tokens sharing a 48-token prefix, 128 output tokens per turn; turn two
    (prompt + answer + 16-64 new tokens) arrives when turn one finishes."""
    import numpy as np
    import torch

    from pagedkv import BlockManager
    from pagedkv.model import PagedQwen2Model, Qwen2Config, random_weights
    from pagedkv.engine import Engine, Seq

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    rank = int(os.environ.get("RANK", "0"))
    cfg = Qwen2Config()
    model = PagedQwen2Model(cfg, random_weights(cfg, seed=5, final_norm_scale=4.0), device="cuda",
                            dtype=torch.float16)
    rng = np.random.default_rng(50 + rank)
    V = cfg.vocab_size
    shared = rng.integers(0, V, size=48).tolist()
    n = args.conversations
    prompts = [shared + rng.integers(0, V, size=int(rng.integers(16, 465))).tolist() for _ in range(n)]
    extra = [rng.integers(0, V, size=int(rng.integers(16, 65))).tolist() for _ in range(n)]
    gaps = rng.exponential(1.0 / args.rate, size=n)
    arrivals = np.cumsum(gaps) - gaps[0]
    out_len = 128
    num_blocks = 24000  # 4.7 GB of fp16 KV for 24 layers
    mgr = BlockManager(num_blocks, 16, cfg.num_hidden_layers, 2, 64, device="cuda", dtype=torch.float16)
    eng = Engine(model, mgr, max_seqs=args.max_num_seqs, token_budget=args.max_batched_tokens,
                 prefix_reuse=True, eos_ids=(), cuda_graphs=not args.no_cuda_graphs)
    t_cap = time.perf_counter()
    if eng.run_step.cuda_graphs:  # every padded step shape, before the timed run
        eng.run_step.step_graphs().capture_all()
    t_cap = time.perf_counter() - t_cap

    def drive(n_conv, arr):
        pending = list(range(n_conv))
        reqs, turn2 = {}, {}
        t0 = time.perf_counter()
        while pending or eng.busy:
            now = time.perf_counter() - t0
            while pending and arr[pending[0]] <= now:
                i = pending.pop(0)
                reqs[i] = eng.submit(Seq(i, list(prompts[i]), limit=out_len))
            if not eng.busy:
                time.sleep(min(1e-3, max(0.0, arr[pending[0]] - now)))
                continue
            eng.step()
            for i, r in list(reqs.items()):
                if r.finish and i not in turn2:
                    turn2[i] = eng.submit(Seq(n_conv + i, r.tokens + extra[i], limit=out_len))
        torch.cuda.synchronize()
        return time.perf_counter() - t0, list(reqs.values()) + list(turn2.values())

    drive(min(4, n), np.zeros(n))  # warm-up: rope tables, TMA descriptors, allocator
    eng.index.clear()   # forget the warm-up prefixes
    for k in list(eng.counts):
        eng.counts[k] = 0
    replays0 = eng.graphs.replays if eng.graphs is not None else 0
    wall, done = drive(n, arrivals)
    replays = (eng.graphs.replays if eng.graphs is not None else 0) - replays0
    mgr.check_errors()
    steps_timed = eng.counts["steps"]
    sched_metrics = dict(eng.counts)
    # attention share, in a separate short run (events around the attention
    # part of every layer would perturb the timed run): fused RoPE + append +
    # attention launches over the whole model step, GPU time
    eng.index.clear()
    model.timing = []
    drive(min(16, n), np.zeros(n))
    torch.cuda.synchronize()
    step_ms = sum(a.elapsed_time(b) for (a, b), _ in model.timing)
    attn_ms = sum(a.elapsed_time(b) for _, layers in model.timing for a, b in layers)
    model.timing = None
    gen = sum(len(r.generated) for r in done)
    ttft = [r.t_first - r.t_arrive for r in done]
    itl = [(r.t_done - r.t_first) / max(1, len(r.generated) - 1) for r in done]
    pct = lambda xs, q: round(1e3 * float(np.percentile(xs, q)), 2)  # noqa: E731
    line = {
        "metric": "end-to-end continuous-batching decode tok/s (config 5)",
        "value": round(gen / wall, 1), "unit": "tok/s", "n_gpus": 1, "steps": steps_timed,
        "warmup": 1, "ms_per_step": round(1e3 * wall / max(1, steps_timed), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic: random-init Qwen2.5-0.5B-shaped weights (seed 5), random token-id prompts",
        "config": {"workload": "config5: Poisson arrivals of 2-turn conversations, prompts 64-512 "
                               "tokens with a shared 48-token prefix, 128 greedy output tokens/turn",
                   "conversations": n, "rate_per_s": args.rate, "max_num_seqs": args.max_num_seqs,
                   "max_batched_tokens": args.max_batched_tokens, "num_blocks": num_blocks,
                   "cuda_graphs": eng.run_step.cuda_graphs},
        "cuda_graphs": {"steps_replayed": replays, "steps": steps_timed,
                        "shapes": len(eng.graphs.graphs) if eng.graphs is not None else 0,
                        "capture_s": round(t_cap, 3)},
        "generated_tokens": gen, "wall_s": round(wall, 3),
        "ttft_ms": {"p50": pct(ttft, 50), "p99": pct(ttft, 99)},
        "itl_ms": {"p50": pct(itl, 50), "p99": pct(itl, 99)},
        "engine": sched_metrics,
        "attention_share": {"value": round(attn_ms / step_ms, 4) if step_ms else None,
                            "what": "GPU time of fused RoPE+append and the attention launches / GPU time "
                                    "of the model step, CUDA events, separate run of 16 conversations"},
    }
    print(json.dumps(line), flush=True)


def run_decode_fp8(args):
    """The config-3 decode step (same contexts, tables, 24 layers) over fp8
    e4m3 pools with per-(token, KV head) fp32 scales: per layer the fp8 append
    of the step's token (pkv_reshape_and_cache_fp8) and the fp8 decode.  One
    GPU; fp16 q / out."""
    import numpy as np
    import torch

    from pagedkv import BlockManager, ops
    from pagedkv import workloads as W

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    L, scale, dt = args.layers, 0.125, torch.float16
    ctx = W.shard_contexts(args.batch, 0, 1)
    B = len(ctx)
    nblk = (ctx + 15) // 16
    nb = int(math.ceil(1.1 * nblk.sum()))
    tabs_np = W.make_tables(ctx, nb, seed=100)
    g = torch.Generator(device=dev)
    g.manual_seed(1234)
    mgr = BlockManager(nb, 16, L, 2, 64, device=dev, dtype=torch.float8_e4m3fn)
    err = ops.new_error_flags(dev)
    all_slots = torch.arange(nb * 16, device=dev, dtype=torch.int64)
    fill = torch.empty((nb * 16, 2, 64), device=dev, dtype=dt)
    for layer in range(L):  # every slot quantised from N(0,1) rows
        fill.normal_(generator=g)
        ops.reshape_and_cache_fp8(fill, fill, mgr.k_pool[layer], mgr.v_pool[layer], mgr.k_scale[layer],
                                  mgr.v_scale[layer], all_slots, err)
    del fill
    q = torch.randn((L, B, 14, 64), generator=g, device=dev, dtype=dt)
    kn = torch.randn((L, B, 2, 64), generator=g, device=dev, dtype=dt)
    vn = torch.randn((L, B, 2, 64), generator=g, device=dev, dtype=dt)
    out = torch.empty_like(q)
    tabs = torch.from_numpy(tabs_np).to(dev)
    ctx_d = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    # per step: the schedule, then the layers' decodes, in which the decode
    # kernel quantises the step's new token into the fp8 pools itself: one
    # multi-layer call whose layers chain (a split-K set per layer), or with
    # --per-layer-calls one call (decode + merge) per layer
    sched = ops.new_decode_schedule(B, tabs.shape[1], dev)
    launches = [ops.bind_decode_schedule(sched, tabs, ctx_d, nb, 14, 2, 64, dt, fp8=True, err=err)]
    if args.per_layer_calls:
        ws = ops.new_decode_workspace(B, 14, 64, dev)
        for l in range(L):
            launches.append(ops.bind_paged_decode_append_attention_fp8(
                q[l], kn[l], vn[l], mgr.k_pool[l], mgr.v_pool[l], mgr.k_scale[l], mgr.v_scale[l], tabs,
                ctx_d, scale, ws, out[l], err, schedule=sched))
    else:
        ws = ops.new_decode_workspace(B, 14, 64, dev, layers=L)
        plan = ops.DecodeAppendFp8LayersPlan(tabs, ctx_d, scale, ws, err, schedule=sched)
        launches.append(lambda: plan(q, kn, vn, mgr.k_cache, mgr.v_cache, mgr.k_scale_cache,
                                     mgr.v_scale_cache, out))
    tot = int(ctx.sum())
    dec_bytes = (tot * 2 * 64 * 2 + tot * 2 * 2 * 4 + B * 14 * 64 * 2 * 2 + int(nblk.sum()) * 4 + B * 4)
    app_bytes = B * (2 * 2 * 64 * 2 + 2 * 2 * 64 + 2 * 2 * 4 + 8)
    step_bytes = L * (dec_bytes + app_bytes)

    def step():
        for f in launches:
            f()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    ops.check_flags(err, "fp8 warm-up")
    sampler = ClockSampler([0])
    time.sleep(0.3)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    t0 = time.time()
    start.record()
    for _ in range(args.steps):
        step()
    end.record()
    torch.cuda.synchronize()
    t1 = time.time()
    sampler.stop()
    ops.check_flags(err, "fp8 timed region")
    ms = start.elapsed_time(end) / args.steps
    peak, kind = peaks()
    line = {
        "metric": "paged decode attn KV GB/s and decode tok/s with fp8 e4m3 KV (config-3 shape)",
        "value": round(step_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s", "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "dtype": "fp8 e4m3 KV (fp32 row scales), f16 q/out",
        "data": "synthetic (seeded normal rows quantised on the device; lognormal contexts)",
        "config": {"workload": "config3 shape: B=256, ctx lognormal(1024, 0.5) in [16,8192], 24 layers x "
                               "(fp8 decode with the fused quantising append), 14q/2kv, d64", "sum_ctx": tot,
                   "bytes_per_token": 2 * 64 * 2 + 2 * 2 * 4},
        "decode_tok_s": round(B / (ms * 1e-3), 1),
        "hbm_frac_step": round(step_bytes / (ms * 1e-3) / 1e9 / peak, 4), "peak": peak, "peak_kind": kind,
        # schedule + (decode with fused append, merge) per layer, or the
        # chained decodes and one merge launch
        "gpu_launches": ((2 * L + 1) if args.per_layer_calls else (L + 2)) * args.steps,
        "calls": "one call per layer" if args.per_layer_calls else "one multi-layer call, layers chained",
        "clocks": sampler.summary(t0, t1),
    }
    print(json.dumps(line), flush=True)


def run_cache_ops(args):
    """reshape_and_cache and copy_blocks at batches large enough to measure HBM
    bandwidth (one GPU).  Append: T tokens of K and V per launch scattered
    to a random permutation of pool slots, one pool per layer (the working
    set of the L layers exceeds L2).  Copy: copy_blocks of P (src, dst) block
    pairs over all L layers in one launch, src and dst disjoint and random
    (a COW fork / preemption-sized batch).  GB/s counts algorithmic bytes:
    every K/V byte read once and written once, plus the slot / pair indices."""
    import numpy as np
    import torch

    from pagedkv import ops
    from pagedkv import workloads as W

    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    L, dt = args.layers, torch.float16
    g = torch.Generator(device=dev)
    g.manual_seed(99)
    rng = np.random.default_rng(99)
    err = ops.new_error_flags(dev)
    peak, kind = peaks()

    def time_calls(calls, reps):
        """Device time per launch of back-to-back launches: each round of
        len(calls) launches is queued behind a short GPU sleep, so the host's
        launch cost does not open gaps between them; one event pair per round."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(reps)]
        for _ in range(args.warmup):
            for c in calls:
                c()
        torch.cuda.synchronize()
        for a, b in evs:
            torch.cuda._sleep(4_000_000)  # ~2 ms of GPU time covers the queueing of the round
            a.record()
            for c in calls:
                c()
            b.record()
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b) for a, b in evs) / (len(evs) * len(calls))

    results = []
    for T in args.append_tokens:
        nb = (T + 15) // 16 + 16
        kp = torch.empty((L, nb, 16, 2, 64), device=dev, dtype=dt)
        vp = torch.empty_like(kp)
        kn = torch.randn((L, T, 2, 64), generator=g, device=dev, dtype=dt)
        vn = torch.randn_like(kn)
        slots = torch.from_numpy(rng.permutation(nb * 16)[:T].astype(np.int64)).to(dev)
        calls = [ops.bind_reshape_and_cache(kn[l], vn[l], kp[l], vp[l], slots, err) for l in range(L)]
        ms = time_calls(calls, max(3, args.steps // L))
        nbytes = W.append_bytes(T)
        results.append({"kernel": "pkv::reshape_and_cache_vec16", "tokens": T, "bytes_per_launch": nbytes,
                        "us": round(ms * 1e3, 3), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                        "frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)})
        # fused RoPE + append of the same tokens from the [T, 18 * 64] projection rows
        from pagedkv.model import Rope

        qkv = torch.randn((L, T, 18 * 64), generator=g, device=dev, dtype=dt)
        pos = torch.from_numpy(rng.integers(0, 8192, size=T).astype(np.int64)).to(dev)
        cos, sin = Rope(64, 1e6, dev, dt).tables(8192)
        qo = torch.empty((L, T, 14, 64), device=dev, dtype=dt)
        rcalls = [lambda l=l: ops.rope_reshape_and_cache(qkv[l], pos, cos, sin, kp[l], vp[l], slots,
                                                         q_out=qo[l], err=err) for l in range(L)]
        ms = time_calls(rcalls, max(3, args.steps // L))
        # per token: the projection row read, rotated q written, k and v rows
        # written, position and slot; the cos / sin tables (2 MB) once
        nbytes = T * (18 * 64 * 2 + 14 * 64 * 2 + 2 * 2 * 64 * 2 + 16) + 2 * cos.numel() * cos.element_size()
        results.append({"kernel": "pkv::rope_reshape_and_cache_vec_kernel<half>", "tokens": T,
                        "bytes_per_launch": nbytes, "us": round(ms * 1e3, 3),
                        "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                        "frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)})
        del kp, vp, kn, vn, qkv, qo
    P = args.copy_pairs
    nb = 2 * P + 16
    kc = torch.randn((L, nb, 16, 2, 64), generator=g, device=dev, dtype=dt)
    vc = torch.randn_like(kc)
    perm = rng.permutation(nb)[:2 * P].astype(np.int32)
    pairs = torch.from_numpy(np.stack([perm[:P], perm[P:]], axis=1).copy()).to(dev)
    ms = time_calls([lambda: ops.copy_blocks(kc, vc, pairs, err)], max(3, args.steps // 50))
    block_bytes = 16 * 2 * 64 * 2
    nbytes = 2 * 2 * L * P * block_bytes + P * 8
    results.append({"kernel": "pkv::copy_blocks_vec16", "pairs": P, "layers": L, "bytes_per_launch": nbytes,
                    "us": round(ms * 1e3, 3), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                    "frac": round(nbytes / (ms * 1e-3) / 1e9 / peak, 4)})
    ops.check_flags(err, "cache_ops")
    line = {"metric": "KV append (reshape_and_cache) and copy_blocks HBM GB/s", "value": results[-2]["gbs"],
            "unit": "GB/s", "n_gpus": 1, "higher_is_better": True, "dtype": "f16",
            "data": "synthetic (seeded normal K/V, random slots and pairs)",
            "config": {"workload": "cache_ops: append T tokens/launch x 24 layer pools; copy_blocks P pairs x 24 layers",
                       "append_tokens": args.append_tokens, "copy_pairs": P, "layers": L},
            "peak": peak, "peak_kind": kind, "kernels": results, "gpu_launches": None}
    print(json.dumps(line), flush=True)


def run_migrate(args):
    """KV block migration between rank pairs (0 -> 1, 2 -> 3, ...) over NVLink.
    Kernel: one pkv_copy_blocks_peer launch moving P blocks x L layers of K
    and V (fp16) from the source's pool to fixed destination blocks of the
    peer's pool, timed with CUDA events on the launching rank.  push: the
    source launches it (its stores cross NVLink); pull: the destination does
    (its loads cross).  GB/s = bytes crossing the link / kernel time.  Then
    the full protocol (allocation, host handshakes, copy, synchronisation) for
    one 1,024-token sequence (64 blocks), host wall time per migration."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from pagedkv import BlockManager, ops
    from pagedkv.migration import PeerPools, migrate_blocks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world < 2:
        print(json.dumps({"metric": "KV block migration GB/s over NVLink", "unavailable":
                          "needs 2 ranks: torchrun --nproc-per-node 2 bench.py --workload migrate"}))
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    L, P = args.layers, args.migrate_blocks
    nb = P + 256
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    mgr = BlockManager(nb, 16, L, 2, 64, device=dev, dtype=torch.float16)
    mgr.k_cache.normal_(generator=g)
    mgr.v_cache.normal_(generator=g)
    src_side = rank % 2 == 0
    peer = rank + 1 if src_side else rank - 1
    rng = np.random.default_rng(5)
    perm_src = rng.permutation(nb)[:P].astype(np.int32)
    perm_dst = rng.permutation(nb)[:P].astype(np.int32)
    pairs = torch.from_numpy(np.stack([perm_src, perm_dst], axis=1).copy()).to(dev)
    nbytes = 2 * L * P * mgr.block_bytes
    res = {}
    for mode in ("push", "pull"):
        peers = PeerPools(mgr, mode=mode)
        launching = src_side == (mode == "push")
        ms = 0.0
        if launching:
            src = peers.refs[rank if src_side else peer]
            dst = peers.refs[peer if src_side else rank]

            def copy():
                ops.copy_blocks_peer(dst.k, dst.v, dst.layer_stride, dst.num_blocks, src.k, src.v,
                                     src.layer_stride, src.num_blocks, L, pairs, dst.block_bytes,
                                     mgr.err)

            for _ in range(args.warmup):
                copy()
            torch.cuda.synchronize()
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in range(args.steps)]
            for a, b in evs:
                a.record()
                copy()
                b.record()
            torch.cuda.synchronize()
            ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)
            ops.check_flags(mgr.err, "migrate bench")
        dist.barrier(group=peers.host_group)
        t = torch.tensor([ms])
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=peers.host_group)
        res[mode] = {"us": round(float(t) * 1e3, 2), "gbs": round(nbytes / (float(t) * 1e-3) / 1e9, 1)}
        # full protocol for a 1,024-token sequence (64 blocks), host wall time
        seq_blocks = list(range(64))
        reps = 20
        dist.barrier(group=peers.host_group)
        t0 = time.perf_counter()
        for _ in range(reps):
            ids = migrate_blocks(peers, rank if src_side else peer, peer if src_side else rank,
                                 seq_blocks if src_side else None)
            if not src_side:
                for b in ids:
                    mgr.decref(b)
        res[mode]["protocol_ms_per_seq"] = round((time.perf_counter() - t0) / reps * 1e3, 3)
        peers.close()
    link_peak = 770.0  # measured peer copy per direction on this pool (GB/s)
    if rank == 0:
        best = max(res.values(), key=lambda r: r["gbs"])
        print(json.dumps({
            "metric": "KV block migration GB/s over NVLink (one copy launch, rank pairs)",
            "value": best["gbs"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "dtype": "f16",
            "data": "synthetic (seeded normal K/V pools, random block pairs)",
            "config": {"workload": f"migrate: {P} blocks x {L} layers x K,V per launch "
                                   f"({nbytes / 1e6:.1f} MB), pairs of ranks 0->1, 2->3, ...",
                       "blocks": P, "layers": L},
            "modes": res,
            "roofline": {"bound": "nvlink", "achieved": best["gbs"], "peak": link_peak,
                         "unit": "GB/s", "frac": round(best["gbs"] / link_peak, 4)},
            "gpu_launches": args.steps}), flush=True)
    dist.destroy_process_group()


def run_model_step(args):
    """GPU time of config 5's model step as the engine replays it: the
    random-init Qwen2.5-0.5B-shaped fp16 model's CUDA graphs
    (pagedkv.graphs.StepGraphs) for a decode-only step of 64 sequences
    (contexts uniform in [300, 900)) and for a mixed step of those 64 decodes
    plus a 128-token chunk after a 300-token prior context.  CUDA events
    around `--steps` replays each; the step's inputs are already on the
    device (the metadata copy of a real step is not in the timed region).
    With --profile-steps N, N replays of the decode-only graph run inside an
    NVTX range "model_step" (for ncu --nvtx-include) and nothing is timed."""
    import numpy as np
    import torch

    from pagedkv import BlockManager, PagedKVCache
    from pagedkv.graphs import StepGraphs
    from pagedkv.model import PagedQwen2Model, Qwen2Config, SequenceForwardInfo, random_weights

    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    cfg = Qwen2Config()
    model = PagedQwen2Model(cfg, random_weights(cfg, seed=5, final_norm_scale=4.0), device="cuda",
                            dtype=torch.float16)
    mgr = BlockManager(8000, 16, cfg.num_hidden_layers, 2, 64, device="cuda", dtype=torch.float16)
    kv = PagedKVCache(mgr)
    rng = np.random.default_rng(0)
    B, chunk = 64, 128
    lens = rng.integers(300, 900, size=B).tolist() + [300]
    for s, n in enumerate(lens):
        kv.add_sequence(s, [mgr.allocate() for _ in range((n + chunk + 16) // 16 + 1)], n)
    runner = StepGraphs(model, kv, max_batch=B, max_tokens=512)

    def infos(mixed):
        out = [SequenceForwardInfo(s, s, 1, np.array([lens[s]])) for s in range(B)]
        if mixed:
            out.append(SequenceForwardInfo(B, B, chunk, np.arange(lens[B], lens[B] + chunk)))
        return out

    res = {}
    for mixed in (False, True):
        inf = infos(mixed)
        ids = torch.tensor(rng.integers(0, cfg.vocab_size, size=B + (chunk if mixed else 0)),
                           device="cuda")
        runner.forward(ids, inf)  # captures the shape and stages the step's metadata
        for s in range(B + 1):    # forward advanced the lengths: restore them
            kv._len[s] = lens[s]
        g = runner.graphs[runner.shape_of(inf)]
        for _ in range(max(3, args.warmup)):
            g.replay()
        if args.profile_steps and not mixed:
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_push("model_step")
            for _ in range(args.profile_steps):
                g.replay()
            torch.cuda.synchronize()
            torch.cuda.nvtx.range_pop()
        if args.profile_steps:
            continue
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        res["mixed" if mixed else "decode"] = {
            "shape": list(runner.shape_of(inf)), "ms_per_step": round(e0.elapsed_time(e1) / args.steps, 4)}
    mgr.check_errors()
    if args.profile_steps:
        return
    print(json.dumps({
        "metric": "config-5 model step GPU time (CUDA-graph replay)", "unit": "ms",
        "value": res["decode"]["ms_per_step"], "higher_is_better": False, "steps": args.steps,
        "data": "synthetic: random-init Qwen2.5-0.5B-shaped weights, random token ids", "dtype": "f16",
        "config": {"workload": "decode-only step of 64 sequences (contexts uniform [300, 900)); "
                               "mixed: + one 128-token chunk after 300 cached tokens"},
        "steps_by_shape": res}), flush=True)


def main():
    args = parse()
    if args.workload == "model_step":
        run_model_step(args)
        return
    if args.workload == "migrate":
        run_migrate(args)
        return
    if args.workload == "e2e" and args.impl == "ours":
        run_e2e(args)
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "cache_ops":
        run_cache_ops(args)
    elif args.workload == "decode_fp8":
        run_decode_fp8(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
