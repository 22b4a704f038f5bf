"""How the timed CPU baseline (the oracle's C port) compares with the
reference's own Python path, on the same config-3 subset and the same cores.

    REF_ROOT=/path/to/llm-inference-scheduler python oracle/compare_reference_cpu.py [seconds]

The workload is the one bench.py's `--impl reference` arm times per step: one
layer of a 32-sequence subset of config 3 (every 8th of rank 0's 256
sequences), fp16 pools scattered through seeded block tables, one new token
per sequence.  Two implementations run it on this machine's host cores:

* reference: the reference's own code, imported read-only from REF_ROOT:
  PagedKVCache.append_and_fetch (mini_engine/paged/block_manager.py:111-141)
  then Qwen2Model._attention (mini_engine/model/qwen2.py:98-128) per
  sequence, with torch.set_num_threads(all cores);
* port: oracle.reshape_and_cache + oracle.paged_attention (C, OpenMP, all
  cores), as bench.py's cpu_baseline and `--impl reference` run it.

Both are reported in the bench metric (algorithmic KV GB/s, workloads.py's
byte count) with the ratio.  This is test infrastructure: it needs the
reference, so it runs where the reference is (not on the GPU box).
"""

from __future__ import annotations

import math
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path[:0] = [HERE, os.path.join(ROOT, "llm-inference-scheduler_b200")]
import oracle  # noqa: E402
from pagedkv import workloads as W  # noqa: E402

sys.path.insert(0, os.environ.get("REF_ROOT", "/root/reference"))
from mini_engine.model.qwen2 import Qwen2Model  # noqa: E402
from mini_engine.paged.block_manager import BlockManager, PagedKVCache  # noqa: E402


class _AttnOnly:
    """What Qwen2Model._attention reads from self: the config's head counts and the scale."""

    class config:  # noqa: N801
        num_attention_heads, num_key_value_heads = 14, 2

    scale = 64 ** -0.5


def workload(n_sub: int = 32):
    ctx = W.shard_contexts(256, 0, 1)
    ctx = ctx[:: max(1, len(ctx) // n_sub)][:n_sub]
    nb = int(math.ceil(1.1 * ((ctx + 15) // 16).sum()))
    tabs = W.make_tables(ctx, nb, seed=100)
    rng = np.random.default_rng(0)
    kp = rng.standard_normal((nb, 16, 2, 64), dtype=np.float32).astype(np.float16)
    vp = rng.standard_normal((nb, 16, 2, 64), dtype=np.float32).astype(np.float16)
    B = len(ctx)
    q = rng.standard_normal((B, 14, 64), dtype=np.float32).astype(np.float16)
    kn = rng.standard_normal((B, 2, 64), dtype=np.float32).astype(np.float16)
    vn = rng.standard_normal((B, 2, 64), dtype=np.float32).astype(np.float16)
    return ctx, nb, tabs, kp, vp, q, kn, vn


def time_reference(seconds: float, threads: int):
    ctx, nb, tabs, kp, vp, q, kn, vn = workload()
    torch.set_num_threads(threads)
    mgr = BlockManager(nb, 16, 1, 2, 64, device="cpu", dtype=torch.float16)
    mgr.k_pool[0].copy_(torch.from_numpy(kp))
    mgr.v_pool[0].copy_(torch.from_numpy(vp))
    nblk = (ctx + 15) // 16
    qt, knt, vnt = (torch.from_numpy(a) for a in (q, kn, vn))
    self_ = _AttnOnly()
    reps, t0 = 0, time.perf_counter()
    while True:
        kv = PagedKVCache(mgr)  # a fresh step: every sequence appends its token at ctx - 1
        for i in range(len(ctx)):
            kv.add_sequence(i, tabs[i, :nblk[i]].tolist(), int(ctx[i]) - 1)
        for i in range(len(ctx)):
            k_all, v_all, prior = kv.append_and_fetch(0, i, knt[i:i + 1], vnt[i:i + 1])
            Qwen2Model._attention(self_, qt[i:i + 1], k_all, v_all, prior)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return W.decode_bytes(ctx) + W.append_bytes(len(ctx)), reps, el


def time_port(seconds: float, threads: int):
    ctx, nb, tabs, kp, vp, q, kn, vn = workload()
    B = len(ctx)
    pos = ctx - 1
    slots = tabs[np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16
    qsl = np.arange(B + 1, dtype=np.int32)
    prior = (ctx - 1).astype(np.int32)
    reps, t0 = 0, time.perf_counter()
    while True:
        oracle.reshape_and_cache(kp, vp, kn, vn, slots, "f16")
        oracle.paged_attention(q, kp, vp, tabs, qsl, prior, "f16", threads=threads)
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return W.decode_bytes(ctx) + W.append_bytes(B), reps, el


def main():
    seconds = float(sys.argv[1]) if len(sys.argv) > 1 else 10.0
    threads = len(os.sched_getaffinity(0))
    res = {}
    for name, fn in (("reference", time_reference), ("port", time_port)):
        fn(1.0, threads)  # warm-up
        nbytes, reps, el = fn(seconds, threads)
        res[name] = nbytes * reps / el / 1e9
        print(f"{name}: {reps} steps in {el:.2f} s, {1e3 * el / reps:.2f} ms/step, "
              f"{res[name]:.3f} GB/s ({threads} threads)", flush=True)
    print(f"port / reference = {res['port'] / res['reference']:.1f}x")


if __name__ == "__main__":
    main()
