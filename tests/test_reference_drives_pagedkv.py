"""The reference's own scheduler and radix cache drive pagedkv unchanged.

north_star: the engine, scheduler and radix cache use the new path "without
other changes".  This test takes the reference's mini_engine/scheduler.py and
mini_engine/paged/radix_cache.py as they are, with one substitution made the
way a maintainer would make it: the module mini_engine.paged.block_manager is
this package's pagedkv.block_manager (BlockManager, PagedKVCache,
OutOfBlocks).  The reference Scheduler then builds its PagedKVCache from
pagedkv, its RadixCache increfs and decrefs pagedkv.BlockManager's blocks,
and the step loop runs over a stand-in model (all logit mass on
cases.fake_next_token; the model's last layer advancing each sequence's
length).  Every scheduling decision -- the sequences and chunk sizes of each
step, the block tables after each step, outputs, preemptions, prefix hits,
metrics and the free-block count -- must equal the reference scheduler over
its own BlockManager (tests/golden/sched_trace.json, make_golden_sched.py).

The reference is read from REF_ROOT (default: the reference checkout next to
this build); without it the test is skipped.  It runs in a child process so
the substituted module never meets the unmodified reference that other
tests import.
"""

import json
import os
import subprocess
import sys
import textwrap

import pytest

from conftest import GOLDEN, PKG_ROOT

REF_ROOT = os.environ.get("REF_ROOT", "/root/reference")

CHILD = textwrap.dedent('''
    import json, sys
    import torch
    sys.path[:0] = [{pkg!r}, {golden!r}]
    import cases as C
    import pagedkv.block_manager as pkv_bm
    sys.modules["mini_engine.paged.block_manager"] = pkv_bm   # the one substitution
    sys.path.insert(0, {ref!r})
    from mini_engine.paged.radix_cache import RadixCache
    from mini_engine.sampling import SamplingParams
    from mini_engine.scheduler import Request, Scheduler
    import mini_engine.scheduler as ref_sched
    assert ref_sched.PagedKVCache is pkv_bm.PagedKVCache and ref_sched.OutOfBlocks is pkv_bm.OutOfBlocks

    class StandIn:
        device = torch.device("cpu")
        def __init__(self, trace):
            self.trace = trace
        def forward(self, input_ids, seq_infos, kv_cache):
            assert isinstance(kv_cache, pkv_bm.PagedKVCache)
            self.trace.append([[s.seq_id, s.num_tokens, int(s.positions[0])] for s in seq_infos])
            logits = torch.full((len(seq_infos), 1024), -1.0)
            for i, s in enumerate(seq_infos):
                kv_cache._len[s.seq_id] += s.num_tokens   # what the last layer does
                last = int(input_ids[s.flat_start + s.num_tokens - 1])
                logits[i, C.fake_next_token(last, int(s.positions[-1]))] = 1.0
            return logits

    class StubTokenizer:
        eos_ids = {{-1}}

    sc = C.sched_scenario()
    trace, tables = [], []
    mgr = pkv_bm.BlockManager(sc["num_blocks"], 16, 1, 1, 1, device=None)
    sched = Scheduler(StandIn(trace), StubTokenizer(), mgr, max_num_seqs=sc["max_num_seqs"],
                      max_batched_tokens=sc["max_batched_tokens"], enable_prefix_cache=True)
    assert isinstance(sched.kv, pkv_bm.PagedKVCache) and isinstance(sched.radix, RadixCache)
    reqs = []
    def add(rid, prompt, n):
        r = Request(req_id=rid, prompt_ids=list(prompt),
                    params=SamplingParams(temperature=0.0, max_new_tokens=n))
        sched.waiting.append(r)
        reqs.append(r)
    for i, (p, n) in enumerate(zip(sc["prompts"], sc["max_new_tokens"])):
        add(i, p, n)
    def drain():
        while sched.has_work:
            sched.step()
            tables.append({{str(r.req_id): list(r.block_table) for r in sched.running}})
    drain()
    for k in sc["turn2"]:
        r0 = reqs[k]
        add(len(reqs), r0.prompt_ids + r0.output_ids + [5, 6, 7], 10)
    drain()
    print(json.dumps(dict(trace=trace, tables=tables, outputs=[r.output_ids for r in reqs],
                          metrics=dict(sched.metrics), preemptions=[r.preemptions for r in reqs],
                          num_prefix_cached=[r.num_prefix_cached for r in reqs], free=mgr.num_free,
                          flushes=mgr.flushes)))
''')


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF_ROOT, "mini_engine")),
                    reason="the reference (REF_ROOT) is not present on this machine")
def test_reference_scheduler_and_radix_cache_over_pagedkv_make_the_same_decisions():
    code = CHILD.format(pkg=PKG_ROOT, golden=GOLDEN, ref=REF_ROOT)
    res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert res.returncode == 0, res.stderr[-3000:]
    got = json.loads(res.stdout.strip().splitlines()[-1])
    with open(f"{GOLDEN}/sched_trace.json") as f:
        want = json.load(f)
    assert want["metrics"]["preemptions"] > 0 and want["metrics"]["prefix_cache_hit_tokens"] > 0
    assert len(got["trace"]) == len(want["trace"])
    for i, (a, b) in enumerate(zip(got["trace"], want["trace"])):
        assert a == b, f"step {i}: scheduled {a}, reference over its own BlockManager {b}"
    assert got["tables"] == want["tables"]
    for key in ("outputs", "metrics", "preemptions", "num_prefix_cached", "free"):
        assert got[key] == want[key], key
