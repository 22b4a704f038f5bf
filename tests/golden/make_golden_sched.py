"""Scheduling decisions of the REFERENCE scheduler under a stand-in model.

    REF_ROOT=/path/to/llm-inference-scheduler python tests/golden/make_golden_sched.py

Drives the reference's Scheduler (mini_engine/scheduler.py) with its
BlockManager / PagedKVCache / RadixCache and a stand-in model whose logits
put all mass on cases.fake_next_token(last token, position); the stand-in
still calls PagedKVCache.append_and_fetch on the last layer so sequence
lengths advance exactly as with the real model.  Records, per step, the
scheduled (seq_id, num_tokens, first position) list and the block tables,
plus outputs and metrics, to tests/golden/sched_trace.json.
"""

import json
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases as C  # noqa: E402

sys.path.insert(0, os.environ.get("REF_ROOT", "/root/reference"))
from mini_engine.paged.block_manager import BlockManager  # noqa: E402
from mini_engine.sampling import SamplingParams  # noqa: E402
from mini_engine.scheduler import Request, Scheduler  # noqa: E402

V = 1024


class StandIn:
    device = torch.device("cpu")

    def __init__(self, trace):
        self.trace = trace

    def forward(self, input_ids, seq_infos, kv_cache):
        self.trace.append([[s.seq_id, s.num_tokens, int(s.positions[0])] for s in seq_infos])
        logits = torch.full((len(seq_infos), V), -1.0)
        for i, s in enumerate(seq_infos):
            z = torch.zeros(s.num_tokens, 1, 1)
            kv_cache.append_and_fetch(0, s.seq_id, z, z)  # single-layer manager: advances lengths
            last = int(input_ids[s.flat_start + s.num_tokens - 1])
            logits[i, C.fake_next_token(last, int(s.positions[-1]))] = 1.0
        return logits


class StubTokenizer:
    eos_ids = {-1}


def main():
    sc = C.sched_scenario()
    trace, tables = [], []
    mgr = BlockManager(sc["num_blocks"], 16, 1, 1, 1)
    sched = Scheduler(StandIn(trace), StubTokenizer(), mgr, max_num_seqs=sc["max_num_seqs"],
                      max_batched_tokens=sc["max_batched_tokens"], enable_prefix_cache=True)
    reqs = []
    for i, (p, n) in enumerate(zip(sc["prompts"], sc["max_new_tokens"])):
        r = Request(req_id=i, prompt_ids=list(p), params=SamplingParams(temperature=0.0, max_new_tokens=n))
        sched.waiting.append(r)
        reqs.append(r)
    while sched.has_work:
        sched.step()
        tables.append({str(r.req_id): list(r.block_table) for r in sched.running})
    for k in sc["turn2"]:
        r0 = reqs[k]
        r = Request(req_id=len(reqs), prompt_ids=r0.prompt_ids + r0.output_ids + [5, 6, 7],
                    params=SamplingParams(temperature=0.0, max_new_tokens=10))
        sched.waiting.append(r)
        reqs.append(r)
    while sched.has_work:
        sched.step()
        tables.append({str(r.req_id): list(r.block_table) for r in sched.running})
    out = dict(trace=trace, tables=tables, outputs=[r.output_ids for r in reqs],
               metrics=dict(sched.metrics), preemptions=[r.preemptions for r in reqs],
               num_prefix_cached=[r.num_prefix_cached for r in reqs], free=mgr.num_free)
    with open(os.path.join(HERE, "sched_trace.json"), "w") as f:
        json.dump(out, f)
    print(out["metrics"], "steps traced", len(trace))


if __name__ == "__main__":
    main()
