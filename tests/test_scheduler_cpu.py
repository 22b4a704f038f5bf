"""Scheduling decisions of pagedkv.scheduler vs the reference scheduler (CPU).

Both schedulers are driven by the same stand-in model (greedy token =
cases.fake_next_token(last token, position)), so only the policy is compared:
the admission order, radix prefix matches and eviction, chunked-prefill
budgets, preemption, copy-on-write and the block tables of every step.  The
reference's decisions were recorded by tests/golden/make_golden_sched.py.
"""

import json

import numpy as np
import torch

import cases as C
from conftest import GOLDEN
from pagedkv import BlockManager
from pagedkv.scheduler import Request, Scheduler


class StandIn:
    """Advances sequence lengths the way forward_layer does on the last layer
    and puts all logit mass on fake_next_token."""

    device = torch.device("cpu")

    def __init__(self, trace):
        self.trace = trace

    def forward(self, ids, infos, kv):
        self.trace.append([[s.seq_id, s.num_tokens, int(s.positions[0])] for s in infos])
        logits = torch.full((len(infos), 1024), -1.0)
        for i, s in enumerate(infos):
            kv._len[s.seq_id] += s.num_tokens
            last = int(ids[s.flat_start + s.num_tokens - 1])
            logits[i, C.fake_next_token(last, int(s.positions[-1]))] = 1.0
        return logits


def run(sc, num_blocks=None):
    trace, tables = [], []
    mgr = BlockManager(num_blocks or sc["num_blocks"], 16, 1, 1, 1, device=None)
    sched = Scheduler(StandIn(trace), mgr, max_num_seqs=sc["max_num_seqs"],
                      max_batched_tokens=sc["max_batched_tokens"], enable_prefix_cache=True,
                      eos_ids={-1})
    reqs = []
    for i, (p, n) in enumerate(zip(sc["prompts"], sc["max_new_tokens"])):
        reqs.append(Request(i, list(p), max_new_tokens=n))
        sched.add_request(reqs[-1])
    while sched.has_work:
        sched.step()
        tables.append({str(r.req_id): list(r.block_table) for r in sched.running})
    for k in sc["turn2"]:
        r0 = reqs[k]
        reqs.append(Request(len(reqs), r0.prompt_ids + r0.output_ids + [5, 6, 7], max_new_tokens=10))
        sched.add_request(reqs[-1])
    while sched.has_work:
        sched.step()
        tables.append({str(r.req_id): list(r.block_table) for r in sched.running})
    return reqs, sched, mgr, trace, tables


def test_decisions_match_reference_step_by_step():
    with open(f"{GOLDEN}/sched_trace.json") as f:
        g = json.load(f)
    reqs, sched, mgr, trace, tables = run(C.sched_scenario())
    assert g["metrics"]["preemptions"] > 0 and g["metrics"]["prefix_cache_hit_tokens"] > 0
    assert len(trace) == len(g["trace"])
    for i, (a, b) in enumerate(zip(trace, g["trace"])):
        assert a == b, f"step {i}: scheduled {a} vs reference {b}"
    assert tables == g["tables"]
    assert [r.output_ids for r in reqs] == g["outputs"]
    assert [r.preemptions for r in reqs] == g["preemptions"]
    assert [r.num_prefix_cached for r in reqs] == g["num_prefix_cached"]
    for k, v in g["metrics"].items():
        assert sched.metrics[k] == v, k
    assert mgr.num_free == g["free"]


def test_eviction_of_a_just_matched_prefix_is_recomputed():
    """With 24 or 18 blocks the reference's radix eviction releases the blocks
    of the prefix it has just matched and its adopt() trips the incref assert;
    here every request still completes with its full output."""
    sc = C.sched_scenario()
    for nb in (24, 18):
        reqs, sched, mgr, trace, _ = run(sc, num_blocks=nb)
        lens = [len(r.output_ids) for r in reqs]
        assert lens == list(sc["max_new_tokens"]) + [10] * len(sc["turn2"])
        assert all(r.finish_reason == "length" for r in reqs)
        # every block is back: free list plus the radix tree's references
        assert mgr.num_free + sched.radix.num_tree_blocks >= 0
        assert sum(1 for c in mgr.ref_count if c > 0) == sched.radix.num_tree_blocks
