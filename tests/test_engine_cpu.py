"""pagedkv.engine and pagedkv.prefix_index on the CPU (no pools, no kernels).

A stand-in model advances sequence lengths as forward_layer does on the last
layer and puts all logit mass on cases.fake_next_token(last token, position),
so every stream is fixed by its tokens alone, whatever the batching.  The
checks:
* the engine's streams equal the reference scheduler's under the same
  stand-in (tests/golden/sched_trace.json, made by make_golden_sched.py),
  on the reference's tight pool and on tighter ones (preemption, prefix
  reuse, eviction);
* the block accounting closes: after the run every block is either free or
  held by the prefix index alone;
* the prefix index: longest-chain lookup, one entry per block, LRU eviction
  of leaves only, in-use blocks never evicted, pinned blocks survive a
  reclaim.
"""

import json

import numpy as np
import torch

import cases as C
from conftest import GOLDEN
from pagedkv import BlockManager
from pagedkv.engine import Engine, Seq
from pagedkv.prefix_index import BlockPrefixIndex


class StandIn:
    device = torch.device("cpu")
    timing = None

    def __init__(self, trace=None):
        self.trace = trace if trace is not None else []

    def forward(self, ids, infos, kv):
        self.trace.append([[s.seq_id, s.num_tokens, int(s.positions[0])] for s in infos])
        logits = torch.full((len(infos), 1024), -1.0)
        for i, s in enumerate(infos):
            kv._len[s.seq_id] += s.num_tokens
            last = int(ids[s.flat_start + s.num_tokens - 1])
            logits[i, C.fake_next_token(last, int(s.positions[-1]))] = 1.0
        return logits


def run(sc, num_blocks=None, prefix_reuse=True):
    nb = num_blocks or sc["num_blocks"]
    mgr = BlockManager(nb, 16, 1, 1, 1, device=None)
    eng = Engine(StandIn(), mgr, max_seqs=sc["max_num_seqs"], token_budget=sc["max_batched_tokens"],
                 prefix_reuse=prefix_reuse, eos_ids={-1})
    seqs = [eng.submit(Seq(i, list(p), limit=n))
            for i, (p, n) in enumerate(zip(sc["prompts"], sc["max_new_tokens"]))]
    eng.run(5000)
    for k in sc["turn2"]:
        s0 = seqs[k]
        seqs.append(eng.submit(Seq(len(seqs), s0.prompt + s0.generated + [5, 6, 7], limit=10)))
    eng.run(5000)
    return seqs, eng, mgr


def test_streams_equal_reference_scheduler_and_accounting_closes():
    with open(f"{GOLDEN}/sched_trace.json") as f:
        g = json.load(f)
    sc = C.sched_scenario()
    for nb, reuse in ((None, True), (24, True), (18, True), (12, True), (None, False), (9, False)):
        seqs, eng, mgr = run(sc, nb, reuse)
        assert not eng.busy
        assert [s.generated for s in seqs] == g["outputs"], (nb, reuse)
        assert all(s.finish == "length" for s in seqs)
        held = len(eng.index) if eng.index is not None else 0
        assert mgr.num_free + held == mgr.num_blocks, (nb, reuse)
        assert all(c in (0, 1) for c in mgr.ref_count)
        if nb == 12:
            assert eng.counts["preemptions"] > 0
        if reuse:
            assert eng.counts["reused_tokens"] > 0
            assert [s.reused > 0 for s in seqs][-2:] == [True, True]  # second turns hit


def test_prefix_index_lookup_publish_and_lru():
    mgr = BlockManager(16, 4, 1, 1, 1, device=None)
    idx = BlockPrefixIndex(mgr)
    a = [mgr.allocate() for _ in range(3)]
    toks = list(range(12)) + [99, 98]          # 3 full blocks + a partial one
    assert idx.publish(toks, a + [mgr.allocate()]) == 3
    assert [mgr.ref_count[b] for b in a] == [2, 2, 2]
    assert idx.lookup(list(range(12)) + [7]) == a
    assert idx.lookup(list(range(8)) + [0, 0, 0, 0]) == a[:2]   # diverges inside block 2
    assert idx.lookup([1] + list(range(1, 12))) == []
    # a sibling that shares block 0 and differs inside block 1
    b = [mgr.allocate() for _ in range(2)]
    assert idx.publish(list(range(4)) + [50, 51, 52, 53], [a[0]] + b) == 1
    assert len(idx) == 4 and mgr.ref_count[a[0]] == 2 and mgr.ref_count[b[1]] == 1
    # the sequences let go: only the index holds the blocks now
    for blk in a + b:
        mgr.decref(blk)
    free0 = mgr.num_free
    idx.lookup(list(range(12)))                  # the first chain is the most recent
    assert idx.reclaim(1) == 1 and mgr.num_free == free0 + 1
    assert idx.lookup(list(range(4)) + [50, 51, 52, 53]) == [a[0]]  # the sibling leaf went
    # a block a running sequence still uses is never evicted, nor its ancestors
    mgr.incref(a[2])
    assert idx.reclaim(10) == 0 and len(idx) == 3
    mgr.decref(a[2])
    assert idx.clear() == 3 and len(idx) == 0
    assert mgr.num_free == mgr.num_blocks - 1    # the partial block is still the test's
    assert all(c == 0 for blk, c in enumerate(mgr.ref_count) if blk != 3)


def test_pinned_prefix_survives_the_allocation_it_triggers():
    """Placing a sequence whose prefix is indexed while the pool is full: the
    matched blocks are pinned before the allocation reclaims index-only blocks,
    so the reclaim takes other blocks, never the ones just matched."""
    mgr = BlockManager(6, 4, 1, 1, 1, device=None)
    eng = Engine(StandIn(), mgr, max_seqs=2, token_budget=64, eos_ids={-1})
    first = eng.submit(Seq(0, list(range(100, 108)), limit=1))    # 2 full blocks + 1 to grow
    other = eng.submit(Seq(1, list(range(200, 208)), limit=1))
    eng.run()
    assert len(eng.index) == 4 and mgr.num_free == 2
    # 17 tokens: 2 matched blocks + 3 fresh ones, one more than the pool has free
    again = eng.submit(Seq(2, list(range(100, 108)) + list(range(1, 10)), limit=2))
    eng.step()
    assert again.reused == 8
    assert eng.index.lookup(list(range(100, 108))) == again.table[:2]  # still indexed
    assert len(eng.index.lookup(list(range(200, 208)))) == 1           # other's leaf went
    eng.run()
    assert again.generated and first.generated and other.generated
    assert mgr.num_free + len(eng.index) == mgr.num_blocks


def test_cancel_releases_blocks_and_keeps_index_clean():
    mgr = BlockManager(32, 16, 1, 1, 1, device=None)
    eng = Engine(StandIn(), mgr, max_seqs=4, token_budget=16, eos_ids={-1})
    a = eng.submit(Seq(0, list(np.arange(3, 60) % 997), limit=50))
    b = eng.submit(Seq(1, [5, 6, 7], limit=50))
    for _ in range(3):
        eng.step()
    eng.cancel(a)
    eng.cancel(b)
    assert a.finish == b.finish == "cancelled" and not eng.busy
    assert mgr.num_free == mgr.num_blocks and len(eng.index) == 0
    assert eng.counts["cancelled"] == 2
