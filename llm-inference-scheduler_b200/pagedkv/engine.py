"""Continuous-batching engine for the paged model (greedy decoding).

The reference's own scheduler (mini_engine/scheduler.py) and radix cache
(mini_engine/paged/radix_cache.py) drive pagedkv.BlockManager / PagedKVCache
and PagedQwen2Model unchanged (tests/test_reference_drives_pagedkv.py shows
it).  They cannot travel to a machine without the reference, so config 5's
runs on the GPU use this engine instead: its own structure, around the
executor that is the part specific to this path.

* `StepExecutor` runs one planned step: the flat token ids go to the device
  with one pinned copy, the step replays a captured CUDA graph when one of
  its padded shapes fits (pagedkv.graphs.StepGraphs) or runs the model
  eagerly (PagedKVCache.prepare_step + one RoPE/append launch and at most
  two attention launches per layer), and the greedy tokens of the whole
  batch come back in one device-to-host copy.
* `Engine` keeps sequences in a FIFO queue and an active list and plans each
  step in four phases:
  1. place: queued sequences join while there is a slot and memory.  The
     prefix index (pagedkv.prefix_index) supplies the blocks of the longest
     indexed run of the sequence's full blocks, at least one token is left
     to compute, those blocks are pinned before anything is allocated, and
     blocks for the rest of the tokens plus one are allocated (evicting
     index-only blocks if the pool is short);
  2. grow: every active sequence gets room for one more token; when the
     pool stays short the youngest active sequence is preempted (its blocks
     released, recomputed later from its tokens), and a sequence that is
     alone and still short sits the step out;
  3. plan: a token budget, sequences that already produced output first,
     each feeding its uncomputed tokens (a long prompt goes in chunks);
     a shared partial tail block is copied first (copy-on-write);
  4. commit: sequences whose tokens are all computed take their greedy
     token; a sequence that hits an EOS id or its token limit publishes its
     full blocks to the index and releases its own references.
  The greedy streams do not depend on these choices: every sequence's
  tokens are computed exactly once per position, whatever the batch.
"""

from __future__ import annotations

import collections
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .block_manager import BlockManager, PagedKVCache
from .model import SequenceForwardInfo
from .prefix_index import BlockPrefixIndex

QUEUED, ACTIVE, DONE = "queued", "active", "done"


@dataclass(eq=False)
class Seq:
    """One request: its prompt, what it generated and where its KV lives."""

    ident: int
    prompt: list[int]
    limit: int = 128                 # tokens to generate at most
    generated: list[int] = field(default_factory=list)
    computed: int = 0                # leading tokens whose KV is in the pool
    table: list[int] = field(default_factory=list)
    status: str = QUEUED
    reused: int = 0                  # tokens taken from the prefix index, over all placements
    preempted: int = 0
    finish: str | None = None        # "stop", "length" or "cancelled"
    t_arrive: float = field(default_factory=time.monotonic)
    t_first: float | None = None
    t_done: float | None = None

    @property
    def tokens(self) -> list[int]:
        return self.prompt + self.generated

    @property
    def length(self) -> int:
        return len(self.prompt) + len(self.generated)


class StepExecutor:
    """One planned step of the paged model -> the greedy token of every
    planned sequence (one host round trip)."""

    def __init__(self, model, kv: PagedKVCache, cuda_graphs: bool = False, max_batch: int = 8,
                 max_tokens: int = 256, graph_max_blocks: int = 64):
        self.model, self.kv = model, kv
        self.cuda_graphs = cuda_graphs and model.device.type == "cuda"
        self.max_batch, self.max_tokens, self.graph_max_blocks = max_batch, max_tokens, graph_max_blocks
        self.graphs = None
        self.last_logits = None

    def step_graphs(self):
        """The CUDA-graph runner (made on first use)."""
        if self.graphs is None:
            from .graphs import StepGraphs

            self.graphs = StepGraphs(self.model, self.kv, self.max_batch, max_tokens=self.max_tokens,
                                     max_blocks_per_seq=self.graph_max_blocks)
        return self.graphs

    def __call__(self, infos: list[SequenceForwardInfo], flat_ids: list[int]) -> list[int]:
        ids = torch.tensor(flat_ids, dtype=torch.long)
        if self.model.device.type == "cuda":
            ids = ids.pin_memory().to(self.model.device, non_blocking=True)
        if self.cuda_graphs and self.model.timing is None and self.step_graphs().supports(infos):
            logits = self.graphs.forward(ids, infos)
        else:
            logits = self.model.forward(ids, infos, self.kv)
        self.last_logits = logits  # [planned sequences, vocab], for Engine.choose
        return logits.float().argmax(dim=-1).tolist()


class Engine:
    """Continuous batching of greedy requests over one BlockManager."""

    def __init__(self, model, manager: BlockManager, max_seqs: int = 8, token_budget: int = 256,
                 prefix_reuse: bool = True, eos_ids=(), cuda_graphs: bool = False,
                 graph_max_blocks: int = 64, choose=None):
        self.mgr = manager
        self.kv = PagedKVCache(manager)
        self.index = BlockPrefixIndex(manager) if prefix_reuse else None
        self.max_seqs, self.token_budget = max_seqs, token_budget
        self.eos_ids = frozenset(eos_ids)
        self.run_step = StepExecutor(model, self.kv, cuda_graphs, max_seqs, token_budget,
                                     graph_max_blocks)
        # choose(seq, greedy_token, logits_row) -> the token appended (a test
        # hook: teacher forcing against another implementation's stream)
        self.choose = choose
        self.queue: collections.deque[Seq] = collections.deque()
        self.active: list[Seq] = []
        self.counts = collections.Counter(steps=0, generated=0, prefill_tokens=0, reused_tokens=0,
                                          preemptions=0, finished=0, cancelled=0)

    # ---- public --------------------------------------------------------------

    @property
    def busy(self) -> bool:
        return bool(self.queue or self.active)

    @property
    def graphs(self):
        return self.run_step.graphs

    def submit(self, seq: Seq) -> Seq:
        seq.status = QUEUED
        self.queue.append(seq)
        return seq

    def cancel(self, seq: Seq) -> None:
        if seq.status == QUEUED:
            self.queue.remove(seq)
        elif seq.status == ACTIVE:
            self.active.remove(seq)
            self._release(seq)
        else:
            return
        self._close(seq, "cancelled")

    @torch.inference_mode()
    def step(self) -> None:
        self.counts["steps"] += 1
        self._place_queued()
        ready = self._grow()
        if not ready:
            return
        plan = self._plan(ready)
        infos, flat = [], []
        for seq, n in plan:
            infos.append(SequenceForwardInfo(seq.ident, len(flat), n,
                                             np.arange(seq.computed, seq.computed + n)))
            flat.extend(seq.tokens[seq.computed:seq.computed + n])
        self._commit(plan, self.run_step(infos, flat))

    def run(self, max_steps: int = 1 << 30) -> int:
        """Step until idle; returns the steps taken."""
        n = 0
        while self.busy and n < max_steps:
            self.step()
            n += 1
        return n

    # ---- memory --------------------------------------------------------------

    def _blocks_for(self, n_tokens: int) -> int:
        return -(-n_tokens // self.mgr.block_size)

    def _take(self, n: int) -> list[int] | None:
        """n fresh blocks, reclaiming index-only blocks if the pool is short."""
        if n <= 0:
            return []
        short = n - self.mgr.num_free
        if short > 0 and self.index is not None:
            self.index.reclaim(short)
        if self.mgr.num_free < n:
            return None
        return [self.mgr.allocate() for _ in range(n)]

    def _release(self, seq: Seq) -> None:
        for b in seq.table:
            self.mgr.decref(b)
        seq.table = []
        self.kv.free_sequence(seq.ident)

    # ---- phase 1: place queued sequences -----------------------------------

    def _place_queued(self) -> None:
        while self.queue and len(self.active) < self.max_seqs:
            if not self._place(self.queue[0]):
                return
            seq = self.queue.popleft()
            seq.status = ACTIVE
            self.active.append(seq)

    def _place(self, seq: Seq) -> bool:
        toks = seq.tokens
        hits = self.index.lookup(toks) if self.index is not None else []
        hits = hits[: (len(toks) - 1) // self.mgr.block_size]  # keep >= 1 token to compute
        for b in hits:  # pinned first: the reclaim below cannot take them
            self.mgr.incref(b)
        fresh = self._take(self._blocks_for(len(toks) + 1) - len(hits))
        if fresh is None:
            for b in hits:
                self.mgr.decref(b)
            return False
        seq.table = hits + fresh
        seq.computed = len(hits) * self.mgr.block_size
        seq.reused += seq.computed
        self.counts["reused_tokens"] += seq.computed
        self.kv.add_sequence(seq.ident, seq.table, seq.computed)
        return True

    # ---- phase 2: room for one more token ----------------------------------

    def _grow(self) -> list[Seq]:
        waiting_out = set()
        for seq in list(self.active):
            while seq.status == ACTIVE:
                missing = self._blocks_for(seq.length + 1) - len(seq.table)
                if missing <= 0:
                    break
                got = self._take(missing)
                if got is not None:
                    seq.table.extend(got)
                    break
                if len(self.active) <= 1:
                    waiting_out.add(seq.ident)
                    break
                self._preempt(self.active[-1])
        return [s for s in self.active if s.ident not in waiting_out]

    def _preempt(self, seq: Seq) -> None:
        """Recompute preemption: release the blocks, requeue at the front."""
        self.active.remove(seq)
        self._release(seq)
        seq.computed = 0
        seq.status = QUEUED
        seq.preempted += 1
        self.counts["preemptions"] += 1
        self.queue.appendleft(seq)

    # ---- phase 3: the step's batch -----------------------------------------

    def _plan(self, ready: list[Seq]) -> list[tuple[Seq, int]]:
        order = [s for s in ready if s.generated] + [s for s in ready if not s.generated]
        budget, plan = self.token_budget, []
        for seq in order:
            if budget <= 0:
                break
            n = min(seq.length - seq.computed, budget)
            budget -= n
            self.kv.ensure_writable_tail(seq.ident)
            plan.append((seq, n))
        return plan

    # ---- phase 4: commit ---------------------------------------------------

    def _commit(self, plan: list[tuple[Seq, int]], tokens: list[int]) -> None:
        now = time.monotonic()
        for row, ((seq, n), tok) in enumerate(zip(plan, tokens)):
            if not seq.generated:
                self.counts["prefill_tokens"] += n
            seq.computed += n
            if seq.computed < seq.length:
                continue  # a chunk of a longer prompt (or recompute): no token yet
            if self.choose is not None:
                tok = self.choose(seq, int(tok), self.run_step.last_logits[row])
            tok = int(tok)
            seq.generated.append(tok)
            self.counts["generated"] += 1
            if seq.t_first is None:
                seq.t_first = now
            if tok in self.eos_ids:
                self._finish(seq, "stop")
            elif len(seq.generated) >= seq.limit:
                self._finish(seq, "length")
        self.active = [s for s in self.active if s.status == ACTIVE]

    def _finish(self, seq: Seq, reason: str) -> None:
        if self.index is not None:
            self.index.publish(seq.tokens[: seq.computed], seq.table)
        self._release(seq)
        self._close(seq, reason)

    def _close(self, seq: Seq, reason: str) -> None:
        seq.status = DONE
        seq.finish = reason
        seq.t_done = time.monotonic()
        self.counts["cancelled" if reason == "cancelled" else "finished"] += 1
