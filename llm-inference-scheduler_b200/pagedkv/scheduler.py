"""Continuous-batching scheduler driving the paged model (greedy sampling).

The scheduling policy is the reference's (mini_engine/scheduler.py:66-292),
restated so that a run here makes the same decisions, token for token:
* admission while running < max_num_seqs, with a radix-cache prefix match
  that always leaves at least one token to compute (scheduler.py:109-135).
  One deliberate difference: when the radix eviction that frees room for the
  new blocks releases part of the prefix just matched, the reference fails
  its incref assert in adopt(); here that prefix is recomputed instead;
* blocks for total_len + 1 tokens, evicting radix leaves first and then
  preempting the most recently admitted running request (recompute, 143-156);
* decode-first token budget: requests that already produced output go
  first, each feeding its uncomputed tokens up to the budget (chunked
  prefill, 226-262);
* copy-on-write of a shared partial tail before the step (250);
* greedy sampling once all known tokens are computed; stop on an EOS id or
  max_new_tokens; finished sequences donate their full blocks to the radix
  cache (158-175, 267-292).
What differs is the execution of a step: the device metadata is built once
(PagedKVCache.prepare_step), every layer runs one append + at most two
attention launches, and the greedy argmax of the whole batch comes back to
the host in one copy.  With cuda_graphs=True a step replays a captured CUDA
graph of the model step (pagedkv.graphs.StepGraphs) when one of its padded
shapes fits: decode-only steps, and mixed steps of up to 4 prefill
sequences; other steps run eagerly.  The decisions are the same either way.
"""

from __future__ import annotations

import enum
import time
from dataclasses import dataclass, field

import numpy as np
import torch

from .block_manager import BlockManager, PagedKVCache
from .model import PagedQwen2Model, SequenceForwardInfo
from .radix_cache import RadixCache


class RequestState(enum.Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"
    CANCELLED = "cancelled"


@dataclass
class Request:
    req_id: int
    prompt_ids: list[int]
    max_new_tokens: int = 128
    state: RequestState = RequestState.WAITING
    output_ids: list[int] = field(default_factory=list)
    num_computed_tokens: int = 0
    block_table: list[int] = field(default_factory=list)
    num_prefix_cached: int = 0
    preemptions: int = 0
    finish_reason: str | None = None
    arrived_at: float = field(default_factory=time.monotonic)
    first_token_at: float | None = None
    finished_at: float | None = None

    @property
    def all_ids(self) -> list[int]:
        return self.prompt_ids + self.output_ids

    @property
    def total_len(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)


class Scheduler:
    def __init__(self, model: PagedQwen2Model, block_manager: BlockManager, max_num_seqs: int = 8,
                 max_batched_tokens: int = 256, enable_prefix_cache: bool = True,
                 eos_ids: set[int] | None = None, cuda_graphs: bool = False,
                 graph_max_blocks: int = 64):
        self.model = model
        self.mgr = block_manager
        self.kv = PagedKVCache(block_manager)
        self.radix = RadixCache(block_manager) if enable_prefix_cache else None
        self.max_num_seqs = max_num_seqs
        self.max_batched_tokens = max_batched_tokens
        self.eos_ids = set(eos_ids or ())
        self.waiting: list[Request] = []
        self.running: list[Request] = []
        self.metrics = dict(requests_finished=0, requests_cancelled=0, preemptions=0, steps=0,
                            tokens_generated=0, prefill_tokens_computed=0, prefix_cache_hit_tokens=0)
        self.cuda_graphs = cuda_graphs and model.device.type == "cuda"
        self.graph_max_blocks = graph_max_blocks
        self.graphs = None  # StepGraphs, made at the first step

    def step_graphs(self):
        """The CUDA-graph runner of the model step (cuda_graphs=True)."""
        if self.graphs is None:
            from .graphs import StepGraphs
            self.graphs = StepGraphs(self.model, self.kv, self.max_num_seqs,
                                     max_tokens=self.max_batched_tokens,
                                     max_blocks_per_seq=self.graph_max_blocks)
        return self.graphs

    # ---- memory ----------------------------------------------------------

    def _blocks_for(self, n_tokens: int) -> int:
        return (n_tokens + self.mgr.block_size - 1) // self.mgr.block_size

    def _try_allocate(self, n: int) -> list[int] | None:
        if self.mgr.num_free < n and self.radix is not None:
            self.radix.evict(n - self.mgr.num_free)
        if self.mgr.num_free < n:
            return None
        return [self.mgr.allocate() for _ in range(n)]

    def _admit(self, req: Request) -> bool:
        feed = req.all_ids
        blocks: list[int] = []
        matched = 0
        if self.radix is not None:
            blocks, matched = self.radix.match_prefix(feed)
            while matched >= len(feed):  # keep at least one token to compute (its logits)
                blocks = blocks[:-1]
                matched -= self.mgr.block_size
        fresh = self._try_allocate(self._blocks_for(len(feed) + 1) - len(blocks))
        if fresh is None:
            return False
        if blocks and any(self.mgr.ref_count[b] == 0 or b in fresh for b in blocks):
            # The radix eviction inside _try_allocate released part of the
            # prefix matched above (the reference would then fail its incref
            # assert in adopt).  Recompute that prefix instead of reusing it.
            more = self._try_allocate(len(blocks))
            if more is None:
                for b in fresh:
                    self.mgr.decref(b)
                return False
            fresh, blocks, matched = fresh + more, [], 0
        if self.radix is not None:
            self.radix.adopt(blocks)
        req.block_table = blocks + fresh
        req.num_computed_tokens = matched
        req.num_prefix_cached += matched
        self.metrics["prefix_cache_hit_tokens"] += matched
        self.kv.add_sequence(req.req_id, req.block_table, matched)
        req.state = RequestState.RUNNING
        self.running.append(req)
        return True

    def _release(self, req: Request):
        for b in req.block_table:
            self.mgr.decref(b)
        req.block_table = []
        self.kv.free_sequence(req.req_id)

    def _preempt_one(self) -> bool:
        cands = [r for r in self.running if r.state is RequestState.RUNNING]
        if len(cands) <= 1:
            return False
        victim = cands[-1]
        self._release(victim)
        victim.num_computed_tokens = 0
        victim.state = RequestState.WAITING
        victim.preemptions += 1
        self.metrics["preemptions"] += 1
        self.running.remove(victim)
        self.waiting.insert(0, victim)
        return True

    def _finish(self, req: Request, reason: str):
        if self.radix is not None and reason != "cancelled":
            self.radix.insert(req.all_ids[: req.num_computed_tokens], req.block_table)
        self._release(req)
        req.state = RequestState.CANCELLED if reason == "cancelled" else RequestState.FINISHED
        req.finish_reason = reason
        req.finished_at = time.monotonic()
        self.metrics["requests_cancelled" if reason == "cancelled" else "requests_finished"] += 1

    def add_request(self, req: Request):
        self.waiting.append(req)

    def cancel(self, req: Request):
        if req.state in (RequestState.FINISHED, RequestState.CANCELLED):
            return
        if req in self.waiting:
            self.waiting.remove(req)
        if req in self.running:
            self.running.remove(req)
        self._finish(req, "cancelled")

    @property
    def has_work(self) -> bool:
        return bool(self.waiting or self.running)

    # ---- one iteration -------------------------------------------------------

    @torch.inference_mode()
    def step(self):
        self.metrics["steps"] += 1
        while self.waiting and len(self.running) < self.max_num_seqs:
            if not self._admit(self.waiting[0]):
                break
            self.waiting.pop(0)
        if not self.running:
            return

        stalled: set[int] = set()
        for req in list(self.running):
            need = self._blocks_for(req.total_len + 1) - len(req.block_table)
            while need > 0 and req.state is RequestState.RUNNING:
                got = self._try_allocate(need)
                if got is not None:
                    req.block_table.extend(got)
                    break
                if not self._preempt_one():
                    stalled.add(req.req_id)
                    break
                need = self._blocks_for(req.total_len + 1) - len(req.block_table)
        active = [r for r in self.running
                  if r.state is RequestState.RUNNING and r.req_id not in stalled]
        if not active:
            return

        budget = self.max_batched_tokens
        flat: list[int] = []
        infos: list[SequenceForwardInfo] = []
        scheduled: list[Request] = []
        for req in sorted(active, key=lambda r: 0 if r.output_ids else 1):
            if budget <= 0:
                break
            chunk = min(req.total_len - req.num_computed_tokens, budget)
            budget -= chunk
            self.kv.ensure_writable_tail(req.req_id)
            start = req.num_computed_tokens
            infos.append(SequenceForwardInfo(req.req_id, len(flat), chunk,
                                             np.arange(start, start + chunk)))
            flat.extend(req.all_ids[start:start + chunk])
            scheduled.append(req)

        ids = torch.tensor(flat, dtype=torch.long)
        if self.model.device.type == "cuda":
            ids = ids.pin_memory().to(self.model.device, non_blocking=True)
        if self.cuda_graphs and self.model.timing is None and self.step_graphs().supports(infos):
            logits = self.graphs.forward(ids, infos)
        else:
            logits = self.model.forward(ids, infos, self.kv)
        tokens = logits.float().argmax(dim=-1).tolist()  # greedy, one D2H per step

        now = time.monotonic()
        for i, req in enumerate(scheduled):
            n_new = infos[i].num_tokens
            if not req.output_ids:
                self.metrics["prefill_tokens_computed"] += n_new
            req.num_computed_tokens += n_new
            if req.num_computed_tokens < req.total_len:
                continue  # chunked prefill / recompute still running
            tok = int(tokens[i])
            req.output_ids.append(tok)
            self.metrics["tokens_generated"] += 1
            if req.first_token_at is None:
                req.first_token_at = now
            if tok in self.eos_ids:
                self._finish(req, "stop")
            elif len(req.output_ids) >= req.max_new_tokens:
                self._finish(req, "length")
        self.running = [r for r in self.running if r.state is RequestState.RUNNING]
