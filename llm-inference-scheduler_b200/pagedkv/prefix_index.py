"""Block-granular prefix index over the paged pool (host side).

Config 5's conversations share a system prompt and grow turn by turn, so a
new request's leading tokens often already have KV in the pool.  This index
finds those blocks.  It is the engine's own structure, not the reference's
radix tree (mini_engine/paged/radix_cache.py, which stays the reference's
prefix cache and drives pagedkv.BlockManager unchanged):

* Granularity is one full block.  Entry i of a chain is keyed by
  (entry id of block i-1, the 16 token ids of block i), so an entry stands
  for the whole prefix that ends with its block, and a lookup is one dict
  probe per block.  Sibling prefixes that differ anywhere inside a block are
  separate entries.
* The index holds one reference (BlockManager.incref) on every block it
  names; a sequence that reuses a block takes its own reference.
* Eviction is least-recently-used over leaf entries (no indexed
  continuation), one block at a time, and only of blocks that nothing but
  the index still references: dropping an entry whose block a running
  sequence uses would free no memory, so such entries stay.  The candidate
  queue is a heap of (last use, entry id) with stale items skipped when
  popped.

The caller pins the blocks a lookup returned (incref) before it allocates,
so an eviction triggered by that allocation cannot take them.
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass

from .block_manager import BlockManager


@dataclass(eq=False)
class _Entry:
    eid: int
    key: tuple
    block: int
    parent: "_Entry | None"
    children: int = 0
    used: int = 0  # logical clock of the last lookup or publish that touched it


class BlockPrefixIndex:
    def __init__(self, manager: BlockManager):
        self.mgr = manager
        self.bs = manager.block_size
        self._by_key: dict[tuple, _Entry] = {}
        self._by_id: dict[int, _Entry] = {}
        self._leaves: list[tuple[int, int]] = []  # heap of (used, eid); stale items skipped
        self._clock = 0
        self._next_id = 0
        self.lookups = 0
        self.hit_blocks = 0

    def __len__(self) -> int:
        return len(self._by_id)

    # ---- queries -------------------------------------------------------------

    def _chunks(self, tokens: list[int], n_blocks: int):
        bs = self.bs
        for i in range(n_blocks):
            yield tuple(tokens[i * bs:(i + 1) * bs])

    def lookup(self, tokens: list[int]) -> list[int]:
        """Blocks holding the longest indexed run of tokens' full blocks, in
        order (possibly empty).  Marks the matched chain as used now."""
        self._clock += 1
        self.lookups += 1
        parent_id, found = None, []
        for chunk in self._chunks(tokens, len(tokens) // self.bs):
            e = self._by_key.get((parent_id, chunk))
            if e is None:
                break
            self._touch(e)
            found.append(e.block)
            parent_id = e.eid
        self.hit_blocks += len(found)
        return found

    # ---- updates -------------------------------------------------------------

    def publish(self, tokens: list[int], blocks: list[int]) -> int:
        """Index the full blocks of a sequence whose first len(tokens) tokens
        have KV in `blocks` (blocks[i] holds tokens [16 i, 16 i + 16)).  A
        prefix already indexed keeps its block; new entries take a reference
        on theirs.  Returns the number of entries added."""
        self._clock += 1
        n = min(len(tokens) // self.bs, len(blocks))
        parent, added = None, 0
        for i, chunk in enumerate(self._chunks(tokens, n)):
            key = (None if parent is None else parent.eid, chunk)
            e = self._by_key.get(key)
            if e is None:
                e = _Entry(self._next_id, key, blocks[i], parent)
                self._next_id += 1
                self.mgr.incref(blocks[i])
                self._by_key[key] = e
                self._by_id[e.eid] = e
                if parent is not None:
                    parent.children += 1
                added += 1
            self._touch(e)
            parent = e
        return added

    def reclaim(self, n_blocks: int) -> int:
        """Drop least-recently-used leaf entries whose block only the index
        holds until n_blocks blocks went back to the free list (or no such
        entry is left).  Returns the number freed."""
        freed, kept = 0, []
        heap = self._leaves
        while freed < n_blocks and heap:
            used, eid = heapq.heappop(heap)
            e = self._by_id.get(eid)
            if e is None or e.children or e.used != used:
                continue  # gone, no longer a leaf, or touched since: a newer item exists
            if self.mgr.ref_count[e.block] > 1:
                kept.append((used, eid))  # a sequence still reads it: dropping frees nothing
                continue
            self._drop(e)
            freed += 1
        for item in kept:
            heapq.heappush(heap, item)
        return freed

    def clear(self) -> int:
        """Drop every entry whose block only the index holds (leaves first,
        repeatedly).  Returns the number of blocks freed."""
        return self.reclaim(len(self._by_id))

    # ---- internals -------------------------------------------------------------

    def _touch(self, e: _Entry) -> None:
        e.used = self._clock
        if not e.children:
            heapq.heappush(self._leaves, (e.used, e.eid))

    def _drop(self, e: _Entry) -> None:
        del self._by_key[e.key]
        del self._by_id[e.eid]
        self.mgr.decref(e.block)
        p = e.parent
        if p is not None:
            p.children -= 1
            if not p.children:  # the parent is a leaf again, with its own last use
                heapq.heappush(self._leaves, (p.used, p.eid))
