"""Block-aligned prefix cache over token ids (host side, ref-count pinned LRU).

Same policy as the reference's RadixCache (mini_engine/paged/radix_cache.py:
35-174), kept host-side as the north star asks: an edge holds whole
16-token blocks only; a lookup returns the longest block-aligned match; an
insert splits an edge at a block boundary; eviction releases least recently
used leaves; the tree holds one reference on every block it points at, so a
block still used by a running sequence is only freed when that sequence
releases it.  The physical blocks it hands out are read in place by the
prefill and decode kernels.
"""

from __future__ import annotations

import time

from .block_manager import BlockManager


class _Node:
    __slots__ = ("tokens", "blocks", "children", "parent", "stamp")

    def __init__(self, tokens: list[int], blocks: list[int], parent):
        self.tokens = tokens      # token ids of the edge into this node
        self.blocks = blocks      # physical blocks holding their KV
        self.children: dict[int, _Node] = {}
        self.parent = parent
        self.stamp = time.monotonic()


def _shared_len(a: list[int], b: list[int]) -> int:
    n = 0
    for x, y in zip(a, b):
        if x != y:
            break
        n += 1
    return n


class RadixCache:
    def __init__(self, manager: BlockManager):
        self.mgr = manager
        self.block_size = manager.block_size
        self.root = _Node([], [], None)
        self.hit_tokens = 0
        self.query_tokens = 0

    def match_prefix(self, token_ids: list[int]) -> tuple[list[int], int]:
        """Longest block-aligned cached prefix: (blocks, n_tokens).  The caller
        takes references on the blocks it keeps with adopt()."""
        self.query_tokens += len(token_ids)
        bs = self.block_size
        node, rest = self.root, token_ids
        blocks: list[int] = []
        while rest:
            child = node.children.get(rest[0])
            if child is None:
                break
            n = _shared_len(child.tokens, rest)
            whole = n // bs
            if whole == 0:
                break
            blocks.extend(child.blocks[:whole])
            child.stamp = time.monotonic()
            if n < len(child.tokens):
                break  # diverges inside this edge
            node, rest = child, rest[n:]
        matched = len(blocks) * bs
        self.hit_tokens += matched
        return blocks, matched

    def adopt(self, blocks: list[int]):
        for b in blocks:
            self.mgr.incref(b)

    def insert(self, token_ids: list[int], blocks: list[int]):
        """Register the full blocks of a computed sequence; the tree takes a
        reference on every block it newly points at."""
        bs = self.block_size
        whole = len(token_ids) // bs
        tokens, blocks = token_ids[: whole * bs], blocks[:whole]
        node = self.root
        while tokens:
            child = node.children.get(tokens[0])
            if child is None:
                node.children[tokens[0]] = _Node(list(tokens), list(blocks), node)
                for b in blocks:
                    self.mgr.incref(b)
                return
            n_blk = _shared_len(child.tokens, tokens) // bs
            if n_blk == 0:
                return  # same first token but < 1 shared block: nothing aligned to add
            if n_blk * bs < len(child.tokens):
                child = self._split(child, n_blk)
            child.stamp = time.monotonic()
            node = child
            tokens, blocks = tokens[n_blk * bs:], blocks[n_blk:]

    def _split(self, node: _Node, n_blk: int) -> _Node:
        """Cut an edge after n_blk blocks; returns the new upper node."""
        cut = n_blk * self.block_size
        upper = _Node(node.tokens[:cut], node.blocks[:n_blk], node.parent)
        upper.stamp = node.stamp
        node.parent.children[node.tokens[0]] = upper
        node.tokens, node.blocks, node.parent = node.tokens[cut:], node.blocks[n_blk:], upper
        upper.children[node.tokens[0]] = node
        return upper

    def evict(self, num_blocks_needed: int) -> int:
        """Release least recently used leaves until num_blocks_needed block
        references were dropped (or nothing is left); returns the count."""
        released = 0
        while released < num_blocks_needed:
            leaves = [n for n in self._nodes() if not n.children and n is not self.root]
            if not leaves:
                break
            victim = min(leaves, key=lambda n: n.stamp)
            for b in victim.blocks:
                self.mgr.decref(b)
            released += len(victim.blocks)
            del victim.parent.children[victim.tokens[0]]
        return released

    def _nodes(self):
        stack = [self.root]
        while stack:
            n = stack.pop()
            yield n
            stack.extend(n.children.values())

    @property
    def num_tree_blocks(self) -> int:
        return sum(len(n.blocks) for n in self._nodes())
