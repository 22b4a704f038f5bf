"""Block pool, ref counts, copy-on-write and the paged KV adapter, with the
pools in HBM and every data movement done by libpagedkv kernels.

Operator surface = the reference's mini_engine/paged/block_manager.py:
`BlockManager(num_blocks, block_size, num_layers, num_kv_heads, head_dim,
device, dtype)` with `.allocate/.incref/.decref/.copy_block/.num_free`,
`.k_pool[l]`, `.v_pool[l]`, `.ref_count`, `.free_list`; `PagedKVCache(mgr)`
with `.add_sequence/.free_sequence/.seq_len/.ensure_writable_tail/
.append_and_fetch` and `.block_tables`.  Names, argument meaning, the LIFO
free list, the ref-count asserts and `OutOfBlocks` behave as there
(block_manager.py:19-141), so the scheduler and the radix cache drive this
class unchanged.

What differs, and why:
* The pools are one [num_layers, num_blocks, block_size, n_kv_heads,
  head_dim] tensor per K and V on a CUDA device; `k_pool[l]` is a view of
  layer l, so `k_pool[l][block, off]` addresses the same bytes as in the
  reference.  `device=None` builds a bookkeeping-only manager (no pools) for
  host-side policy code and tests.
* `copy_block` returns the new block at once and queues the (src, dst) pair;
  all queued pairs are copied by ONE `copy_blocks` launch over every layer
  before the next kernel that touches the pool (stream order keeps the
  reference's copy-before-use semantics).  A pair that would read or
  overwrite a block of a still-queued pair flushes the queue first, so the
  batched copy equals the reference's sequential one.
* The hot path is batched: `prepare_step` builds the step's device metadata
  (slot mapping, block tables, context lengths, query offsets) once per step
  with one host-to-device copy, and `forward_layer` runs one fused
  append + decode-attention call for the leading one-token sequences and one
  append + one chunked-prefill launch for the rest,
  replacing the per-sequence append_and_fetch + gather + _attention loop of
  mini_engine/model/qwen2.py:158-166.  `append_and_fetch` keeps the
  reference's contract (gathered K/V) for callers that still attend
  themselves.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from . import ops


class OutOfBlocks(Exception):
    """Allocation failed; scheduler must preempt or wait."""


class BlockManager:
    def __init__(self, num_blocks: int, block_size: int, num_layers: int, num_kv_heads: int,
                 head_dim: int, device="cuda", dtype=torch.float16):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        if device is None:
            self.device = None
            self.k_cache = self.v_cache = None
            self.k_pool = self.v_pool = None
        else:
            self.device = torch.device(device)
            if self.device.type != "cuda":
                raise RuntimeError(
                    "pagedkv.BlockManager keeps its pools in GPU memory; pass a CUDA device "
                    "(or device=None for a bookkeeping-only manager)")
            ops.dtype_code(dtype)
            shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
            self.k_cache = torch.zeros(shape, device=self.device, dtype=dtype)
            self.v_cache = torch.zeros(shape, device=self.device, dtype=dtype)
            self.k_pool = [self.k_cache[layer] for layer in range(num_layers)]
            self.v_pool = [self.v_cache[layer] for layer in range(num_layers)]
            self.err = ops.new_error_flags(self.device)
        self.ref_count = [0] * num_blocks
        self.free_list = list(range(num_blocks - 1, -1, -1))  # pop() from the end
        self._pending: list[tuple[int, int]] = []
        self._pending_src: set[int] = set()
        self._pending_dst: set[int] = set()
        self.flushes = 0           # non-empty flushes of the COW queue
        self.copies_launched = 0   # copy_blocks launches issued by them

    @property
    def num_free(self) -> int:
        return len(self.free_list)

    @property
    def block_bytes(self) -> int:
        """Bytes of one block of one layer's K (or V) pool."""
        esize = torch.tensor([], dtype=self.dtype).element_size()
        return self.block_size * self.num_kv_heads * self.head_dim * esize

    def allocate(self) -> int:
        if not self.free_list:
            raise OutOfBlocks()
        block = self.free_list.pop()
        assert self.ref_count[block] == 0
        self.ref_count[block] = 1
        return block

    def incref(self, block: int):
        assert self.ref_count[block] > 0, f"incref on free block {block}"
        self.ref_count[block] += 1

    def decref(self, block: int):
        assert self.ref_count[block] > 0, f"decref on free block {block}"
        self.ref_count[block] -= 1
        if self.ref_count[block] == 0:
            self.free_list.append(block)

    def copy_block(self, src: int) -> int:
        """Copy-on-write: give the caller a private copy of a shared block.

        The copy of every layer's K and V block is queued and issued by
        flush_copies() (called by every pool-touching method of PagedKVCache).
        """
        dst = self.allocate()
        if dst in self._pending_src or dst in self._pending_dst or src in self._pending_dst:
            self.flush_copies()
        self._pending.append((src, dst))
        self._pending_src.add(src)
        self._pending_dst.add(dst)
        return dst

    @property
    def pending_copies(self) -> list[tuple[int, int]]:
        return list(self._pending)

    def flush_copies(self):
        """Issue every queued COW pair as one copy_blocks launch."""
        if not self._pending:
            return
        pairs = self._pending
        self._pending, self._pending_src, self._pending_dst = [], set(), set()
        self.flushes += 1
        if self.k_cache is None:
            return
        host = torch.tensor(pairs, dtype=torch.int32).pin_memory()
        dev = host.to(self.device, non_blocking=True)
        ops.copy_blocks(self.k_cache, self.v_cache, dev, self.err)
        self.copies_launched += 1

    def check_errors(self):
        """Synchronise and raise if any kernel recorded a device-side error."""
        if self.k_cache is not None:
            ops.check_flags(self.err, "BlockManager")


@dataclass
class StepMetadata:
    """Device-side description of one forward step (built once, used by every layer).

    Sequences are in flat-batch order.  The leading run of sequences with one
    new token (ongoing decodes, which the reference scheduler orders first,
    scheduler.py:242) is served by the decode kernel; every other sequence by
    the chunked-prefill kernel.
    """

    seq_ids: list[int]
    num_new: list[int]
    num_prior: list[int]
    n_tokens: int
    n_decode: int            # leading sequences with num_new == 1
    max_query_len: int       # over the prefill part
    slot_mapping: torch.Tensor      # int64 [n_tokens]
    block_tables: torch.Tensor      # int32 [B, W]
    context_lens: torch.Tensor      # int32 [B] = num_prior + num_new
    query_start_loc: torch.Tensor   # int32 [B - n_decode + 1], relative to the prefill rows
    num_prior_dev: torch.Tensor     # int32 [B]

    @property
    def n_seqs(self) -> int:
        return len(self.seq_ids)


class PagedKVCache:
    """The model-facing adapter: same append_and_fetch contract as the
    reference's ContiguousKVCache / PagedKVCache, plus the batched
    prepare_step / forward_layer path that the paged model uses."""

    def __init__(self, manager: BlockManager):
        self.mgr = manager
        self.block_tables: dict[int, list[int]] = {}
        self._len: dict[int, int] = {}
        self._workspace: torch.Tensor | None = None

    def add_sequence(self, seq_id: int, block_table: list[int], num_cached_tokens: int):
        """num_cached_tokens = tokens already present via prefix-cache reuse."""
        self.block_tables[seq_id] = block_table
        self._len[seq_id] = num_cached_tokens

    def free_sequence(self, seq_id: int):
        self.block_tables.pop(seq_id, None)
        self._len.pop(seq_id, None)

    def seq_len(self, seq_id: int) -> int:
        return self._len[seq_id]

    def ensure_writable_tail(self, seq_id: int):
        """COW check before a step: if the block we are about to append into
        is shared (ref > 1), replace it with a private copy."""
        length = self._len[seq_id]
        table = self.block_tables[seq_id]
        idx = length // self.mgr.block_size
        if idx < len(table) and length % self.mgr.block_size != 0:
            block = table[idx]
            if self.mgr.ref_count[block] > 1:
                table[idx] = self.mgr.copy_block(block)
                self.mgr.decref(block)

    # ---- reference contract: one sequence, one layer -----------------------

    def _slots(self, table: list[int], start: int, n: int) -> np.ndarray:
        bs = self.mgr.block_size
        pos = np.arange(start, start + n, dtype=np.int64)
        tab = np.asarray(table, dtype=np.int64)
        return tab[pos // bs] * bs + pos % bs

    def append_and_fetch(self, layer: int, seq_id: int, k_new: torch.Tensor, v_new: torch.Tensor):
        """Write k_new/v_new ([n_new, Hkv, D]) after the sequence's cached
        tokens and return (K, V, num_prior) with K/V = all of the sequence's
        keys/values for this layer.  Reference: block_manager.py:111-141."""
        mgr = self.mgr
        bs = mgr.block_size
        table = self.block_tables[seq_id]
        num_prior = self._len[seq_id]
        n_new = k_new.shape[0]
        total = num_prior + n_new
        assert total <= len(table) * bs, (
            f"seq {seq_id}: {total} tokens but only {len(table)} blocks allocated")
        mgr.flush_copies()
        if n_new:
            slots = torch.from_numpy(self._slots(table, num_prior, n_new)).to(mgr.device)
            ops.reshape_and_cache(k_new.to(mgr.dtype), v_new.to(mgr.dtype), mgr.k_pool[layer],
                                  mgr.v_pool[layer], slots, mgr.err)
        if layer == mgr.num_layers - 1:
            self._len[seq_id] = total
        used = (total + bs - 1) // bs
        idx = torch.tensor(table[:used], device=mgr.device, dtype=torch.long)
        k = mgr.k_pool[layer][idx].reshape(used * bs, *k_new.shape[1:])[:total]
        v = mgr.v_pool[layer][idx].reshape(used * bs, *v_new.shape[1:])[:total]
        return k, v, num_prior

    # ---- batched hot path ---------------------------------------------------

    def step_arrays(self, seqs: list[tuple[int, int]]) -> dict:
        """Host half of prepare_step (no device work): numpy arrays of the step.

        Returns dict(ints=int32 [B*W + 2B + n_prefill + 1] = block tables (B x W,
        zero padded) | context lens | num_prior | prefill query_start_loc,
        slots=int64 [T], plus the scalar fields of StepMetadata).
        """
        bs = self.mgr.block_size
        B = len(seqs)
        seq_ids = [s for s, _ in seqs]
        num_new = [int(n) for _, n in seqs]
        num_prior = [self._len[s] for s in seq_ids]
        totals = [p + n for p, n in zip(num_prior, num_new)]
        used = [(t + bs - 1) // bs for t in totals]
        for s, t in zip(seq_ids, totals):
            assert t <= len(self.block_tables[s]) * bs, (
                f"seq {s}: {t} tokens but only {len(self.block_tables[s])} blocks allocated")
        W = max(1, max(used, default=1))
        n_dec = 0
        while n_dec < B and num_new[n_dec] == 1:
            n_dec += 1
        pre_new = num_new[n_dec:]
        n_pre = B - n_dec
        ints = np.zeros(B * W + 2 * B + n_pre + 1, dtype=np.int32)
        tabs = ints[: B * W].reshape(B, W)
        for i, (s, u) in enumerate(zip(seq_ids, used)):
            tabs[i, :u] = self.block_tables[s][:u]
        ints[B * W: B * W + B] = totals
        ints[B * W + B: B * W + 2 * B] = num_prior
        if n_pre:
            ints[B * W + 2 * B + 1:] = np.cumsum(pre_new)
        T = sum(num_new)
        slots = np.empty(T, dtype=np.int64)
        o = 0
        for s, p, n in zip(seq_ids, num_prior, num_new):
            slots[o:o + n] = self._slots(self.block_tables[s], p, n)
            o += n
        return dict(ints=ints, slots=slots, seq_ids=seq_ids, num_new=num_new, num_prior=num_prior,
                    n_tokens=T, n_decode=n_dec, max_query_len=max(pre_new, default=0), B=B, W=W)

    def prepare_step(self, seqs: list[tuple[int, int]]) -> StepMetadata:
        """Build the device metadata of a step with one pinned host-to-device
        copy of the int32 arrays and one of the slot mapping.  seqs =
        [(seq_id, num_new)] in flat-batch order.  Flushes queued COW copies."""
        self.mgr.flush_copies()
        a = self.step_arrays(seqs)
        B, W = a["B"], a["W"]
        dev = self.mgr.device
        ints_d = torch.from_numpy(a["ints"]).pin_memory().to(dev, non_blocking=True)
        slots_d = torch.from_numpy(a["slots"]).pin_memory().to(dev, non_blocking=True)
        return StepMetadata(
            seq_ids=a["seq_ids"], num_new=a["num_new"], num_prior=a["num_prior"],
            n_tokens=a["n_tokens"], n_decode=a["n_decode"], max_query_len=a["max_query_len"],
            slot_mapping=slots_d,
            block_tables=ints_d[: B * W].view(B, W),
            context_lens=ints_d[B * W: B * W + B],
            num_prior_dev=ints_d[B * W + B: B * W + 2 * B],
            query_start_loc=ints_d[B * W + 2 * B:])

    def decode_workspace(self, n_seqs: int, n_q_heads: int, head_dim: int) -> torch.Tensor:
        need = ops.decode_workspace_bytes(n_seqs, n_q_heads, head_dim)
        if self._workspace is None or self._workspace.numel() < need:
            self._workspace = torch.empty(need, dtype=torch.uint8, device=self.mgr.device)
        return self._workspace

    def forward_layer(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                      meta: StepMetadata, scale: float, out: torch.Tensor | None = None,
                      advance: bool = True) -> torch.Tensor:
        """Append this step's K/V for `layer` and attend: q [T, Hq, D] ->
        out [T, Hq, D].  After the last layer the sequences' lengths advance
        (block_manager.py:133-134 semantics); advance=False replays a step
        without moving the lengths (benchmarks re-running one step)."""
        mgr = self.mgr
        mgr.flush_copies()
        if out is None:
            out = torch.empty((meta.n_tokens,) + tuple(q.shape[1:]), dtype=q.dtype, device=q.device)
        nd = meta.n_decode
        if nd:
            # decode sequences: append fused into the decode kernel
            ws = self.decode_workspace(nd, q.shape[1], q.shape[2])
            ops.paged_decode_append_attention(q[:nd], k_new[:nd], v_new[:nd], mgr.k_pool[layer],
                                              mgr.v_pool[layer], meta.block_tables[:nd],
                                              meta.context_lens[:nd], scale, workspace=ws,
                                              out=out[:nd], err=mgr.err)
        if nd < meta.n_seqs:
            ops.reshape_and_cache(k_new[nd:], v_new[nd:], mgr.k_pool[layer], mgr.v_pool[layer],
                                  meta.slot_mapping[nd:], mgr.err)
            ops.paged_prefill_attention(q[nd:], mgr.k_pool[layer], mgr.v_pool[layer],
                                        meta.block_tables[nd:], meta.query_start_loc,
                                        meta.num_prior_dev[nd:], meta.max_query_len, scale,
                                        out=out[nd:], err=mgr.err)
        if advance and layer == mgr.num_layers - 1:
            for s, p, n in zip(meta.seq_ids, meta.num_prior, meta.num_new):
                self._len[s] = p + n
        return out
