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
    """Block pools in HBM plus the reference's host-side allocator.

    dtype=torch.float8_e4m3fn keeps fp8 e4m3 pools (no counterpart in the
    reference): k_cache / v_cache hold the bytes (uint8) and k_scale_cache /
    v_scale_cache [L, NB, block_size, n_kv_heads] one fp32 scale per (slot,
    KV head) row; copy_block copies both.
    """

    def __init__(self, num_blocks: int, block_size: int, num_layers: int, num_kv_heads: int,
                 head_dim: int, device="cuda", dtype=torch.float16):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.fp8 = dtype == torch.float8_e4m3fn
        self.k_scale_cache = self.v_scale_cache = None
        self.k_scale = self.v_scale = None
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
            shape = (num_layers, num_blocks, block_size, num_kv_heads, head_dim)
            if self.fp8:
                pool_dt = torch.uint8
                sshape = shape[:-1]
                self.k_scale_cache = torch.zeros(sshape, device=self.device, dtype=torch.float32)
                self.v_scale_cache = torch.zeros(sshape, device=self.device, dtype=torch.float32)
                self.k_scale = [self.k_scale_cache[layer] for layer in range(num_layers)]
                self.v_scale = [self.v_scale_cache[layer] for layer in range(num_layers)]
            else:
                ops.dtype_code(dtype)
                pool_dt = dtype
            self.k_cache = torch.zeros(shape, device=self.device, dtype=pool_dt)
            self.v_cache = torch.zeros(shape, device=self.device, dtype=pool_dt)
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
        esize = 1 if self.fp8 else torch.tensor([], dtype=self.dtype).element_size()
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
        if self.fp8:  # the rows' scales travel with their bytes
            ops.copy_blocks(self.k_scale_cache, self.v_scale_cache, dev, self.err)
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
    decode_plan: ops.DecodeAppendPlan | None = None  # built by the first forward_layer
    layers_plan: ops.DecodeAppendLayersPlan | None = None  # built by the first forward_layers
    decode_plain_plan: ops.DecodePlan | None = None   # built by the first forward_layer_qkv
    decode_schedule: torch.Tensor | None = None       # the step's decode schedule (first layer)
    rope_plan: ops.RopePlan | None = None             # built by the first forward_layer_qkv
    prefill_plan: ops.PrefillPlan | None = None       # built by the first prefill layer

    @property
    def n_seqs(self) -> int:
        return len(self.seq_ids)


class _TableMirror:
    """Host int32 copy of the live block tables: one zero-padded row per
    sequence in a 2-D buffer, so that a step's table matrix and decode slots
    are single vectorised gathers instead of per-sequence list conversions.

    A row follows its Python list by length: entries appended since the last
    step are copied in; a list replaced by a new object, one that shrank, or
    one whose last entry disagrees with the row is copied in full.  Entries
    rewritten in place other than the last must go through
    PagedKVCache.ensure_writable_tail (which updates the row) or a new
    add_sequence."""

    def __init__(self):
        self.buf = np.zeros((64, 64), dtype=np.int32)
        self.state: dict[int, list] = {}  # seq_id -> [row, synced length, list object, last entry]
        self.free_rows: list[int] = []
        self.next_row = 0

    def _fit(self, rows: int, cols: int):
        r, c = self.buf.shape
        if rows > r or cols > c:
            nb = np.zeros((max(r, 1 << (rows - 1).bit_length()), max(c, 1 << (cols - 1).bit_length())),
                          dtype=np.int32)
            nb[:r, :c] = self.buf
            self.buf = nb

    def add(self, seq_id: int, table: list[int]):
        if seq_id in self.state:
            self.remove(seq_id)
        if self.free_rows:
            row = self.free_rows.pop()
        else:
            row = self.next_row
            self.next_row += 1
            self._fit(row + 1, 1)
        self.state[seq_id] = [row, 0, table, None]

    def remove(self, seq_id: int):
        st = self.state.pop(seq_id, None)
        if st is not None:
            self.buf[st[0], : st[1]] = 0
            self.free_rows.append(st[0])

    def set(self, seq_id: int, idx: int, block: int):
        st = self.state.get(seq_id)
        if st is not None and idx < st[1]:
            self.buf[st[0], idx] = block
            if idx == st[1] - 1:
                st[3] = block

    def resync(self, st: list, table: list[int]):
        row, k = st[0], st[1]
        n = len(table)
        self._fit(row + 1, n)
        self.buf[row, :k] = 0
        self.buf[row, :n] = table
        st[1], st[2], st[3] = n, table, (table[-1] if n else None)

class PagedKVCache:
    """The model-facing adapter: same append_and_fetch contract as the
    reference's ContiguousKVCache / PagedKVCache, plus the batched
    prepare_step / forward_layer path that the paged model uses.

    Block tables are the caller's lists (the reference's contract).  A live
    sequence's table grows by appending; copy-on-write replaces its tail
    block through ensure_writable_tail; any other rewrite of an existing entry
    is followed by add_sequence (the reference scheduler does exactly this)."""

    def __init__(self, manager: BlockManager):
        self.mgr = manager
        self.block_tables: dict[int, list[int]] = {}
        self._len: dict[int, int] = {}
        self._workspace: torch.Tensor | None = None
        self._schedule_buf: torch.Tensor | None = None
        self._fp8_scratch: torch.Tensor | None = None
        self._mirror = _TableMirror()
        self._stage_ring: list = [[None, None] for _ in range(4)]
        self._stage_next = 0

    def add_sequence(self, seq_id: int, block_table: list[int], num_cached_tokens: int):
        """num_cached_tokens = tokens already present via prefix-cache reuse."""
        self.block_tables[seq_id] = block_table
        self._len[seq_id] = num_cached_tokens
        self._mirror.add(seq_id, block_table)

    def free_sequence(self, seq_id: int):
        self.block_tables.pop(seq_id, None)
        self._len.pop(seq_id, None)
        self._mirror.remove(seq_id)

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
                self._mirror.set(seq_id, idx, table[idx])
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
            if mgr.fp8:
                ops.reshape_and_cache_fp8(k_new, v_new, mgr.k_pool[layer], mgr.v_pool[layer],
                                          mgr.k_scale[layer], mgr.v_scale[layer], slots, mgr.err)
            else:
                ops.reshape_and_cache(k_new.to(mgr.dtype), v_new.to(mgr.dtype), mgr.k_pool[layer],
                                      mgr.v_pool[layer], slots, mgr.err)
        if layer == mgr.num_layers - 1:
            self._len[seq_id] = total
        used = (total + bs - 1) // bs
        idx = torch.tensor(table[:used], device=mgr.device, dtype=torch.long)
        k = mgr.k_pool[layer][idx].reshape(used * bs, *k_new.shape[1:])[:total]
        v = mgr.v_pool[layer][idx].reshape(used * bs, *v_new.shape[1:])[:total]
        if mgr.fp8:  # dequantised, in the dtype of the new rows
            ks = mgr.k_scale[layer][idx].reshape(used * bs, -1, 1)[:total]
            vs = mgr.v_scale[layer][idx].reshape(used * bs, -1, 1)[:total]
            k = (k.view(torch.float8_e4m3fn).float() * ks).to(k_new.dtype)
            v = (v.view(torch.float8_e4m3fn).float() * vs).to(v_new.dtype)
        return k, v, num_prior

    # ---- batched hot path ---------------------------------------------------

    def step_arrays(self, seqs: list[tuple[int, int]], out=None, width: int | None = None,
                    pad_to: int | None = None) -> dict:
        """Host half of prepare_step (no device work): numpy arrays of the step.

        Returns dict(ints=int32 [B*W + 2B + n_prefill + 1] = block tables (B x W;
        row s holds the sequence's first ceil(len/16) blocks, the entries after
        them are unspecified) | context lens | num_prior | prefill query_start_loc,
        slots=int64 [T], plus the scalar fields of StepMetadata).  With
        out(n_ints, n_slots) -> (int32 array, int64 array), the two arrays are
        written into the buffers it returns (prepare_step: its pinned staging
        buffer) instead of fresh ones.

        width fixes W (AssertionError if a sequence needs more blocks).
        pad_to (decode-only steps) lays the arrays out for pad_to >= B rows:
        the rows past B are padding, context length 0, slot -1 and an all-zero
        table row, which the kernels skip (a CUDA-graph step of fixed shape).
        """
        bs = self.mgr.block_size
        B = len(seqs)
        seq_ids = [s for s, _ in seqs]
        mirror, tables, lens = self._mirror, self.block_tables, self._len
        rows, n_blocks, prior = [0] * B, [0] * B, [0] * B
        state, buf = mirror.state, mirror.buf
        for i, s_id in enumerate(seq_ids):
            st = state[s_id]
            table = tables[s_id]
            n, k = len(table), st[1]
            if table is not st[2] or n < k or (n == k and n and table[-1] != st[3]):
                mirror.resync(st, table)
                buf = mirror.buf
            elif n > k:
                mirror._fit(st[0] + 1, n)
                buf = mirror.buf
                buf[st[0], k:n] = table[k:]
                st[1], st[3] = n, table[-1]
            rows[i], n_blocks[i], prior[i] = st[0], n, lens[s_id]
        rows = np.asarray(rows, dtype=np.int64)
        num_new = np.fromiter((n for _, n in seqs), dtype=np.int64, count=B)
        num_prior = np.asarray(prior, dtype=np.int64)
        n_blocks = np.asarray(n_blocks, dtype=np.int64)
        totals = num_prior + num_new
        bad = np.nonzero(totals > n_blocks * bs)[0]
        assert not len(bad), (f"seq {seq_ids[bad[0]]}: {totals[bad[0]]} tokens but only "
                              f"{n_blocks[bad[0]]} blocks allocated")
        used = (totals + bs - 1) // bs
        W = max(1, int(used.max(initial=1)))
        if width is not None:
            assert W <= width, f"a sequence needs {W} blocks, more than the fixed width {width}"
            W = width
        ones = num_new == 1
        n_dec = B if ones.all() else int(np.argmin(ones))
        pre_new = num_new[n_dec:]
        n_pre = B - n_dec
        T = int(num_new.sum())
        R = B if pad_to is None else pad_to  # rows of the layout
        assert R >= B and (R == B or n_pre == 0), "pad_to is for decode-only steps of <= pad_to rows"
        n_ints = R * W + 2 * R + n_pre + 1
        if out is None:
            ints, slots = np.empty(n_ints, dtype=np.int32), np.empty(T + R - B, dtype=np.int64)
        else:
            ints, slots = out(n_ints, T + R - B)
        tabs = ints[: R * W].reshape(R, W)
        mirror._fit(1, W)
        # entries past a sequence's used blocks are left as the mirror holds
        # them (allocated-ahead block ids or zeros): no kernel reads them
        np.take(mirror.buf[:, :W], rows, axis=0, out=tabs[:B])
        ints[R * W: R * W + B] = totals
        ints[R * W + R: R * W + R + B] = num_prior
        if R > B:
            tabs[B:] = 0
            ints[R * W + B: R * W + R] = 0
            ints[R * W + R + B: R * W + 2 * R] = 0
            slots[T:] = -1
        ints[R * W + 2 * R] = 0
        if n_pre:
            ints[R * W + 2 * R + 1:] = np.cumsum(pre_new)
        # decode sequences: one slot each, gathered in one step
        pos = num_prior[:n_dec]
        slots[:n_dec] = mirror.buf[rows[:n_dec], pos // bs].astype(np.int64) * bs + pos % bs
        o = n_dec
        for i in range(n_dec, B):
            n = int(num_new[i])
            pos = np.arange(num_prior[i], num_prior[i] + n, dtype=np.int64)
            slots[o:o + n] = mirror.buf[rows[i], pos // bs].astype(np.int64) * bs + pos % bs
            o += n
        return dict(ints=ints, slots=slots, seq_ids=seq_ids, num_new=num_new.tolist(),
                    num_prior=num_prior.tolist(), n_tokens=T, n_decode=n_dec,
                    max_query_len=int(pre_new.max(initial=0)), B=B, W=W, R=R)

    def _staging(self, nbytes: int) -> torch.Tensor:
        """A pinned host buffer of >= nbytes from a small ring; waits (normally
        not at all) until the copy last issued from that buffer has finished."""
        ring = self._stage_ring
        i = self._stage_next = (self._stage_next + 1) % len(ring)
        buf, ev = ring[i]
        if ev is not None:
            ev.synchronize()
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 16, 2 * (0 if buf is None else buf.numel())),
                              dtype=torch.uint8).pin_memory()
        ring[i] = [buf, None]
        return i, buf

    def prepare_step(self, seqs: list[tuple[int, int]]) -> StepMetadata:
        """Build the device metadata of a step with one host-to-device copy:
        the int32 arrays and the int64 slot mapping packed in one pinned
        staging buffer.  seqs = [(seq_id, num_new)] in flat-batch order.
        Flushes queued COW copies."""
        self.mgr.flush_copies()
        dev = self.mgr.device
        staged = []

        def into_staging(n_ints: int, n_slots: int):
            # int32 arrays first, then the int64 slots 16-byte aligned
            off = (4 * n_ints + 15) // 16 * 16
            i, stage = self._staging(off + 8 * n_slots)
            host = stage.numpy()
            staged.append((i, stage, off, off + 8 * n_slots))
            return host[: 4 * n_ints].view(np.int32), host[off: off + 8 * n_slots].view(np.int64)

        a = self.step_arrays(seqs, out=into_staging if dev.type == "cuda" else None)
        B, W = a["B"], a["W"]
        ints, slots = a["ints"], a["slots"]
        n_int = ints.nbytes
        off = (n_int + 15) // 16 * 16  # the slots start 16-byte aligned
        nbytes = off + slots.nbytes
        if dev.type == "cuda":
            i, stage, _, _ = staged[0]
            dbuf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            dbuf.copy_(stage[:nbytes], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(dev))
            self._stage_ring[i][1] = ev
        else:
            dbuf = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            dbuf[:n_int] = torch.from_numpy(ints.view(np.uint8))
            dbuf[off:nbytes] = torch.from_numpy(slots.view(np.uint8))
        ints_d = dbuf[:n_int].view(torch.int32)
        return StepMetadata(
            seq_ids=a["seq_ids"], num_new=a["num_new"], num_prior=a["num_prior"],
            n_tokens=a["n_tokens"], n_decode=a["n_decode"], max_query_len=a["max_query_len"],
            slot_mapping=dbuf[off:nbytes].view(torch.int64),
            block_tables=ints_d[: B * W].view(B, W),
            context_lens=ints_d[B * W: B * W + B],
            num_prior_dev=ints_d[B * W + B: B * W + 2 * B],
            query_start_loc=ints_d[B * W + 2 * B:])

    def _step_schedule(self, meta: StepMetadata, q: torch.Tensor) -> torch.Tensor:
        """The step's decode schedule, built on its first decode layer into a
        buffer this cache reuses from step to step (stream order keeps a
        step's build behind the previous step's decode launches)."""
        if meta.decode_schedule is None:
            nd, W = meta.n_decode, meta.block_tables.shape[1]
            need = ops.decode_schedule_bytes(nd, W)
            if self._schedule_buf is None or self._schedule_buf.numel() < need:
                self._schedule_buf = ops.new_decode_schedule(nd, W, self.mgr.device)
            meta.decode_schedule = ops.build_decode_schedule(
                self._schedule_buf, meta.block_tables[:nd], meta.context_lens[:nd],
                self.mgr.num_blocks, q.shape[1], self.mgr.num_kv_heads, q.shape[2], q.dtype,
                fp8=self.mgr.fp8, err=self.mgr.err)
        return meta.decode_schedule

    def _prefill_scratch(self, meta: StepMetadata, q: torch.Tensor) -> torch.Tensor:
        """16-bit scratch pool of the fp8 tensor-core prefill, reused across
        layers and steps (stream order keeps each use behind the previous)."""
        n_pre = meta.n_seqs - meta.n_decode
        need = ops.prefill_fp8_scratch_bytes(n_pre, meta.block_tables.shape[1], self.mgr.num_kv_heads,
                                             q.shape[2])
        if self._fp8_scratch is None or self._fp8_scratch.numel() < need:
            self._fp8_scratch = torch.empty(need, dtype=torch.uint8, device=self.mgr.device)
        return self._fp8_scratch

    def decode_workspace(self, n_seqs: int, n_q_heads: int, head_dim: int,
                         layers: int = 1) -> torch.Tensor:
        """The cache's split-K scratch (grown on demand); layers > 1: one set
        per layer, so a multi-layer decode call chains its layers."""
        need = ops.decode_workspace_bytes(n_seqs, n_q_heads, head_dim) * max(1, layers)
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
        if mgr._pending:
            mgr.flush_copies()
        if out is None:
            out = torch.empty((meta.n_tokens,) + tuple(q.shape[1:]), dtype=q.dtype, device=q.device)
        if mgr.fp8:
            return self._forward_layer_fp8(layer, q, k_new, v_new, meta, scale, out, advance)
        nd = meta.n_decode
        plan = meta.decode_plan
        if nd == meta.n_tokens and plan is not None and plan.scale == scale:
            # a decode-only step after its first layer: one launch, no slicing
            plan(q, k_new, v_new, mgr.k_pool[layer], mgr.v_pool[layer], out)
            if advance and layer == mgr.num_layers - 1:
                self._advance(meta)
            return out
        if nd:
            # decode sequences: append fused into the decode kernel; the
            # step's plan validates once and then only swaps layer pointers
            plan = meta.decode_plan
            if plan is None or plan.scale != scale:
                ws = self.decode_workspace(nd, q.shape[1], q.shape[2])
                plan = meta.decode_plan = ops.DecodeAppendPlan(
                    meta.block_tables[:nd], meta.context_lens[:nd], scale, ws, mgr.err,
                    schedule=self._step_schedule(meta, q))
            whole = nd == meta.n_tokens
            plan(q if whole else q[:nd], k_new if whole else k_new[:nd],
                 v_new if whole else v_new[:nd], mgr.k_pool[layer], mgr.v_pool[layer],
                 out if whole else out[:nd])
        if nd < meta.n_seqs:
            ops.reshape_and_cache(k_new[nd:], v_new[nd:], mgr.k_pool[layer], mgr.v_pool[layer],
                                  meta.slot_mapping[nd:], mgr.err)
            self._prefill(layer, q, meta, scale, out)
        if advance and layer == mgr.num_layers - 1:
            self._advance(meta)
        return out

    def forward_layers(self, first_layer: int, q: torch.Tensor, k_new: torch.Tensor,
                       v_new: torch.Tensor, meta: StepMetadata, scale: float,
                       out: torch.Tensor | None = None, advance: bool = True,
                       input_ready: torch.Tensor | None = None,
                       defer_first: bool = False) -> torch.Tensor:
        """forward_layer for the n consecutive layers first_layer ..
        first_layer + n - 1 at once, with layer-major inputs: q [n, T, Hq, D],
        k_new / v_new [n, T, Hkv, D] -> out [n, T, Hq, D].  A decode-only step
        is one C call for the whole run (pkv_paged_decode_append_attention_layers,
        or _fp8_layers over fp8 pools: the fused append + decode of every
        layer, chained, then one merge launch); other steps run forward_layer
        layer by layer.  The results are those of forward_layer either way.
        input_ready (one-call form only): an int32 device tensor of one word
        per layer; layer l's kernels wait, bounded, until a copy on another
        stream has set word l nonzero after that layer's q / k_new / v_new.
        defer_first (one-call form over 16-bit pools): the run's first decode
        kernel continues the launch chain of the run enqueued just before it,
        whose layers used other split-K sets (meta.layers_plan must hold this
        run's own workspace slice)."""
        mgr = self.mgr
        n = q.shape[0]
        last = first_layer + n
        assert 0 <= first_layer and last <= mgr.num_layers, "layers outside the pools"
        if out is None:
            out = torch.empty((n, meta.n_tokens) + tuple(q.shape[2:]), dtype=q.dtype, device=q.device)
        if mgr._pending:
            mgr.flush_copies()
        nd = meta.n_decode
        if defer_first and (meta.layers_plan is None or mgr.fp8):
            raise ValueError("pagedkv: defer_first needs meta.layers_plan over this run's own "
                             "split-K sets (16-bit pools)")
        if 0 < nd == meta.n_tokens:
            plan = meta.layers_plan
            kind = ops.DecodeAppendFp8LayersPlan if mgr.fp8 else ops.DecodeAppendLayersPlan
            if plan is None or plan.scale != scale or not isinstance(plan, kind):
                ws = self.decode_workspace(nd, q.shape[2], q.shape[3], layers=mgr.num_layers)
                plan = meta.layers_plan = kind(meta.block_tables, meta.context_lens, scale, ws, mgr.err,
                                               schedule=self._step_schedule(meta, q[0]))
            if mgr.fp8:
                if input_ready is not None:
                    raise ValueError("pagedkv: input_ready serves 16-bit pools")
                plan(q, k_new, v_new, mgr.k_cache[first_layer:last], mgr.v_cache[first_layer:last],
                     mgr.k_scale_cache[first_layer:last], mgr.v_scale_cache[first_layer:last], out)
            else:
                plan(q, k_new, v_new, mgr.k_cache[first_layer:last], mgr.v_cache[first_layer:last], out,
                     input_ready=input_ready, defer_first=defer_first)
            if advance and last == mgr.num_layers:
                self._advance(meta)
            return out
        if input_ready is not None:
            raise ValueError("pagedkv: input_ready serves decode-only steps over 16-bit pools")
        for i in range(n):
            self.forward_layer(first_layer + i, q[i], k_new[i], v_new[i], meta, scale, out=out[i],
                               advance=advance)
        return out

    def _prefill(self, layer: int, q: torch.Tensor, meta: StepMetadata, scale: float,
                 out: torch.Tensor) -> None:
        """The step's chunked-prefill launch over the 16-bit pools for the rows
        after the decode sequences (arguments validated on the first layer)."""
        nd, mgr = meta.n_decode, self.mgr
        plan = meta.prefill_plan
        if plan is None or plan.scale != scale:
            plan = meta.prefill_plan = ops.PrefillPlan(
                meta.block_tables[nd:], meta.query_start_loc, meta.num_prior_dev[nd:],
                meta.max_query_len, scale, mgr.err)
        plan(q[nd:], mgr.k_pool[layer], mgr.v_pool[layer], out[nd:])

    def _advance(self, meta: StepMetadata):
        """After the last layer: the step's tokens count as cached
        (block_manager.py:133-134 semantics)."""
        for s, p, n in zip(meta.seq_ids, meta.num_prior, meta.num_new):
            self._len[s] = p + n

    def _forward_layer_fp8(self, layer, q, k_new, v_new, meta, scale, out, advance):
        """forward_layer over fp8 pools: the decode kernel quantises the decode
        tokens itself; the chunk tokens take the quantising append; then the
        chunked prefill over the fp8 pools."""
        mgr = self.mgr
        ks, vs = mgr.k_scale[layer], mgr.v_scale[layer]
        nd = meta.n_decode
        if nd:
            ws = self.decode_workspace(nd, q.shape[1], q.shape[2])
            ops.paged_decode_append_attention_fp8(
                q[:nd], k_new[:nd], v_new[:nd], mgr.k_pool[layer], mgr.v_pool[layer], ks, vs,
                meta.block_tables[:nd], meta.context_lens[:nd], scale, workspace=ws, out=out[:nd],
                err=mgr.err, schedule=self._step_schedule(meta, q))
        if nd < meta.n_seqs:
            ops.reshape_and_cache_fp8(k_new[nd:], v_new[nd:], mgr.k_pool[layer], mgr.v_pool[layer],
                                      ks, vs, meta.slot_mapping[nd:], mgr.err)
            ops.paged_prefill_attention_fp8(q[nd:], mgr.k_pool[layer], mgr.v_pool[layer], ks, vs,
                                            meta.block_tables[nd:], meta.query_start_loc,
                                            meta.num_prior_dev[nd:], meta.max_query_len, scale,
                                            out=out[nd:], err=mgr.err,
                                            scratch=self._prefill_scratch(meta, q))
        if advance and layer == mgr.num_layers - 1:
            self._advance(meta)
        return out

    def _attend_fp8(self, layer, q, meta, scale, out, advance):
        """The step's attention launches over fp8 pools whose rows are already
        appended: decode (with the step's schedule) and chunked prefill."""
        mgr = self.mgr
        ks, vs = mgr.k_scale[layer], mgr.v_scale[layer]
        nd = meta.n_decode
        if nd:
            ws = self.decode_workspace(nd, q.shape[1], q.shape[2])
            ops.paged_decode_attention_fp8(q[:nd], mgr.k_pool[layer], mgr.v_pool[layer], ks, vs,
                                           meta.block_tables[:nd], meta.context_lens[:nd], scale,
                                           workspace=ws, out=out[:nd], err=mgr.err,
                                           schedule=self._step_schedule(meta, q))
        if nd < meta.n_seqs:
            ops.paged_prefill_attention_fp8(q[nd:], mgr.k_pool[layer], mgr.v_pool[layer], ks, vs,
                                            meta.block_tables[nd:], meta.query_start_loc,
                                            meta.num_prior_dev[nd:], meta.max_query_len, scale,
                                            out=out[nd:], err=mgr.err,
                                            scratch=self._prefill_scratch(meta, q))
        if advance and layer == mgr.num_layers - 1:
            self._advance(meta)
        return out

    def forward_layer_qkv(self, layer: int, qkv: torch.Tensor, positions: torch.Tensor,
                          cos: torch.Tensor, sin: torch.Tensor, meta: StepMetadata, scale: float,
                          out: torch.Tensor | None = None, advance: bool = True) -> torch.Tensor:
        """forward_layer for the rows of the fused q|k|v projection, qkv
        [T, (Hq + 2 Hkv) D]: one launch rotates q and k at `positions` (RoPE
        tables cos/sin [max_pos, D]) and appends the rotated k and v; then the
        step's attention launches (decode without a second append, chunked
        prefill).  Returns out [T, Hq, D].  Same results as rotating q and k
        with Rope.rotate and calling forward_layer."""
        mgr = self.mgr
        if mgr._pending:
            mgr.flush_copies()
        rope = meta.rope_plan
        if rope is None or not rope.uses(positions, cos, sin):
            rope = meta.rope_plan = ops.RopePlan(positions, cos, sin, meta.slot_mapping, mgr.err)
        if mgr.fp8:  # rotated k and v quantised into the fp8 pools in the same launch
            q = rope(qkv, mgr.k_pool[layer], mgr.v_pool[layer], mgr.k_scale[layer], mgr.v_scale[layer])
            return self._attend_fp8(layer, q, meta, scale, torch.empty_like(q) if out is None else out,
                                    advance)
        q = rope(qkv, mgr.k_pool[layer], mgr.v_pool[layer])
        if out is None:
            out = torch.empty_like(q)
        nd = meta.n_decode
        if nd:
            plan = meta.decode_plain_plan
            if plan is None or plan.scale != scale:
                ws = self.decode_workspace(nd, q.shape[1], q.shape[2])
                plan = meta.decode_plain_plan = ops.DecodePlan(
                    meta.block_tables[:nd], meta.context_lens[:nd], scale, ws, mgr.err,
                    schedule=self._step_schedule(meta, q))
            whole = nd == meta.n_tokens
            plan(q if whole else q[:nd], mgr.k_pool[layer], mgr.v_pool[layer],
                 out if whole else out[:nd])
        if nd < meta.n_seqs:
            self._prefill(layer, q, meta, scale, out)
        if advance and layer == mgr.num_layers - 1:
            self._advance(meta)
        return out
