"""CUDA graphs of the model step (decode-only and mixed decode + prefill).

A step of the 24-layer model is about 11 launches per layer, some 270 in
all.  Issued from Python one by one they cost more host time than the GPU
spends on them (about 4 ms of host time for a step of 96 decodes and a
128-token chunk, against under 2 ms of kernels).  `StepGraphs` captures the
whole step once per padded shape and replays it: a step then costs one
host-to-device copy of its metadata, one or two small device copies of the
token ids, and one graph launch.

Shapes.  A graph is keyed (R, P):
* P = 0: a decode-only step of up to R sequences (R in `buckets`);
* P > 0: a mixed step of up to R decode sequences (R in `mixed_rows`) and up
  to `prefill_seqs` prefill sequences with up to P new tokens in all (P in
  `prefill_tokens`).  The flat batch is R decode rows, then P prefill rows.

Fixed shapes make a replay valid for any step that fits:
* the step's metadata lives in one device buffer laid out for S = R +
  prefill_seqs sequence rows and a block-table width of W blocks: tables
  [S, W] | context lens [S] | num_prior [S] | query_start_loc [prefill_seqs
  + 1] (int32), then slots [R + P], positions [R + P] and the LM-head rows
  [R + prefill_seqs] (int64).  The host fills a pinned staging copy; one copy
  moves it;
* padding decode rows have context length 0 (the decode kernel gives them no
  blocks, the merge writes zero rows) and slot -1 (the RoPE + append launch
  stores nothing); padding prefill sequences have no query rows (their
  prefill CTAs return at once); padding prefill rows belong to no sequence
  and have slot -1;
* the decode schedule is built inside the graph from that metadata, so the
  stream-K partition follows the step's real lengths; the chunked-prefill
  launch is sized for P query rows and prefill_seqs sequences, and its CTAs
  past a sequence's rows return;
* the LM head runs on the rows listed in the metadata: the decode rows, then
  each prefill sequence's last row, so the first B logits rows are the
  step's sequences in order;
* the runner owns the decode schedule, the RoPE tables (sized for W * 16
  positions) and the logits buffer; the cache's split-K workspace and fp8
  prefill scratch are sized for the largest graph before the first capture
  and held here, so a later reallocation by an eager step cannot free them
  under a graph.

Padding does not change the real rows: the attention kernels give padding
rows no keys and no output, and every other operation of the step (GEMMs,
RMSNorm, SwiGLU, the LM head) is row-independent.  The GEMMs see padded M,
so the library may pick another algorithm: logits agree with the eager step
to rounding, not bit for bit.

Graphs are captured lazily (or all at once by `capture_all`) into one
memory pool, largest first.  A step whose sequences need more than W blocks
doubles W and drops the graphs.  Replays and eager steps share the current
stream.

Reference: the step of mini_engine/scheduler.py step() +
mini_engine/model/qwen2.py forward (one Python call per sequence and layer
there).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib, ops
from .block_manager import PagedKVCache, StepMetadata
from .model import PagedQwen2Model, SequenceForwardInfo


def default_buckets(max_batch: int) -> list[int]:
    """Padded batch sizes of decode-only steps: 1, 2, 4, 8, then steps of 16
    up to 128 and of 32 beyond, and max_batch itself."""
    out = [b for b in (1, 2, 4, 8) if b < max_batch]
    b = 16
    while b < max_batch:
        out.append(b)
        b += 16 if b < 128 else 32
    out.append(max_batch)
    return sorted(set(out))


def mixed_row_buckets(max_batch: int) -> list[int]:
    """Padded decode-row counts of mixed steps: 16, 32, then steps of 32, and
    max_batch (padding decode rows cost little: no keys, and GEMM rows)."""
    out = [b for b in (16, 32) if b < max_batch]
    b = 64
    while b < max_batch:
        out.append(b)
        b += 32
    out.append(max_batch)
    return sorted(set(out))


def prefill_token_buckets(max_tokens: int) -> list[int]:
    """Padded prefill-token counts of mixed steps: 32, 64, then steps of 64,
    and max_tokens (padding rows cost GEMM work, so the steps are finer)."""
    out = [b for b in (32, 64) if b < max_tokens]
    b = 128
    while b < max_tokens:
        out.append(b)
        b += 64
    out.append(max_tokens)
    return sorted(set(out))


def graph_keys(buckets: list[int], mixed_rows: list[int], prefill_tokens: list[int],
               max_tokens: int) -> list[tuple[int, int]]:
    """Every (R, P) shape to capture: (R, 0) for the decode-only buckets, and
    (R, P) for the mixed ones that the token budget can reach (the smallest
    step of the shape, one more decode row than the bucket below and one
    more prefill token than the bucket below, fits max_tokens)."""
    out = [(R, 0) for R in buckets]
    for i, R in enumerate(mixed_rows):
        r_lo = mixed_rows[i - 1] + 1 if i else 0
        for j, P in enumerate(prefill_tokens):
            p_lo = prefill_tokens[j - 1] + 1 if j else 1
            if r_lo + p_lo <= max_tokens:
                out.append((R, P))
    return out


def _align16(n: int) -> int:
    return (n + 15) // 16 * 16


def _bucket(buckets: list[int], n: int) -> int | None:
    for b in buckets:
        if b >= n:
            return b
    return None


class StepGraphs:
    """Captured steps of `model` over `kv_cache`: decode-only steps of up to
    max_batch sequences, and (max_tokens given: the scheduler's token budget)
    mixed steps of up to max_batch decodes plus up to prefill_seqs prefill
    sequences of up to max_tokens new tokens, for contexts that fit
    max_blocks_per_seq blocks (grown by doubling when a step needs more)."""

    def __init__(self, model: PagedQwen2Model, kv_cache: PagedKVCache, max_batch: int,
                 max_tokens: int | None = None, max_blocks_per_seq: int = 64,
                 buckets: list[int] | None = None, prefill_seqs: int = 4):
        if model.device.type != "cuda":
            raise RuntimeError("pagedkv: CUDA graphs need the model on a CUDA device")
        self.model, self.kv = model, kv_cache
        self.buckets = sorted(buckets or default_buckets(max_batch))
        self.max_batch = self.buckets[-1]
        self.prefill_seqs = prefill_seqs if max_tokens else 0
        self.mixed_rows = mixed_row_buckets(self.max_batch) if max_tokens else []
        self.prefill_tokens = prefill_token_buckets(max_tokens) if max_tokens else []
        self.max_tokens = max_tokens or 0
        self.W = max(1, int(max_blocks_per_seq))
        self.graphs: dict[tuple[int, int], torch.cuda.CUDAGraph] = {}
        self.replays = 0
        self._key_set = set(self.keys())
        self._alloc()

    # ---- shapes and buffers ---------------------------------------------------

    def keys(self) -> list[tuple[int, int]]:
        return graph_keys(self.buckets, self.mixed_rows, self.prefill_tokens, self.max_tokens)

    def _layout(self, R: int, P: int) -> dict:
        """Byte offsets of an (R, P) step's metadata."""
        NP = self.prefill_seqs if P else 0
        S = R + NP
        n_ints = S * self.W + 2 * S + NP + 1
        o64 = _align16(4 * n_ints)
        T = R + P
        return dict(NP=NP, S=S, T=T, n_ints=n_ints, slots=o64, pos=o64 + 8 * T,
                    last=o64 + 16 * T, end=o64 + 16 * T + 8 * (R + NP))

    def _alloc(self) -> None:
        m, kv = self.model, self.kv
        mgr, cfg, dev = kv.mgr, m.cfg, m.device
        keys = self.keys()
        nbytes = max(self._layout(R, P)["end"] for R, P in keys)
        rows = max(R + P for R, P in keys)
        heads = max(R + self._layout(R, P)["NP"] for R, P in keys)
        self.graphs = {}
        self.pool = torch.cuda.graph_pool_handle()
        self.meta_dev = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self.stage = [[torch.empty(nbytes, dtype=torch.uint8).pin_memory(), None] for _ in range(2)]
        self._stage_next = 0
        self.ids = torch.zeros(rows, dtype=torch.long, device=dev)
        self.logits = torch.empty((heads, cfg.vocab_size), dtype=m.dtype, device=dev)
        Rm = max(R for R, _ in keys)
        self.schedule = ops.new_decode_schedule(Rm, self.W, dev)
        self.workspace = kv.decode_workspace(Rm, cfg.num_attention_heads, cfg.head_dim)
        self.scratch = None
        if mgr.fp8 and self.prefill_seqs:
            need = ops.prefill_fp8_scratch_bytes(self.prefill_seqs, self.W, mgr.num_kv_heads,
                                                 cfg.head_dim)
            if kv._fp8_scratch is None or kv._fp8_scratch.numel() < need:
                kv._fp8_scratch = torch.empty(need, dtype=torch.uint8, device=dev)
            self.scratch = kv._fp8_scratch
        cos, sin = m.rope.tables(self.W * mgr.block_size)
        self.cos, self.sin = cos, sin  # held: an eager step that grows the tables drops them

    def _views(self, R: int, P: int) -> dict:
        L, W, buf = self._layout(R, P), self.W, self.meta_dev
        S, NP, T = L["S"], L["NP"], L["T"]
        ints = buf[: 4 * L["n_ints"]].view(torch.int32)
        return dict(tables=ints[: S * W].view(S, W), ctx=ints[S * W: S * W + S],
                    prior=ints[S * W + S: S * W + 2 * S], qsl=ints[S * W + 2 * S:],
                    slots=buf[L["slots"]: L["slots"] + 8 * T].view(torch.int64),
                    positions=buf[L["pos"]: L["pos"] + 8 * T].view(torch.int64),
                    last=buf[L["last"]: L["last"] + 8 * (R + NP)].view(torch.int64))

    def _meta(self, R: int, P: int) -> StepMetadata:
        v, S = self._views(R, P), self._layout(R, P)["S"]
        return StepMetadata(seq_ids=list(range(S)), num_new=[1] * S, num_prior=[0] * S,
                            n_tokens=R + P, n_decode=R, max_query_len=P, slot_mapping=v["slots"],
                            block_tables=v["tables"], context_lens=v["ctx"],
                            query_start_loc=v["qsl"], num_prior_dev=v["prior"])

    # ---- the captured step -------------------------------------------------

    def _step(self, R: int, P: int) -> None:
        """The step over the (R, P) metadata (what a graph holds)."""
        m, kv = self.model, self.kv
        mgr, cfg = kv.mgr, m.cfg
        meta = self._meta(R, P)
        v = self._views(R, P)
        pos = v["positions"]
        meta.decode_schedule = ops.build_decode_schedule(
            self.schedule, meta.block_tables[:R], meta.context_lens[:R], mgr.num_blocks,
            cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, m.dtype,
            fp8=mgr.fp8, err=mgr.err)
        rot = None
        if not m.fused_rope:
            rot = (self.cos[pos].unsqueeze(1), self.sin[pos].unsqueeze(1))
        h = m._layers(m.embed[self.ids[:R + P]], pos, self.cos, self.sin, rot, meta, kv, advance=False)
        if P:
            h = h[v["last"]]
        h = torch.nn.functional.rms_norm(h, (cfg.hidden_size,), m.final_norm, cfg.rms_norm_eps)
        torch.mm(h, m.embed.t(), out=self.logits[:h.shape[0]])

    def capture(self, R: int, P: int = 0) -> None:
        """Capture the (R, P) step.  Runs it once uncaptured first, on
        all-padding metadata, which reads and writes no KV."""
        if (R, P) not in self._key_set:
            raise ValueError(f"pagedkv: ({R}, {P}) is not a captured shape of this runner")
        self.kv.mgr.flush_copies()
        v = self._views(R, P)
        cur = torch.cuda.current_stream(self.model.device)
        # all rows padding: zero tables / lengths / positions / query starts /
        # LM-head rows, slots -1
        self.meta_dev.zero_()
        v["slots"].fill_(-1)
        side = torch.cuda.Stream(self.model.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            self._step(R, P)  # library handles, kernel attributes, argument caches
        cur.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool, capture_error_mode="thread_local"):
            self._step(R, P)
        self.graphs[(R, P)] = g

    def capture_all(self) -> None:
        for key in sorted(self._key_set, key=lambda k: -(k[0] + k[1])):
            if key not in self.graphs:
                self.capture(*key)

    # ---- a step -------------------------------------------------------------

    def shape_of(self, seq_infos: list[SequenceForwardInfo]) -> tuple[int, int] | None:
        """The (R, P) graph that serves this step (decode sequences first, as
        the scheduler orders them), or None if none does."""
        B = len(seq_infos)
        nd = 0
        while nd < B and seq_infos[nd].num_tokens == 1:
            nd += 1
        if nd == B:
            R = _bucket(self.buckets, B)
            return None if R is None or B == 0 else (R, 0)
        if B - nd > self.prefill_seqs:
            return None
        R = _bucket(self.mixed_rows, nd)
        P = _bucket(self.prefill_tokens, sum(s.num_tokens for s in seq_infos[nd:]))
        if R is None or P is None or (R, P) not in self._key_set:
            return None
        return R, P

    def supports(self, seq_infos: list[SequenceForwardInfo]) -> bool:
        return self.shape_of(seq_infos) is not None

    def forward(self, input_ids: torch.Tensor, seq_infos: list[SequenceForwardInfo]) -> torch.Tensor:
        """PagedQwen2Model.forward by graph replay, for a step that `supports`.

        input_ids [T] on the device (flat: the decode tokens, then each
        prefill sequence's chunk).  Returns the logits [B, vocab] of each
        sequence's last new token as a view of the runner's buffer, valid
        until the next replay.  The sequences' lengths advance as after an
        eager step."""
        kv, bs = self.kv, self.kv.mgr.block_size
        shape = self.shape_of(seq_infos)
        if shape is None:
            raise ValueError("pagedkv: StepGraphs.forward: no captured shape serves this step")
        need = max((kv._len[s.seq_id] + s.num_tokens + bs - 1) // bs for s in seq_infos)
        if need > self.W:
            w = self.W
            while w < need:
                w *= 2
            self.W = w
            self._alloc()
        R, P = shape
        if shape not in self.graphs:
            self.capture(R, P)
        kv.mgr.flush_copies()
        i = self._stage_next = (self._stage_next + 1) % len(self.stage)
        host, ev = self.stage[i]
        if ev is not None:
            ev.synchronize()
        hnp = host.numpy()
        L = self._layout(R, P)
        B = len(seq_infos)
        seqs = [(s.seq_id, s.num_tokens) for s in seq_infos]
        if P == 0:
            def into(n_ints: int, n_slots: int):
                return (hnp[: 4 * n_ints].view(np.int32),
                        hnp[L["slots"]: L["slots"] + 8 * n_slots].view(np.int64))

            a = kv.step_arrays(seqs, out=into, width=self.W, pad_to=R)
            pos = hnp[L["pos"]: L["pos"] + 8 * R].view(np.int64)
            pos[:B] = [int(s.positions[0]) for s in seq_infos]
            pos[B:] = 0
        else:
            a = kv.step_arrays(seqs, width=self.W)
            self._lay_mixed(hnp, L, R, a, seq_infos)
        self.meta_dev[: L["end"]].copy_(host[: L["end"]], non_blocking=True)
        cur = torch.cuda.current_stream(self.model.device)
        ev = torch.cuda.Event()
        ev.record(cur)
        self.stage[i][1] = ev
        nd = a["n_decode"]
        if P == 0:
            self.ids[:B].copy_(input_ids, non_blocking=True)
        else:
            if nd:
                self.ids[:nd].copy_(input_ids[:nd], non_blocking=True)
            self.ids[R: R + input_ids.shape[0] - nd].copy_(input_ids[nd:], non_blocking=True)
        self.graphs[shape].replay()
        self.replays += 1
        for s_id, p, n in zip(a["seq_ids"], a["num_prior"], a["num_new"]):
            kv._len[s_id] = p + n
        return self.logits[:B]

    def _lay_mixed(self, hnp, L, R, a, seq_infos) -> None:
        """Write step_arrays' unpadded arrays into the staging buffer in the
        (R, P) layout: decode rows 0..nd-1 then padding up to R, prefill
        sequences R..R+n_pre-1 then empty ones; tokens likewise."""
        W, S, NP = self.W, L["S"], L["NP"]
        B, nd = a["B"], a["n_decode"]
        n_pre = B - nd
        src = a["ints"]
        ints = hnp[: 4 * L["n_ints"]].view(np.int32)
        tabs = ints[: S * W].reshape(S, W)
        stabs = src[: B * W].reshape(B, W)
        tabs[:nd] = stabs[:nd]
        tabs[nd:R] = 0
        tabs[R: R + n_pre] = stabs[nd:]
        tabs[R + n_pre:] = 0
        for k, off in ((0, S * W), (1, S * W + S)):  # context lens, num_prior
            col = src[B * W + k * B: B * W + (k + 1) * B]
            dst = ints[off: off + S]
            dst[:nd] = col[:nd]
            dst[nd:R] = 0
            dst[R: R + n_pre] = col[nd:]
            dst[R + n_pre:] = 0
        qsl = src[B * W + 2 * B:]  # n_pre + 1 entries, qsl[0] = 0
        dq = ints[S * W + 2 * S: S * W + 2 * S + NP + 1]
        dq[: n_pre + 1] = qsl
        dq[n_pre + 1:] = qsl[-1]
        t_pre = int(qsl[-1])
        sl = a["slots"]
        slots = hnp[L["slots"]: L["slots"] + 8 * L["T"]].view(np.int64)
        slots[:nd] = sl[:nd]
        slots[nd:R] = -1
        slots[R: R + t_pre] = sl[nd:]
        slots[R + t_pre:] = -1
        pos = hnp[L["pos"]: L["pos"] + 8 * L["T"]].view(np.int64)
        pos[:nd] = [int(s.positions[0]) for s in seq_infos[:nd]]
        pos[nd:R] = 0
        pos[R: R + t_pre] = np.concatenate([s.positions for s in seq_infos[nd:]])
        pos[R + t_pre:] = 0
        last = hnp[L["last"]: L["last"] + 8 * (R + NP)].view(np.int64)
        last[:nd] = np.arange(nd)
        last[nd: nd + n_pre] = R + qsl[1:] - 1
        last[nd + n_pre:] = 0


DecodeGraphs = StepGraphs  # decode-only use: StepGraphs(model, kv, max_batch)


class DecodeStepGraph:
    """A decode-only step over every layer of a cache's pools, fed from and
    returned to caller-owned pinned host buffers, captured as one CUDA graph.

    For hosts that hold one step's q / new K / new V of every layer together,
    as layer-major rows host_qkv [L, R, Hq + 2 Hkv, D] (pinned), and want every
    layer's attention output back in host_out [L, R, Hq, D] (pinned).  Issued
    from Python one by one, such a step is about 100 launches, copies and
    event operations, which cost more host time than the GPU spends on them.
    Here the host builds the step's metadata (PagedKVCache.step_arrays into a
    pinned staging buffer, padded to R rows), copies it with one H2D copy and
    launches one graph holding:
    * the decode schedule build;
    * on a copy stream, the H2D copies of the rows (copy_chunks: one layer,
      then three, then four at a time), each followed by one copy that sets
      its layers' ready words (cleared at the step's start);
    * per chunk of layers, one pkv_paged_decode_append_attention_layers call
      with a split-K set per layer: the layers' decode kernels chain (each
      later one starts on the SMs the previous one's tail frees) and one merge
      launch follows them.  Every layer of the step has its own set, so a
      chunk's first decode continues the chain too (PKV_LAYERS_DEFER_FIRST):
      it starts beside the previous chunk's merge instead of after it.  Each layer's kernels wait, bounded, for its ready
      word before reading its rows.  An event wait on the copy stream would
      instead end the programmatic overlap between two launches (about 5 us
      each); the ready words keep the step one launch chain;
    * per chunk, on a second copy stream, the D2H copy of the chunk's outputs
      once its merge is done.
    The pipeline's fill is one layer's copy in; the drain is the last chunk's
    copy out, so the default chunks taper at the end (ready_chunks).  Where
    the tensor-core decode does not serve the shapes (the ready words are
    then refused), chunks wait on copy events instead, in event_chunks'
    sizes unless chunks were given.

    A step of B <= R sequences (one new token each, host rows 0 .. B-1) pads
    rows B .. R-1: context length 0, slot -1, so they read and write no KV
    and their outputs are zeros.  The block-table width W is fixed at capture
    and doubled (with a new capture) when a step needs more.  With
    advance=True the sequences' lengths advance as after forward_layer's last
    layer (block_manager.py:133-134 semantics).  Results equal
    PagedKVCache.forward_layers over the same rows bit for bit.
    Reference: the per-layer loop of Qwen2Model.forward (qwen2.py:159-166)
    over PagedKVCache.append_and_fetch + _attention, for decode steps.
    """

    def __init__(self, kv_cache: PagedKVCache, host_qkv: torch.Tensor, host_out: torch.Tensor,
                 scale: float, chunks: tuple[int, ...] | None = None, max_blocks_per_seq: int = 64):
        mgr = kv_cache.mgr
        if mgr.fp8 or mgr.device is None or mgr.device.type != "cuda":
            raise RuntimeError("pagedkv: DecodeStepGraph serves 16-bit pools on a CUDA device")
        L, R, width, D = host_qkv.shape
        hkv = mgr.num_kv_heads
        hq = width - 2 * hkv
        if L != mgr.num_layers or D != mgr.head_dim or hq <= 0 or host_qkv.dtype != mgr.dtype:
            raise ValueError("pagedkv: host_qkv must be [num_layers, rows, Hq + 2 Hkv, head_dim] "
                             "in the pool dtype")
        if tuple(host_out.shape) != (L, R, hq, D) or host_out.dtype != mgr.dtype:
            raise ValueError("pagedkv: host_out must be [num_layers, rows, Hq, head_dim]")
        if not (host_qkv.is_pinned() and host_out.is_pinned() and host_qkv.is_contiguous()
                and host_out.is_contiguous()):
            raise ValueError("pagedkv: host_qkv / host_out must be contiguous pinned host tensors")
        self._chunks_given = chunks is not None
        # input copies of about 2.4 MB (4 layers at config 3); compute chunks
        # taper towards the end (ready_chunks)
        esz = host_qkv.element_size()
        chunks = tuple(chunks or ready_chunks(L))
        if sum(chunks) != L or min(chunks) <= 0:
            raise ValueError(f"pagedkv: chunks {chunks} must be positive and sum to {L}")
        self.kv, self.scale = kv_cache, float(scale)
        self.host_qkv, self.host_out = host_qkv, host_out
        self.R, self.hq, self.L = R, hq, L
        self.bounds = [(sum(chunks[:i]), sum(chunks[:i + 1])) for i in range(len(chunks))]
        self.W = max(1, int(max_blocks_per_seq))
        self.graph: torch.cuda.CUDAGraph | None = None
        self.replays = 0
        dev = mgr.device
        self.dev_qkv = torch.empty((L, R, width, D), dtype=mgr.dtype, device=dev)
        self.dev_out = torch.empty((L, R, hq, D), dtype=mgr.dtype, device=dev)
        self.h2d, self.d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        # one split-K set per layer of the step: a chunk's layers chain, and a
        # chunk's first layer continues the chain of the chunk before it
        # (PKV_LAYERS_DEFER_FIRST), whose merge may still read its own sets
        self.ws1 = ops.decode_workspace_bytes(R, hq, D)
        self.workspace = kv_cache.decode_workspace(R, hq, D, layers=L)
        # per layer: nonzero once its rows are on the device (set by the copy stream)
        self.ready = torch.zeros(L, dtype=torch.int32, device=dev)
        self._ones = torch.ones(L, dtype=torch.int32).pin_memory()
        # the input copies (each followed by one copy of its layers' ready
        # words): one layer first, so compute starts after one layer's copy,
        # then larger copies (every copy costs the copy engine a fixed time)
        cc = copy_chunks(L, pieces_for(L, R * width * D * esz, 2_400_000))
        self.copy_bounds = [(sum(cc[:i]), sum(cc[:i + 1])) for i in range(len(cc))]
        self.gated = True
        self._alloc()

    def _layout(self) -> dict:
        R, W = self.R, self.W
        n_ints = R * W + 2 * R + 1
        o64 = _align16(4 * n_ints)
        return dict(n_ints=n_ints, slots=o64, end=o64 + 8 * R)

    def _alloc(self) -> None:
        dev = self.kv.mgr.device
        end = self._layout()["end"]
        self.meta_dev = torch.zeros(end, dtype=torch.uint8, device=dev)
        self.stage = [[torch.empty(end, dtype=torch.uint8).pin_memory(), None] for _ in range(2)]
        self._stage_next = 0
        self.schedule = ops.new_decode_schedule(self.R, self.W, dev)
        self.graph = None

    def _meta(self) -> StepMetadata:
        R, W, lay = self.R, self.W, self._layout()
        ints = self.meta_dev[: 4 * lay["n_ints"]].view(torch.int32)
        return StepMetadata(seq_ids=list(range(R)), num_new=[1] * R, num_prior=[0] * R,
                            n_tokens=R, n_decode=R, max_query_len=0,
                            slot_mapping=self.meta_dev[lay["slots"]: lay["end"]].view(torch.int64),
                            block_tables=ints[: R * W].view(R, W), context_lens=ints[R * W: R * W + R],
                            query_start_loc=ints[R * W + 2 * R:],
                            num_prior_dev=ints[R * W + R: R * W + 2 * R])

    def _step(self) -> None:
        """What the graph holds (on the current stream, forking to the copy streams)."""
        kv, mgr = self.kv, self.kv.mgr
        meta = self._meta()
        cur = torch.cuda.current_stream(mgr.device)
        hkv, q = mgr.num_kv_heads, self.dev_qkv
        # the input copies first: they depend on nothing in the step and run
        # beside the schedule build
        if self.gated:
            self.ready.zero_()
        self.h2d.wait_stream(cur)
        ev_in = [torch.cuda.Event() for _ in self.bounds]
        with torch.cuda.stream(self.h2d):
            if self.gated:  # each copy followed by its layers' ready words
                for a, b in self.copy_bounds:
                    q[a:b].copy_(self.host_qkv[a:b], non_blocking=True)
                    self.ready[a:b].copy_(self._ones[: b - a], non_blocking=True)
            else:
                for (a, b), ev in zip(self.bounds, ev_in):
                    q[a:b].copy_(self.host_qkv[a:b], non_blocking=True)
                    ev.record(self.h2d)
        meta.decode_schedule = ops.build_decode_schedule(
            self.schedule, meta.block_tables, meta.context_lens, mgr.num_blocks, self.hq,
            mgr.num_kv_heads, mgr.head_dim, mgr.dtype, err=mgr.err)
        for c, ((a, b), ev) in enumerate(zip(self.bounds, ev_in)):
            if not self.gated:
                cur.wait_event(ev)
            # chunk c's layers use split-K sets a .. b-1 of the step's workspace
            meta.layers_plan = ops.DecodeAppendLayersPlan(
                meta.block_tables, meta.context_lens, self.scale,
                self.workspace[a * self.ws1: b * self.ws1], mgr.err, schedule=meta.decode_schedule)
            kv.forward_layers(a, q[a:b, :, :self.hq], q[a:b, :, self.hq:self.hq + hkv],
                              q[a:b, :, self.hq + hkv:], meta, self.scale, out=self.dev_out[a:b],
                              advance=False, input_ready=self.ready[a:b] if self.gated else None,
                              defer_first=self.gated and c > 0)
            done = torch.cuda.Event()
            done.record(cur)
            self.d2h.wait_event(done)
            with torch.cuda.stream(self.d2h):
                self.host_out[a:b].copy_(self.dev_out[a:b], non_blocking=True)
        cur.wait_stream(self.h2d)
        cur.wait_stream(self.d2h)

    def capture(self) -> None:
        """Capture the step.  Runs it once uncaptured first, on all-padding
        metadata (no KV read or written), so every library handle, kernel
        attribute and argument cache exists before the capture."""
        mgr = self.kv.mgr
        mgr.flush_copies()
        lay = self._layout()
        self.meta_dev.zero_()
        self.meta_dev[lay["slots"]: lay["end"]].view(torch.int64).fill_(-1)
        cur = torch.cuda.current_stream(mgr.device)
        side = torch.cuda.Stream(mgr.device)
        side.wait_stream(cur)
        try:
            with torch.cuda.stream(side):
                self._step()
        except _lib.PagedKVError as e:
            if not self.gated or e.status != _lib.ERR_UNSUPPORTED:
                raise
            torch.cuda.synchronize(mgr.device)
            self.gated = False  # shapes outside the tensor-core decode: event waits
            if not self._chunks_given:
                ch = event_chunks(self.L)
                self.bounds = [(sum(ch[:i]), sum(ch[:i + 1])) for i in range(len(ch))]
            with torch.cuda.stream(side):
                self._step()
        cur.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        # thread-local capture: other threads of the process (a process
        # group's watchdog) may query their events while this one captures
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            self._step()
        self.graph = g

    def run(self, seqs: list[tuple[int, int]], advance: bool = False) -> None:
        """One decode step for seqs = [(seq_id, 1)] * B (B <= R, in the host
        rows' order): host_out receives every layer's output when the
        current stream reaches the end of the step."""
        kv, bs = self.kv, self.kv.mgr.block_size
        B = len(seqs)
        if B > self.R or any(n != 1 for _, n in seqs):
            raise ValueError(f"pagedkv: DecodeStepGraph serves up to {self.R} one-token sequences")
        need = max(((kv._len[s] + 1 + bs - 1) // bs for s, _ in seqs), default=1)
        if need > self.W:
            while self.W < need:
                self.W *= 2
            self._alloc()
        if self.graph is None:
            self.capture()
        kv.mgr.flush_copies()
        i = self._stage_next = (self._stage_next + 1) % len(self.stage)
        host, ev = self.stage[i]
        if ev is not None:
            ev.synchronize()
        hnp = host.numpy()
        lay = self._layout()

        def into(n_ints: int, n_slots: int):
            return (hnp[: 4 * n_ints].view(np.int32),
                    hnp[lay["slots"]: lay["slots"] + 8 * n_slots].view(np.int64))

        a = kv.step_arrays(seqs, out=into, width=self.W, pad_to=self.R)
        cur = torch.cuda.current_stream(kv.mgr.device)
        self.meta_dev.copy_(host, non_blocking=True)
        ev = torch.cuda.Event()
        ev.record(cur)
        self.stage[i][1] = ev
        self.graph.replay()
        self.replays += 1
        if advance:
            for s_id, p in zip(a["seq_ids"], a["num_prior"]):
                kv._len[s_id] = p + 1


def copy_chunks(n_layers: int, per_copy: int = 4) -> list[int]:
    """Layers per input copy of DecodeStepGraph (24 layers, per_copy 4: 1, 3,
    4, 4, 4, 4, 4): the first compute waits for one layer's copy only, and
    the copy engine stays ahead of the compute (at config 3 a layer's copy
    takes about 11 us at 54 GB/s, its decode 26 us) with few copies (each
    costs a fixed few us, so small layers go in larger pieces)."""
    out, left = [], n_layers
    for size in (1, per_copy - 1):
        if left > 0 and size > 0:
            out.append(min(size, left))
            left -= out[-1]
    while left > 0:
        out.append(min(per_copy, left))
        left -= out[-1]
    return out


def ready_chunks(n_layers: int) -> list[int]:
    """Chunks of layers for DecodeStepGraph with ready words (24 layers: 16,
    4, 2, 1, 1).  Within a chunk the layers' decode kernels chain and one
    merge launch ends it; each chunk boundary still costs a few microseconds,
    so chunks are few.  A chunk's outputs go back while the chunks after it
    compute, and the last chunk's copy out is the pipeline's drain: from the
    end, chunks of 1, 1, 2, 4, ... layers (each as many as all after it),
    the remaining layers in front as one chunk of up to twice the layers
    after it.  On one B200 box (config 3, e2e ms per step): 16, 4, 2, 1, 1:
    0.729; 12, 6, 3, 2, 1: 0.734; 8, 8, 4, 2, 1, 1: 0.737; 6, 6, 6, 3, 2, 1:
    0.740; 4, 4, 4, 4, 4, 2, 1, 1: 0.748; 2 x 10, 1 x 4: 0.770."""
    tail: list[int] = []
    left = n_layers
    while left > 0:
        after = sum(tail)
        if left <= 2 * max(after, 1) and after >= 2:
            tail.append(left)  # the head: up to twice the layers after it
            break
        c = min(left, max(1, after))
        tail.append(c)
        left -= c
    return tail[::-1]


def pieces_for(n_layers: int, layer_bytes: int, target_bytes: int) -> int:
    """Layers per copy piece: about target_bytes of copy each, 1 .. n_layers."""
    return max(1, min(n_layers, round(target_bytes / max(1, layer_bytes))))


def event_chunks(n_layers: int) -> list[int]:
    """Chunks of layers for a copy pipeline whose chunks wait on copy events
    (24 layers: 1, 2, 4, 5, 5, 4, 2, 1).  Small first and last chunks shorten
    the fill (first copy in) and the drain (last copy out).  Every chunk
    boundary costs the first decode of the chunk its overlap with the kernel
    before it (it waits on a copy event), so finer chunks that would track the
    host-to-device rate more closely (1, 1, 2, 3, 4, 5, 5, 2, 1) measured
    slower: 0.826 against 0.810 ms per step.  With ready words (no event
    waits) a boundary costs nothing and DecodeStepGraph takes one layer per
    chunk."""
    head, tail = [1, 2, 4], [4, 2, 1]
    mid = n_layers - sum(head) - sum(tail)
    if mid < 0:
        return [n_layers]
    out = list(head)
    while mid > 0:
        out.append(min(5, mid))
        mid -= out[-1]
    return out + tail
