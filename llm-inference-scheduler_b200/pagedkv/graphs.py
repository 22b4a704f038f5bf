"""CUDA graphs of the decode-only model step.

A decode-only step (every scheduled sequence adds one token) of the 24-layer
model is about 11 launches per layer, some 270 in all.  Issued from Python
one by one they cost more host time than the GPU spends on them.  `DecodeGraphs` captures
the whole step (embedding gather, 24 layers with the fused RoPE + append and
the scheduled decode attention, final norm, LM head) once per padded batch
size and replays it: a step then costs one host-to-device copy of its
metadata and one graph launch.

Fixed shapes make the replay valid for any decode step of up to R
sequences:
* the step's metadata lives in one device buffer, laid out for R rows and a
  block-table width of W blocks: tables [R, W] | context lens [R] |
  num_prior [R] | query_start_loc [1] (int32), then slots [R] and positions
  [R] (int64).  `PagedKVCache.step_arrays(width=W, pad_to=R)` writes it into a
  pinned staging buffer; one copy moves it;
* rows past the step's B sequences are padding: context length 0 (the
  decode kernel gives them no blocks and the merge writes zero rows), slot
  -1 (the RoPE + append launch stores nothing), positions 0;
* the decode schedule is built inside the graph from that metadata, so the
  stream-K partition follows the step's real lengths;
* the runner owns the decode schedule, the RoPE tables (sized for W * 16
  positions) and the logits buffer; the split-K workspace is the cache's,
  sized for R rows before the first capture and held here so a later
  reallocation by an eager step cannot free it under a graph.

Padding rows do not change the real rows: the schedule gives them no
blocks, and every other operation of the step (GEMMs, RMSNorm, SwiGLU, the
LM head) is row-independent.  The GEMMs see M = R instead of B, so the
library may pick another algorithm: logits agree with the eager step to
rounding, not bit for bit.

Graphs are captured lazily (or all at once by `capture_all`) into one
memory pool, largest first.  A step whose sequences need more than W
blocks doubles W and drops the graphs.  Replays and eager steps share the
current stream.

Reference: the decode path of mini_engine/scheduler.py step() +
mini_engine/model/qwen2.py forward (one Python call per sequence and layer
there).
"""

from __future__ import annotations

import numpy as np
import torch

from . import ops
from .block_manager import PagedKVCache, StepMetadata
from .model import PagedQwen2Model, SequenceForwardInfo


def default_buckets(max_batch: int) -> list[int]:
    """Padded batch sizes: 1, 2, 4, 8, then steps of 16 up to 128 and of 32
    beyond, and max_batch itself."""
    out = [b for b in (1, 2, 4, 8) if b < max_batch]
    b = 16
    while b < max_batch:
        out.append(b)
        b += 16 if b < 128 else 32
    out.append(max_batch)
    return sorted(set(out))


def _align16(n: int) -> int:
    return (n + 15) // 16 * 16


class DecodeGraphs:
    """Captured decode-only steps of `model` over `kv_cache`, one CUDA graph
    per padded batch size (buckets), for steps of up to max(buckets)
    sequences whose contexts fit max_blocks_per_seq blocks (grown by doubling
    when a step needs more)."""

    def __init__(self, model: PagedQwen2Model, kv_cache: PagedKVCache, max_batch: int,
                 max_blocks_per_seq: int = 64, buckets: list[int] | None = None):
        if model.device.type != "cuda":
            raise RuntimeError("pagedkv: CUDA graphs need the model on a CUDA device")
        self.model, self.kv = model, kv_cache
        self.buckets = sorted(buckets or default_buckets(max_batch))
        self.max_batch = self.buckets[-1]
        self.W = max(1, int(max_blocks_per_seq))
        self.graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self.replays = 0
        self._alloc()

    # ---- buffers ----------------------------------------------------------

    def _layout(self, R: int) -> tuple[int, int, int]:
        """(int32 count, byte offset of the slots, total bytes) of an R-row step."""
        n_ints = R * self.W + 2 * R + 1
        s_off = _align16(4 * n_ints)
        return n_ints, s_off, s_off + 16 * R

    def _alloc(self) -> None:
        m, mgr = self.model, self.kv.mgr
        cfg, dev = m.cfg, m.device
        Rm = self.max_batch
        nbytes = self._layout(Rm)[2]
        self.graphs = {}
        self.pool = torch.cuda.graph_pool_handle()
        self.meta_dev = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        self.stage = [[torch.empty(nbytes, dtype=torch.uint8).pin_memory(), None] for _ in range(2)]
        self._stage_next = 0
        self.ids = torch.zeros(Rm, dtype=torch.long, device=dev)
        self.logits = torch.empty((Rm, cfg.vocab_size), dtype=m.dtype, device=dev)
        self.schedule = ops.new_decode_schedule(Rm, self.W, dev)
        self.workspace = self.kv.decode_workspace(Rm, cfg.num_attention_heads, cfg.head_dim)
        cos, sin = m.rope.tables(self.W * mgr.block_size)
        self.cos, self.sin = cos, sin  # held: an eager step that grows the tables drops them

    def _views(self, R: int) -> dict:
        n_ints, s_off, _ = self._layout(R)
        W, buf = self.W, self.meta_dev
        ints = buf[: 4 * n_ints].view(torch.int32)
        return dict(tables=ints[: R * W].view(R, W), ctx=ints[R * W: R * W + R],
                    prior=ints[R * W + R: R * W + 2 * R], qsl=ints[R * W + 2 * R:],
                    slots=buf[s_off: s_off + 8 * R].view(torch.int64),
                    positions=buf[s_off + 8 * R: s_off + 16 * R].view(torch.int64))

    def _meta(self, R: int) -> StepMetadata:
        v = self._views(R)
        return StepMetadata(seq_ids=list(range(R)), num_new=[1] * R, num_prior=[0] * R, n_tokens=R,
                            n_decode=R, max_query_len=0, slot_mapping=v["slots"],
                            block_tables=v["tables"], context_lens=v["ctx"],
                            query_start_loc=v["qsl"], num_prior_dev=v["prior"])

    # ---- the captured step -------------------------------------------------

    def _step(self, R: int) -> None:
        """The decode-only step over the R-row metadata (what a graph holds)."""
        m, kv = self.model, self.kv
        mgr, cfg = kv.mgr, m.cfg
        meta = self._meta(R)
        pos = self._views(R)["positions"]
        meta.decode_schedule = ops.build_decode_schedule(
            self.schedule, meta.block_tables, meta.context_lens, mgr.num_blocks,
            cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, m.dtype,
            fp8=mgr.fp8, err=mgr.err)
        rot = None
        if not m.fused_rope:
            rot = (self.cos[pos].unsqueeze(1), self.sin[pos].unsqueeze(1))
        h = m._layers(m.embed[self.ids[:R]], pos, self.cos, self.sin, rot, meta, kv, advance=False)
        h = torch.nn.functional.rms_norm(h, (cfg.hidden_size,), m.final_norm, cfg.rms_norm_eps)
        torch.mm(h, m.embed.t(), out=self.logits[:R])

    def capture(self, R: int) -> None:
        """Capture the R-row step (R a bucket).  Runs it once uncaptured
        first, on all-padding metadata, which reads and writes no KV."""
        if R not in self.buckets:
            raise ValueError(f"pagedkv: {R} is not one of the buckets {self.buckets}")
        self.kv.mgr.flush_copies()
        v = self._views(R)
        cur = torch.cuda.current_stream(self.model.device)
        # all rows padding: zero tables / lengths / positions, slots -1
        self.meta_dev.zero_()
        v["slots"].fill_(-1)
        side = torch.cuda.Stream(self.model.device)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            self._step(R)  # library handles, kernel attributes, argument caches
        cur.wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self.pool):
            self._step(R)
        self.graphs[R] = g

    def capture_all(self) -> None:
        for R in reversed(self.buckets):
            if R not in self.graphs:
                self.capture(R)

    # ---- a step -------------------------------------------------------------

    def bucket(self, B: int) -> int:
        for R in self.buckets:
            if R >= B:
                return R
        raise ValueError(f"pagedkv: {B} sequences, more than the largest bucket {self.max_batch}")

    def supports(self, seq_infos: list[SequenceForwardInfo]) -> bool:
        """A decode-only step of at most max_batch sequences."""
        return 0 < len(seq_infos) <= self.max_batch and all(s.num_tokens == 1 for s in seq_infos)

    def forward(self, input_ids: torch.Tensor, seq_infos: list[SequenceForwardInfo]) -> torch.Tensor:
        """PagedQwen2Model.forward for a decode-only step, by graph replay.

        input_ids [B] on the device, one token per sequence.  Returns the
        logits [B, vocab] as a view of the runner's buffer, valid until the
        next replay.  The sequences' lengths advance as after an eager step."""
        kv, bs = self.kv, self.kv.mgr.block_size
        B = len(seq_infos)
        if not self.supports(seq_infos):
            raise ValueError("pagedkv: DecodeGraphs.forward takes decode-only steps of <= "
                             f"{self.max_batch} sequences")
        need = (max(kv._len[s.seq_id] for s in seq_infos) + bs) // bs  # blocks incl. the new token
        if need > self.W:
            w = self.W
            while w < need:
                w *= 2
            self.W = w
            self._alloc()
        R = self.bucket(B)
        if R not in self.graphs:
            self.capture(R)
        kv.mgr.flush_copies()
        i = self._stage_next = (self._stage_next + 1) % len(self.stage)
        host, ev = self.stage[i]
        if ev is not None:
            ev.synchronize()
        hnp = host.numpy()
        _, s_off, nbytes = self._layout(R)

        def into(n_ints: int, n_slots: int):
            return hnp[: 4 * n_ints].view(np.int32), hnp[s_off: s_off + 8 * n_slots].view(np.int64)

        a = kv.step_arrays([(s.seq_id, 1) for s in seq_infos], out=into, width=self.W, pad_to=R)
        pos = hnp[s_off + 8 * R: s_off + 16 * R].view(np.int64)
        pos[:B] = [int(s.positions[0]) for s in seq_infos]
        pos[B:] = 0
        self.meta_dev[:nbytes].copy_(host[:nbytes], non_blocking=True)
        cur = torch.cuda.current_stream(self.model.device)
        ev = torch.cuda.Event()
        ev.record(cur)
        self.stage[i][1] = ev
        self.ids[:B].copy_(input_ids, non_blocking=True)
        self.graphs[R].replay()
        self.replays += 1
        for s_id, p in zip(a["seq_ids"], a["num_prior"]):
            kv._len[s_id] = p + 1
        return self.logits[:B]
