"""Torch-facing wrappers of the paged-KV kernels (one C-ABI call each).

All tensors must live on a CUDA device: there is no CPU implementation.  The
kernels run asynchronously on the current torch stream of that device.
Device-side bounds problems (bad slot, block id, context length) never fault:
they are recorded in an optional int32 `err` tensor of one element (see
pagedkv._lib.FLAG_*), which callers check with `check_flags` after a sync.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported KV dtype {dt}; use float32, float16 or bfloat16") from None


def _cuda(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"pagedkv: `{name}` must be a CUDA tensor (no CPU path exists)")
    return t


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _raw_stream(t: torch.Tensor) -> int:
    """The current stream of t's device as a handle (cheaper than _stream)."""
    return torch._C._cuda_getCurrentRawStream(t.get_device())


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _row_stride(t: torch.Tensor, name: str) -> int:
    """Token-row stride of a [T, H, D] tensor whose inner [H, D] is dense."""
    if t.dim() != 3 or t.stride(2) != 1 or t.stride(1) != t.shape[2]:
        raise ValueError(f"pagedkv: `{name}` must be [tokens, heads, head_dim] with dense heads")
    return t.stride(0) if t.shape[0] > 1 else t.shape[1] * t.shape[2]


def new_error_flags(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def check_flags(err: torch.Tensor, where: str = "pagedkv") -> None:
    """Raise if a kernel recorded a device-side error (synchronises)."""
    v = int(err.item())
    if v:
        raise _lib.PagedKVError(v, where + " (device error flags)")


def _reshape_and_cache_args(k, v, k_pool, v_pool, slot_mapping, err):
    for t, n in ((k, "k"), (v, "v"), (k_pool, "k_pool"), (v_pool, "v_pool"), (slot_mapping, "slot_mapping")):
        _cuda(t, n)
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
        raise TypeError("pagedkv: slot_mapping must be a contiguous int64 tensor")
    if k_pool.dtype != k.dtype or v_pool.dtype != v.dtype or k.dtype != v.dtype:
        raise TypeError("pagedkv: k, v and the pools must share one dtype")
    if not (k_pool.is_contiguous() and v_pool.is_contiguous()):
        raise ValueError("pagedkv: pools must be contiguous")
    nb, bs, hkv, d = k_pool.shape
    T = slot_mapping.shape[0]
    if k.shape[0] != T or v.shape[0] != T or tuple(k.shape[1:]) != (hkv, d) or tuple(v.shape[1:]) != (hkv, d):
        raise ValueError("pagedkv: k/v shape does not match the pool and slot_mapping")
    return (k.data_ptr(), v.data_ptr(), _row_stride(k, "k"), _row_stride(v, "v"), k_pool.data_ptr(),
            v_pool.data_ptr(), slot_mapping.data_ptr(), T, nb, bs, hkv, d, dtype_code(k.dtype),
            _ptr(err), _stream(k))


def reshape_and_cache(k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                      slot_mapping: torch.Tensor, err: torch.Tensor | None = None) -> None:
    """k_pool.view(-1, Hkv, D)[slot_mapping[t]] = k[t] (same for v); slot -1 skipped.

    k, v: [T, Hkv, D]; pools: [num_blocks, block_size, Hkv, D] (one layer);
    slot_mapping: int64 [T].  Reference: block_manager.py:121-131.
    """
    args = _reshape_and_cache_args(k, v, k_pool, v_pool, slot_mapping, err)
    if args[7] == 0:
        return
    _lib.check(_lib.load().pkv_reshape_and_cache(*args), "pkv_reshape_and_cache")


def copy_blocks(k_cache: torch.Tensor, v_cache: torch.Tensor, pairs: torch.Tensor,
                err: torch.Tensor | None = None) -> None:
    """For every (src, dst) row of `pairs` (int32 [N, 2]) and every layer:
    k_cache[l, dst] = k_cache[l, src] (same for v).  Reference: block_manager.py:65-71.

    k_cache, v_cache: [L, num_blocks, block_size, Hkv, D] contiguous.
    """
    _cuda(k_cache, "k_cache"), _cuda(v_cache, "v_cache"), _cuda(pairs, "pairs")
    if pairs.dtype != torch.int32 or not pairs.is_contiguous() or pairs.dim() != 2 or pairs.shape[1] != 2:
        raise TypeError("pagedkv: pairs must be a contiguous int32 [N, 2] tensor")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()) or k_cache.shape != v_cache.shape:
        raise ValueError("pagedkv: k_cache / v_cache must be contiguous and equally shaped")
    L, nb = k_cache.shape[:2]
    block_bytes = k_cache[0, 0].numel() * k_cache.element_size()
    if pairs.shape[0] == 0:
        return
    rc = _lib.load().pkv_copy_blocks(
        k_cache.data_ptr(), v_cache.data_ptr(), nb * block_bytes, L, pairs.data_ptr(),
        pairs.shape[0], nb, block_bytes, _ptr(err), _stream(k_cache))
    _lib.check(rc, "pkv_copy_blocks")


def ipc_export(t: torch.Tensor) -> tuple[bytes, int]:
    """CUDA IPC handle of the device allocation that holds t's data, and the
    byte offset of t.data_ptr() in it (pkv_ipc_export)."""
    _cuda(t, "tensor")
    h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    off = ctypes.c_uint64(0)
    _lib.check(_lib.load().pkv_ipc_export(t.data_ptr(), h, ctypes.byref(off)), "pkv_ipc_export")
    return h.raw, int(off.value)


def ipc_open(handle: bytes) -> int:
    """Map an allocation exported by another process; returns its base address
    on the current device (pkv_ipc_open).  Open each allocation once."""
    if len(handle) != _lib.IPC_HANDLE_BYTES:
        raise ValueError(f"pagedkv: an IPC handle has {_lib.IPC_HANDLE_BYTES} bytes")
    base = ctypes.c_void_p(0)
    _lib.check(_lib.load().pkv_ipc_open(handle, ctypes.byref(base)), "pkv_ipc_open")
    return int(base.value)


def ipc_close(base: int) -> None:
    _lib.check(_lib.load().pkv_ipc_close(base), "pkv_ipc_close")


def copy_blocks_peer(dst_k: int, dst_v: int, dst_layer_stride: int, dst_num_blocks: int,
                     src_k: int, src_v: int, src_layer_stride: int, src_num_blocks: int,
                     n_layers: int, pairs: torch.Tensor, block_bytes: int,
                     err: torch.Tensor | None = None) -> None:
    """For every (src, dst) row of `pairs` (int32 [N, 2] on the current device)
    and every layer, block dst of the destination K / V pools becomes a copy of
    block src of the source pools (pkv_copy_blocks_peer).  Pools are given by
    device addresses, so either side may be a peer GPU's pool mapped with
    ipc_open; the kernel runs on the current device's current stream."""
    _cuda(pairs, "pairs")
    if pairs.dtype != torch.int32 or not pairs.is_contiguous() or pairs.dim() != 2 or pairs.shape[1] != 2:
        raise TypeError("pagedkv: pairs must be a contiguous int32 [N, 2] tensor")
    if pairs.shape[0] == 0:
        return
    rc = _lib.load().pkv_copy_blocks_peer(
        dst_k, dst_v, dst_layer_stride, dst_num_blocks, src_k, src_v, src_layer_stride,
        src_num_blocks, n_layers, pairs.data_ptr(), pairs.shape[0], block_bytes, _ptr(err),
        _stream(pairs))
    _lib.check(rc, "pkv_copy_blocks_peer")


def decode_workspace_bytes(n_seqs: int, n_q_heads: int, head_dim: int) -> int:
    return int(_lib.load().pkv_decode_workspace_bytes(n_seqs, n_q_heads, head_dim))


def new_decode_workspace(n_seqs: int, n_q_heads: int, head_dim: int, device,
                         layers: int = 1) -> torch.Tensor:
    """Split-K scratch of paged_decode_attention (any initial contents).
    layers > 1: one set per layer, for a multi-layer call
    (pkv_paged_decode_append_attention_layers) to chain its layers."""
    return torch.empty(decode_workspace_bytes(n_seqs, n_q_heads, head_dim) * max(1, layers),
                       dtype=torch.uint8, device=device)


def rope_reshape_and_cache(qkv: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor,
                           sin: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                           slot_mapping: torch.Tensor, q_out: torch.Tensor | None = None,
                           err: torch.Tensor | None = None, k_scale: torch.Tensor | None = None,
                           v_scale: torch.Tensor | None = None) -> torch.Tensor:
    """Rotary embedding of q and k fused with the append.

    qkv: [T, (Hq + 2 Hkv) * D] rows of the fused q/k/v projection (unit inner
    stride); positions: int64 [T]; cos, sin: [max_pos, D] tables in the pool
    dtype.  Writes the rotated k and the v of token t to the pools at
    slot_mapping[t] (-1 skips) and returns the rotated q [T, Hq, D] (into
    q_out when given).  Bit-identical to rotating q and k with separate
    elementwise multiply/add operations (pagedkv.model.Rope.rotate) followed
    by reshape_and_cache.  Reference: qwen2.py:152-158 (RoPE before the
    append, K cached post-RoPE) + block_manager.py:121-131.

    fp8 e4m3 pools (uint8 k_pool / v_pool, fp32 k_scale / v_scale [NB, bs,
    Hkv]): the rotated k and the v rows are quantised as reshape_and_cache_fp8
    quantises them, bit-identical to rotating and calling it.
    """
    for t, n in ((qkv, "qkv"), (positions, "positions"), (cos, "cos"), (sin, "sin"),
                 (k_pool, "k_pool"), (v_pool, "v_pool"), (slot_mapping, "slot_mapping")):
        _cuda(t, n)
    if qkv.dim() != 2 or qkv.stride(1) != 1:
        raise ValueError("pagedkv: qkv must be [tokens, (n_q + 2 n_kv) * head_dim] with unit inner stride")
    if positions.dtype != torch.int64 or slot_mapping.dtype != torch.int64 or \
            not positions.is_contiguous() or not slot_mapping.is_contiguous():
        raise TypeError("pagedkv: positions and slot_mapping must be contiguous int64 tensors")
    if not (k_pool.is_contiguous() and v_pool.is_contiguous() and cos.is_contiguous() and sin.is_contiguous()):
        raise ValueError("pagedkv: pools and rope tables must be contiguous")
    dt = qkv.dtype
    fp8 = k_scale is not None or v_scale is not None
    if fp8:
        _check_fp8_pools(k_pool, v_pool, k_scale, v_scale)
        if cos.dtype != dt or sin.dtype != dt:
            raise TypeError("pagedkv: the rope tables must have the qkv dtype")
    elif any(t.dtype != dt for t in (cos, sin, k_pool, v_pool)):
        raise TypeError("pagedkv: qkv, the rope tables and the pools must share one dtype")
    nb, bs, hkv, d = k_pool.shape
    T, W = qkv.shape
    hq = W // d - 2 * hkv if W % d == 0 else 0
    if hq <= 0 or cos.dim() != 2 or cos.shape != sin.shape or cos.shape[1] != d or \
            positions.shape[0] != T or slot_mapping.shape[0] != T:
        raise ValueError("pagedkv: qkv / tables / positions / slot_mapping shapes disagree")
    if q_out is None:
        q_out = torch.empty((T, hq, d), dtype=dt, device=qkv.device)
    elif q_out.dtype != dt or tuple(q_out.shape) != (T, hq, d):
        raise ValueError("pagedkv: q_out must be [tokens, n_q_heads, head_dim] in the qkv dtype")
    if T == 0:
        return q_out
    name, args = _rope_args(qkv, positions, cos, sin, k_pool, v_pool, slot_mapping, q_out, err,
                            k_scale, v_scale, hq)
    _lib.check(getattr(_lib.load(), name)(*args), name)
    return q_out


def _rope_args(qkv, positions, cos, sin, k_pool, v_pool, slot_mapping, q_out, err, k_scale, v_scale,
               hq):
    """C arguments of pkv_rope_reshape_and_cache(_fp8) for validated tensors:
    (entry point name, argument tuple)."""
    nb, bs, hkv, d = k_pool.shape
    T = qkv.shape[0]
    head = (q_out.data_ptr(), _row_stride(q_out, "q_out"), qkv.data_ptr(), qkv.stride(0),
            positions.data_ptr(), cos.data_ptr(), sin.data_ptr(), cos.shape[0], k_pool.data_ptr(),
            v_pool.data_ptr())
    tail = (slot_mapping.data_ptr(), T, nb, bs, hq, hkv, d, dtype_code(qkv.dtype), _ptr(err),
            _stream(qkv))
    if k_scale is not None:
        return "pkv_rope_reshape_and_cache_fp8", head + (k_scale.data_ptr(), v_scale.data_ptr()) + tail
    return "pkv_rope_reshape_and_cache", head + tail


class RopePlan:
    """rope_reshape_and_cache for the layers of one step, which share
    positions, RoPE tables, slot mapping and error word.  The first call (and
    any call whose tensors differ in dtype, shape, stride or stream from the
    previous one) validates through rope_reshape_and_cache; the others only
    fill in the layer's pointers (q_out, qkv, pools, fp8 scales)."""

    def __init__(self, positions, cos, sin, slot_mapping, err=None):
        self._static = (positions, cos, sin, slot_mapping, err)
        self._key = None
        self._args: list = []

    def uses(self, positions, cos, sin) -> bool:
        """Whether this plan was made for these positions and tables."""
        st = self._static
        return st[0] is positions and st[1] is cos and st[2] is sin

    def __call__(self, qkv, k_pool, v_pool, k_scale=None, v_scale=None) -> torch.Tensor:
        key = (qkv.dtype, qkv.shape, qkv.stride(), k_pool.dtype, k_pool.shape, k_pool.stride(),
               v_pool.shape, v_pool.stride(), k_scale is None, v_scale is None, qkv.get_device(),
               _raw_stream(qkv))
        if key != self._key:
            positions, cos, sin, slots, err = self._static
            q_out = rope_reshape_and_cache(qkv, positions, cos, sin, k_pool, v_pool, slots, err=err,
                                           k_scale=k_scale, v_scale=v_scale)
            if qkv.shape[0] and (k_scale is None) == (v_scale is None):
                name, args = _rope_args(qkv, positions, cos, sin, k_pool, v_pool, slots, q_out, err,
                                        k_scale, v_scale, q_out.shape[1])
                self._fn, self._name, self._args = getattr(_lib.load(), name), name, list(args)
                self._qshape, self._key = tuple(q_out.shape), key
            return q_out
        q_out = torch.empty(self._qshape, dtype=qkv.dtype, device=qkv.device)
        a = self._args
        a[0], a[2], a[8], a[9] = q_out.data_ptr(), qkv.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr()
        if k_scale is not None:
            a[10], a[11] = k_scale.data_ptr(), v_scale.data_ptr()
        rc = self._fn(*a)
        if rc:
            _lib.check(rc, self._name)
        return q_out


def _check_tables(block_tables: torch.Tensor) -> None:
    _cuda(block_tables, "block_tables")
    if block_tables.dtype != torch.int32 or block_tables.dim() != 2 or block_tables.stride(1) != 1:
        raise TypeError("pagedkv: block_tables must be int32 [n_seqs, max_blocks] with unit inner stride")


def _decode_args(q, k_pool, v_pool, block_tables, context_lens, scale, workspace, out, err):
    for t, n in ((q, "q"), (k_pool, "k_pool"), (v_pool, "v_pool"), (context_lens, "context_lens")):
        _cuda(t, n)
    _check_tables(block_tables)
    if context_lens.dtype != torch.int32 or not context_lens.is_contiguous():
        raise TypeError("pagedkv: context_lens must be a contiguous int32 tensor")
    if q.dtype != k_pool.dtype or k_pool.dtype != v_pool.dtype:
        raise TypeError("pagedkv: q and the pools must share one dtype")
    nb, bs, hkv, d = k_pool.shape
    B, hq, dq = q.shape
    if dq != d or block_tables.shape[0] < B or context_lens.shape[0] < B:
        raise ValueError("pagedkv: q / block_tables / context_lens shapes disagree")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    if workspace is None:
        workspace = new_decode_workspace(B, hq, d, q.device)
    args = (out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
            k_pool.data_ptr(), v_pool.data_ptr(), nb, block_tables.data_ptr(), block_tables.stride(0),
            block_tables.shape[1], context_lens.data_ptr(), B, hq, hkv, d, bs, float(scale),
            dtype_code(q.dtype), workspace.data_ptr(), workspace.numel() * workspace.element_size(),
            _ptr(err), _stream(q))
    return args, out


def decode_schedule_bytes(n_seqs: int, max_blocks_per_seq: int) -> int:
    return int(_lib.load().pkv_decode_schedule_bytes(n_seqs, max_blocks_per_seq))


def new_decode_schedule(n_seqs: int, max_blocks_per_seq: int, device) -> torch.Tensor:
    """Buffer for a per-step decode schedule (any initial contents)."""
    return torch.empty(max(16, decode_schedule_bytes(n_seqs, max_blocks_per_seq)), dtype=torch.uint8,
                       device=device)


def build_decode_schedule(schedule: torch.Tensor, block_tables: torch.Tensor,
                          context_lens: torch.Tensor, num_blocks: int, n_q_heads: int,
                          n_kv_heads: int, head_dim: int, dtype: torch.dtype, fp8: bool = False,
                          err: torch.Tensor | None = None) -> torch.Tensor:
    """The step's stream-K partition for the decode kernel, computed once and
    read by every layer's `schedule=` decode call (pkv_decode_schedule).
    dtype is the q / out dtype of those calls; fp8=True for the fp8 decode."""
    _cuda(schedule, "schedule"), _cuda(context_lens, "context_lens")
    _check_tables(block_tables)
    if context_lens.dtype != torch.int32 or not context_lens.is_contiguous():
        raise TypeError("pagedkv: context_lens must be a contiguous int32 tensor")
    B = context_lens.shape[0]
    rc = _lib.load().pkv_decode_schedule(
        schedule.data_ptr(), schedule.numel() * schedule.element_size(), block_tables.data_ptr(),
        block_tables.stride(0), block_tables.shape[1], context_lens.data_ptr(), B, num_blocks,
        n_q_heads, n_kv_heads, head_dim, 16, dtype_code(dtype), int(bool(fp8)), _ptr(err),
        _stream(context_lens))
    _lib.check(rc, "pkv_decode_schedule")
    return schedule


def _sched_fn(name: str, schedule):
    return getattr(_lib.load(), name + "_scheduled" if schedule is not None else name)


def _sched_args(args: tuple, schedule) -> tuple:
    return args + (schedule.data_ptr(),) if schedule is not None else args


def paged_decode_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                           block_tables: torch.Tensor, context_lens: torch.Tensor, scale: float,
                           workspace: torch.Tensor | None = None, out: torch.Tensor | None = None,
                           err: torch.Tensor | None = None,
                           schedule: torch.Tensor | None = None) -> torch.Tensor:
    """out[s] = softmax(scale * q[s] K_s^T) V_s over context_lens[s] tokens of
    sequence s, read in place through block_tables[s] (GQA: q head h uses kv
    head h // (Hq // Hkv)).  q: [B, Hq, D]; returns [B, Hq, D].
    Reference: block_manager.py:136-141 + qwen2.py:98-128 (num_new == 1).
    """
    args, out = _decode_args(q, k_pool, v_pool, block_tables, context_lens, scale, workspace, out, err)
    _lib.check(_sched_fn("pkv_paged_decode_attention", schedule)(*_sched_args(args, schedule)),
               "pkv_paged_decode_attention")
    return out


def _decode_append_args(q, k_new, v_new, k_pool, v_pool, block_tables, context_lens, scale,
                        workspace, out, err):
    args, out = _decode_args(q, k_pool, v_pool, block_tables, context_lens, scale, workspace, out,
                             err)
    _cuda(k_new, "k_new"), _cuda(v_new, "v_new")
    nb, bs, hkv, d = k_pool.shape
    B = q.shape[0]
    if k_new.dtype != q.dtype or v_new.dtype != q.dtype:
        raise TypeError("pagedkv: k_new / v_new must have the pool dtype")
    if k_new.shape[0] < B or v_new.shape[0] < B or tuple(k_new.shape[1:]) != (hkv, d) \
            or tuple(v_new.shape[1:]) != (hkv, d):
        raise ValueError("pagedkv: k_new / v_new must be [n_seqs, n_kv_heads, head_dim]")
    # decode-call argument order with the new rows inserted after q
    args = args[:4] + (k_new.data_ptr(), v_new.data_ptr(), _row_stride(k_new, "k_new"),
                       _row_stride(v_new, "v_new")) + args[4:]
    return args, out


def paged_decode_append_attention(q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                                  k_pool: torch.Tensor, v_pool: torch.Tensor,
                                  block_tables: torch.Tensor, context_lens: torch.Tensor,
                                  scale: float, workspace: torch.Tensor | None = None,
                                  out: torch.Tensor | None = None,
                                  err: torch.Tensor | None = None,
                                  schedule: torch.Tensor | None = None) -> torch.Tensor:
    """One decode step of one layer: write k_new[s] / v_new[s] at position
    context_lens[s] - 1 of sequence s (slot from its block table), then the
    paged attention over context_lens[s] tokens.  Reference:
    PagedKVCache.append_and_fetch + Qwen2Model._attention (num_new == 1)."""
    args, out = _decode_append_args(q, k_new, v_new, k_pool, v_pool, block_tables, context_lens,
                                    scale, workspace, out, err)
    _lib.check(_sched_fn("pkv_paged_decode_append_attention", schedule)(*_sched_args(args, schedule)),
               "pkv_paged_decode_append_attention")
    return out


# ---------------------------------------------------------------- fp8 e4m3 pools

def _check_fp8_pools(k_pool, v_pool, k_scale, v_scale):
    for t, n in ((k_pool, "k_pool"), (v_pool, "v_pool"), (k_scale, "k_scale"), (v_scale, "v_scale")):
        _cuda(t, n)
    if k_pool.dtype != torch.uint8 or v_pool.dtype != torch.uint8:
        raise TypeError("pagedkv: fp8 pools are uint8 tensors of e4m3 bytes")
    if k_scale.dtype != torch.float32 or v_scale.dtype != torch.float32:
        raise TypeError("pagedkv: fp8 pool scales are float32")
    if not all(t.is_contiguous() for t in (k_pool, v_pool, k_scale, v_scale)):
        raise ValueError("pagedkv: fp8 pools and scales must be contiguous")
    nb, bs, hkv, d = k_pool.shape
    if tuple(v_pool.shape) != (nb, bs, hkv, d) or tuple(k_scale.shape) != (nb, bs, hkv) or \
            tuple(v_scale.shape) != (nb, bs, hkv):
        raise ValueError("pagedkv: fp8 pools [nb, bs, hkv, d] and scales [nb, bs, hkv] disagree")
    return nb, bs, hkv, d


def reshape_and_cache_fp8(k: torch.Tensor, v: torch.Tensor, k_pool: torch.Tensor,
                          v_pool: torch.Tensor, k_scale: torch.Tensor, v_scale: torch.Tensor,
                          slot_mapping: torch.Tensor, err: torch.Tensor | None = None) -> None:
    """reshape_and_cache into fp8 e4m3 pools: each (token, KV head) row of
    k / v ([T, Hkv, D], fp32/fp16/bf16) is quantised with scale =
    absmax / 448, byte = e4m3(x / scale) (nearest even, saturated); the bytes
    go to k_pool / v_pool (uint8 [NB, bs, Hkv, D]) and the scales to
    k_scale / v_scale (fp32 [NB, bs, Hkv]) at slot_mapping[t] (-1 skips)."""
    nb, bs, hkv, d = _check_fp8_pools(k_pool, v_pool, k_scale, v_scale)
    for t, n in ((k, "k"), (v, "v"), (slot_mapping, "slot_mapping")):
        _cuda(t, n)
    if slot_mapping.dtype != torch.int64 or not slot_mapping.is_contiguous():
        raise TypeError("pagedkv: slot_mapping must be a contiguous int64 tensor")
    T = slot_mapping.shape[0]
    if k.dtype != v.dtype or k.shape[0] != T or v.shape[0] != T or tuple(k.shape[1:]) != (hkv, d) \
            or tuple(v.shape[1:]) != (hkv, d):
        raise ValueError("pagedkv: k/v shape does not match the pool and slot_mapping")
    if T == 0:
        return
    rc = _lib.load().pkv_reshape_and_cache_fp8(
        k.data_ptr(), v.data_ptr(), _row_stride(k, "k"), _row_stride(v, "v"), k_pool.data_ptr(),
        v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), slot_mapping.data_ptr(), T, nb, bs,
        hkv, d, dtype_code(k.dtype), _ptr(err), _stream(k))
    _lib.check(rc, "pkv_reshape_and_cache_fp8")


def paged_decode_attention_fp8(q, k_pool, v_pool, k_scale, v_scale, block_tables, context_lens,
                               scale, workspace=None, out=None, err=None,
                               schedule=None) -> torch.Tensor:
    """paged_decode_attention over fp8 e4m3 pools (value = e4m3(byte) *
    scale of its row); q / out in fp16, bf16 or fp32."""
    nb, bs, hkv, d = _check_fp8_pools(k_pool, v_pool, k_scale, v_scale)
    _cuda(q, "q"), _cuda(context_lens, "context_lens")
    _check_tables(block_tables)
    if context_lens.dtype != torch.int32 or not context_lens.is_contiguous():
        raise TypeError("pagedkv: context_lens must be a contiguous int32 tensor")
    B, hq, dq = q.shape
    if dq != d or block_tables.shape[0] < B or context_lens.shape[0] < B:
        raise ValueError("pagedkv: q / block_tables / context_lens shapes disagree")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    if workspace is None:
        workspace = new_decode_workspace(B, hq, d, q.device)
    if B == 0:
        return out
    args = (out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
            k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), nb,
            block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
            context_lens.data_ptr(), B, hq, hkv, d, bs, float(scale), dtype_code(q.dtype),
            workspace.data_ptr(), workspace.numel() * workspace.element_size(), _ptr(err), _stream(q))
    rc = _sched_fn("pkv_paged_decode_attention_fp8", schedule)(*_sched_args(args, schedule))
    _lib.check(rc, "pkv_paged_decode_attention_fp8")
    return out


def _decode_append_fp8_args(q, k_new, v_new, k_pool, v_pool, k_scale, v_scale, block_tables,
                            context_lens, scale, workspace, out, err):
    nb, bs, hkv, d = _check_fp8_pools(k_pool, v_pool, k_scale, v_scale)
    for t, n in ((q, "q"), (k_new, "k_new"), (v_new, "v_new"), (context_lens, "context_lens")):
        _cuda(t, n)
    _check_tables(block_tables)
    if context_lens.dtype != torch.int32 or not context_lens.is_contiguous():
        raise TypeError("pagedkv: context_lens must be a contiguous int32 tensor")
    B, hq, dq = q.shape
    if dq != d or block_tables.shape[0] < B or context_lens.shape[0] < B:
        raise ValueError("pagedkv: q / block_tables / context_lens shapes disagree")
    if k_new.dtype != q.dtype or v_new.dtype != q.dtype:
        raise TypeError("pagedkv: k_new / v_new must have the q dtype")
    if k_new.shape[0] < B or v_new.shape[0] < B or tuple(k_new.shape[1:]) != (hkv, d) \
            or tuple(v_new.shape[1:]) != (hkv, d):
        raise ValueError("pagedkv: k_new / v_new must be [n_seqs, n_kv_heads, head_dim]")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    if workspace is None:
        workspace = new_decode_workspace(B, hq, d, q.device)
    args = (out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
            k_new.data_ptr(), v_new.data_ptr(), _row_stride(k_new, "k_new"), _row_stride(v_new, "v_new"),
            k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), nb,
            block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
            context_lens.data_ptr(), B, hq, hkv, d, bs, float(scale), dtype_code(q.dtype),
            workspace.data_ptr(), workspace.numel() * workspace.element_size(), _ptr(err), _stream(q))
    return args, out


def paged_decode_append_attention_fp8(q, k_new, v_new, k_pool, v_pool, k_scale, v_scale,
                                      block_tables, context_lens, scale, workspace=None, out=None,
                                      err=None, schedule=None) -> torch.Tensor:
    """One fp8 decode step of one layer: the decode kernel quantises
    k_new[s] / v_new[s] into the fp8 pools at position context_lens[s] - 1
    (reshape_and_cache_fp8's quantisation, scales included), then attends
    (paged_decode_attention_fp8)."""
    args, out = _decode_append_fp8_args(q, k_new, v_new, k_pool, v_pool, k_scale, v_scale,
                                        block_tables, context_lens, scale, workspace, out, err)
    if q.shape[0] == 0:
        return out
    rc = _sched_fn("pkv_paged_decode_append_attention_fp8", schedule)(*_sched_args(args, schedule))
    _lib.check(rc, "pkv_paged_decode_append_attention_fp8")
    return out


def prefill_fp8_scratch_bytes(n_seqs: int, max_blocks_per_seq: int, n_kv_heads: int,
                              head_dim: int) -> int:
    return int(_lib.load().pkv_prefill_fp8_scratch_bytes(n_seqs, max_blocks_per_seq, n_kv_heads,
                                                          head_dim))


def paged_prefill_attention_fp8(q, k_pool, v_pool, k_scale, v_scale, block_tables, query_start_loc,
                                num_prior, max_query_len, scale, out=None, err=None,
                                tensor_cores: bool = True, scratch=None,
                                scratch_free: bool = False) -> torch.Tensor:
    """paged_prefill_attention over fp8 e4m3 pools.

    tensor_cores=True: the tcgen05 prefill over 16-bit rows.  By default the
    blocks the step sees are first written as 16-bit rows (e4m3 x scale,
    rounded once to q's dtype) into `scratch` (prefill_fp8_scratch_bytes;
    allocated here when None).  scratch_free=True (fp16 q only): the kernel
    converts the e4m3 tiles in shared memory itself
    (pkv_paged_prefill_attention_fp8_tc), no scratch; slower at config 4's
    shape (each CTA converts the tiles it reads, where the scratch pass
    converts each visible block once).  tensor_cores=False: the CUDA-core
    kernel dequantises on load (no scratch, no extra rounding)."""
    nb, bs, hkv, d = _check_fp8_pools(k_pool, v_pool, k_scale, v_scale)
    for t, n in ((q, "q"), (query_start_loc, "query_start_loc"), (num_prior, "num_prior")):
        _cuda(t, n)
    _check_tables(block_tables)
    T, hq, dq = q.shape
    n_seqs = query_start_loc.shape[0] - 1
    if dq != d or num_prior.shape[0] < n_seqs:
        raise ValueError("pagedkv: q / num_prior shapes disagree")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    if T == 0 or n_seqs == 0:
        return out
    if tensor_cores and scratch_free:
        rc = _lib.load().pkv_paged_prefill_attention_fp8_tc(
            out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
            k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), nb,
            block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
            query_start_loc.data_ptr(), num_prior.data_ptr(), n_seqs, T, int(max_query_len), hq, hkv,
            d, bs, float(scale), dtype_code(q.dtype), _ptr(err), _stream(q))
        _lib.check(rc, "pkv_paged_prefill_attention_fp8_tc")
        return out
    if tensor_cores and q.dtype in (torch.float16, torch.bfloat16):
        need = prefill_fp8_scratch_bytes(n_seqs, block_tables.shape[1], hkv, d)
        if scratch is None:
            scratch = torch.empty(need, dtype=torch.uint8, device=q.device)
        _cuda(scratch, "scratch")
        rc = _lib.load().pkv_paged_prefill_attention_fp8_scratch(
            out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
            k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), nb,
            block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
            query_start_loc.data_ptr(), num_prior.data_ptr(), n_seqs, T, int(max_query_len), hq, hkv,
            d, bs, float(scale), dtype_code(q.dtype), scratch.data_ptr(),
            scratch.numel() * scratch.element_size(), _ptr(err), _stream(q))
        _lib.check(rc, "pkv_paged_prefill_attention_fp8_scratch")
        return out
    rc = _lib.load().pkv_paged_prefill_attention_fp8(
        out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"), k_pool.data_ptr(),
        v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), nb, block_tables.data_ptr(),
        block_tables.stride(0), block_tables.shape[1], query_start_loc.data_ptr(), num_prior.data_ptr(),
        n_seqs, T, int(max_query_len), hq, hkv, d, bs, float(scale), dtype_code(q.dtype), _ptr(err),
        _stream(q))
    _lib.check(rc, "pkv_paged_prefill_attention_fp8")
    return out


class DecodeAppendPlan:
    """pkv_paged_decode_append_attention for the layers of one step, which
    share block tables, context lengths, scale, workspace and error word.

    The first call (and any call whose tensors differ in dtype, shape, stride
    or stream from the previous one) builds the arguments through the regular
    validating path; the others reuse them and only fill in the layer's
    pointers (q, k_new, v_new, pools, out), so a layer costs one ctypes call
    and a few attribute reads instead of a full argument check."""

    _PTRS = (0, 2, 4, 5, 8, 9)  # out, q, k_new, v_new, k_pool, v_pool in the C argument list

    def __init__(self, block_tables, context_lens, scale, workspace, err=None, schedule=None):
        self._static = (block_tables, context_lens, scale, workspace, err)
        self.scale = scale
        self.schedule = schedule  # the step's decode schedule (build_decode_schedule) or None
        self._key = None
        self._args: list = []
        self._fn = _sched_fn("pkv_paged_decode_append_attention", schedule)

    def __call__(self, q, k_new, v_new, k_pool, v_pool, out) -> torch.Tensor:
        # everything the validated arguments depend on besides the six pointers
        key = (q.dtype, k_new.dtype, v_new.dtype, k_pool.dtype, v_pool.dtype, out.dtype,
               q.shape, q.stride(), k_new.shape, k_new.stride(), v_new.shape, v_new.stride(),
               k_pool.shape, k_pool.stride(), v_pool.shape, v_pool.stride(), out.shape, out.stride(),
               q.get_device(), _raw_stream(q))
        if key != self._key:
            tables, ctx, scale, ws, err = self._static
            args, out = _decode_append_args(q, k_new, v_new, k_pool, v_pool, tables, ctx, scale, ws,
                                            out, err)
            self._args, self._key = list(_sched_args(args, self.schedule)), key
        else:
            a = self._args
            a[0], a[2], a[4], a[5], a[8], a[9] = (out.data_ptr(), q.data_ptr(), k_new.data_ptr(),
                                                  v_new.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr())
        rc = self._fn(*self._args)
        if rc:
            _lib.check(rc, "pkv_paged_decode_append_attention")
        return out


class DecodeAppendLayersPlan:
    """pkv_paged_decode_append_attention_layers for runs of consecutive layers
    of one decode-only step: one C call per run issues every layer's decode
    (with the fused append) and merge.  Layer-major inputs: q and out
    [n, B, Hq, D], k_new and v_new [n, B, Hkv, D] (dense [heads, dims]), the
    pools the layer slices [n, NB, bs, Hkv, D] of the step's contiguous
    [L, NB, bs, Hkv, D] caches.  Validated arguments are reused as
    DecodeAppendPlan reuses them, with the run's pointers and length swapped
    in."""

    def __init__(self, block_tables, context_lens, scale, workspace, err=None, schedule=None):
        self._static = (block_tables, context_lens, scale, workspace, err)
        self.scale = scale
        self.schedule = schedule
        self._key = None
        self._args: list = []
        self._fn = _lib.load().pkv_paged_decode_append_attention_layers_flags

    @staticmethod
    def _layer_stride(t: torch.Tensor, name: str) -> int:
        if t.dim() != 4:
            raise ValueError(f"pagedkv: `{name}` must be [layers, rows, heads, head_dim]")
        return t.stride(0)

    def __call__(self, q, k_new, v_new, k_pools, v_pools, out, input_ready=None,
                 defer_first: bool = False) -> torch.Tensor:
        """input_ready: None, or an int32 device tensor of one word per layer:
        layer l's kernels wait (bounded) until input_ready[l] is nonzero
        before reading its q, k_new and v_new (set by a copy on another
        stream after that layer's rows).  defer_first: PKV_LAYERS_DEFER_FIRST
        (the run continues the chain of a run just enqueued over other layers
        and other split-K sets; nothing still running touches this run's
        data)."""
        n = q.shape[0]
        if k_new.shape[0] != n or v_new.shape[0] != n or out.shape[0] != n or \
                k_pools.shape[0] != n or v_pools.shape[0] != n:
            raise ValueError("pagedkv: q, k_new, v_new, out and the pools must cover the same layers")
        if n == 0:
            return out
        key = (q.dtype, k_new.dtype, v_new.dtype, k_pools.dtype, out.dtype, q.shape[1:], q.stride(),
               k_new.shape[1:], k_new.stride(), v_new.stride(), k_pools.shape[1:], k_pools.stride(),
               v_pools.stride(), out.shape[1:], out.stride(), q.get_device(), _raw_stream(q))
        if key != self._key:
            if k_new.stride(0) != v_new.stride(0):
                raise ValueError("pagedkv: k_new and v_new must share one layer stride")
            if k_pools.stride() != v_pools.stride() or not k_pools[0].is_contiguous():
                raise ValueError("pagedkv: the K and V pools must be equally strided, layers dense")
            tables, ctx, scale, ws, err = self._static
            # the per-layer checks of the single-layer call, on layer 0
            args, _ = _decode_append_args(q[0], k_new[0], v_new[0], k_pools[0], v_pools[0], tables,
                                          ctx, scale, ws, out[0], err)
            (o, o_rs, qp, q_rs, kn, vn, kn_rs, vn_rs, kp, vp, nb, bt, bt_s, mb, cl, B, hq, hkv, d, bs,
             sc, dt, wsp, wsb, errp, st) = args
            self._args = [n, o, self._layer_stride(out, "out"), o_rs, qp, self._layer_stride(q, "q"),
                          q_rs, kn, vn, self._layer_stride(k_new, "k_new"), kn_rs, vn_rs, kp, vp,
                          k_pools.stride(0) * k_pools.element_size(), nb, bt, bt_s, mb, cl, B, hq,
                          hkv, d, bs, sc, dt, wsp, wsb, errp, st,
                          None if self.schedule is None else self.schedule.data_ptr(), None, 0]
            self._key = key
        a = self._args
        a[0], a[1], a[4], a[7], a[8], a[12], a[13] = (n, out.data_ptr(), q.data_ptr(), k_new.data_ptr(),
                                                      v_new.data_ptr(), k_pools.data_ptr(),
                                                      v_pools.data_ptr())
        if input_ready is not None:
            _cuda(input_ready, "input_ready")
            if input_ready.dtype != torch.int32 or input_ready.numel() != n or not input_ready.is_contiguous():
                raise ValueError("pagedkv: input_ready must hold one contiguous int32 word per layer")
        a[-2] = None if input_ready is None else input_ready.data_ptr()
        a[-1] = _lib.LAYERS_DEFER_FIRST if defer_first else 0
        rc = self._fn(*a)
        if rc:
            _lib.check(rc, "pkv_paged_decode_append_attention_layers")
        return out


class DecodePlan(DecodeAppendPlan):
    """pkv_paged_decode_attention (no append: the step's K/V are already in
    the pools) for the layers of one step, with the same reuse of validated
    arguments as DecodeAppendPlan."""

    def __init__(self, block_tables, context_lens, scale, workspace, err=None, schedule=None):
        super().__init__(block_tables, context_lens, scale, workspace, err, schedule)
        self._fn = _sched_fn("pkv_paged_decode_attention", schedule)

    def __call__(self, q, k_pool, v_pool, out) -> torch.Tensor:
        key = (q.dtype, k_pool.dtype, v_pool.dtype, out.dtype, q.shape, q.stride(), k_pool.shape,
               k_pool.stride(), v_pool.shape, v_pool.stride(), out.shape, out.stride(),
               q.get_device(), _raw_stream(q))
        if key != self._key:
            tables, ctx, scale, ws, err = self._static
            args, out = _decode_args(q, k_pool, v_pool, tables, ctx, scale, ws, out, err)
            self._args, self._key = list(_sched_args(args, self.schedule)), key
        else:
            a = self._args
            a[0], a[2], a[4], a[5] = out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr()
        rc = self._fn(*self._args)
        if rc:
            _lib.check(rc, "pkv_paged_decode_attention")
        return out


class BoundLaunch:
    """A validated launch with its C-ABI arguments fixed (pointers, sizes and
    the stream that was current when it was bound).  Calling it re-issues the
    kernel with no Python-side checks: for loops that replay one step, where
    per-call validation would dominate the launch cost.  The tensors it was
    bound to must stay alive and unchanged in shape."""

    def __init__(self, fn, args, name, keep):
        self._fn, self._args, self._name, self._keep = fn, args, name, keep

    def __call__(self) -> None:
        rc = self._fn(*self._args)
        if rc:
            _lib.check(rc, self._name)


def bind_paged_decode_append_attention_fp8(q, k_new, v_new, k_pool, v_pool, k_scale, v_scale,
                                           block_tables, context_lens, scale, workspace, out, err=None,
                                           schedule=None) -> BoundLaunch:
    args, out = _decode_append_fp8_args(q, k_new, v_new, k_pool, v_pool, k_scale, v_scale,
                                        block_tables, context_lens, scale, workspace, out, err)
    return BoundLaunch(_sched_fn("pkv_paged_decode_append_attention_fp8", schedule),
                       _sched_args(args, schedule), "pkv_paged_decode_append_attention_fp8",
                       (q, k_new, v_new, k_pool, v_pool, k_scale, v_scale, block_tables, context_lens,
                        workspace, out, err, schedule))


class DecodeAppendFp8LayersPlan:
    """pkv_paged_decode_append_attention_fp8_layers for runs of consecutive
    layers of one decode-only step over fp8 pools: q / out [n, B, Hq, D] and
    k_new / v_new [n, B, Hkv, D] in the 16-bit model dtype, the uint8 pools
    [n, NB, bs, Hkv, D] and fp32 scales [n, NB, bs, Hkv] of the step's
    contiguous caches.  A workspace of one split-K set per layer chains the
    run's layers.  Validated arguments are reused, with the run's pointers and
    length swapped in."""

    def __init__(self, block_tables, context_lens, scale, workspace, err=None, schedule=None):
        self._static = (block_tables, context_lens, scale, workspace, err)
        self.scale = scale
        self.schedule = schedule
        self._key = None
        self._args: list = []
        self._fn = _lib.load().pkv_paged_decode_append_attention_fp8_layers

    def __call__(self, q, k_new, v_new, k_pools, v_pools, k_scales, v_scales, out) -> torch.Tensor:
        n = q.shape[0]
        if any(t.shape[0] != n for t in (k_new, v_new, out, k_pools, v_pools, k_scales, v_scales)):
            raise ValueError("pagedkv: the inputs, pools, scales and out must cover the same layers")
        if n == 0:
            return out
        key = (q.dtype, q.shape[1:], q.stride(), k_new.shape[1:], k_new.stride(), v_new.stride(),
               k_pools.shape[1:], k_pools.stride(), v_pools.stride(), k_scales.stride(),
               v_scales.stride(), out.shape[1:], out.stride(), q.get_device(), _raw_stream(q))
        if key != self._key:
            if k_new.stride(0) != v_new.stride(0) or k_scales.stride() != v_scales.stride():
                raise ValueError("pagedkv: k_new / v_new and the two scale arrays must be equally strided")
            if k_pools.stride() != v_pools.stride() or not k_pools[0].is_contiguous():
                raise ValueError("pagedkv: the K and V pools must be equally strided, layers dense")
            tables, ctx, scale, ws, err = self._static
            # the per-layer checks of the single-layer call, on layer 0
            args, _ = _decode_append_fp8_args(q[0], k_new[0], v_new[0], k_pools[0], v_pools[0],
                                              k_scales[0], v_scales[0], tables, ctx, scale, ws, out[0], err)
            (o, o_rs, qp, q_rs, kn, vn, kn_rs, vn_rs, kp, vp, ksp, vsp, nb, bt, bt_s, mb, cl, B, hq, hkv, d,
             bs, sc, dt, wsp, wsb, errp, st) = args
            self._args = [n, o, DecodeAppendLayersPlan._layer_stride(out, "out"), o_rs, qp,
                          DecodeAppendLayersPlan._layer_stride(q, "q"), q_rs, kn, vn,
                          DecodeAppendLayersPlan._layer_stride(k_new, "k_new"), kn_rs, vn_rs, kp, vp,
                          k_pools.stride(0) * k_pools.element_size(), ksp, vsp, k_scales.stride(0), nb, bt,
                          bt_s, mb, cl, B, hq, hkv, d, bs, sc, dt, wsp, wsb, errp, st,
                          None if self.schedule is None else self.schedule.data_ptr()]
            self._key = key
        a = self._args
        a[0], a[1], a[4], a[7], a[8], a[12], a[13], a[15], a[16] = (
            n, out.data_ptr(), q.data_ptr(), k_new.data_ptr(), v_new.data_ptr(), k_pools.data_ptr(),
            v_pools.data_ptr(), k_scales.data_ptr(), v_scales.data_ptr())
        rc = self._fn(*a)
        if rc:
            _lib.check(rc, "pkv_paged_decode_append_attention_fp8_layers")
        return out


def bind_paged_prefill_attention_fp8(q, k_pool, v_pool, k_scale, v_scale, block_tables,
                                     query_start_loc, num_prior, max_query_len, scale, out, scratch,
                                     err=None) -> BoundLaunch:
    """The tensor-core fp8 prefill bound to fixed tensors: scratch pass +
    tcgen05 kernel, or with scratch=None the scratch-free entry (fp16 q)."""
    paged_prefill_attention_fp8(q, k_pool, v_pool, k_scale, v_scale, block_tables, query_start_loc,
                                num_prior, max_query_len, scale, out=out, err=err, scratch=scratch,
                                scratch_free=scratch is None)
    nb, bs, hkv, d = k_pool.shape
    T, hq, _ = q.shape
    if scratch is None:
        args = (out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
                k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), nb,
                block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
                query_start_loc.data_ptr(), num_prior.data_ptr(), query_start_loc.shape[0] - 1, T,
                int(max_query_len), hq, hkv, d, bs, float(scale), dtype_code(q.dtype), _ptr(err),
                _stream(q))
        return BoundLaunch(_lib.load().pkv_paged_prefill_attention_fp8_tc, args,
                           "pkv_paged_prefill_attention_fp8_tc",
                           (q, k_pool, v_pool, k_scale, v_scale, block_tables, query_start_loc,
                            num_prior, out, err))
    args = (out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
            k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), nb,
            block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
            query_start_loc.data_ptr(), num_prior.data_ptr(), query_start_loc.shape[0] - 1, T,
            int(max_query_len), hq, hkv, d, bs, float(scale), dtype_code(q.dtype), scratch.data_ptr(),
            scratch.numel() * scratch.element_size(), _ptr(err), _stream(q))
    return BoundLaunch(_lib.load().pkv_paged_prefill_attention_fp8_scratch, args,
                       "pkv_paged_prefill_attention_fp8_scratch",
                       (q, k_pool, v_pool, k_scale, v_scale, block_tables, query_start_loc, num_prior,
                        out, scratch, err))


def bind_decode_schedule(schedule, block_tables, context_lens, num_blocks, n_q_heads, n_kv_heads,
                         head_dim, dtype, fp8=False, err=None) -> BoundLaunch:
    build_decode_schedule(schedule, block_tables, context_lens, num_blocks, n_q_heads, n_kv_heads,
                          head_dim, dtype, fp8, err)  # validates (and runs once)
    args = (schedule.data_ptr(), schedule.numel() * schedule.element_size(), block_tables.data_ptr(),
            block_tables.stride(0), block_tables.shape[1], context_lens.data_ptr(),
            context_lens.shape[0], num_blocks, n_q_heads, n_kv_heads, head_dim, 16, dtype_code(dtype),
            int(bool(fp8)), _ptr(err), _stream(context_lens))
    return BoundLaunch(_lib.load().pkv_decode_schedule, args, "pkv_decode_schedule",
                       (schedule, block_tables, context_lens, err))


def bind_reshape_and_cache(k, v, k_pool, v_pool, slot_mapping, err=None) -> BoundLaunch:
    args = _reshape_and_cache_args(k, v, k_pool, v_pool, slot_mapping, err)
    return BoundLaunch(_lib.load().pkv_reshape_and_cache, args, "pkv_reshape_and_cache",
                       (k, v, k_pool, v_pool, slot_mapping, err))


def bind_paged_decode_attention(q, k_pool, v_pool, block_tables, context_lens, scale, workspace,
                                out, err=None, schedule=None) -> BoundLaunch:
    args, out = _decode_args(q, k_pool, v_pool, block_tables, context_lens, scale, workspace, out, err)
    return BoundLaunch(_sched_fn("pkv_paged_decode_attention", schedule), _sched_args(args, schedule),
                       "pkv_paged_decode_attention",
                       (q, k_pool, v_pool, block_tables, context_lens, workspace, out, err, schedule))


def bind_paged_decode_append_attention(q, k_new, v_new, k_pool, v_pool, block_tables, context_lens,
                                       scale, workspace, out, err=None, schedule=None) -> BoundLaunch:
    args, out = _decode_append_args(q, k_new, v_new, k_pool, v_pool, block_tables, context_lens,
                                    scale, workspace, out, err)
    return BoundLaunch(_sched_fn("pkv_paged_decode_append_attention", schedule),
                       _sched_args(args, schedule), "pkv_paged_decode_append_attention",
                       (q, k_new, v_new, k_pool, v_pool, block_tables, context_lens, workspace, out,
                        err, schedule))


def _prefill_args(q, k_pool, v_pool, block_tables, query_start_loc, num_prior, max_query_len,
                  scale, out, err):
    for t, n in ((q, "q"), (k_pool, "k_pool"), (v_pool, "v_pool"),
                 (query_start_loc, "query_start_loc"), (num_prior, "num_prior")):
        _cuda(t, n)
    _check_tables(block_tables)
    for t, n in ((query_start_loc, "query_start_loc"), (num_prior, "num_prior")):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise TypeError(f"pagedkv: {n} must be a contiguous int32 tensor")
    if q.dtype != k_pool.dtype or k_pool.dtype != v_pool.dtype:
        raise TypeError("pagedkv: q and the pools must share one dtype")
    nb, bs, hkv, d = k_pool.shape
    T, hq, dq = q.shape
    B = num_prior.shape[0]
    if dq != d or query_start_loc.shape[0] != B + 1 or block_tables.shape[0] < B:
        raise ValueError("pagedkv: q / query_start_loc / num_prior / block_tables shapes disagree")
    if out is None:
        out = torch.empty_like(q, memory_format=torch.contiguous_format)
    args = (out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
            k_pool.data_ptr(), v_pool.data_ptr(), nb, block_tables.data_ptr(), block_tables.stride(0),
            block_tables.shape[1], query_start_loc.data_ptr(), num_prior.data_ptr(), B, T,
            int(max_query_len), hq, hkv, d, bs, float(scale), dtype_code(q.dtype), _ptr(err),
            _stream(q))
    return args, out


def paged_prefill_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor,
                            block_tables: torch.Tensor, query_start_loc: torch.Tensor,
                            num_prior: torch.Tensor, max_query_len: int, scale: float,
                            out: torch.Tensor | None = None,
                            err: torch.Tensor | None = None) -> torch.Tensor:
    """Chunked prefill: sequence s owns q rows [qsl[s], qsl[s+1]); its new token
    i attends to keys 0 .. num_prior[s] + i through block_tables[s].
    max_query_len must be >= every chunk length.
    Reference: qwen2.py:98-128 causal mask with the num_prior offset.
    """
    args, out = _prefill_args(q, k_pool, v_pool, block_tables, query_start_loc, num_prior,
                              max_query_len, scale, out, err)
    if args[13] == 0:
        return out
    _lib.check(_lib.load().pkv_paged_prefill_attention(*args), "pkv_paged_prefill_attention")
    return out


class PrefillPlan:
    """paged_prefill_attention for the layers of one step, which share block
    tables, query_start_loc, num_prior, max_query_len, scale and error word,
    with the same reuse of validated arguments as DecodePlan (pointers
    swapped: out, q, pools)."""

    def __init__(self, block_tables, query_start_loc, num_prior, max_query_len, scale, err=None):
        self._static = (block_tables, query_start_loc, num_prior, max_query_len, scale, err)
        self.scale = scale
        self._key = None
        self._args: list = []

    def __call__(self, q, k_pool, v_pool, out) -> torch.Tensor:
        key = (q.dtype, k_pool.dtype, v_pool.dtype, out.dtype, q.shape, q.stride(), k_pool.shape,
               k_pool.stride(), v_pool.shape, v_pool.stride(), out.shape, out.stride(),
               q.get_device(), _raw_stream(q))
        if key != self._key:
            tables, qsl, prior, mql, scale, err = self._static
            args, out = _prefill_args(q, k_pool, v_pool, tables, qsl, prior, mql, scale, out, err)
            self._args, self._key = list(args), key
        else:
            a = self._args
            a[0], a[2], a[4], a[5] = out.data_ptr(), q.data_ptr(), k_pool.data_ptr(), v_pool.data_ptr()
        if self._args[13] == 0:
            return out
        rc = _lib.load().pkv_paged_prefill_attention(*self._args)
        if rc:
            _lib.check(rc, "pkv_paged_prefill_attention")
        return out


def bind_paged_prefill_attention(q, k_pool, v_pool, block_tables, query_start_loc, num_prior,
                                 max_query_len, scale, out, err=None) -> BoundLaunch:
    args, out = _prefill_args(q, k_pool, v_pool, block_tables, query_start_loc, num_prior,
                              max_query_len, scale, out, err)
    return BoundLaunch(_lib.load().pkv_paged_prefill_attention, args, "pkv_paged_prefill_attention",
                       (q, k_pool, v_pool, block_tables, query_start_loc, num_prior, out, err))


def set_decode_impl(impl: int) -> None:
    _lib.check(_lib.load().pkv_set_decode_impl(int(impl)), "pkv_set_decode_impl")


def bind_reshape_and_cache_fp8(k, v, k_pool, v_pool, k_scale, v_scale, slot_mapping,
                               err=None) -> BoundLaunch:
    nb, bs, hkv, d = _check_fp8_pools(k_pool, v_pool, k_scale, v_scale)
    reshape_and_cache_fp8(k, v, k_pool, v_pool, k_scale, v_scale, slot_mapping, err)  # validates
    args = (k.data_ptr(), v.data_ptr(), _row_stride(k, "k"), _row_stride(v, "v"), k_pool.data_ptr(),
            v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), slot_mapping.data_ptr(),
            slot_mapping.shape[0], nb, bs, hkv, d, dtype_code(k.dtype), _ptr(err), _stream(k))
    return BoundLaunch(_lib.load().pkv_reshape_and_cache_fp8, args, "pkv_reshape_and_cache_fp8",
                       (k, v, k_pool, v_pool, k_scale, v_scale, slot_mapping, err))


def bind_paged_decode_attention_fp8(q, k_pool, v_pool, k_scale, v_scale, block_tables, context_lens,
                                    scale, workspace, out, err=None, schedule=None) -> BoundLaunch:
    nb, bs, hkv, d = _check_fp8_pools(k_pool, v_pool, k_scale, v_scale)
    paged_decode_attention_fp8(q, k_pool, v_pool, k_scale, v_scale, block_tables, context_lens, scale,
                               workspace, out, err, schedule)  # validates (and runs once)
    B, hq, _ = q.shape
    args = (out.data_ptr(), _row_stride(out, "out"), q.data_ptr(), _row_stride(q, "q"),
            k_pool.data_ptr(), v_pool.data_ptr(), k_scale.data_ptr(), v_scale.data_ptr(), nb,
            block_tables.data_ptr(), block_tables.stride(0), block_tables.shape[1],
            context_lens.data_ptr(), B, hq, hkv, d, bs, float(scale), dtype_code(q.dtype),
            workspace.data_ptr(), workspace.numel() * workspace.element_size(), _ptr(err), _stream(q))
    return BoundLaunch(_sched_fn("pkv_paged_decode_attention_fp8", schedule),
                       _sched_args(args, schedule), "pkv_paged_decode_attention_fp8",
                       (q, k_pool, v_pool, k_scale, v_scale, block_tables, context_lens, workspace,
                        out, err, schedule))
