"""Qwen2-architecture forward pass whose attention runs on the paged-KV kernels.

The layer math follows the reference's Qwen2Model.forward
(mini_engine/model/qwen2.py:130-183): embedding -> per layer [RMSNorm ->
q/k/v projections with bias -> RoPE (K rotated before it is cached) ->
attention -> o_proj -> residual -> RMSNorm -> SwiGLU MLP -> residual] ->
final RMSNorm -> tied LM head on the last new token of each sequence.  The
weights use the reference's (Hugging Face) names, so one weight dict drives
both this model and the reference's.

What changes is the attention call site (qwen2.py:152-166): instead of RoPE
on q and k and a Python loop of append_and_fetch + _attention per sequence,
each layer makes one fused q/k/v projection GEMM and calls
PagedKVCache.forward_layer_qkv with the step metadata built by prepare_step:
one launch rotates q and k and appends k and v (bit-identical to the torch
RoPE + append), then one decode launch for the leading one-token sequences
and one chunked-prefill launch for the rest.  fused_rope=False keeps RoPE as
torch operations and calls forward_layer (the same results).  RMSNorm, the
MLP and the LM head stay torch operations (out of scope of the KV path).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from .block_manager import PagedKVCache


@dataclass
class Qwen2Config:
    """Qwen2.5-0.5B geometry (the reference's mini_engine/model/config.py:13-23)."""

    vocab_size: int = 151936
    hidden_size: int = 896
    intermediate_size: int = 4864
    num_hidden_layers: int = 24
    num_attention_heads: int = 14
    num_key_value_heads: int = 2
    head_dim: int = 64
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1000000.0


@dataclass
class SequenceForwardInfo:
    """One sequence's slice of the flat token batch (reference qwen2.py:22-29)."""

    seq_id: int
    flat_start: int
    num_tokens: int
    positions: np.ndarray  # absolute positions of the new tokens


def random_weights(cfg: Qwen2Config, seed: int = 0, std: float = 0.02,
                   final_norm_scale: float = 1.0) -> dict[str, torch.Tensor]:
    """Seeded random weights with the reference's names, fp32 on the CPU.

    Matrices and biases ~ N(0, std^2), layer RMSNorm weights 1; the final
    RMSNorm weight is final_norm_scale, which spreads the tied-embedding
    logits so greedy choices are well separated.  Generated with a CPU
    torch.Generator so every machine with the same torch build gets the same
    tensors.
    """
    g = torch.Generator().manual_seed(seed)
    H, I, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    qd = cfg.num_attention_heads * cfg.head_dim
    kd = cfg.num_key_value_heads * cfg.head_dim

    def n(*shape):
        return torch.randn(*shape, generator=g) * std

    w = {"model.embed_tokens.weight": n(V, H)}
    for layer in range(cfg.num_hidden_layers):
        p = f"model.layers.{layer}"
        w[f"{p}.input_layernorm.weight"] = torch.ones(H)
        w[f"{p}.self_attn.q_proj.weight"] = n(qd, H)
        w[f"{p}.self_attn.q_proj.bias"] = n(qd)
        w[f"{p}.self_attn.k_proj.weight"] = n(kd, H)
        w[f"{p}.self_attn.k_proj.bias"] = n(kd)
        w[f"{p}.self_attn.v_proj.weight"] = n(kd, H)
        w[f"{p}.self_attn.v_proj.bias"] = n(kd)
        w[f"{p}.self_attn.o_proj.weight"] = n(H, qd)
        w[f"{p}.post_attention_layernorm.weight"] = torch.ones(H)
        w[f"{p}.mlp.gate_proj.weight"] = n(I, H)
        w[f"{p}.mlp.up_proj.weight"] = n(I, H)
        w[f"{p}.mlp.down_proj.weight"] = n(H, I)
    w["model.norm.weight"] = torch.full((H,), final_norm_scale)
    return w


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """The reference's RMSNorm as written (qwen2.py:32-35): fp32 math, the
    weight applied in fp32, one rounding to x's dtype.  The model's forward
    uses torch's fused F.rms_norm, the same formula in one kernel."""
    dt = x.dtype
    xf = x.float()
    xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * weight.float()).to(dt)


class Rope:
    """Rotary embedding tables: angle(pos, i) = pos * theta^(-2i/d), the two
    halves of the head dimension rotated as a pair (cos/sin computed in fp32,
    stored in the model dtype; tables grow by doubling)."""

    def __init__(self, head_dim: int, theta: float, device, dtype):
        self.inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))
        self.device, self.dtype = device, dtype
        self.cos = self.sin = None
        self.n = 0

    def tables(self, max_pos: int):
        if max_pos > self.n:
            n = max(max_pos, 4096, 2 * self.n)
            ang = torch.outer(torch.arange(n, device=self.device).float(), self.inv_freq)
            ang = torch.cat((ang, ang), dim=-1)
            self.cos, self.sin, self.n = ang.cos().to(self.dtype), ang.sin().to(self.dtype), n
        return self.cos, self.sin

    @staticmethod
    def rotate(x, cos, sin):
        half = x.shape[-1] // 2
        rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
        return x * cos + rot * sin


class PagedQwen2Model:
    """Qwen2 forward over a flat token batch with paged attention."""

    def __init__(self, cfg: Qwen2Config, weights: dict[str, torch.Tensor], device="cuda",
                 dtype=torch.float16, fused_rope: bool = True):
        self.cfg, self.device, self.dtype = cfg, torch.device(device), dtype
        self.fused_rope = fused_rope
        # when a list: forward() appends (step start, step end, [(attn start,
        # attn end) per layer]) CUDA events -- the attention share diagnostic
        self.timing: list | None = None
        dev = self.device
        w = {k: v.to(device=dev, dtype=dtype) for k, v in weights.items()}
        self.embed = w["model.embed_tokens.weight"]
        self.final_norm = w["model.norm.weight"]
        self.layers = []
        for layer in range(cfg.num_hidden_layers):
            p = f"model.layers.{layer}"
            self.layers.append(dict(
                ln1=w[f"{p}.input_layernorm.weight"],
                wqkv=torch.cat([w[f"{p}.self_attn.q_proj.weight"], w[f"{p}.self_attn.k_proj.weight"],
                                w[f"{p}.self_attn.v_proj.weight"]]),
                bqkv=torch.cat([w[f"{p}.self_attn.q_proj.bias"], w[f"{p}.self_attn.k_proj.bias"],
                                w[f"{p}.self_attn.v_proj.bias"]]),
                wo=w[f"{p}.self_attn.o_proj.weight"],
                ln2=w[f"{p}.post_attention_layernorm.weight"],
                # gate and up projections as one [2 I, H] GEMM operand
                wgu=torch.cat([w[f"{p}.mlp.gate_proj.weight"], w[f"{p}.mlp.up_proj.weight"]]),
                wdown=w[f"{p}.mlp.down_proj.weight"]))
        self.rope = Rope(cfg.head_dim, cfg.rope_theta, dev, dtype)
        self.scale = cfg.head_dim ** -0.5

    @torch.inference_mode()
    def forward(self, input_ids: torch.Tensor, seq_infos: list[SequenceForwardInfo],
                kv_cache: PagedKVCache) -> torch.Tensor:
        """input_ids [T] (flat over sequences, on the device) -> logits of the
        last new token of each sequence [n_seqs, vocab]."""
        cfg = self.cfg
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        meta = kv_cache.prepare_step([(s.seq_id, s.num_tokens) for s in seq_infos])
        pos_np = np.concatenate([s.positions for s in seq_infos]).astype(np.int64)
        positions = torch.from_numpy(pos_np).pin_memory().to(self.device, non_blocking=True)
        cos_t, sin_t = self.rope.tables(int(pos_np.max()) + 1)
        fused = self.fused_rope
        if not fused:
            cos, sin = cos_t[positions].unsqueeze(1), sin_t[positions].unsqueeze(1)
        timing = self.timing
        if timing is not None:
            ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
            t_step = (ev(), ev())
            t_attn = [(ev(), ev()) for _ in self.layers]
            t_step[0].record()
        h = self._layers(self.embed[input_ids], positions, cos_t, sin_t,
                         None if fused else (cos, sin), meta, kv_cache,
                         t_attn if timing is not None else None)
        h = F.rms_norm(h, (cfg.hidden_size,), self.final_norm, cfg.rms_norm_eps)
        last = torch.tensor([s.flat_start + s.num_tokens - 1 for s in seq_infos])
        if self.device.type == "cuda":  # a pageable copy would wait for the whole step
            last = last.pin_memory().to(self.device, non_blocking=True)
        logits = F.linear(h[last], self.embed)
        if timing is not None:
            t_step[1].record()
            timing.append((t_step, t_attn))
        return logits

    def _layers(self, h, positions, cos_t, sin_t, rot, meta, kv_cache, t_attn=None, advance=True):
        """The 24 decoder layers over the flat batch h [T, hidden] (the step's
        metadata in `meta`); rot = (cos, sin) per token for the unfused RoPE,
        None for the fused RoPE + append launch.

        The reference's layer math (qwen2.py:143-176) in fewer launches, all
        torch operations outside the attention: fused F.rms_norm; the residual
        adds folded into the o_proj and down_proj GEMMs (addmm: the sum is
        rounded once); gate and up as one GEMM."""
        cfg = self.cfg
        hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        H, I, eps = cfg.hidden_size, cfg.intermediate_size, cfg.rms_norm_eps
        T = h.shape[0]
        for li, lw in enumerate(self.layers):
            residual = h
            x = F.rms_norm(h, (H,), lw["ln1"], eps)
            qkv = F.linear(x, lw["wqkv"], lw["bqkv"])
            if t_attn is not None:
                t_attn[li][0].record()
            if rot is None:
                attn = kv_cache.forward_layer_qkv(li, qkv, positions, cos_t, sin_t, meta, self.scale,
                                                  advance=advance)
            else:
                cos, sin = rot
                q = Rope.rotate(qkv[:, : hq * d].view(T, hq, d), cos, sin)
                k = Rope.rotate(qkv[:, hq * d: (hq + hkv) * d].view(T, hkv, d), cos, sin)
                v = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
                attn = kv_cache.forward_layer(li, q, k, v, meta, self.scale, advance=advance)
            if t_attn is not None:
                t_attn[li][1].record()
            h = torch.addmm(residual, attn.view(T, hq * d), lw["wo"].t())
            residual = h
            x = F.rms_norm(h, (H,), lw["ln2"], eps)
            gu = torch.mm(x, lw["wgu"].t())
            h = torch.addmm(residual, F.silu(gu[:, :I]) * gu[:, I:], lw["wdown"].t())
        return h
