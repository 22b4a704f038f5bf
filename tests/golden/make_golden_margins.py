"""Top-1 minus top-2 logit margins of the reference's greedy tokens.

    python tests/golden/make_golden_margins.py

Reads the reference's token streams (tests/golden/e2e_greedy.json) and, for
every generated token, records how far the chosen logit was above the
runner-up, from a dense fp32 teacher-forced forward pass over prompt + outputs
with the same seeded weights (plain torch on the CPU: embedding, 24 x
[RMSNorm, q/k/v with bias, RoPE, causal GQA attention, o_proj, SwiGLU MLP],
final RMSNorm, tied LM head -- the math of mini_engine/model/qwen2.py:130-183
without the paged cache).  That forward reproduces every reference token.

An fp16 run moves a top-1/top-2 gap by up to ~0.026 logits on these weights
(measured the same way with the dense forward in fp16), so an fp16 stream can
legitimately part from the fp32 reference at a token whose margin is that
small; tests/test_e2e_gpu.py uses these margins to tell such a near-tie from a
real error.  Writes tests/golden/e2e_margins.json.
"""

import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(ROOT, "llm-inference-scheduler_b200"))
import cases as C  # noqa: E402
from pagedkv.model import Qwen2Config, Rope, random_weights, rms_norm  # noqa: E402


def dense_logits(w, cfg: Qwen2Config, ids: list[int], dtype=torch.float32) -> torch.Tensor:
    """Logits [len(ids), vocab] of a dense causal forward (no KV cache)."""
    W = {k: v.to(dtype) for k, v in w.items()}
    T = len(ids)
    hq, hkv, d = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
    cos, sin = Rope(d, cfg.rope_theta, "cpu", dtype).tables(T)
    cos, sin = cos[:T].unsqueeze(1), sin[:T].unsqueeze(1)
    h = W["model.embed_tokens.weight"][torch.tensor(ids)]
    for layer in range(cfg.num_hidden_layers):
        p = f"model.layers.{layer}"
        x = rms_norm(h, W[f"{p}.input_layernorm.weight"], cfg.rms_norm_eps)
        q = F.linear(x, W[f"{p}.self_attn.q_proj.weight"], W[f"{p}.self_attn.q_proj.bias"]).view(T, hq, d)
        k = F.linear(x, W[f"{p}.self_attn.k_proj.weight"], W[f"{p}.self_attn.k_proj.bias"]).view(T, hkv, d)
        v = F.linear(x, W[f"{p}.self_attn.v_proj.weight"], W[f"{p}.self_attn.v_proj.bias"]).view(T, hkv, d)
        q, k = Rope.rotate(q, cos, sin), Rope.rotate(k, cos, sin)
        k = k.repeat_interleave(hq // hkv, dim=1)
        v = v.repeat_interleave(hq // hkv, dim=1)
        a = F.scaled_dot_product_attention(q.transpose(0, 1).float(), k.transpose(0, 1).float(),
                                           v.transpose(0, 1).float(), is_causal=True)
        a = a.transpose(0, 1).to(dtype).reshape(T, hq * d)
        h = h + F.linear(a, W[f"{p}.self_attn.o_proj.weight"])
        x = rms_norm(h, W[f"{p}.post_attention_layernorm.weight"], cfg.rms_norm_eps)
        h = h + F.linear(F.silu(F.linear(x, W[f"{p}.mlp.gate_proj.weight"])) *
                         F.linear(x, W[f"{p}.mlp.up_proj.weight"]), W[f"{p}.mlp.down_proj.weight"])
    h = rms_norm(h, W["model.norm.weight"], cfg.rms_norm_eps)
    return F.linear(h, W["model.embed_tokens.weight"]).float()


def main():
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    cfg = Qwen2Config()
    w = random_weights(cfg, seed=C.E2E_SEED, final_norm_scale=C.E2E_FINAL_NORM_SCALE)
    with open(os.path.join(HERE, "e2e_greedy.json")) as f:
        g = json.load(f)
    out = {}
    for name, sc in C.e2e_scenarios().items():
        outs = g[name]["outputs"]
        prompts = list(sc["prompts"])
        if sc["turn2_extra"] is not None:
            prompts.append(prompts[0] + outs[0] + sc["turn2_extra"])
        margins = []
        for prompt, gen in zip(prompts, outs):
            ids = prompt + gen
            logits = dense_logits(w, cfg, ids[:-1])
            pos = np.arange(len(prompt) - 1, len(ids) - 1)
            top = logits[pos].topk(2, dim=-1)
            assert top.indices[:, 0].tolist() == gen, "dense forward disagrees with the reference"
            margins.append([round(float(m), 5) for m in (top.values[:, 0] - top.values[:, 1])])
        out[name] = margins
        print(name, [min(m) for m in margins], flush=True)
    with open(os.path.join(HERE, "e2e_margins.json"), "w") as f:
        json.dump(out, f)


if __name__ == "__main__":
    main()
