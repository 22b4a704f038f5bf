"""End-to-end greedy decoding through the paged path vs the reference.

The golden streams come from the reference's own Scheduler + Qwen2Model +
BlockManager on the CPU, with seeded random Qwen2.5-0.5B-shaped weights:
* tests/golden/e2e_greedy.json: fp32 (make_golden_e2e.py);
* tests/golden/e2e_greedy_f16.json: fp16 weights and fp16 KV pools, with the
  reference's top-2 token ids and fp16 logits at every generated token
  (make_golden_e2e_f16.py).
Here the same weights drive PagedQwen2Model through pagedkv.engine on the GPU:
every attention call goes through prepare_step / forward_layer(_qkv) (RoPE +
append, decode and chunked-prefill kernels), reused prefix blocks come from
the prefix index, copies from copy_blocks.  Greedy streams depend only on
each sequence's tokens, not on how the engine batches them.

* fp32: every stream is identical to the reference's.
* fp16, teacher-forced: the engine is fed the reference's fp16 tokens and
  reports its own logits at every generated token.  The gap between the
  reference's top-1 and top-2 tokens must agree with the reference's fp16 gap
  within FP16_GAP_TOL at every token; the engine's own greedy choice may
  differ from the reference's only where the reference's gap is itself within
  FP16_GAP_TOL, and at most once per request.
* fp16, free running: each stream equals the reference's fp16 stream up to
  its first divergence, which must fall on such a near-tie.

FP16_GAP_TOL: the reference's fp16 logits are rounded to fp16 (1 ulp =
0.0078 for logits in [8, 16), 0.0039 in [4, 8)), and its hidden states carry
fp16 rounding at every GEMM, norm and attention output (scores rounded to
fp16, probabilities cast to fp16 before PV, qwen2.py:116-127) that this
path's kernels, accumulating in fp32, do not repeat.  Measured between the
two on these weights: a gap differs by at most 0.03 logits (the test prints
its maximum).  The tolerance is 0.0625, 8 ulps of a logit in [8, 16).
"""

import json

import pytest
import torch

import cases as C
from conftest import GOLDEN
from pagedkv import BlockManager
from pagedkv.engine import Engine, Seq
from pagedkv.model import PagedQwen2Model, Qwen2Config, random_weights

pytestmark = pytest.mark.gpu

FP16_GAP_TOL = 0.0625


@pytest.fixture(scope="module")
def golden_e2e():
    with open(f"{GOLDEN}/e2e_greedy.json") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def golden_f16():
    with open(f"{GOLDEN}/e2e_greedy_f16.json") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def weights():
    return random_weights(Qwen2Config(), seed=C.E2E_SEED, final_norm_scale=C.E2E_FINAL_NORM_SCALE)


def run_engine(model, sc, dtype, **kw):
    mgr = BlockManager(sc["num_blocks"], 16, 24, 2, 64, device="cuda", dtype=dtype)
    eng = Engine(model, mgr, max_seqs=sc["max_num_seqs"], token_budget=sc["max_batched_tokens"],
                 prefix_reuse=sc["prefix_cache"], eos_ids={-1}, **kw)
    seqs = [eng.submit(Seq(i, list(p), limit=sc["max_new_tokens"])) for i, p in enumerate(sc["prompts"])]
    eng.run(5000)
    if sc["turn2_extra"] is not None:
        s0 = seqs[0]
        seqs.append(eng.submit(Seq(len(seqs), s0.prompt + s0.generated + sc["turn2_extra"],
                                   limit=sc["max_new_tokens"])))
        eng.run(5000)
    mgr.check_errors()
    assert not eng.busy
    return seqs, eng


def first_divergence(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None if len(a) == len(b) else min(len(a), len(b))


@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "graphs"])
@pytest.mark.parametrize("scenario", ["prefix", "preempt"])
def test_fp32_greedy_streams_identical_to_reference(golden_e2e, weights, scenario, graphs):
    """graphs: steps replay CUDA graphs (pagedkv.graphs); the table width
    starts at 2 blocks so the runner also regrows and recaptures."""
    sc = C.e2e_scenarios()[scenario]
    g = golden_e2e[scenario]
    model = PagedQwen2Model(Qwen2Config(), weights, device="cuda", dtype=torch.float32)
    seqs, eng = run_engine(model, sc, torch.float32, cuda_graphs=graphs, graph_max_blocks=2)
    if graphs:
        assert eng.graphs.replays > 0 and eng.graphs.W > 2
    for s, ref in zip(seqs, g["outputs"]):
        assert s.generated == ref, (
            f"seq {s.ident}: first divergence at token {first_divergence(s.generated, ref)}")
    assert eng.counts["generated"] == g["metrics"]["tokens_generated"]
    assert eng.counts["finished"] == g["metrics"]["requests_finished"]
    if scenario == "prefix":   # the second turn reuses the first turn's blocks
        assert seqs[-1].reused > 0
    else:                      # the 11-block pool forces recompute preemption
        assert eng.counts["preemptions"] > 0


@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "graphs"])
def test_fp32_unfused_rope_path_identical_to_reference(golden_e2e, weights, graphs):
    """The same fp32 parity through the unfused path (torch RoPE +
    forward_layer with the decode kernel's own append)."""
    sc = C.e2e_scenarios()["prefix"]
    g = golden_e2e["prefix"]
    model = PagedQwen2Model(Qwen2Config(), weights, device="cuda", dtype=torch.float32,
                            fused_rope=False)
    seqs, eng = run_engine(model, sc, torch.float32, cuda_graphs=graphs)
    assert not graphs or eng.graphs.replays > 0
    for s, ref in zip(seqs, g["outputs"]):
        assert s.generated == ref, (
            f"seq {s.ident}: first divergence at token {first_divergence(s.generated, ref)}")


@pytest.mark.parametrize("graphs", [False, True], ids=["eager", "graphs"])
@pytest.mark.parametrize("scenario", ["prefix", "preempt"])
def test_fp16_teacher_forced_logit_gaps_match_reference_fp16(golden_f16, weights, scenario, graphs):
    sc = C.e2e_scenarios()[scenario]
    g = golden_f16[scenario]
    model = PagedQwen2Model(Qwen2Config(), weights, device="cuda", dtype=torch.float16)
    seen = {}  # seq -> [(our greedy token, our gap between the reference's top-2)]

    def force(seq, token, row):
        t = len(seq.generated)
        i1, _, i2, _ = g["top2"][seq.ident][t]
        gap = float(row[i1].float() - row[i2].float())
        seen.setdefault(seq.ident, []).append((token, gap))
        return g["outputs"][seq.ident][t]

    seqs, eng = run_engine(model, sc, torch.float16, cuda_graphs=graphs, choose=force)
    assert not graphs or eng.graphs.replays > 0
    worst, flips = 0.0, []
    for s in seqs:
        assert s.generated == g["outputs"][s.ident]
        mine = seen[s.ident]
        assert len(mine) == len(g["top2"][s.ident])
        n_flip = 0
        for t, ((tok, gap), (i1, v1, _, v2)) in enumerate(zip(mine, g["top2"][s.ident])):
            ref_gap = v1 - v2
            worst = max(worst, abs(gap - ref_gap))
            assert abs(gap - ref_gap) <= FP16_GAP_TOL, (
                f"seq {s.ident} token {t}: gap {gap:.4f} vs the reference's fp16 {ref_gap:.4f}")
            if tok != i1:
                n_flip += 1
                flips.append((s.ident, t, round(ref_gap, 4)))
                assert ref_gap <= FP16_GAP_TOL, (s.ident, t, ref_gap)
        assert n_flip <= 1, f"seq {s.ident}: {n_flip} greedy choices differ from the reference's"
    print(f"\n{scenario}/{'graphs' if graphs else 'eager'}: max |gap - reference fp16 gap| = "
          f"{worst:.4f}; greedy choices that differ (seq, token, reference gap): {flips}")


@pytest.mark.parametrize("scenario", ["prefix", "preempt"])
def test_fp16_greedy_streams_match_reference_fp16(golden_f16, weights, scenario):
    sc = C.e2e_scenarios()[scenario]
    g = golden_f16[scenario]
    model = PagedQwen2Model(Qwen2Config(), weights, device="cuda", dtype=torch.float16)
    seqs, eng = run_engine(model, sc, torch.float16, cuda_graphs=True)
    for s, ref, marg in zip(seqs, g["outputs"], g["margins"]):
        assert len(s.generated) == len(ref)
        d = first_divergence(s.generated, ref)
        if d is not None:
            assert marg[d] <= FP16_GAP_TOL, (
                f"seq {s.ident}: token {d} differs where the reference's fp16 gap is {marg[d]}")
