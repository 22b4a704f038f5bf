"""CUDA-graph steps (pagedkv.graphs.StepGraphs) against the eager step.

Steps of a random-init Qwen2.5-0.5B-shaped model over pools of random K/V,
run twice from the same state: eagerly (PagedQwen2Model.forward) and by graph
replay, with batches that are not bucket sizes so padding is in the graph:
* decode-only: 13 sequences (bucket 16), two steps;
* mixed: 13 decodes and two prefill chunks (40 tokens after a 37-token
  prior context, 100 tokens of a fresh prompt) in the (16, 192) graph, then
  a decode-only step of all 15 sequences.
Checks:
* the logits agree to rounding (the GEMMs see padded M, so the library may
  pick another algorithm) and the greedy tokens are equal where the top two
  logits are apart;
* each run changes the pools only at the steps' appended slots (padding rows
  and padding sequences write nothing), and both runs write every one of
  them, to rounding (16-bit pools) or to the fp8 scale tolerance;
* the lengths advance as after the eager steps.
"""

import numpy as np
import pytest
import torch

from pagedkv import BlockManager, PagedKVCache
from pagedkv.graphs import StepGraphs
from pagedkv.model import PagedQwen2Model, Qwen2Config, SequenceForwardInfo, random_weights

pytestmark = pytest.mark.gpu

V = Qwen2Config().vocab_size


@pytest.fixture(scope="module")
def model():
    cfg = Qwen2Config()
    return PagedQwen2Model(cfg, random_weights(cfg, seed=3, final_norm_scale=4.0), device="cuda",
                           dtype=torch.float16)


def _state(kv_dtype, lens, extra, seed):
    """Pools of random K/V and tables that already hold blocks for
    lens[s] + extra[s] tokens (no allocation during the runs)."""
    mgr = BlockManager(1200, 16, 24, 2, 64, device="cuda", dtype=kv_dtype)
    g = torch.Generator(device="cuda").manual_seed(seed)
    if kv_dtype == torch.float8_e4m3fn:
        mgr.k_cache.random_(0, 120, generator=g)  # finite e4m3 bytes
        mgr.v_cache.random_(0, 120, generator=g)
        mgr.k_scale_cache.uniform_(0.001, 0.01, generator=g)
        mgr.v_scale_cache.uniform_(0.001, 0.01, generator=g)
    else:
        mgr.k_cache.normal_(generator=g)
        mgr.v_cache.normal_(generator=g)
    tables = [[mgr.allocate() for _ in range((n + e + 15) // 16)] for n, e in zip(lens, extra)]
    return mgr, tables


def _pools(mgr):
    out = [mgr.k_cache, mgr.v_cache]
    if mgr.fp8:
        out += [mgr.k_scale_cache, mgr.v_scale_cache]
    return out


def _rows(mask):
    """(block, row) pairs where a [layers, blocks, 16, ...] mask is set."""
    m = mask.reshape(mask.shape[0], mask.shape[1], mask.shape[2], -1).any(-1).any(0)
    return {(int(b), int(r)) for b, r in torch.nonzero(m).tolist()}


def _run(model, mgr, lens, tables, steps, graphs: bool, seed: int):
    """steps: per step, [(sequence index, new tokens)] in flat order."""
    rng = np.random.default_rng(seed)
    kv = PagedKVCache(mgr)
    for s, (n, t) in enumerate(zip(lens, tables)):
        kv.add_sequence(100 + s, list(t), n)
    runner = StepGraphs(model, kv, max_batch=32, max_tokens=256) if graphs else None
    logits = []
    for step in steps:
        infos, flat = [], 0
        for s, n in step:
            p = kv.seq_len(100 + s)
            infos.append(SequenceForwardInfo(100 + s, flat, n, np.arange(p, p + n)))
            flat += n
        x = torch.tensor(rng.integers(0, V, size=flat), dtype=torch.long, device="cuda")
        if graphs:
            assert runner.supports(infos)
            out = runner.forward(x, infos)
        else:
            out = model.forward(x, infos, kv)
        logits.append(out.float().clone())
    torch.cuda.synchronize()
    mgr.check_errors()
    return logits, [p.clone() for p in _pools(mgr)], [kv.seq_len(100 + s) for s in range(len(lens))], runner


def _compare(model, kv_dtype, lens, steps, seed):
    extra = [0] * len(lens)
    for step in steps:
        for s, n in step:
            extra[s] += n
    mgr, tables = _state(kv_dtype, lens, extra, seed)
    before = [p.clone() for p in _pools(mgr)]
    le, pe, len_e, _ = _run(model, mgr, lens, tables, steps, graphs=False, seed=seed)
    for p, b in zip(_pools(mgr), before):
        p.copy_(b)
    lg, pg, len_g, runner = _run(model, mgr, lens, tables, steps, graphs=True, seed=seed)
    assert runner.replays == len(steps)
    assert len_g == len_e == [n + e for n, e in zip(lens, extra)]
    for a, b in zip(le, lg):
        # fp16 rounding through 24 layers of GEMMs that may run another
        # algorithm (padded M): measured max 0.037 on logits of magnitude ~5;
        # a systematic error would move the mean
        torch.testing.assert_close(b, a, atol=8e-2, rtol=2e-2)
        assert (b - a).abs().mean().item() < 5e-3
        top2 = a.topk(2, dim=-1).values
        clear = (top2[:, 0] - top2[:, 1]) > 0.1
        assert torch.equal(a.argmax(-1)[clear], b.argmax(-1)[clear])
    appended = {(t[p // 16], p % 16) for t, n, e in zip(tables, lens, extra) for p in range(n, n + e)}
    u8 = lambda x: x.view(torch.uint8)  # noqa: E731
    for i, (a, b, b0) in enumerate(zip(pe, pg, before)):
        assert _rows(u8(a) != u8(b0)) <= appended, f"pool {i}: the eager steps wrote elsewhere"
        assert _rows(u8(b) != u8(b0)) <= appended, f"pool {i}: the graph steps wrote elsewhere"
        if a.dtype == torch.float16:
            assert _rows(a != b0) == appended == _rows(b != b0)  # every appended row was written
            torch.testing.assert_close(b.float(), a.float(), atol=2e-2, rtol=1e-2)
        elif a.dtype == torch.float32:  # fp8 scales
            torch.testing.assert_close(b, a, atol=1e-4, rtol=2e-2)
    return runner


KV_DTYPES = pytest.mark.parametrize("kv_dtype", [torch.float16, torch.float8_e4m3fn], ids=["f16", "fp8"])


@KV_DTYPES
def test_graph_decode_steps_match_eager(model, kv_dtype):
    lens = np.random.default_rng(11).integers(1, 400, size=13).tolist()
    steps = [[(s, 1) for s in range(13)]] * 2
    runner = _compare(model, kv_dtype, lens, steps, seed=11)
    assert set(runner.graphs) == {(16, 0)}


@KV_DTYPES
def test_graph_mixed_step_matches_eager(model, kv_dtype):
    lens = np.random.default_rng(12).integers(1, 400, size=13).tolist() + [37, 0]
    steps = [[(s, 1) for s in range(13)] + [(13, 40), (14, 100)],
             [(s, 1) for s in range(15)]]
    runner = _compare(model, kv_dtype, lens, steps, seed=12)
    assert set(runner.graphs) == {(16, 192), (16, 0)}


# ---------------------------------------------------------------- DecodeStepGraph

def _decode_state(dt, ctx, nb, seed):
    """Two identical caches of one-layer-per-pool random K/V and scattered tables."""
    from pagedkv.graphs import DecodeStepGraph  # noqa: F401  (import check)

    L = 5
    g = torch.Generator(device="cuda").manual_seed(seed)
    kp = torch.randn((L, nb, 16, 2, 64), generator=g, device="cuda").to(dt)
    vp = torch.randn((L, nb, 16, 2, 64), generator=g, device="cuda").to(dt)
    perm = np.random.default_rng(seed).permutation(nb)
    out = []
    for _ in range(2):
        m = BlockManager(nb, 16, L, 2, 64, device="cuda", dtype=dt)
        m.k_cache.copy_(kp)
        m.v_cache.copy_(vp)
        kv = PagedKVCache(m)
        o = 0
        for s, c in enumerate(ctx):
            n = (int(c) + 16) // 16  # room for the step's token and one more
            kv.add_sequence(s, perm[o:o + n].tolist(), int(c) - 1)
            o += n
        out.append((m, kv))
    assert o <= nb
    return out


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_decode_step_graph_equals_forward_layers(dt):
    """DecodeStepGraph.run (host rows in, host outputs back, one graph replay)
    against forward_layers on a copy of the same cache: outputs and pools
    bit-identical, padding rows zero, lengths advanced, and a step that needs
    a wider table recaptures."""
    from pagedkv.graphs import DecodeStepGraph

    rng = np.random.default_rng(5)
    ctx = rng.integers(1, 300, size=21)
    ctx[:2] = [16, 17]
    (m1, kv1), (m2, kv2) = _decode_state(dt, ctx, 1024, 9)
    L, R, B = 5, 24, len(ctx)
    hqkv = torch.randn((L, R, 18, 64), dtype=torch.float32).to(dt).pin_memory()
    hout = torch.full((L, R, 14, 64), 7.0, dtype=dt).pin_memory()
    runner = DecodeStepGraph(kv1, hqkv, hout, 0.125, chunks=(1, 2, 2), max_blocks_per_seq=4)
    seqs = [(s, 1) for s in range(B)]
    for step in range(2):
        runner.run(seqs, advance=True)
        torch.cuda.synchronize()
        meta = kv2.prepare_step(seqs)
        d = hqkv.cuda()
        ref = kv2.forward_layers(0, d[:, :B, :14], d[:, :B, 14:16], d[:, :B, 16:18], meta, 0.125)
        torch.cuda.synchronize()
        m1.check_errors()
        assert torch.equal(hout[:, :B], ref.cpu()), step
        assert not hout[:, B:].float().abs().sum()  # padding rows: no keys, zero output
        assert torch.equal(m1.k_cache, m2.k_cache) and torch.equal(m1.v_cache, m2.v_cache)
        assert [kv1.seq_len(s) for s in range(B)] == [kv2.seq_len(s) for s in range(B)]
        assert [kv1.seq_len(s) for s in range(B)] == [int(c) + step for c in ctx]
    assert runner.replays == 2 and runner.W >= 32  # 300-token contexts outgrew 4 blocks
