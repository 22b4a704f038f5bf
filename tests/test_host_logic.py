"""Host-side bookkeeping of pagedkv.BlockManager / PagedKVCache against the
reference's behaviour (no GPU needed: bookkeeping-only managers, device=None).

The reference scenarios are mini_engine tests/test_block_manager.py:16-83 and
the config-2 fork/COW flow; their recorded outcomes live in tests/golden.
"""

import json
import os

import numpy as np
import pytest
import torch

import cases as C
from conftest import GOLDEN
from pagedkv import BlockManager, OutOfBlocks, PagedKVCache
from pagedkv import ops


def mgr(num_blocks=8, block_size=4, layers=2, heads=1, dim=2):
    return BlockManager(num_blocks, block_size, layers, heads, dim, device=None)


def test_allocate_free_cycle():
    """test_block_manager.py:16-24"""
    m = mgr(num_blocks=4)
    blocks = [m.allocate() for _ in range(4)]
    assert blocks == [0, 1, 2, 3]  # LIFO over range(n-1, -1, -1)
    assert m.num_free == 0
    with pytest.raises(OutOfBlocks):
        m.allocate()
    for b in blocks:
        m.decref(b)
    assert m.num_free == 4


def test_ref_counting_delays_free():
    """test_block_manager.py:27-34"""
    m = mgr()
    b = m.allocate()
    m.incref(b)
    m.decref(b)
    assert m.ref_count[b] == 1 and b not in m.free_list
    m.decref(b)
    assert m.num_free == m.num_blocks


def test_asserts_on_free_blocks():
    m = mgr()
    with pytest.raises(AssertionError):
        m.decref(3)
    with pytest.raises(AssertionError):
        m.incref(3)


def test_reference_scenarios_bookkeeping():
    """Tables, free list and COW outcome of the reference's own unit scenarios."""
    with open(f"{GOLDEN}/block_manager_ref.json") as f:
        g = json.load(f)
    m = mgr()
    kv = PagedKVCache(m)
    table = [m.allocate() for _ in range(3)]
    assert table == g["roundtrip"]["table"]
    kv.add_sequence(0, table, 0)
    assert list(m.free_list) == g["roundtrip"]["free_list"]

    m = mgr()
    kv = PagedKVCache(m)
    table = [m.allocate()]
    kv.add_sequence(0, table, 2)
    for b in table:
        m.incref(b)
    kv.add_sequence(1, list(table), 2)
    kv.ensure_writable_tail(1)
    assert {str(k): v for k, v in kv.block_tables.items()} == g["cow"]["tables_after_cow"]
    assert list(m.ref_count) == g["cow"]["ref_count"]
    assert list(m.free_list) == g["cow"]["free_list"]
    assert m.pending_copies == [(table[0], kv.block_tables[1][0])]


def test_config2_cow_pairs_match_reference():
    """The fork flow of config 2 allocates the same COW destinations, in the
    same order, as the reference's LIFO allocator over the seeded free list."""
    c = C.make_append_cow_case()
    with open(f"{GOLDEN}/append_cow_c2_f16.json") as f:
        g = json.load(f)
    m = BlockManager(c["num_blocks"], C.BS, c["n_layers"], C.HKV, C.D, device=None)
    m.free_list = list(c["free_list"])
    kv = PagedKVCache(m)
    n = len(c["ctx"])
    for s in range(n):
        ctx = int(c["ctx"][s])
        kv.add_sequence(s, [m.allocate() for _ in range((ctx + 15) // 16)], ctx)
    assert [kv.block_tables[s] for s in range(n)] == g["tables"]
    for i, s in enumerate(c["forked"]):
        s = int(s)
        for b in kv.block_tables[s]:
            m.incref(b)
        kv.add_sequence(n + i, list(kv.block_tables[s]), kv.seq_len(s))
        kv.ensure_writable_tail(n + i)
    assert [list(p) for p in m.pending_copies] == g["pairs"]
    assert {str(k): v for k, v in kv.block_tables.items() if k >= n} == g["child_tables"]
    assert list(m.ref_count) == g["ref_count"]
    assert list(m.free_list) == g["free_list"]
    assert m.flushes == 0  # 32 independent pairs fit one copy_blocks launch


def test_cow_queue_flushes_on_conflict():
    """A freed COW source that is re-allocated as a destination in the same
    step must not share a launch with the copy that reads it."""
    m = mgr(num_blocks=8)
    a = m.allocate()           # 0
    b = m.allocate()           # 1
    m.incref(a)                # shared
    d1 = m.copy_block(a)       # (0 -> 2) queued
    m.decref(a)
    m.decref(a)                # block 0 free again, top of the free list
    d2 = m.copy_block(b)       # allocates block 0, which the queued pair still reads
    assert d1 == 2 and d2 == a
    assert m.flushes == 1
    assert m.pending_copies == [(b, d2)]


def test_step_arrays_slots_tables_and_split():
    m = mgr(num_blocks=64, block_size=16)
    kv = PagedKVCache(m)
    kv.add_sequence(10, [m.allocate() for _ in range(3)], 33)   # decode at position 33
    kv.add_sequence(11, [m.allocate() for _ in range(2)], 15)   # decode at 15 (block edge)
    kv.add_sequence(12, [m.allocate() for _ in range(2)], 5)    # 20-token chunk
    kv.add_sequence(13, [m.allocate()], 0)                      # 3-token prompt
    a = kv.step_arrays([(10, 1), (11, 1), (12, 20), (13, 3)])
    assert a["n_decode"] == 2 and a["n_tokens"] == 25 and a["max_query_len"] == 20
    B, W = a["B"], a["W"]
    ints = a["ints"]
    tabs = ints[:B * W].reshape(B, W)
    assert tabs[0, :3].tolist() == kv.block_tables[10]
    assert ints[B * W:B * W + B].tolist() == [34, 16, 25, 3]
    assert ints[B * W + B:B * W + 2 * B].tolist() == [33, 15, 5, 0]
    assert ints[B * W + 2 * B:].tolist() == [0, 20, 23]

    # slots: the reference's scatter writes position p to table[p // bs], offset p % bs
    def ref_slots(seq, start, n):
        t = kv.block_tables[seq]
        return [t[p // 16] * 16 + p % 16 for p in range(start, start + n)]

    expect = ref_slots(10, 33, 1) + ref_slots(11, 15, 1) + ref_slots(12, 5, 20) + ref_slots(13, 0, 3)
    assert a["slots"].tolist() == expect


def test_step_arrays_capacity_assert():
    m = mgr(num_blocks=8, block_size=16)
    kv = PagedKVCache(m)
    kv.add_sequence(0, [m.allocate()], 16)
    with pytest.raises(AssertionError):
        kv.step_arrays([(0, 1)])


def test_step_arrays_padded_fixed_width_layout():
    """step_arrays(width=W, pad_to=R) (the CUDA-graph decode step): the real
    rows as in the unpadded arrays, re-laid for R rows of W blocks; padding
    rows have a zero table row, context length 0, num_prior 0 and slot -1."""
    m = mgr(num_blocks=64, block_size=16)
    kv = PagedKVCache(m)
    kv.add_sequence(10, [m.allocate() for _ in range(3)], 33)
    kv.add_sequence(11, [m.allocate() for _ in range(2)], 15)
    kv.add_sequence(12, [m.allocate() for _ in range(1)], 0)
    seqs = [(10, 1), (11, 1), (12, 1)]
    base = kv.step_arrays(seqs)
    B, W0 = base["B"], base["W"]
    bt0 = base["ints"][:B * W0].reshape(B, W0)
    R, W = 8, 5
    a = kv.step_arrays(seqs, width=W, pad_to=R)
    assert a["W"] == W and a["R"] == R and a["B"] == B and a["n_decode"] == B
    ints = a["ints"]
    assert ints.size == R * W + 2 * R + 1
    tabs = ints[:R * W].reshape(R, W)
    for i, (s, _) in enumerate(seqs):
        u = (kv.seq_len(s) + 1 + 15) // 16
        assert tabs[i, :u].tolist() == bt0[i, :u].tolist() == kv.block_tables[s][:u]
    assert not tabs[B:].any()
    assert ints[R * W:R * W + R].tolist() == [34, 16, 1] + [0] * (R - B)
    assert ints[R * W + R:R * W + 2 * R].tolist() == [33, 15, 0] + [0] * (R - B)
    assert ints[R * W + 2 * R:].tolist() == [0]
    assert a["slots"].tolist() == base["slots"].tolist() + [-1] * (R - B)
    with pytest.raises(AssertionError):  # a sequence needs 3 blocks
        kv.step_arrays(seqs, width=2, pad_to=R)
    with pytest.raises(AssertionError):  # padding is for decode-only steps
        kv.step_arrays([(10, 1), (12, 4)], pad_to=R)


def test_graph_buckets():
    from pagedkv.graphs import default_buckets, graph_keys, mixed_row_buckets, prefill_token_buckets
    assert default_buckets(1) == [1]
    assert default_buckets(6) == [1, 2, 4, 6]
    assert default_buckets(128) == [1, 2, 4, 8, 16, 32, 48, 64, 80, 96, 112, 128]
    assert default_buckets(200) == [1, 2, 4, 8, 16, 32, 48, 64, 80, 96, 112, 128, 160, 192, 200]
    assert mixed_row_buckets(3) == [3]
    assert mixed_row_buckets(128) == [16, 32, 64, 96, 128]
    assert prefill_token_buckets(48) == [32, 48]
    assert prefill_token_buckets(512) == [32, 64, 128, 192, 256, 320, 384, 448, 512]
    rows, toks = mixed_row_buckets(128), prefill_token_buckets(512)
    keys = graph_keys(default_buckets(128), rows, toks, 512)
    assert keys[:12] == [(b, 0) for b in default_buckets(128)]
    mixed = set(keys[12:])
    # a shape is kept iff its smallest step (one more than the buckets below) fits 512 tokens
    for i, R in enumerate(rows):
        for j, P in enumerate(toks):
            lo = (rows[i - 1] + 1 if i else 0) + (toks[j - 1] + 1 if j else 1)
            assert ((R, P) in mixed) == (lo <= 512), (R, P)
    assert (128, 448) in mixed and (128, 512) not in mixed and (16, 512) in mixed


def test_graph_mixed_layout():
    """StepGraphs._lay_mixed: the unpadded step arrays re-laid for an (R, P)
    graph: decode rows, padding to R, prefill sequences, empty ones; token
    rows likewise; LM-head rows = the decode rows then each chunk's last row."""
    from pagedkv.graphs import StepGraphs
    from pagedkv.model import SequenceForwardInfo
    m = mgr(num_blocks=64, block_size=16)
    kv = PagedKVCache(m)
    kv.add_sequence(1, [m.allocate() for _ in range(3)], 33)   # decode
    kv.add_sequence(2, [m.allocate() for _ in range(2)], 15)   # decode
    kv.add_sequence(3, [m.allocate() for _ in range(2)], 5)    # 20-token chunk
    kv.add_sequence(4, [m.allocate()], 0)                      # 3-token prompt
    seqs = [(1, 1), (2, 1), (3, 20), (4, 3)]
    infos, flat = [], 0
    for s, n in seqs:
        p = kv.seq_len(s)
        infos.append(SequenceForwardInfo(s, flat, n, np.arange(p, p + n)))
        flat += n
    g = StepGraphs.__new__(StepGraphs)  # layout only: no device state
    g.W, g.prefill_seqs = 4, 4
    R, P = 16, 32
    L = g._layout(R, P)
    a = kv.step_arrays(seqs, width=g.W)
    hnp = np.full(L["end"], 0x5A, dtype=np.uint8)  # stale bytes everywhere
    g._lay_mixed(hnp, L, R, a, infos)
    S, W = L["S"], g.W
    assert S == 20 and L["T"] == 48
    ints = hnp[:4 * L["n_ints"]].view(np.int32)
    tabs = ints[:S * W].reshape(S, W)
    assert tabs[0, :3].tolist() == kv.block_tables[1] and tabs[1, :2].tolist() == kv.block_tables[2]
    assert tabs[R, :2].tolist() == kv.block_tables[3] and tabs[R + 1, :1].tolist() == kv.block_tables[4]
    assert not tabs[2:R].any() and not tabs[R + 2:].any()
    ctx, prior = ints[S * W:S * W + S], ints[S * W + S:S * W + 2 * S]
    assert ctx.tolist() == [34, 16] + [0] * 14 + [25, 3, 0, 0]
    assert prior.tolist() == [33, 15] + [0] * 14 + [5, 0, 0, 0]
    assert ints[S * W + 2 * S:].tolist() == [0, 20, 23, 23, 23]
    slots = hnp[L["slots"]:L["slots"] + 8 * 48].view(np.int64)
    assert slots[:2].tolist() == a["slots"][:2].tolist()
    assert (slots[2:R] == -1).all() and (slots[R + 23:] == -1).all()
    assert slots[R:R + 23].tolist() == a["slots"][2:].tolist()
    pos = hnp[L["pos"]:L["pos"] + 8 * 48].view(np.int64)
    assert pos[:2].tolist() == [33, 15] and not pos[2:R].any()
    assert pos[R:R + 23].tolist() == list(range(5, 25)) + [0, 1, 2] and not pos[R + 23:].any()
    last = hnp[L["last"]:L["last"] + 8 * (R + 4)].view(np.int64)
    assert last.tolist() == [0, 1, R + 19, R + 22] + [0] * (R + 4 - 4)


def test_no_cpu_pools():
    with pytest.raises(RuntimeError):
        BlockManager(8, 16, 1, 2, 64, device="cpu")


def test_ops_refuse_cpu_tensors():
    k = torch.zeros(2, 2, 64, dtype=torch.float16)
    pool = torch.zeros(4, 16, 2, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.reshape_and_cache(k, k, pool, pool, torch.zeros(2, dtype=torch.int64))
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.paged_decode_attention(torch.zeros(2, 14, 64, dtype=torch.float16), pool, pool,
                                   torch.zeros(2, 1, dtype=torch.int32),
                                   torch.ones(2, dtype=torch.int32), 0.125)


def test_to_dtype_bf16_matches_torch():
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 37.0
    ours = C.to_dtype(x, "bf16")
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


def test_e2e_margin_fixture_matches_streams():
    """Every reference token of the e2e golden has its top-1/top-2 margin."""
    import json

    from conftest import GOLDEN

    with open(f"{GOLDEN}/e2e_greedy.json") as f:
        g = json.load(f)
    with open(f"{GOLDEN}/e2e_margins.json") as f:
        m = json.load(f)
    for name in ("prefix", "preempt"):
        assert [len(x) for x in m[name]] == [len(o) for o in g[name]["outputs"]]
        assert all(v >= 0 for x in m[name] for v in x)


def test_exp2_polynomial_error_bound():
    """exp2_poly3 (csrc/pkv_common.cuh), the FMA-pipe 2^x that takes a quarter
    of the prefill softmax's exponentials, restated step by step in float32:
    relative error below 1e-4 on [-125, 16] (fp16 rounding is 4.9e-4), and
    2^n exact at integers."""
    import re

    import numpy as np

    from conftest import ROOT

    src = open(os.path.join(ROOT, "llm-inference-scheduler_b200", "csrc", "pkv_common.cuh")).read()
    c = {int(k): np.float32(float.fromhex(v))
         for k, v in re.findall(r"kExp2C(\d) = (0x[0-9a-fp.+-]+)f;", src)}
    assert sorted(c) == [0, 1, 2, 3]
    f32 = np.float32

    def fma(a, b, d):  # a*b is exact in float64; one rounding to float32 after the add
        return (a.astype(np.float64) * b + d).astype(np.float32)

    x = np.concatenate([np.linspace(-125, 16, 2_000_001, dtype=np.float32),
                        np.arange(-125, 17, dtype=np.float32)])
    xc = np.maximum(x, f32(-125))
    t = (xc + f32(12582912.0)).astype(np.float32)
    f = (xc - (t - f32(12582912.0)).astype(np.float32)).astype(np.float32)
    assert np.all(np.abs(f) <= 0.5)
    p = fma(fma(fma(np.full_like(f, c[3]), f, c[2]), f, c[1]), f, c[0])
    bits = (p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)) & 0xFFFFFFFF
    y = bits.astype(np.uint32).view(np.float32).astype(np.float64)
    rel = np.abs(y / np.exp2(xc.astype(np.float64)) - 1)
    assert rel.max() < 1e-4, rel.max()


def _step_arrays_direct(kv, seqs):
    """The step arrays built directly from the block-table lists, sequence by
    sequence, zero padded (what PagedKVCache.step_arrays computes through its
    mirror, whose padding is unspecified)."""
    bs = kv.mgr.block_size
    B = len(seqs)
    num_new = [n for _, n in seqs]
    num_prior = [kv.seq_len(s) for s, _ in seqs]
    totals = [p + n for p, n in zip(num_prior, num_new)]
    used = [(t + bs - 1) // bs for t in totals]
    W = max(1, max(used))
    n_dec = 0
    while n_dec < B and num_new[n_dec] == 1:
        n_dec += 1
    ints = np.zeros(B * W + 2 * B + (B - n_dec) + 1, dtype=np.int32)
    for i, ((s, _), u) in enumerate(zip(seqs, used)):
        ints[i * W: i * W + u] = kv.block_tables[s][:u]
    ints[B * W: B * W + B] = totals
    ints[B * W + B: B * W + 2 * B] = num_prior
    if B - n_dec:
        ints[B * W + 2 * B + 1:] = np.cumsum(num_new[n_dec:])
    slots = np.concatenate([kv._slots(kv.block_tables[s], p, n)
                            for (s, n), p in zip(seqs, num_prior)])
    return ints, slots, n_dec, W


def test_step_arrays_track_table_changes():
    """PagedKVCache.step_arrays (host mirror of the tables) equals the arrays
    built directly from the lists while tables grow, fork, copy-on-write,
    are replaced, freed and re-added, over mixed decode / chunk steps."""
    rng = np.random.default_rng(7)
    mgr = BlockManager(4096, 16, 1, 1, 1, device=None)
    kv = PagedKVCache(mgr)
    live = {}
    next_id = 0
    for it in range(300):
        op = rng.integers(0, 10)
        if op < 3 or not live:  # new sequence with a fresh table
            n = int(rng.integers(0, 40))
            table = [mgr.allocate() for _ in range((n + 16) // 16 + 1)]
            kv.add_sequence(next_id, table, n)
            live[next_id] = table
            next_id += 1
        elif op == 3:  # fork a sequence (shared blocks), then copy-on-write its tail
            s = int(rng.choice(list(live)))
            for b in kv.block_tables[s]:
                mgr.incref(b)
            kv.add_sequence(next_id, list(kv.block_tables[s]), kv.seq_len(s))
            live[next_id] = kv.block_tables[next_id]
            kv.ensure_writable_tail(next_id)
            next_id += 1
        elif op == 4 and len(live) > 1:  # free
            s = int(rng.choice(list(live)))
            for b in kv.block_tables[s]:
                mgr.decref(b)
            kv.free_sequence(s)
            del live[s]
        elif op == 5:  # the caller replaces a table with a new list object
            s = int(rng.choice(list(live)))
            kv.block_tables[s] = list(kv.block_tables[s])
        # one step over a random subset: decodes first, then chunks
        ids = [int(x) for x in rng.permutation(list(live))[: int(rng.integers(1, len(live) + 1))]]
        seqs = []
        for s in ids:
            n = 1 if rng.random() < 0.7 else int(rng.integers(2, 40))
            need = (kv.seq_len(s) + n + 15) // 16
            while len(kv.block_tables[s]) < need:
                kv.block_tables[s].append(mgr.allocate())  # the scheduler grows tables in place
            seqs.append((s, n))
        seqs.sort(key=lambda x: x[1] != 1)
        a = kv.step_arrays(seqs)
        ints, slots, n_dec, W = _step_arrays_direct(kv, seqs)
        assert a["n_decode"] == n_dec and a["W"] == W
        B = len(seqs)
        got, want = a["ints"][: B * W].reshape(B, W), ints[: B * W].reshape(B, W)
        for i, (s, n) in enumerate(seqs):  # the used blocks of each row (the rest is unspecified)
            u = (kv.seq_len(s) + n + 15) // 16
            np.testing.assert_array_equal(got[i, :u], want[i, :u])
        np.testing.assert_array_equal(a["ints"][B * W:], ints[B * W:])
        np.testing.assert_array_equal(a["slots"], slots)
        for s, n in seqs:  # advance, as the last layer of forward_layer does
            kv._len[s] += n


def test_decode_step_graph_chunk_sizes():
    """DecodeStepGraph's default compute chunks: they cover every layer once,
    end in chunks of 1, 1, 2, 4 ... layers (each chunk's copy out overlaps the
    compute of the chunks after it), and the front chunk holds at most twice
    the layers after it; 24 layers (config 3) give 16, 4, 2, 1, 1."""
    from pagedkv.graphs import ready_chunks

    assert ready_chunks(24) == [16, 4, 2, 1, 1]
    for n in range(1, 100):
        ch = ready_chunks(n)
        assert sum(ch) == n and min(ch) >= 1
        assert ch[-1] == 1
        for i, c in enumerate(ch[1:], 1):
            assert c <= max(1, sum(ch[i + 1:]))  # the tail doubles at most
        assert ch[0] <= 2 * max(1, sum(ch[1:]))
