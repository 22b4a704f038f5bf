"""Seeded synthetic inputs for the paged-KV parity cases (test infrastructure).

Every case is generated from a numpy PCG64 seed, so the golden-fixture script
(which runs the reference's own Python path) and the tests (which run the CUDA
path and the C oracle) see byte-identical inputs without committing megabytes
of pool data.  Each golden fixture stores `input_sha256` of the arrays built
here; a test that regenerates a case checks that digest first, so a change in
numpy's generator streams fails loudly instead of silently comparing different
inputs.

Shapes follow the reference's pool layout `[num_blocks, block_size,
num_kv_heads, head_dim]` (mini_engine/paged/block_manager.py:37) and the
Qwen2.5-0.5B attention geometry 14 q heads / 2 kv heads / head_dim 64
(mini_engine/model/config.py:13-23).

dtype tags: "f32", "f16", "bf16".  bf16 arrays are carried as uint16 bit
patterns (numpy has no bfloat16); `to_dtype` rounds float32 to bf16 with
round-to-nearest-even, the same rounding torch's `.to(torch.bfloat16)` uses.
"""

from __future__ import annotations

import hashlib

import numpy as np

HQ, HKV, D, BS = 14, 2, 64, 16

DTYPE_CODE = {"f32": 0, "f16": 1, "bf16": 2}
ESIZE = {"f32": 4, "f16": 2, "bf16": 2}


def to_dtype(x: np.ndarray, dt: str) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    if dt == "f32":
        return x
    if dt == "f16":
        return x.astype(np.float16)
    if dt == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        rounding = ((u >> 16) & 1) + 0x7FFF
        return ((u + rounding) >> 16).astype(np.uint16)
    raise ValueError(dt)


def to_float32(x: np.ndarray, dt: str) -> np.ndarray:
    if dt == "bf16":
        return (x.astype(np.uint32) << 16).view(np.float32)
    return x.astype(np.float32)


def _normal(rng, shape, dt):
    return to_dtype(rng.standard_normal(shape, dtype=np.float32), dt)


def digest(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode())
        h.update(str(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


def pad_tables(tables: list[list[int]], width: int | None = None) -> np.ndarray:
    width = max(1, max((len(t) for t in tables), default=1)) if width is None else width
    out = np.zeros((len(tables), width), dtype=np.int32)
    for i, t in enumerate(tables):
        out[i, : len(t)] = t
    return out


# --------------------------------------------------------------------------
# decode: one new token per sequence, attention over the whole context
# --------------------------------------------------------------------------

def make_decode_case(seed: int, n_seqs: int, ctx_lo: int, ctx_hi: int, num_blocks: int,
                     dt: str, ctx_list=None, lognormal_median: float | None = None,
                     lognormal_sigma: float = 0.5, pool_slack: float | None = None):
    """A decode step: sequence s holds ctx_s - 1 prior tokens in its blocks and
    appends one new token (position ctx_s - 1); attention covers ctx_s tokens.

    Block tables are consecutive slices of a seeded permutation of the pool,
    so they are scattered and disjoint (BASELINE configs 1 and 3).  With
    `lognormal_median`, contexts are clip(round(exp(N(ln median, sigma^2))),
    ctx_lo, ctx_hi) and the pool is sized to the blocks needed times
    `pool_slack` (config 3: median 1024, sigma 0.5, [16, 8192], +10%).
    """
    rng = np.random.default_rng(seed)
    if ctx_list is not None:
        ctx = np.asarray(ctx_list, dtype=np.int64)
    elif lognormal_median is not None:
        z = rng.standard_normal(n_seqs)
        ctx = np.clip(np.round(np.exp(np.log(lognormal_median) + lognormal_sigma * z)),
                      ctx_lo, ctx_hi).astype(np.int64)
    else:
        ctx = rng.integers(ctx_lo, ctx_hi + 1, size=n_seqs).astype(np.int64)
    nblk = (ctx + BS - 1) // BS
    if pool_slack is not None:
        num_blocks = int(np.ceil(pool_slack * nblk.sum()))
    assert nblk.sum() <= num_blocks
    perm = rng.permutation(num_blocks).astype(np.int32)
    tables, o = [], 0
    for n in nblk:
        tables.append(perm[o:o + n].tolist())
        o += n
    k_pool = _normal(rng, (num_blocks, BS, HKV, D), dt)
    v_pool = _normal(rng, (num_blocks, BS, HKV, D), dt)
    q = _normal(rng, (n_seqs, HQ, D), dt)
    k_new = _normal(rng, (n_seqs, HKV, D), dt)
    v_new = _normal(rng, (n_seqs, HKV, D), dt)
    return dict(kind="decode", dt=dt, ctx=ctx, tables=tables, k_pool=k_pool, v_pool=v_pool,
                q=q, k_new=k_new, v_new=v_new, num_blocks=num_blocks)


def decode_digest(c) -> str:
    return digest(c["ctx"], pad_tables(c["tables"]), c["k_pool"], c["v_pool"], c["q"],
                  c["k_new"], c["v_new"])


def decode_slots(c) -> np.ndarray:
    """slot = table[pos // 16] * 16 + pos % 16 for the appended position ctx - 1."""
    pos = c["ctx"] - 1
    return np.array([c["tables"][s][p // BS] * BS + p % BS for s, p in enumerate(pos)],
                    dtype=np.int64)


# --------------------------------------------------------------------------
# chunked prefill over a radix-shared prefix
# --------------------------------------------------------------------------

def make_prefill_case(seed: int, chunk_lens, private_priors, shared_tokens: int,
                      num_blocks: int, dt: str):
    """Sequence s has num_prior_s = shared_tokens + private_priors[s] cached
    tokens and feeds chunk_lens[s] new tokens (causal inside the chunk).

    The first shared_tokens // 16 blocks are the same physical blocks in
    every table (a radix-cache hit, ref count = number of sequences); the rest
    of each table is private, drawn from a seeded permutation of the
    remaining pool.  shared_tokens must be block-aligned, as radix matches are
    (mini_engine/paged/radix_cache.py:62).
    """
    assert shared_tokens % BS == 0
    rng = np.random.default_rng(seed)
    chunk = np.asarray(chunk_lens, dtype=np.int64)
    prior = shared_tokens + np.asarray(private_priors, dtype=np.int64)
    n_shared = shared_tokens // BS
    perm = rng.permutation(num_blocks).astype(np.int32)
    shared = perm[:n_shared].tolist()
    o = n_shared
    tables = []
    for s in range(len(chunk)):
        need = (prior[s] + chunk[s] + BS - 1) // BS - n_shared
        tables.append(shared + perm[o:o + need].tolist())
        o += need
    assert o <= num_blocks
    k_pool = _normal(rng, (num_blocks, BS, HKV, D), dt)
    v_pool = _normal(rng, (num_blocks, BS, HKV, D), dt)
    T = int(chunk.sum())
    q = _normal(rng, (T, HQ, D), dt)
    k_new = _normal(rng, (T, HKV, D), dt)
    v_new = _normal(rng, (T, HKV, D), dt)
    qsl = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    return dict(kind="prefill", dt=dt, chunk=chunk, prior=prior, tables=tables, qsl=qsl,
                k_pool=k_pool, v_pool=v_pool, q=q, k_new=k_new, v_new=v_new,
                num_blocks=num_blocks, shared_tokens=shared_tokens)


def prefill_digest(c) -> str:
    return digest(c["chunk"], c["prior"], pad_tables(c["tables"]), c["k_pool"], c["v_pool"],
                  c["q"], c["k_new"], c["v_new"])


def prefill_slots(c) -> np.ndarray:
    out = []
    for s in range(len(c["chunk"])):
        for p in range(int(c["prior"][s]), int(c["prior"][s] + c["chunk"][s])):
            out.append(c["tables"][s][p // BS] * BS + p % BS)
    return np.array(out, dtype=np.int64)


def make_c4_case(seed: int = 4, dt: str = "f16", n_seqs: int = 16, chunk_len: int = 512,
                 prior_hi: int = 4096):
    """16 sequences, 512-token chunks, a 48-token shared
    system prompt (3 blocks, ref count 16) plus a private prior ~ U[0, 4096]."""
    rng = np.random.default_rng(seed + 1000)
    priv = rng.integers(0, prior_hi + 1, size=n_seqs)
    need = 3 + sum((48 + int(p) + chunk_len + BS - 1) // BS - 3 for p in priv)
    return make_prefill_case(seed, [chunk_len] * n_seqs, priv.tolist(), 48,
                             int(need * 1.1) + 8, dt)


# --------------------------------------------------------------------------
# append + copy-on-write
# --------------------------------------------------------------------------

def make_append_cow_case(seed: int = 2, n_seqs: int = 64, num_blocks: int = 4096,
                         n_layers: int = 4, n_forks: int = 32, dt: str = "f16"):
    """64 sequences each append one token per layer; then 32 of them are forked
    while their tail block is partially filled (ref count 2) and the child's
    ensure_writable_tail triggers a copy-on-write.

    The allocator's free list is a seeded permutation, so the blocks that the
    reference's LIFO allocator hands out (and therefore the COW destination
    blocks) are scattered.  Pool contents are random so a wrong copy is visible.
    """
    rng = np.random.default_rng(seed)
    free_list = rng.permutation(num_blocks).astype(np.int64).tolist()
    # context lengths whose tail block is partial for the forked sequences
    ctx = rng.integers(1, 600, size=n_seqs).astype(np.int64)
    forked = np.sort(rng.choice(n_seqs, size=n_forks, replace=False)).astype(np.int64)
    for s in forked:
        if ctx[s] % BS == 0:
            ctx[s] += 1
    k_pools = _normal(rng, (n_layers, num_blocks, BS, HKV, D), dt)
    v_pools = _normal(rng, (n_layers, num_blocks, BS, HKV, D), dt)
    k_new = _normal(rng, (n_layers, n_seqs, HKV, D), dt)
    v_new = _normal(rng, (n_layers, n_seqs, HKV, D), dt)
    return dict(kind="append_cow", dt=dt, free_list=free_list, ctx=ctx, forked=forked,
                k_pools=k_pools, v_pools=v_pools, k_new=k_new, v_new=v_new,
                num_blocks=num_blocks, n_layers=n_layers)


def append_cow_digest(c) -> str:
    return digest(np.asarray(c["free_list"]), c["ctx"], c["forked"], c["k_pools"],
                  c["v_pools"], c["k_new"], c["v_new"])


# --------------------------------------------------------------------------
# end-to-end greedy decoding (BASELINE config 5 geometry, shortened runs)
# --------------------------------------------------------------------------

E2E_SEED = 5
E2E_FINAL_NORM_SCALE = 4.0  # spreads the tied-embedding logits (well-separated argmax)
E2E_VOCAB = 151936


def e2e_scenarios():
    """Two scheduler runs over the same seeded random-init Qwen2.5-0.5B weights.

    "prefix": 4 requests sharing a 48-token prompt prefix, prefix cache on,
    max_batched_tokens small enough that prompts are prefilled in chunks,
    followed by a second turn of request 0 (its prompt + answer + new tokens)
    that hits the radix cache.
    "preempt": 3 requests on an 11-block pool with the prefix cache off, which
    forces recompute preemption (the reference's test_scheduler.py:104-128
    setup).
    """
    rng = np.random.default_rng(E2E_SEED)
    shared = rng.integers(0, E2E_VOCAB, size=48).tolist()
    prompts = [shared + rng.integers(0, E2E_VOCAB, size=n).tolist() for n in (22, 61, 103, 7)]
    turn2_extra = rng.integers(0, E2E_VOCAB, size=19).tolist()
    pre = [rng.integers(0, E2E_VOCAB, size=n).tolist() for n in (30, 41, 25)]
    return {
        "prefix": dict(num_blocks=256, max_num_seqs=4, max_batched_tokens=48, prefix_cache=True,
                       prompts=prompts, max_new_tokens=12, turn2_extra=turn2_extra),
        "preempt": dict(num_blocks=11, max_num_seqs=3, max_batched_tokens=64, prefix_cache=False,
                        prompts=pre, max_new_tokens=48, turn2_extra=None),
    }


# --------------------------------------------------------------------------
# scheduler decisions with a deterministic stand-in model (no attention)
# --------------------------------------------------------------------------

def fake_next_token(last_id: int, position: int) -> int:
    """Deterministic 'greedy' token of the stand-in model used to compare
    scheduling decisions: depends only on the last fed token and its position."""
    return (last_id * 31 + position * 7) % 997 + 3


def sched_scenario():
    """Admission under a tight pool with the prefix cache on: shared prompt
    prefixes, chunked prefill, radix eviction, preemption, a second turn."""
    rng = np.random.default_rng(77)
    shared = rng.integers(3, 1000, size=40).tolist()
    prompts = [shared + rng.integers(3, 1000, size=n).tolist() for n in (9, 30, 55, 17, 70, 3)]
    return dict(num_blocks=20, max_num_seqs=4, max_batched_tokens=40, prompts=prompts,
                max_new_tokens=[20, 35, 12, 40, 25, 30], turn2=[0, 3])
