"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle and the
reference's golden vectors.  Marked gpu: run with `pytest -m gpu` on a B200.

Bars (written here, as the north star states them):
* append / copy: bit-exact (pool SHA-256 equal to the reference's);
* attention: max |cuda - oracle| <= 1e-5 (fp32), 2e-3 (fp16), 1.6e-2 (bf16),
  and the same bound against the reference's golden outputs.
"""

import json

import numpy as np
import pytest
import torch

import cases as C
from conftest import GOLDEN, PRODUCT_ATOL, as_f32, golden, max_abs_diff
from pagedkv import BlockManager, PagedKVCache, _lib, ops

pytestmark = pytest.mark.gpu

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
DTS = ("f32", "f16", "bf16")


def dev(a: np.ndarray, dt: str | None = None) -> torch.Tensor:
    a = np.ascontiguousarray(a)
    if dt == "bf16":
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(a).cuda()


def host(t: torch.Tensor, dt: str) -> np.ndarray:
    t = t.contiguous().cpu()
    if dt == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


@pytest.fixture(params=["auto", "generic"])
def decode_impl(request):
    ops.set_decode_impl(_lib.DECODE_AUTO if request.param == "auto" else _lib.DECODE_GENERIC)
    yield request.param
    ops.set_decode_impl(_lib.DECODE_AUTO)


def run_decode_gpu(c, err=None, scale=0.125):
    """Append the new token (reshape_and_cache) then decode-attend."""
    dt = c["dt"]
    kp, vp = dev(c["k_pool"], dt), dev(c["v_pool"], dt)
    slots = torch.from_numpy(C.decode_slots(c)).cuda()
    err = ops.new_error_flags("cuda") if err is None else err
    ops.reshape_and_cache(dev(c["k_new"], dt), dev(c["v_new"], dt), kp, vp, slots, err)
    tabs = dev(C.pad_tables(c["tables"]))
    ctx = dev(c["ctx"].astype(np.int32))
    out = ops.paged_decode_attention(dev(c["q"], dt), kp, vp, tabs, ctx, scale, err=err)
    torch.cuda.synchronize()
    return host(out, dt), kp, vp, int(err.item())


def run_prefill_gpu(c, scale=0.125):
    dt = c["dt"]
    kp, vp = dev(c["k_pool"], dt), dev(c["v_pool"], dt)
    err = ops.new_error_flags("cuda")
    ops.reshape_and_cache(dev(c["k_new"], dt), dev(c["v_new"], dt), kp, vp,
                          torch.from_numpy(C.prefill_slots(c)).cuda(), err)
    out = ops.paged_prefill_attention(dev(c["q"], dt), kp, vp, dev(C.pad_tables(c["tables"])),
                                      dev(c["qsl"]), dev(c["prior"].astype(np.int32)),
                                      int(c["chunk"].max()), scale, err=err)
    torch.cuda.synchronize()
    return host(out, dt), int(err.item())


# ---------------------------------------------------------------- append / copy

def test_append_and_cow_config2_bit_exact():
    """Config 2 through the product path: reshape_and_cache per layer, then the
    BlockManager's batched copy_blocks; pool digests equal the reference's."""
    c = C.make_append_cow_case()
    with open(f"{GOLDEN}/append_cow_c2_f16.json") as f:
        g = json.load(f)
    L, dt = c["n_layers"], "f16"
    m = BlockManager(c["num_blocks"], C.BS, L, C.HKV, C.D, device="cuda", dtype=torch.float16)
    m.k_cache.copy_(dev(c["k_pools"], dt))
    m.v_cache.copy_(dev(c["v_pools"], dt))
    m.free_list = list(c["free_list"])
    kv = PagedKVCache(m)
    n = len(c["ctx"])
    for s in range(n):
        ctx = int(c["ctx"][s])
        kv.add_sequence(s, [m.allocate() for _ in range((ctx + 15) // 16)], ctx - 1)
    meta = kv.prepare_step([(s, 1) for s in range(n)])
    for layer in range(L):
        ops.reshape_and_cache(dev(c["k_new"][layer], dt), dev(c["v_new"][layer], dt),
                              m.k_pool[layer], m.v_pool[layer], meta.slot_mapping, m.err)
    torch.cuda.synchronize()
    assert C.digest(*host(m.k_cache, dt), *host(m.v_cache, dt)) == g["pools_after_append_sha256"]
    for s in range(n):
        kv._len[s] = int(c["ctx"][s])
    for i, s in enumerate(c["forked"]):
        s = int(s)
        for b in kv.block_tables[s]:
            m.incref(b)
        kv.add_sequence(n + i, list(kv.block_tables[s]), kv.seq_len(s))
        kv.ensure_writable_tail(n + i)
    assert [list(p) for p in m.pending_copies] == g["pairs"]
    m.flush_copies()
    torch.cuda.synchronize()
    assert m.copies_launched == 1
    assert C.digest(*host(m.k_cache, dt), *host(m.v_cache, dt)) == g["pools_after_cow_sha256"]
    m.check_errors()


@pytest.mark.parametrize("dt", DTS)
def test_reshape_and_cache_matches_oracle(oracle_mod, dt):
    rng = np.random.default_rng(7)
    nb = 64
    kp = C.to_dtype(rng.standard_normal((nb, 16, 2, 64), dtype=np.float32), dt)
    vp = C.to_dtype(rng.standard_normal((nb, 16, 2, 64), dtype=np.float32), dt)
    T = 300
    k = C.to_dtype(rng.standard_normal((T, 2, 64), dtype=np.float32), dt)
    v = C.to_dtype(rng.standard_normal((T, 2, 64), dtype=np.float32), dt)
    slots = rng.permutation(nb * 16)[:T].astype(np.int64)
    slots[::7] = -1  # padding tokens are skipped
    kd, vd = dev(kp, dt), dev(vp, dt)
    err = ops.new_error_flags("cuda")
    ops.reshape_and_cache(dev(k, dt), dev(v, dt), kd, vd, torch.from_numpy(slots).cuda(), err)
    assert oracle_mod.reshape_and_cache(kp, vp, k, v, slots, dt) == 0
    torch.cuda.synchronize()
    assert np.array_equal(host(kd, dt), kp) and np.array_equal(host(vd, dt), vp)
    assert int(err.item()) == 0


def test_reshape_and_cache_strided_input(oracle_mod):
    """K/V as strided views of a fused [T, (14+2+2)*64] projection output."""
    rng = np.random.default_rng(8)
    T, nb = 40, 8
    qkv = torch.randn(T, 18 * 64, dtype=torch.float16, device="cuda")
    k = qkv[:, 14 * 64:16 * 64].view(T, 2, 64)
    v = qkv[:, 16 * 64:].view(T, 2, 64)
    kp = torch.zeros(nb, 16, 2, 64, dtype=torch.float16, device="cuda")
    vp = torch.zeros_like(kp)
    slots = torch.from_numpy(rng.permutation(nb * 16)[:T].astype(np.int64)).cuda()
    ops.reshape_and_cache(k, v, kp, vp, slots)
    ref_k, ref_v = torch.zeros_like(kp).view(-1, 2, 64), torch.zeros_like(vp).view(-1, 2, 64)
    ref_k[slots] = k
    ref_v[slots] = v
    assert torch.equal(kp.view(-1, 2, 64), ref_k) and torch.equal(vp.view(-1, 2, 64), ref_v)


def test_reshape_and_cache_flags_bad_slot():
    kp = torch.zeros(4, 16, 2, 64, dtype=torch.float16, device="cuda")
    vp = torch.zeros_like(kp)
    k = torch.ones(3, 2, 64, dtype=torch.float16, device="cuda")
    slots = torch.tensor([0, 4 * 16, 5], dtype=torch.int64, device="cuda")  # middle one out of range
    err = ops.new_error_flags("cuda")
    ops.reshape_and_cache(k, k, kp, vp, slots, err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.FLAG_SLOT_OUT_OF_RANGE
    flat = kp.view(-1, 2, 64)
    assert flat[0].eq(1).all() and flat[5].eq(1).all() and flat[1].eq(0).all()


def test_copy_blocks_flags_bad_pair():
    kc = torch.randn(2, 8, 16, 2, 64, dtype=torch.float16, device="cuda")
    vc = torch.randn_like(kc)
    k0, v0 = kc.clone(), vc.clone()
    pairs = torch.tensor([[1, 2], [3, 99]], dtype=torch.int32, device="cuda")
    err = ops.new_error_flags("cuda")
    ops.copy_blocks(kc, vc, pairs, err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.FLAG_BLOCK_OUT_OF_RANGE
    assert torch.equal(kc[:, 2], k0[:, 1]) and torch.equal(vc[:, 2], v0[:, 1])
    assert torch.equal(kc[:, 3], k0[:, 3])


# ---------------------------------------------------------------- decode

@pytest.mark.parametrize("dt", DTS)
def test_decode_config1(oracle_mod, decode_impl, dt):
    c = C.make_decode_case(1, 8, 32, 600, 512, dt)
    out, _, _, err = run_decode_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_decode_case(c)
    assert max_abs_diff(out, ref, dt) <= PRODUCT_ATOL[dt]
    assert max_abs_diff(out, golden(f"decode_c1_{dt}.npz")["out"], dt) <= PRODUCT_ATOL[dt]


@pytest.mark.parametrize("dt", DTS)
def test_decode_edge_contexts(oracle_mod, decode_impl, dt):
    c = C.make_decode_case(11, 9, 0, 0, 128, dt, ctx_list=[1, 2, 15, 16, 17, 31, 32, 33, 600])
    out, _, _, err = run_decode_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_decode_case(c)
    assert max_abs_diff(out, ref, dt) <= PRODUCT_ATOL[dt]
    assert max_abs_diff(out, golden(f"decode_edge_{dt}.npz")["out"], dt) <= PRODUCT_ATOL[dt]


@pytest.mark.parametrize("dt", ("f16", "bf16"))
def test_decode_config3_full(oracle_mod, decode_impl, dt):
    """BASELINE config 3 at full size (B=256, lognormal contexts to 8192)."""
    c = C.make_decode_case(3, 256, 16, 8192, 0, dt, lognormal_median=1024.0, pool_slack=1.1)
    out, _, _, err = run_decode_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_decode_case(c)
    assert max_abs_diff(out, ref, dt) <= PRODUCT_ATOL[dt]
    if dt == "f16":
        assert max_abs_diff(out, golden("decode_c3_f16.npz")["out"], dt) <= PRODUCT_ATOL[dt]


@pytest.mark.parametrize("name,dt,make", [
    ("c1", "f32", lambda: C.make_decode_case(1, 8, 32, 600, 512, "f32")),
    ("c1", "bf16", lambda: C.make_decode_case(1, 8, 32, 600, 512, "bf16")),
    ("edge", "f16", lambda: C.make_decode_case(11, 9, 0, 0, 128, "f16",
                                              ctx_list=[1, 2, 15, 16, 17, 31, 32, 33, 600])),
    ("c3", "f16", lambda: C.make_decode_case(3, 256, 16, 8192, 0, "f16", lognormal_median=1024.0,
                                            pool_slack=1.1)),
])
def test_decode_append_fused_matches_oracle(oracle_mod, decode_impl, name, dt, make):
    """pkv_paged_decode_append_attention: the decode kernel writes the new
    token itself (slot from the block table); the pools must equal the
    oracle's bit for bit and the output match within tolerance."""
    c = make()
    kp, vp = dev(c["k_pool"], dt), dev(c["v_pool"], dt)
    err = ops.new_error_flags("cuda")
    out = ops.paged_decode_append_attention(dev(c["q"], dt), dev(c["k_new"], dt), dev(c["v_new"], dt),
                                            kp, vp, dev(C.pad_tables(c["tables"])),
                                            dev(c["ctx"].astype(np.int32)), 0.125, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref, ref_k, ref_v = oracle_mod.run_decode_case(c)
    assert np.array_equal(host(kp, dt), ref_k) and np.array_equal(host(vp, dt), ref_v)
    assert max_abs_diff(host(out, dt), ref, dt) <= PRODUCT_ATOL[dt]


def test_decode_many_short_and_long(oracle_mod, decode_impl):
    """Ragged batch: many 1-block sequences around a few very long ones, so
    the stream-K ranges split sequences at every kind of boundary."""
    rng = np.random.default_rng(31)
    ctx = rng.integers(1, 40, size=700).tolist()
    ctx[5], ctx[300], ctx[699] = 8192, 5000, 4097
    c = C.make_decode_case(31, len(ctx), 0, 0, sum((x + 15) // 16 for x in ctx) + 5, "f16",
                           ctx_list=ctx)
    out, _, _, err = run_decode_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_decode_case(c)
    assert max_abs_diff(out, ref, "f16") <= PRODUCT_ATOL["f16"]


def test_decode_repeated_launches_reuse_workspace(oracle_mod):
    """The workspace needs no initialisation and carries nothing between
    calls: ten launches on one garbage-filled workspace give identical outputs."""
    c = C.make_decode_case(3, 256, 16, 8192, 0, "f16", lognormal_median=1024.0, pool_slack=1.1)
    kp, vp = dev(c["k_pool"], "f16"), dev(c["v_pool"], "f16")
    ops.reshape_and_cache(dev(c["k_new"], "f16"), dev(c["v_new"], "f16"), kp, vp,
                          torch.from_numpy(C.decode_slots(c)).cuda())
    q, tabs, ctx = dev(c["q"], "f16"), dev(C.pad_tables(c["tables"])), dev(c["ctx"].astype(np.int32))
    ws = torch.randint(0, 255, (ops.decode_workspace_bytes(256, 14, 64),), dtype=torch.uint8,
                       device="cuda")
    outs = [ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, workspace=ws).clone()
            for _ in range(10)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref, _, _ = oracle_mod.run_decode_case(c)
    assert max_abs_diff(host(outs[0], "f16"), ref, "f16") <= PRODUCT_ATOL["f16"]


def test_decode_zero_context_and_flags(decode_impl):
    kp = torch.randn(8, 16, 2, 64, dtype=torch.float16, device="cuda")
    vp = torch.randn_like(kp)
    q = torch.randn(3, 14, 64, dtype=torch.float16, device="cuda")
    tabs = torch.tensor([[0, 1], [2, 3], [4, 5]], dtype=torch.int32, device="cuda")
    ctx = torch.tensor([20, 0, 5], dtype=torch.int32, device="cuda")
    err = ops.new_error_flags("cuda")
    out = torch.full_like(q, 7.0)  # rows of empty sequences must be overwritten with zeros
    ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, out=out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert out[1].eq(0).all() and torch.isfinite(out).all() and not out[0].eq(7.0).any()
    # every sequence empty: no KV block to stream, all rows zero
    out = torch.full_like(q, 7.0)
    ops.paged_decode_attention(q, kp, vp, tabs, torch.zeros(3, dtype=torch.int32, device="cuda"),
                               0.125, out=out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and out.eq(0).all()
    # context beyond the table: flagged and clamped, no fault
    ctx = torch.tensor([20, 40, 5], dtype=torch.int32, device="cuda")
    ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.FLAG_CONTEXT_EXCEEDS_TABLE
    # block id outside the pool: flagged, no fault
    err.zero_()
    bad = torch.tensor([[0, 1], [2, 77], [4, 5]], dtype=torch.int32, device="cuda")
    ops.paged_decode_attention(q, kp, vp, bad, torch.tensor([20, 30, 5], dtype=torch.int32,
                                                            device="cuda"), 0.125, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.FLAG_BLOCK_OUT_OF_RANGE


# ---------------------------------------------------------------- prefill

@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("name,args", [
    ("prefill_small", (21, [1, 7, 33, 64, 16], [0, 5, 37, 100, 11], 48, 256)),
    ("prefill_noshare", (22, [20, 3, 48], [0, 16, 1], 0, 64)),
])
def test_prefill_small(oracle_mod, decode_impl, dt, name, args):
    c = C.make_prefill_case(*args, dt)
    out, err = run_prefill_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_prefill_case(c)
    assert max_abs_diff(out, ref, dt) <= PRODUCT_ATOL[dt]
    assert max_abs_diff(out, golden(f"{name}_{dt}.npz")["out"], dt) <= PRODUCT_ATOL[dt]


@pytest.mark.parametrize("dt", ("f16", "bf16"))
def test_prefill_ragged_multi_tile(oracle_mod, decode_impl, dt):
    """Chunks spanning several 128-query tiles with ragged ends, priors that
    are not block aligned, and a one-token chunk behind them."""
    c = C.make_prefill_case(23, [300, 129, 1, 257], [37, 0, 500, 1000], 32, 512, dt)
    out, err = run_prefill_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_prefill_case(c)
    assert max_abs_diff(out, ref, dt) <= PRODUCT_ATOL[dt]


@pytest.mark.parametrize("dt", ("f16", "bf16"))
def test_prefill_equal_lengths_and_many_sequences(oracle_mod, dt):
    """The tensor-core kernel maps CTAs longest-sequence-first: five sequences
    of the same total length (ties ranked by index) beside a longer one, and
    a batch of 70 sequences, beyond the ranked limit (natural order)."""
    c = C.make_prefill_case(24, [100, 100, 100, 100, 50, 260], [10, 10, 10, 10, 60, 0], 16, 256, dt)
    out, err = run_prefill_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_prefill_case(c)
    assert max_abs_diff(out, ref, dt) <= PRODUCT_ATOL[dt]
    rng = np.random.default_rng(25)
    chunks = rng.integers(1, 300, size=70).tolist()
    priors = rng.integers(0, 200, size=70).tolist()
    c = C.make_prefill_case(25, chunks, priors, 32, 4096, dt)
    out, err = run_prefill_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_prefill_case(c)
    assert max_abs_diff(out, ref, dt) <= PRODUCT_ATOL[dt]


def prefill_fp64(c, scale=0.125):
    """Causal attention of a prefill case in float64 from its stored (16-bit)
    inputs: scores and probabilities unrounded.  A yardstick for cases whose
    scores are too large for the reference's rounding points (the oracle
    rounds Q.K^T to the KV dtype, an ulp of several percent of P there)."""
    dt = c["dt"]
    f64 = lambda a: C.to_float32(a, dt).astype(np.float64)  # noqa: E731
    kp, vp, q, kn, vn = f64(c["k_pool"]), f64(c["v_pool"]), f64(c["q"]), f64(c["k_new"]), f64(c["v_new"])
    out = np.zeros_like(q)
    g = C.HQ // C.HKV
    for s in range(len(c["chunk"])):
        P, a, b = int(c["prior"][s]), int(c["qsl"][s]), int(c["qsl"][s + 1])
        pos = np.arange(P)
        blocks = np.asarray(c["tables"][s], dtype=np.int64)[pos // C.BS]
        K = np.concatenate([kp[blocks, pos % C.BS], kn[a:b]])  # [P + n, HKV, D]
        V = np.concatenate([vp[blocks, pos % C.BS], vn[a:b]])
        visible = np.arange(P + b - a)[None, :] <= (P + np.arange(b - a))[:, None]
        for h in range(C.HQ):
            sc = np.where(visible, q[a:b, h] @ K[:, h // g].T * scale, -np.inf)
            w = np.exp(sc - sc.max(axis=1, keepdims=True))
            out[a:b, h] = (w / w.sum(axis=1, keepdims=True)) @ V[:, h // g]
    return out


@pytest.mark.parametrize("dt", ("f16", "bf16"))
def test_prefill_running_max_jumps(dt):
    """Scores that grow along the keys: K rows of a sequence's blocks 8-23
    scaled by 4 and from block 24 on by 16 (the new rows too, by the block
    they land in), so rows' maxima jump by far more than the rescale slack
    (2^8) in later key tiles.  The tensor-core kernel runs a tile's
    exponentials against the running max and redoes the tile when a row's
    max moved; the redone tiles and the O rescales with them, against float64
    attention of the same inputs.  Tolerance: the output's rounding plus P
    rounded to the pool dtype (relative 2^-11 for fp16, 2^-8 for bf16) over
    |V| < 5."""
    c = C.make_prefill_case(31, [300, 200, 129], [700, 300, 0], 32, 256, dt)
    factor = lambda j: 16.0 if j >= 24 else 4.0 if j >= 8 else 1.0  # noqa: E731
    scale_of = {}
    for s, tab in enumerate(c["tables"]):
        for j, b in enumerate(tab):
            if j >= 2:  # the shared prefix blocks stay as they are
                scale_of[b] = factor(j)
    kp = C.to_float32(c["k_pool"], dt).copy()
    for b, f in scale_of.items():
        kp[b] *= f  # powers of two: exact in every dtype
    c["k_pool"] = C.to_dtype(kp, dt)
    kn = C.to_float32(c["k_new"], dt).copy()
    for s in range(len(c["chunk"])):
        for i in range(int(c["chunk"][s])):
            kn[c["qsl"][s] + i] *= factor((int(c["prior"][s]) + i) // 16)
    c["k_new"] = C.to_dtype(kn, dt)
    out, err = run_prefill_gpu(c)
    assert err == 0
    ref = prefill_fp64(c)
    tol = {"f16": 4e-3, "bf16": 3.2e-2}[dt]
    assert float(np.max(np.abs(as_f32(out, dt).astype(np.float64) - ref))) <= tol


def test_prefill_config4_full(oracle_mod, decode_impl):
    c = C.make_c4_case()
    out, err = run_prefill_gpu(c)
    assert err == 0
    ref, _, _ = oracle_mod.run_prefill_case(c)
    assert max_abs_diff(out, ref, "f16") <= PRODUCT_ATOL["f16"]
    g = golden("prefill_c4_f16_rows.npz")
    assert max_abs_diff(out[g["rows"]], g["out"], "f16") <= PRODUCT_ATOL["f16"]


# ---------------------------------------------------------------- operator surface

def test_append_and_fetch_roundtrip_reference_scenario():
    """The reference's test_paged_write_read_roundtrip (test_block_manager.py:37-55),
    fp32, block_size 4, 1 kv head, head_dim 2, through the CUDA pools."""
    with open(f"{GOLDEN}/block_manager_ref.json") as f:
        g = json.load(f)["roundtrip"]
    m = BlockManager(8, 4, 2, 1, 2, device="cuda", dtype=torch.float32)
    kv = PagedKVCache(m)
    table = [m.allocate() for _ in range(3)]
    kv.add_sequence(0, table, 0)
    k1 = torch.arange(10, dtype=torch.float32, device="cuda").reshape(5, 1, 2)
    for layer in range(2):
        k, v, prior = kv.append_and_fetch(layer, 0, k1, k1 * 10)
        assert prior == g["step1"][layer]["prior"]
        assert k.cpu().tolist() == g["step1"][layer]["k"] and v.cpu().tolist() == g["step1"][layer]["v"]
    k2 = torch.arange(100, 106, dtype=torch.float32, device="cuda").reshape(3, 1, 2)
    for layer in range(2):
        k, v, prior = kv.append_and_fetch(layer, 0, k2, k2 * 10)
        assert prior == g["step2"][layer]["prior"]
        assert k.cpu().tolist() == g["step2"][layer]["k"] and v.cpu().tolist() == g["step2"][layer]["v"]
    assert kv.seq_len(0) == g["seq_len"]
    m.check_errors()


def test_cow_isolates_shared_tail_reference_scenario():
    """test_block_manager.py:58-83 on the GPU pools (COW through copy_blocks)."""
    with open(f"{GOLDEN}/block_manager_ref.json") as f:
        g = json.load(f)["cow"]
    m = BlockManager(8, 4, 2, 1, 2, device="cuda", dtype=torch.float32)
    kv = PagedKVCache(m)
    table = [m.allocate()]
    kv.add_sequence(0, table, 0)
    k = torch.ones(2, 1, 2, device="cuda")
    for layer in range(2):
        kv.append_and_fetch(layer, 0, k, k)
    for b in table:
        m.incref(b)
    kv.add_sequence(1, list(table), 2)
    kv.ensure_writable_tail(1)
    k_new = torch.full((1, 1, 2), 7.0, device="cuda")
    for layer in range(2):
        kv.append_and_fetch(layer, 1, k_new, k_new)
    z = torch.zeros(0, 1, 2, device="cuda")
    k0, _, _ = kv.append_and_fetch(0, 0, z, z)
    k1, _, _ = kv.append_and_fetch(0, 1, z, z)
    assert k0.cpu().tolist() == g["k_seq0"] and k1.cpu().tolist() == g["k_seq1"]
    assert [p.cpu().tolist() for p in m.k_pool] == g["k_pool"]
    assert [p.cpu().tolist() for p in m.v_pool] == g["v_pool"]


@pytest.mark.parametrize("dt", ("f16", "bf16"))
def test_forward_layer_mixed_batch(oracle_mod, dt):
    """prepare_step + forward_layer on a batch of decodes followed by chunks:
    one append launch, one decode launch, one prefill launch."""
    rng = np.random.default_rng(41)
    L, nb = 2, 256
    m = BlockManager(nb, 16, L, 2, 64, device="cuda", dtype=TORCH_DT[dt])
    pools_k = C.to_dtype(rng.standard_normal((L, nb, 16, 2, 64), dtype=np.float32), dt)
    pools_v = C.to_dtype(rng.standard_normal((L, nb, 16, 2, 64), dtype=np.float32), dt)
    m.k_cache.copy_(dev(pools_k, dt))
    m.v_cache.copy_(dev(pools_v, dt))
    kv = PagedKVCache(m)
    plan = [(0, 100, 1), (1, 17, 1), (2, 0, 1), (3, 48, 30), (4, 5, 64), (5, 31, 1)]
    for s, prior, n in plan:
        kv.add_sequence(s, [m.allocate() for _ in range((prior + n + 15) // 16)], prior)
    meta = kv.prepare_step([(s, n) for s, _, n in plan])
    assert meta.n_decode == 3
    T = meta.n_tokens
    for layer in range(L):
        q = C.to_dtype(rng.standard_normal((T, 14, 64), dtype=np.float32), dt)
        k = C.to_dtype(rng.standard_normal((T, 2, 64), dtype=np.float32), dt)
        v = C.to_dtype(rng.standard_normal((T, 2, 64), dtype=np.float32), dt)
        out = kv.forward_layer(layer, dev(q, dt), dev(k, dt), dev(v, dt), meta, 0.125)
        torch.cuda.synchronize()
        slots = np.concatenate([kv._slots(kv.block_tables[s], p, n) for s, p, n in plan])
        assert oracle_mod.reshape_and_cache(pools_k[layer], pools_v[layer], k, v, slots, dt) == 0
        qsl = np.concatenate([[0], np.cumsum([n for _, _, n in plan])]).astype(np.int32)
        tabs = C.pad_tables([kv.block_tables[s] for s, _, _ in plan])
        ref = oracle_mod.paged_attention(q, pools_k[layer], pools_v[layer], tabs, qsl,
                                         np.array([p for _, p, _ in plan], dtype=np.int32), dt)
        assert max_abs_diff(host(out, dt), ref, dt) <= PRODUCT_ATOL[dt]
    assert [kv.seq_len(s) for s, _, _ in plan] == [p + n for _, p, n in plan]
    m.check_errors()


@pytest.mark.parametrize("dt", ["f16", "bf16"])
def test_forward_layers_equals_forward_layer_and_oracle(oracle_mod, dt):
    """PagedKVCache.forward_layers (one pkv_paged_decode_append_attention_layers
    call per run of layers) against forward_layer layer by layer on a copy of
    the same pools: outputs and pools bit-identical; outputs within the
    product tolerance of the oracle.  Layer-major inputs are strided views of
    one [L, B, Hq + 2 Hkv, D] buffer, as the end-to-end bench stages them.  A
    mixed step (not decode-only) takes the per-layer path and still matches."""
    rng = np.random.default_rng(43)
    L, nb, tdt = 5, 1024, TORCH_DT[dt]
    ctx = rng.integers(1, 700, size=37)
    ctx[:3] = [1, 16, 17]
    assert int(((ctx + 15) // 16).sum()) <= nb - 8  # the last 8 blocks stay for the mixed step
    pools_k = C.to_dtype(rng.standard_normal((L, nb, 16, 2, 64), dtype=np.float32), dt)
    pools_v = C.to_dtype(rng.standard_normal((L, nb, 16, 2, 64), dtype=np.float32), dt)
    managers = []
    for _ in range(2):
        m = BlockManager(nb, 16, L, 2, 64, device="cuda", dtype=tdt)
        m.k_cache.copy_(dev(pools_k, dt))
        m.v_cache.copy_(dev(pools_v, dt))
        kv = PagedKVCache(m)
        perm = np.random.default_rng(7).permutation(nb - 8)
        o = 0
        for s, c in enumerate(ctx):
            n = (int(c) + 15) // 16
            kv.add_sequence(s, perm[o:o + n].tolist(), int(c) - 1)
            o += n
        managers.append((m, kv))
    B = len(ctx)
    qkv = C.to_dtype(rng.standard_normal((L, B, 18, 64), dtype=np.float32), dt)
    dqkv = dev(qkv, dt)
    (m1, kv1), (m2, kv2) = managers
    meta1 = kv1.prepare_step([(s, 1) for s in range(B)])
    meta2 = kv2.prepare_step([(s, 1) for s in range(B)])
    out1 = torch.empty((L, B, 14, 64), dtype=tdt, device="cuda")
    out2 = torch.empty_like(out1)
    # runs of 2 and 3 layers
    for a, b in ((0, 2), (2, 5)):
        kv1.forward_layers(a, dqkv[a:b, :, :14], dqkv[a:b, :, 14:16], dqkv[a:b, :, 16:18], meta1,
                           0.125, out=out1[a:b])
    for layer in range(L):
        kv2.forward_layer(layer, dqkv[layer, :, :14], dqkv[layer, :, 14:16], dqkv[layer, :, 16:18],
                          meta2, 0.125, out=out2[layer])
    torch.cuda.synchronize()
    m1.check_errors()
    assert torch.equal(out1, out2)
    assert torch.equal(m1.k_cache, m2.k_cache) and torch.equal(m1.v_cache, m2.v_cache)
    assert [kv1.seq_len(s) for s in range(B)] == [int(c) for c in ctx]
    tabs = C.pad_tables([kv1.block_tables[s] for s in range(B)])
    for layer in (0, L - 1):
        slots = np.array([kv1._slots(kv1.block_tables[s], int(c) - 1, 1)[0] for s, c in enumerate(ctx)])
        kp, vp = pools_k[layer].copy(), pools_v[layer].copy()
        kn_l, vn_l = (np.ascontiguousarray(qkv[layer, :, a:b]) for a, b in ((14, 16), (16, 18)))
        assert oracle_mod.reshape_and_cache(kp, vp, kn_l, vn_l, slots, dt) == 0
        ref = oracle_mod.paged_attention(np.ascontiguousarray(qkv[layer, :, :14]), kp, vp, tabs,
                                         np.arange(B + 1, dtype=np.int32),
                                         (ctx - 1).astype(np.int32), dt)
        assert max_abs_diff(host(out1[layer], dt), ref, dt) <= PRODUCT_ATOL[dt]
        assert np.array_equal(host(m1.k_cache[layer], dt), kp)
    # a mixed step goes layer by layer and equals forward_layer
    kv1.add_sequence(B, [nb - 8, nb - 7, nb - 6], 5)
    kv2.add_sequence(B, [nb - 8, nb - 7, nb - 6], 5)
    # decode sequences whose last block has room for one more token
    seqs = [(s, 1) for s in range(B) if ctx[s] % 16] + [(B, 20)]
    meta1, meta2 = kv1.prepare_step(seqs), kv2.prepare_step(seqs)
    T = meta1.n_tokens
    x = dev(C.to_dtype(rng.standard_normal((2, T, 18, 64), dtype=np.float32), dt), dt)
    o1 = kv1.forward_layers(0, x[:, :, :14], x[:, :, 14:16], x[:, :, 16:18], meta1, 0.125)
    o2 = torch.stack([kv2.forward_layer(layer, x[layer, :, :14], x[layer, :, 14:16],
                                        x[layer, :, 16:18], meta2, 0.125) for layer in range(2)])
    torch.cuda.synchronize()
    assert torch.equal(o1, o2)


def test_decode_layers_abi_rejects_overlapping_pools():
    """pkv_paged_decode_append_attention_layers refuses a pool layer stride
    smaller than one layer's pool (the layers would overlap) before any launch."""
    from pagedkv import _lib

    nb, B, L = 8, 2, 2
    kc = torch.zeros((L, nb, 16, 2, 64), dtype=torch.float16, device="cuda")
    vc = torch.zeros_like(kc)
    q = torch.zeros((L, B, 14, 64), dtype=torch.float16, device="cuda")
    kn = torch.zeros((L, B, 2, 64), dtype=torch.float16, device="cuda")
    out = torch.full_like(q, 7.0)
    tabs = torch.zeros((B, 1), dtype=torch.int32, device="cuda")
    ctx = torch.ones(B, dtype=torch.int32, device="cuda")
    ws = ops.new_decode_workspace(B, 14, 64, "cuda")
    lib = _lib.load()
    pool_bytes = nb * 16 * 2 * 64 * 2
    for stride, want in ((pool_bytes - 16, _lib.ERR_BAD_SHAPE), (pool_bytes + 8, _lib.ERR_MISALIGNED)):
        rc = lib.pkv_paged_decode_append_attention_layers(
            L, out.data_ptr(), q.stride(0), 14 * 64, q.data_ptr(), q.stride(0), 14 * 64,
            kn.data_ptr(), kn.data_ptr(), kn.stride(0), 128, 128, kc.data_ptr(), vc.data_ptr(), stride,
            nb, tabs.data_ptr(), 1, 1, ctx.data_ptr(), B, 14, 2, 64, 16, 0.125, _lib.F16,
            ws.data_ptr(), ws.numel(), None, torch.cuda.current_stream().cuda_stream, None, None)
        assert rc == want, (stride, rc)
    torch.cuda.synchronize()
    assert bool((out == 7.0).all()) and not kc.any()


def test_decode_layers_input_ready_word():
    """forward_layers with input_ready (the word a copy stream sets after the
    inputs; the kernels wait for it before reading them):
    * a set word: outputs and pools bit-identical to the call without it;
    * a word that nothing sets: the bounded wait runs out (about a second)
      and the call flags PKV_FLAG_PIPELINE_TIMEOUT (its outputs are then
      unspecified); the next call on the same context is clean and exact;
    * shapes outside the tensor-core decode (fp32) refuse it before launching."""
    from pagedkv import _lib

    rng = np.random.default_rng(47)
    L, nb = 2, 512
    ctx = rng.integers(1, 600, size=21)
    pk = rng.standard_normal((L, nb, 16, 2, 64), dtype=np.float32)
    pv = rng.standard_normal((L, nb, 16, 2, 64), dtype=np.float32)
    qkv = rng.standard_normal((L, len(ctx), 18, 64), dtype=np.float32)

    def setup(tdt):
        m = BlockManager(nb, 16, L, 2, 64, device="cuda", dtype=tdt)
        m.k_cache.copy_(torch.from_numpy(pk).to(tdt))
        m.v_cache.copy_(torch.from_numpy(pv).to(tdt))
        kv = PagedKVCache(m)
        o = 0
        for s, c in enumerate(ctx):
            n = (int(c) + 15) // 16
            kv.add_sequence(s, list(range(o, o + n)), int(c) - 1)
            o += n
        x = torch.from_numpy(qkv).to(tdt).cuda()
        meta = kv.prepare_step([(s, 1) for s in range(len(ctx))])
        return m, kv, x, meta

    def call(kv, x, meta, ready=None, layers=L):
        return kv.forward_layers(0, x[:layers, :, :14], x[:layers, :, 14:16], x[:layers, :, 16:18],
                                 meta, 0.125, advance=False, input_ready=ready)

    m1, kv1, x1, meta1 = setup(torch.float16)
    m2, kv2, x2, meta2 = setup(torch.float16)
    set_word = torch.ones(L, dtype=torch.int32, device="cuda")  # one word per layer
    o1 = call(kv1, x1, meta1, set_word)
    o2 = call(kv2, x2, meta2)
    torch.cuda.synchronize()
    m1.check_errors()
    assert torch.equal(o1, o2)
    assert torch.equal(m1.k_cache, m2.k_cache) and torch.equal(m1.v_cache, m2.v_cache)
    # a word nothing sets: one layer, so one bounded wait
    never = torch.zeros(1, dtype=torch.int32, device="cuda")
    o3 = call(kv1, x1, meta1, never, layers=1)  # layer 0's word
    torch.cuda.synchronize()
    flags = int(m1.err.item())
    assert flags & _lib.FLAG_PIPELINE_TIMEOUT, flags
    assert o3.shape == o2[:1].shape
    m1.err.zero_()
    o4 = call(kv1, x1, meta1)
    torch.cuda.synchronize()
    m1.check_errors()
    assert torch.equal(o4, o2)
    # fp32: the CUDA-core decode serves it, which does not wait on a word
    m5, kv5, x5, meta5 = setup(torch.float32)
    with pytest.raises(_lib.PagedKVError) as e:
        call(kv5, x5, meta5, set_word)
    assert e.value.status == _lib.ERR_UNSUPPORTED


@pytest.mark.parametrize("dt", ("f16", "bf16"))
def test_decode_layers_chained_equals_per_layer_merges(dt):
    """pkv_paged_decode_append_attention_layers with one split-K set per
    layer (the layers' decodes chained, one merge launch for all) against the
    same call with a single set (each layer's decode followed by its merge),
    on copies of the same pools, twice in a row: outputs and pools
    bit-identical, and equal to the single-layer entry point."""
    rng = np.random.default_rng(49)
    L, nb, tdt = 4, 1024, TORCH_DT[dt]
    ctx = rng.integers(1, 900, size=41)
    ctx[:2] = [1, 16]
    tabs_np = C.pad_tables([list(x) for x in np.split(rng.permutation(nb)[:int(((ctx + 15) // 16).sum())],
                                                     np.cumsum((ctx + 15) // 16)[:-1])])
    B = len(ctx)
    pools = [dev(C.to_dtype(rng.standard_normal((L, nb, 16, 2, 64), dtype=np.float32), dt), dt)
             for _ in range(2)]
    x = dev(C.to_dtype(rng.standard_normal((L, B, 18, 64), dtype=np.float32), dt), dt)
    tabs, ctx_d = dev(tabs_np), dev(ctx.astype(np.int32))
    err = ops.new_error_flags("cuda")
    outs, caches = [], []
    for layers_ws in (L, 1):
        kc, vc = pools[0].clone(), pools[1].clone()
        ws = ops.new_decode_workspace(B, 14, 64, "cuda", layers=layers_ws)
        plan = ops.DecodeAppendLayersPlan(tabs, ctx_d, 0.125, ws, err)
        out = torch.empty((L, B, 14, 64), dtype=tdt, device="cuda")
        for _ in range(2):
            plan(x[:, :, :14], x[:, :, 14:16], x[:, :, 16:18], kc, vc, out)
        outs.append(out)
        caches.append((kc, vc))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(caches[0][0], caches[1][0]) and torch.equal(caches[0][1], caches[1][1])
    kc, vc = pools[0].clone(), pools[1].clone()
    for layer in range(L):
        for _ in range(2):
            single = ops.paged_decode_append_attention(x[layer, :, :14], x[layer, :, 14:16], x[layer, :, 16:18],
                                                       kc[layer], vc[layer], tabs, ctx_d, 0.125, err=err)
        assert torch.equal(single, outs[0][layer])


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ("f16", "bf16"))
def test_decode_layers_defer_first_runs_equal_one_chain(dt):
    """Consecutive runs of layers as one launch chain: runs of 3, 1, 2 and 1
    layers, each after the first with PKV_LAYERS_DEFER_FIRST over its own
    slice of a workspace of one split-K set per layer, twice in a row, against
    one call over all layers on copies of the same pools: outputs and pools
    bit-identical.  An unknown flag bit is refused before any launch."""
    rng = np.random.default_rng(53)
    L, nb, tdt = 7, 1024, TORCH_DT[dt]
    ctx = rng.integers(1, 700, size=37)
    ctx[:3] = [1, 16, 17]
    tabs_np = C.pad_tables([list(x) for x in np.split(rng.permutation(nb)[:int(((ctx + 15) // 16).sum())],
                                                     np.cumsum((ctx + 15) // 16)[:-1])])
    B = len(ctx)
    pools = [dev(C.to_dtype(rng.standard_normal((L, nb, 16, 2, 64), dtype=np.float32), dt), dt)
             for _ in range(2)]
    x = dev(C.to_dtype(rng.standard_normal((L, B, 18, 64), dtype=np.float32), dt), dt)
    tabs, ctx_d = dev(tabs_np), dev(ctx.astype(np.int32))
    err = ops.new_error_flags("cuda")
    ws1 = ops.decode_workspace_bytes(B, 14, 64)
    ws = ops.new_decode_workspace(B, 14, 64, "cuda", layers=L)
    ref_ws = ops.new_decode_workspace(B, 14, 64, "cuda", layers=L)
    ref_k, ref_v = pools[0].clone(), pools[1].clone()
    ref = torch.empty((L, B, 14, 64), dtype=tdt, device="cuda")
    one = ops.DecodeAppendLayersPlan(tabs, ctx_d, 0.125, ref_ws, err)
    kc, vc = pools[0].clone(), pools[1].clone()
    out = torch.empty_like(ref)
    runs = [(0, 3), (3, 4), (4, 6), (6, 7)]
    plans = [ops.DecodeAppendLayersPlan(tabs, ctx_d, 0.125, ws[a * ws1: b * ws1], err) for a, b in runs]
    for _ in range(2):
        one(x[:, :, :14], x[:, :, 14:16], x[:, :, 16:18], ref_k, ref_v, ref)
        for i, ((a, b), plan) in enumerate(zip(runs, plans)):
            plan(x[a:b, :, :14], x[a:b, :, 14:16], x[a:b, :, 16:18], kc[a:b], vc[a:b], out[a:b],
                 defer_first=i > 0)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(out, ref)
    assert torch.equal(kc, ref_k) and torch.equal(vc, ref_v)
    a = list(plans[1]._args)
    a[-1] = 2  # not a defined flag
    assert _lib.load().pkv_paged_decode_append_attention_layers_flags(*a) == _lib.ERR_UNSUPPORTED


# ---------------------------------------------------------------- fused RoPE + append

def qkv_rows(T, width, g, tdt, layout, mul=1.0):
    """[T, width] projection rows: "packed" (row stride = width: 16-byte
    aligned rows, the vectorised RoPE kernel) or "padded" (row stride width +
    2 elements: rows off the 16-byte grid, the warp-per-head kernel)."""
    pad = 2 if layout == "padded" else 0
    big = (mul * torch.randn((T, width + pad), generator=g, device="cuda")).to(tdt)
    return big[:, :width]


@pytest.mark.parametrize("layout", ("packed", "padded"))
@pytest.mark.parametrize("dt", DTS)
def test_rope_reshape_and_cache_bit_identical_to_torch_rope(dt, layout):
    """pkv_rope_reshape_and_cache against the unfused path it replaces:
    Rope.rotate on q and k (separate torch multiply / add) then
    reshape_and_cache.  Rotated q and both pools must be identical bit for
    bit; a padding slot (-1) writes q only; a position outside the tables is
    flagged and that token skipped.  Both kernel forms (qkv_rows)."""
    from pagedkv.model import Rope

    tdt = TORCH_DT[dt]
    g = torch.Generator(device="cuda").manual_seed(61)
    T, hq, hkv, d, nb = 200, 14, 2, 64, 64
    rope = Rope(d, 1e6, "cuda", tdt)
    cos, sin = rope.tables(5000)
    qkv = qkv_rows(T, (hq + 2 * hkv) * d, g, tdt, layout)
    pos = torch.randint(0, 5000, (T,), generator=g, device="cuda")
    slots = torch.randperm(nb * 16, generator=g, device="cuda")[:T]
    slots[7] = -1
    kp = torch.randn((nb, 16, hkv, d), generator=g, device="cuda").to(tdt)
    vp = torch.randn_like(kp)
    kp_ref, vp_ref = kp.clone(), vp.clone()
    err = ops.new_error_flags("cuda")
    q = ops.rope_reshape_and_cache(qkv, pos, cos, sin, kp, vp, slots, err=err)
    c, s = cos[pos].unsqueeze(1), sin[pos].unsqueeze(1)
    q_ref = Rope.rotate(qkv[:, : hq * d].view(T, hq, d), c, s)
    k_ref = Rope.rotate(qkv[:, hq * d: (hq + hkv) * d].view(T, hkv, d), c, s)
    v_ref = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
    ops.reshape_and_cache(k_ref.contiguous(), v_ref.contiguous(), kp_ref, vp_ref, slots)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(q, q_ref)
    assert torch.equal(kp, kp_ref) and torch.equal(vp, vp_ref)
    # a position past the tables: flagged, token skipped, the rest written
    pos[3] = 5000
    q2 = torch.zeros_like(q)
    ops.rope_reshape_and_cache(qkv, pos, cos, sin, kp, vp, slots, q_out=q2, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.FLAG_POSITION_OUT_OF_RANGE
    assert q2[3].eq(0).all() and torch.equal(q2[4:], q_ref[4:])


@pytest.mark.parametrize("dt", ("f16", "f32"))
def test_forward_layer_qkv_equals_forward_layer(dt):
    """The fused RoPE + append path (forward_layer_qkv: rope kernel, decode
    without append, prefill) gives the same outputs and pools as rotating in
    torch and calling forward_layer (decode kernel with the fused append)."""
    from pagedkv.model import Rope

    tdt = TORCH_DT[dt]
    g = torch.Generator(device="cuda").manual_seed(62)
    L, nb, hq, hkv, d = 2, 256, 14, 2, 64
    plan = [(0, 100, 1), (1, 17, 1), (2, 0, 1), (3, 48, 30), (4, 5, 64), (5, 31, 1)]
    caches = []
    for _ in range(2):
        m = BlockManager(nb, 16, L, hkv, d, device="cuda", dtype=tdt)
        kv = PagedKVCache(m)
        o = 0
        for s, prior, n in plan:  # disjoint consecutive blocks
            nblk = (prior + n + 15) // 16
            kv.add_sequence(s, list(range(o, o + nblk)), prior)
            o += nblk
        caches.append((m, kv))
    base_k = torch.randn((L, nb, 16, hkv, d), generator=g, device="cuda").to(tdt)
    base_v = torch.randn_like(base_k)
    for m, _ in caches:
        m.k_cache.copy_(base_k)
        m.v_cache.copy_(base_v)
    metas = [kv.prepare_step([(s, n) for s, _, n in plan]) for _, kv in caches]
    T = metas[0].n_tokens
    pos = torch.from_numpy(np.concatenate([np.arange(p, p + n) for _, p, n in plan])).cuda()
    rope = Rope(d, 1e6, "cuda", tdt)
    cos, sin = rope.tables(4096)
    for layer in range(L):
        qkv = torch.randn((T, (hq + 2 * hkv) * d), generator=g, device="cuda").to(tdt)
        out_a = caches[0][1].forward_layer_qkv(layer, qkv, pos, cos, sin, metas[0], 0.125)
        c, s_ = cos[pos].unsqueeze(1), sin[pos].unsqueeze(1)
        q = Rope.rotate(qkv[:, : hq * d].view(T, hq, d), c, s_)
        k = Rope.rotate(qkv[:, hq * d: (hq + hkv) * d].view(T, hkv, d), c, s_)
        v = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
        out_b = caches[1][1].forward_layer(layer, q, k, v, metas[1], 0.125)
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b)
    assert torch.equal(caches[0][0].k_cache, caches[1][0].k_cache)
    assert torch.equal(caches[0][0].v_cache, caches[1][0].v_cache)
    for m, _ in caches:
        m.check_errors()


# ---------------------------------------------------------------- fp8 e4m3 pools

def fp8_atol(dt: str, ref: np.ndarray) -> float:
    """Tolerance of attention over fp8 pools against the fp32 oracle over the
    dequantised pools.  fp8 KV has no reference path to emulate, so the oracle
    keeps every step in fp32; the kernels compute in the query dtype and
    round one extra product to it -- P times the token's V scale -- so the bar
    is the 16-bit tolerance of that dtype plus one rounding (2^-8 relative for
    bf16, 2^-10 for fp16) of the largest output."""
    eps = {"f16": 2.0 ** -10, "bf16": 2.0 ** -8, "f32": 0.0}[dt]
    return PRODUCT_ATOL[dt] + eps * float(np.abs(ref).max())


def _fp8_case(seed, ctx, src_dt, nb=None):
    """Pools filled through pkv_reshape_and_cache_fp8 with every context token
    of every sequence (random block tables); returns the device pools plus the
    source rows, tables and slots."""
    rng = np.random.default_rng(seed)
    ctx = np.asarray(ctx, dtype=np.int64)
    nblk = (ctx + 15) // 16
    nb = nb or int(nblk.sum()) + 8
    perm = rng.permutation(nb).astype(np.int32)
    tables, o = [], 0
    for n in nblk:
        tables.append(perm[o:o + n].tolist())
        o += n
    T = int(ctx.sum())
    k = C.to_dtype(rng.standard_normal((T, 2, 64), dtype=np.float32) * 3, src_dt)
    v = C.to_dtype(rng.standard_normal((T, 2, 64), dtype=np.float32), src_dt)
    slots = np.concatenate([np.array(t, np.int64)[np.arange(c) // 16] * 16 + np.arange(c) % 16
                            for t, c in zip(tables, ctx)])
    kp = torch.zeros((nb, 16, 2, 64), dtype=torch.uint8, device="cuda")
    vp = torch.zeros_like(kp)
    ks = torch.zeros((nb, 16, 2), dtype=torch.float32, device="cuda")
    vs = torch.zeros_like(ks)
    err = ops.new_error_flags("cuda")
    ops.reshape_and_cache_fp8(dev(k, src_dt), dev(v, src_dt), kp, vp, ks, vs,
                              torch.from_numpy(slots).cuda(), err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return dict(ctx=ctx, tables=tables, k=k, v=v, slots=slots, kp=kp, vp=vp, ks=ks, vs=vs, nb=nb, rng=rng)


@pytest.mark.parametrize("src_dt", DTS)
def test_reshape_and_cache_fp8_matches_oracle(oracle_mod, src_dt):
    """Quantisation on the device equals the oracle's restatement bit for bit:
    the e4m3 bytes and the per-(token, KV head) scales, from fp32 / fp16 /
    bf16 rows; a padding slot writes nothing."""
    c = _fp8_case(71, [37, 300, 5, 129], src_dt)
    for name, rows in (("k", c["k"]), ("v", c["v"])):
        b, s = oracle_mod.fp8_quantize_rows(as_f32(rows, src_dt))
        pool = (c["kp"] if name == "k" else c["vp"]).view(-1, 2, 64).cpu().numpy()[c["slots"]]
        sc = (c["ks"] if name == "k" else c["vs"]).view(-1, 2).cpu().numpy()[c["slots"]]
        assert np.array_equal(pool, b), f"{name} bytes differ at {np.argwhere(pool != b)[:4]}"
        assert np.array_equal(sc, s), f"{name} scales differ"
    # slot -1: skipped
    kp0 = c["kp"].clone()
    ones = torch.ones((1, 2, 64), dtype=TORCH_DT[src_dt], device="cuda")
    ops.reshape_and_cache_fp8(ones, ones, c["kp"], c["vp"], c["ks"], c["vs"],
                              torch.tensor([-1], dtype=torch.int64, device="cuda"))
    torch.cuda.synchronize()
    assert torch.equal(kp0, c["kp"])


@pytest.mark.parametrize("q_dt", ("f16", "bf16"))
def test_decode_fp8_matches_oracle(oracle_mod, decode_impl, q_dt):
    """Decode over fp8 pools (tensor-core kernel and CUDA-core kernel) against
    the oracle's attention over the dequantised pools, with the 16-bit
    tolerance of the query dtype."""
    ctx = [1, 15, 16, 17, 33, 600, 1000, 2047, 64, 5000, 3, 250]
    c = _fp8_case(72, ctx, "f16")
    B = len(ctx)
    q = C.to_dtype(c["rng"].standard_normal((B, 14, 64), dtype=np.float32), q_dt)
    tabs = C.pad_tables(c["tables"])
    err = ops.new_error_flags("cuda")
    out = ops.paged_decode_attention_fp8(dev(q, q_dt), c["kp"], c["vp"], c["ks"], c["vs"], dev(tabs),
                                         dev(c["ctx"].astype(np.int32)), 0.125, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    qsl = np.arange(B + 1, dtype=np.int32)
    prior = (c["ctx"] - 1).astype(np.int32)
    q32 = as_f32(q, q_dt)
    ref = oracle_mod.paged_attention_fp8(q32, c["kp"].cpu().numpy(), c["vp"].cpu().numpy(),
                                         c["ks"].cpu().numpy(), c["vs"].cpu().numpy(), tabs, qsl, prior)
    got = as_f32(host(out, q_dt), q_dt)
    assert np.abs(got - ref).max() <= fp8_atol(q_dt, ref)


@pytest.mark.parametrize("q_dt,path", [("f16", "scratch"), ("bf16", "scratch"), ("f16", "in_kernel"),
                                         ("f16", "cuda_cores"), ("bf16", "cuda_cores")])
def test_prefill_fp8_matches_oracle(oracle_mod, q_dt, path):
    """Chunked prefill over fp8 pools, chunks over a prior: the tensor-core
    path (16-bit scratch pool + tcgen05 kernel; fp16 q also with the e4m3
    tiles converted inside the tcgen05 kernel) and the CUDA-core kernel."""
    prior = np.array([48, 0, 300, 17, 1000], dtype=np.int64)
    chunk = np.array([64, 130, 1, 40, 300], dtype=np.int64)
    c = _fp8_case(73, prior + chunk, "f16")
    T = int(chunk.sum())
    q = C.to_dtype(c["rng"].standard_normal((T, 14, 64), dtype=np.float32), q_dt)
    tabs = C.pad_tables(c["tables"])
    qsl = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    err = ops.new_error_flags("cuda")
    out = ops.paged_prefill_attention_fp8(dev(q, q_dt), c["kp"], c["vp"], c["ks"], c["vs"], dev(tabs),
                                          dev(qsl), dev(prior.astype(np.int32)), int(chunk.max()), 0.125,
                                          err=err, tensor_cores=path != "cuda_cores",
                                          scratch_free=path == "in_kernel")
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    ref = oracle_mod.paged_attention_fp8(as_f32(q, q_dt), c["kp"].cpu().numpy(),
                                         c["vp"].cpu().numpy(), c["ks"].cpu().numpy(),
                                         c["vs"].cpu().numpy(), tabs, qsl, prior.astype(np.int32))
    got = as_f32(host(out, q_dt), q_dt)
    assert np.abs(got - ref).max() <= fp8_atol(q_dt, ref)


def test_prefill_fp8_tensor_cores_config4_shape():
    """Config-4 shape over fp8 pools (16 chunks of 512 over a 48-token shared
    prefix plus private priors): the tensor-core paths (scratch pass, and
    in-kernel conversion) against the CUDA-core kernel, within the fp16 fp8
    tolerance; the scratch is reused across two calls with different pools
    (no state carried)."""
    rng = np.random.default_rng(74)
    prior = 48 + rng.integers(0, 4096, size=16)
    chunk = np.full(16, 512)
    c = _fp8_case(74, prior + chunk, "f16")
    T = int(chunk.sum())
    tabs = dev(C.pad_tables(c["tables"]))
    qsl = dev(np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32))
    pr = dev(prior.astype(np.int32))
    err = ops.new_error_flags("cuda")
    scratch = torch.full((ops.prefill_fp8_scratch_bytes(16, tabs.shape[1], 2, 64),), 255,
                         dtype=torch.uint8, device="cuda")
    for seed in (1, 2):
        g = torch.Generator(device="cuda").manual_seed(seed)
        q = torch.randn((T, 14, 64), generator=g, device="cuda").half()
        kp = c["kp"] if seed == 1 else torch.roll(c["kp"], 1, dims=0)
        a = ops.paged_prefill_attention_fp8(q, kp, c["vp"], c["ks"], c["vs"], tabs, qsl, pr, 512, 0.125,
                                            err=err, scratch=scratch)
        b = ops.paged_prefill_attention_fp8(q, kp, c["vp"], c["ks"], c["vs"], tabs, qsl, pr, 512, 0.125,
                                            err=err, tensor_cores=False)
        k = ops.paged_prefill_attention_fp8(q, kp, c["vp"], c["ks"], c["vs"], tabs, qsl, pr, 512, 0.125,
                                            err=err, scratch_free=True)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        ref = b.float().cpu().numpy()
        assert np.abs(a.float().cpu().numpy() - ref).max() <= 2 * fp8_atol("f16", ref)
        assert np.abs(k.float().cpu().numpy() - ref).max() <= 2 * fp8_atol("f16", ref)


def test_prefill_fp8_in_kernel_conversion_ignores_unused_slots(oracle_mod):
    """The tcgen05 prefill converting e4m3 tiles itself: the slots past each
    sequence's last key (the tail of its last block) may hold any bytes and
    scales, here +448-magnitude bytes and an infinite scale; the converters
    write those rows as zeros, so the output is bit-identical to the run over
    clean pools and matches the oracle.  bf16 queries are refused by the
    scratch-free entry point (PKV_ERR_UNSUPPORTED)."""
    prior = np.array([5, 0, 77, 200], dtype=np.int64)
    chunk = np.array([19, 33, 130, 3], dtype=np.int64)
    c = _fp8_case(91, prior + chunk, "f16")
    T = int(chunk.sum())
    q = dev(C.to_dtype(c["rng"].standard_normal((T, 14, 64), dtype=np.float32), "f16"), "f16")
    tabs = C.pad_tables(c["tables"])
    qsl = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    args = (dev(tabs), dev(qsl), dev(prior.astype(np.int32)), int(chunk.max()), 0.125)
    err = ops.new_error_flags("cuda")
    clean = ops.paged_prefill_attention_fp8(q, c["kp"], c["vp"], c["ks"], c["vs"], *args, err=err,
                                            scratch_free=True)
    torch.cuda.synchronize()
    kp, vp, ks, vs = c["kp"].clone(), c["vp"].clone(), c["ks"].clone(), c["vs"].clone()
    for t, n in zip(c["tables"], c["ctx"]):
        last, used = t[-1], int(n) - 16 * (len(t) - 1)
        kp[last, used:] = 0x7E
        vp[last, used:] = 0xFE
        ks[last, used:] = float("inf")
        vs[last, used:] = float("inf")
    dirty = ops.paged_prefill_attention_fp8(q, kp, vp, ks, vs, *args, err=err, scratch_free=True)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(clean, dirty)
    ref = oracle_mod.paged_attention_fp8(host(q, "f16").astype(np.float32), c["kp"].cpu().numpy(),
                                         c["vp"].cpu().numpy(), c["ks"].cpu().numpy(),
                                         c["vs"].cpu().numpy(), tabs, qsl, prior.astype(np.int32))
    assert np.abs(clean.float().cpu().numpy() - ref).max() <= fp8_atol("f16", ref)
    qb = q.to(torch.bfloat16)
    out = torch.empty_like(qb)
    nb = c["kp"].shape[0]
    rc = _lib.load().pkv_paged_prefill_attention_fp8_tc(
        out.data_ptr(), 14 * 64, qb.data_ptr(), 14 * 64, c["kp"].data_ptr(), c["vp"].data_ptr(),
        c["ks"].data_ptr(), c["vs"].data_ptr(), nb, args[0].data_ptr(), args[0].stride(0),
        args[0].shape[1], args[1].data_ptr(), args[2].data_ptr(), len(chunk), T, int(chunk.max()), 14, 2,
        64, 16, 0.125, _lib.BF16, None, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_UNSUPPORTED


def test_forward_layer_fp8_pools_and_cow(oracle_mod):
    """BlockManager(dtype=float8_e4m3fn) + forward_layer on a mixed batch
    (decodes then chunks): outputs against the oracle over the pools it left
    (dequantised), and a copy-on-write copies bytes and scales."""
    L, nb = 2, 128
    m = BlockManager(nb, 16, L, 2, 64, device="cuda", dtype=torch.float8_e4m3fn)
    assert m.fp8 and m.k_cache.dtype == torch.uint8 and m.block_bytes == 16 * 2 * 64
    kv = PagedKVCache(m)
    g = torch.Generator(device="cuda").manual_seed(74)
    plan = [(0, 40, 1), (1, 17, 1), (2, 48, 30), (3, 5, 20)]
    for s, prior, n in plan:
        kv.add_sequence(s, [m.allocate() for _ in range((prior + n + 15) // 16)], 0)
    # prefill the priors through the same path (chunks only), then the mixed step
    meta0 = kv.prepare_step([(s, prior) for s, prior, _ in plan])
    T0 = meta0.n_tokens
    for layer in range(L):
        q = torch.randn((T0, 14, 64), generator=g, device="cuda", dtype=torch.float16)
        k = torch.randn((T0, 2, 64), generator=g, device="cuda", dtype=torch.float16)
        kv.forward_layer(layer, q, k, k * 0.5, meta0, 0.125)
    meta = kv.prepare_step([(s, n) for s, _, n in plan])
    assert meta.n_decode == 2
    T = meta.n_tokens
    qsl = np.concatenate([[0], np.cumsum([n for _, _, n in plan])]).astype(np.int32)
    tabs = C.pad_tables([kv.block_tables[s] for s, _, _ in plan])
    for layer in range(L):
        q = torch.randn((T, 14, 64), generator=g, device="cuda", dtype=torch.float16)
        k = torch.randn((T, 2, 64), generator=g, device="cuda", dtype=torch.float16)
        v = torch.randn((T, 2, 64), generator=g, device="cuda", dtype=torch.float16)
        out = kv.forward_layer(layer, q, k, v, meta, 0.125)
        torch.cuda.synchronize()
        ref = oracle_mod.paged_attention_fp8(
            q.float().cpu().numpy(), m.k_pool[layer].cpu().numpy(), m.v_pool[layer].cpu().numpy(),
            m.k_scale[layer].cpu().numpy(), m.v_scale[layer].cpu().numpy(), tabs, qsl,
            np.array([p for _, p, _ in plan], dtype=np.int32))
        assert np.abs(out.float().cpu().numpy() - ref).max() <= fp8_atol("f16", ref)
    m.check_errors()
    # fork sequence 2 and copy-on-write its partial tail block: bytes and scales follow
    s = 2
    for b in kv.block_tables[s]:
        m.incref(b)
    kv.add_sequence(9, list(kv.block_tables[s]), kv.seq_len(s))
    kv.ensure_writable_tail(9)
    m.flush_copies()
    torch.cuda.synchronize()
    src, dst = kv.block_tables[s][-1], kv.block_tables[9][-1]
    assert src != dst
    assert torch.equal(m.k_cache[:, dst], m.k_cache[:, src])
    assert torch.equal(m.v_scale_cache[:, dst], m.v_scale_cache[:, src])


# ---------------------------------------------------------------- per-step decode schedule

def _sched_for(tabs, ctx, q, fp8=False, err=None):
    s = ops.new_decode_schedule(ctx.shape[0], tabs.shape[1], "cuda")
    s.random_(0, 255)  # the builder needs no initialised buffer
    return ops.build_decode_schedule(s, tabs, ctx, NB_SCHED[0], q.shape[1], 2, q.shape[2], q.dtype,
                                     fp8=fp8, err=err)


NB_SCHED = [0]


@pytest.mark.parametrize("dt", ("f16", "bf16"))
@pytest.mark.parametrize("case", ("c3", "ragged", "edge"))
def test_scheduled_decode_bit_identical(oracle_mod, dt, case):
    """pkv_decode_schedule + the _scheduled decode calls (plain and fused
    append) give the same bits as the unscheduled calls (the same stream-K
    partition and arithmetic), and match the oracle."""
    if case == "c3":
        c = C.make_decode_case(3, 256, 16, 8192, 0, dt, lognormal_median=1024.0, pool_slack=1.1)
    elif case == "ragged":
        rng = np.random.default_rng(31)
        ctx = rng.integers(1, 40, size=700).tolist()
        ctx[5], ctx[300], ctx[699] = 8192, 5000, 4097
        c = C.make_decode_case(31, len(ctx), 0, 0, sum((x + 15) // 16 for x in ctx) + 5, dt,
                               ctx_list=ctx)
    else:
        c = C.make_decode_case(11, 9, 0, 0, 128, dt, ctx_list=[1, 2, 15, 16, 17, 31, 32, 33, 600])
    NB_SCHED[0] = c["k_pool"].shape[0]
    tabs, ctx = dev(C.pad_tables(c["tables"])), dev(c["ctx"].astype(np.int32))
    q, kn, vn = dev(c["q"], dt), dev(c["k_new"], dt), dev(c["v_new"], dt)
    err = ops.new_error_flags("cuda")
    sched = _sched_for(tabs, ctx, q, err=err)
    outs = {}
    for mode in ("plain", "sched"):
        kp, vp = dev(c["k_pool"], dt), dev(c["v_pool"], dt)
        s = sched if mode == "sched" else None
        o1 = ops.paged_decode_append_attention(q, kn, vn, kp, vp, tabs, ctx, 0.125, err=err,
                                               schedule=s)
        o2 = ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, err=err, schedule=s)
        outs[mode] = (o1, o2, kp, vp)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for a, b in zip(outs["plain"], outs["sched"]):
        assert torch.equal(a, b)
    ref, ref_k, _ = oracle_mod.run_decode_case(c)
    assert np.array_equal(host(outs["sched"][2], dt), ref_k)
    assert max_abs_diff(host(outs["sched"][0], dt), ref, dt) <= PRODUCT_ATOL[dt]


def test_scheduled_decode_reused_across_layers_and_fp8(oracle_mod):
    """One schedule serves several layers' pools (the step's 24 calls), and
    an fp8 schedule serves the fp8 decode bit-identically."""
    c = C.make_decode_case(3, 256, 16, 8192, 0, "f16", lognormal_median=1024.0, pool_slack=1.1)
    NB_SCHED[0] = c["k_pool"].shape[0]
    tabs, ctx = dev(C.pad_tables(c["tables"])), dev(c["ctx"].astype(np.int32))
    q = dev(c["q"], "f16")
    err = ops.new_error_flags("cuda")
    sched = _sched_for(tabs, ctx, q, err=err)
    g = torch.Generator(device="cuda").manual_seed(5)
    for _ in range(3):
        kp = torch.randn(dev(c["k_pool"], "f16").shape, generator=g, device="cuda", dtype=torch.float16)
        vp = torch.randn_like(kp)
        a = ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, err=err)
        b = ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, err=err, schedule=sched)
        assert torch.equal(a, b)
    k8 = torch.randint(0, 256, kp.shape, generator=g, device="cuda", dtype=torch.uint8)
    k8[(k8 & 0x7f) == 0x7f] = 0  # no NaN encodings in live rows
    v8 = torch.randint(0, 256, kp.shape, generator=g, device="cuda", dtype=torch.uint8)
    v8[(v8 & 0x7f) == 0x7f] = 0
    ks = torch.rand(kp.shape[:3], generator=g, device="cuda") + 0.5
    vs = torch.rand(kp.shape[:3], generator=g, device="cuda") + 0.5
    s8 = _sched_for(tabs, ctx, q, fp8=True, err=err)
    a = ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, tabs, ctx, 0.125, err=err)
    b = ops.paged_decode_attention_fp8(q, k8, v8, ks, vs, tabs, ctx, 0.125, err=err, schedule=s8)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(a, b)


def test_scheduled_decode_rejects_foreign_schedule():
    """A schedule built for another batch size: the decode call sets
    PKV_FLAG_BAD_SCHEDULE (its output rows are then unspecified)."""
    c = C.make_decode_case(11, 9, 0, 0, 128, "f16", ctx_list=[1, 2, 15, 16, 17, 31, 32, 33, 600])
    NB_SCHED[0] = c["k_pool"].shape[0]
    tabs, ctx = dev(C.pad_tables(c["tables"])), dev(c["ctx"].astype(np.int32))
    q = dev(c["q"], "f16")
    kp, vp = dev(c["k_pool"], "f16"), dev(c["v_pool"], "f16")
    sched = _sched_for(tabs[:5], ctx[:5], q[:5])
    err = ops.new_error_flags("cuda")
    out = torch.full_like(q, 7.0)
    ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, out=out, err=err, schedule=sched)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.FLAG_BAD_SCHEDULE


def test_scheduled_decode_rejects_schedule_of_another_table_width():
    """A schedule built over block tables of another width (so another row
    length and buffer size) is not read: PKV_FLAG_BAD_SCHEDULE, and the
    decode call with the matching width still gives the unscheduled bits."""
    c = C.make_decode_case(12, 9, 0, 0, 128, "f16", ctx_list=[1, 2, 15, 16, 17, 31, 32, 33, 600])
    NB_SCHED[0] = c["k_pool"].shape[0]
    tabs, ctx = dev(C.pad_tables(c["tables"])), dev(c["ctx"].astype(np.int32))
    wide = torch.zeros((tabs.shape[0], tabs.shape[1] + 64), dtype=torch.int32, device="cuda")
    wide[:, :tabs.shape[1]] = tabs
    q = dev(c["q"], "f16")
    kp, vp = dev(c["k_pool"], "f16"), dev(c["v_pool"], "f16")
    sched = _sched_for(tabs, ctx, q)
    err = ops.new_error_flags("cuda")
    out = torch.full_like(q, 7.0)
    ops.paged_decode_attention(q, kp, vp, wide, ctx, 0.125, out=out, err=err, schedule=sched)
    torch.cuda.synchronize()
    assert int(err.item()) & _lib.FLAG_BAD_SCHEDULE
    err2 = ops.new_error_flags("cuda")
    got = ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, err=err2, schedule=sched)
    want = ops.paged_decode_attention(q, kp, vp, tabs, ctx, 0.125, err=err2)
    torch.cuda.synchronize()
    assert int(err2.item()) == 0
    assert torch.equal(got, want)


# ---------------------------------------------------------------- fused RoPE + fp8 append

@pytest.mark.parametrize("layout", ("packed", "padded"))
@pytest.mark.parametrize("dt", DTS)
def test_rope_reshape_and_cache_fp8_bit_identical(dt, layout):
    """pkv_rope_reshape_and_cache_fp8 against the unfused path: Rope.rotate in
    the model dtype, then reshape_and_cache_fp8.  Rotated q, the e4m3 bytes
    and the scales must be identical bit for bit; a padding slot (-1) writes
    q only.  Both kernel forms (qkv_rows)."""
    from pagedkv.model import Rope

    tdt = TORCH_DT[dt]
    g = torch.Generator(device="cuda").manual_seed(64)
    T, hq, hkv, d, nb = 200, 14, 2, 64, 64
    rope = Rope(d, 1e6, "cuda", tdt)
    cos, sin = rope.tables(5000)
    qkv = qkv_rows(T, (hq + 2 * hkv) * d, g, tdt, layout, mul=3.0)
    pos = torch.randint(0, 5000, (T,), generator=g, device="cuda")
    slots = torch.randperm(nb * 16, generator=g, device="cuda")[:T]
    slots[7] = -1
    kp = torch.randint(0, 255, (nb, 16, hkv, d), generator=g, device="cuda", dtype=torch.uint8)
    vp = torch.randint(0, 255, (nb, 16, hkv, d), generator=g, device="cuda", dtype=torch.uint8)
    ks = torch.rand((nb, 16, hkv), generator=g, device="cuda")
    vs = torch.rand((nb, 16, hkv), generator=g, device="cuda")
    ref = [t.clone() for t in (kp, vp, ks, vs)]
    err = ops.new_error_flags("cuda")
    q = ops.rope_reshape_and_cache(qkv, pos, cos, sin, kp, vp, slots, err=err, k_scale=ks, v_scale=vs)
    c, s = cos[pos].unsqueeze(1), sin[pos].unsqueeze(1)
    q_ref = Rope.rotate(qkv[:, : hq * d].view(T, hq, d), c, s)
    k_ref = Rope.rotate(qkv[:, hq * d: (hq + hkv) * d].view(T, hkv, d), c, s)
    v_ref = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
    ops.reshape_and_cache_fp8(k_ref.contiguous(), v_ref.contiguous(), *ref, slots)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(q, q_ref)
    for a, b in zip((kp, vp, ks, vs), ref):
        assert torch.equal(a, b)


def test_forward_layers_fp8_equals_forward_layer_fp8():
    """PagedKVCache.forward_layers over fp8 pools (one
    pkv_paged_decode_append_attention_fp8_layers call per run of layers, the
    layers chained on a split-K set each) against forward_layer layer by
    layer on a copy of the same pools: outputs, e4m3 bytes and scales
    bit-identical.  Two consecutive runs share the workspace."""
    rng = np.random.default_rng(48)
    L, nb = 5, 768
    ctx = rng.integers(1, 600, size=29)
    ctx[:3] = [1, 16, 17]
    managers = []
    for _ in range(2):
        m = BlockManager(nb, 16, L, 2, 64, device="cuda", dtype=torch.float8_e4m3fn)
        kv = PagedKVCache(m)
        o = 0
        for s_, c in enumerate(ctx):
            n = (int(c) + 15) // 16
            kv.add_sequence(s_, list(range(o, o + n)), int(c) - 1)
            o += n
        managers.append((m, kv))
    (m1, kv1), (m2, kv2) = managers
    g = torch.Generator(device="cuda").manual_seed(48)
    fill = torch.randn((nb * 16, 2, 64), generator=g, device="cuda").half()
    slots = torch.arange(nb * 16, device="cuda", dtype=torch.int64)
    for layer in range(L):  # identical quantised pools in both caches
        for m in (m1, m2):
            ops.reshape_and_cache_fp8(fill, fill * 0.5, m.k_pool[layer], m.v_pool[layer], m.k_scale[layer],
                                      m.v_scale[layer], slots, m.err)
    B = len(ctx)
    x = torch.randn((L, B, 18, 64), generator=g, device="cuda").half()
    meta1 = kv1.prepare_step([(s_, 1) for s_ in range(B)])
    meta2 = kv2.prepare_step([(s_, 1) for s_ in range(B)])
    out1 = torch.empty((L, B, 14, 64), dtype=torch.float16, device="cuda")
    for a, b in ((0, 2), (2, 5)):
        kv1.forward_layers(a, x[a:b, :, :14], x[a:b, :, 14:16], x[a:b, :, 16:18], meta1, 0.125,
                           out=out1[a:b])
    out2 = torch.stack([kv2.forward_layer(layer, x[layer, :, :14], x[layer, :, 14:16], x[layer, :, 16:18],
                                          meta2, 0.125) for layer in range(L)])
    torch.cuda.synchronize()
    m1.check_errors()
    m2.check_errors()
    assert torch.equal(out1, out2)
    assert torch.equal(m1.k_cache, m2.k_cache) and torch.equal(m1.v_cache, m2.v_cache)
    assert torch.equal(m1.k_scale_cache, m2.k_scale_cache) and torch.equal(m1.v_scale_cache, m2.v_scale_cache)


def test_forward_layer_qkv_fp8_equals_forward_layer_fp8():
    """Over fp8 pools, forward_layer_qkv (fused RoPE + quantising append, then
    the fp8 decode and prefill) equals rotating in torch and calling
    forward_layer, bit for bit (pools, scales and outputs)."""
    from pagedkv.model import Rope

    tdt = torch.float16
    g = torch.Generator(device="cuda").manual_seed(65)
    L, nb, hq, hkv, d = 2, 256, 14, 2, 64
    plan = [(0, 100, 1), (1, 17, 1), (2, 0, 1), (3, 48, 30), (4, 5, 64), (5, 31, 1)]
    caches = []
    for _ in range(2):
        m = BlockManager(nb, 16, L, hkv, d, device="cuda", dtype=torch.float8_e4m3fn)
        kv = PagedKVCache(m)
        o = 0
        for s, prior, n in plan:
            nblk = (prior + n + 15) // 16
            kv.add_sequence(s, list(range(o, o + nblk)), prior)
            o += nblk
        caches.append((m, kv))
    src = torch.randn((L, nb * 16, hkv, d), generator=g, device="cuda").to(tdt)
    allslots = torch.arange(nb * 16, device="cuda")
    for m, _ in caches:
        for layer in range(L):
            ops.reshape_and_cache_fp8(src[layer], src[layer], m.k_pool[layer], m.v_pool[layer],
                                      m.k_scale[layer], m.v_scale[layer], allslots)
    metas = [kv.prepare_step([(s, n) for s, _, n in plan]) for _, kv in caches]
    T = metas[0].n_tokens
    pos = torch.from_numpy(np.concatenate([np.arange(p, p + n) for _, p, n in plan])).cuda()
    cos, sin = Rope(d, 1e6, "cuda", tdt).tables(4096)
    for layer in range(L):
        qkv = torch.randn((T, (hq + 2 * hkv) * d), generator=g, device="cuda").to(tdt)
        out_a = caches[0][1].forward_layer_qkv(layer, qkv, pos, cos, sin, metas[0], 0.125)
        c, s_ = cos[pos].unsqueeze(1), sin[pos].unsqueeze(1)
        q = Rope.rotate(qkv[:, : hq * d].view(T, hq, d), c, s_)
        k = Rope.rotate(qkv[:, hq * d: (hq + hkv) * d].view(T, hkv, d), c, s_)
        v = qkv[:, (hq + hkv) * d:].view(T, hkv, d)
        out_b = caches[1][1].forward_layer(layer, q, k.contiguous(), v.contiguous(), metas[1], 0.125)
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b)
    for a, b in ((caches[0][0].k_cache, caches[1][0].k_cache), (caches[0][0].v_cache, caches[1][0].v_cache),
                 (caches[0][0].k_scale_cache, caches[1][0].k_scale_cache),
                 (caches[0][0].v_scale_cache, caches[1][0].v_scale_cache)):
        assert torch.equal(a, b)
    for m, _ in caches:
        m.check_errors()


@pytest.mark.parametrize("q_dt", ("f16", "bf16"))
@pytest.mark.parametrize("impl", ("auto", "generic"))
def test_decode_append_fp8_fused_equals_unfused(q_dt, impl):
    """pkv_paged_decode_append_attention_fp8 (the tensor-core decode kernel
    quantises the new token itself; the CUDA-core path appends with a
    separate kernel) gives the same pool bytes, scales and outputs, bit for
    bit, as reshape_and_cache_fp8 at the newest slot followed by
    paged_decode_attention_fp8, with and without a schedule."""
    ops.set_decode_impl(_lib.DECODE_AUTO if impl == "auto" else _lib.DECODE_GENERIC)
    try:
        ctx = [1, 15, 16, 17, 33, 600, 1000, 2047, 64, 5000, 3, 250]
        c = _fp8_case(73, ctx, "f16")
        B = len(ctx)
        tdt = TORCH_DT[q_dt]
        g = torch.Generator(device="cuda").manual_seed(9)
        q = torch.randn((B, 14, 64), generator=g, device="cuda").to(tdt)
        kn = (2 * torch.randn((B, 2, 64), generator=g, device="cuda")).to(tdt)
        vn = torch.randn((B, 2, 64), generator=g, device="cuda").to(tdt)
        tabs_np = C.pad_tables(c["tables"])
        tabs, ctx_d = dev(tabs_np), dev(c["ctx"].astype(np.int32))
        pos = c["ctx"] - 1
        slots = torch.from_numpy(tabs_np[np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16).cuda()
        err = ops.new_error_flags("cuda")
        ref = [t.clone() for t in (c["kp"], c["vp"], c["ks"], c["vs"])]
        ops.reshape_and_cache_fp8(kn, vn, *ref, slots, err)
        out_ref = ops.paged_decode_attention_fp8(q, *ref, tabs, ctx_d, 0.125, err=err)
        for use_sched in (False, True):
            pools = [t.clone() for t in (c["kp"], c["vp"], c["ks"], c["vs"])]
            sched = None
            if use_sched:
                NB_SCHED[0] = pools[0].shape[0]
                sched = _sched_for(tabs, ctx_d, q, fp8=True, err=err)
            out = ops.paged_decode_append_attention_fp8(q, kn, vn, *pools, tabs, ctx_d, 0.125, err=err,
                                                        schedule=sched)
            torch.cuda.synchronize()
            assert int(err.item()) == 0
            for a, b in zip(pools, ref):
                assert torch.equal(a, b)
            assert torch.equal(out, out_ref)
    finally:
        ops.set_decode_impl(_lib.DECODE_AUTO)
