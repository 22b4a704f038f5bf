"""Pin the CPU oracle to the reference: every golden vector the reference's own
Python path produced (tests/golden/make_golden.py) must be reproduced.

* decode / prefill attention: within about one ulp of the output dtype
  (ORACLE_ATOL), and with most elements bit-identical;
* append + copy-on-write (config 2): the pools after the reference's scatter
  and after its COW copies have the same SHA-256 as the oracle's, i.e. the
  data path is bit-exact.
"""

import json

import numpy as np
import pytest

import cases as C
from conftest import GOLDEN, ORACLE_ATOL, as_f32, golden, max_abs_diff

DTS = ("f32", "f16", "bf16")


def _check(out, g, dt, max_mismatch_frac):
    assert out.shape == g["out"].shape
    d = max_abs_diff(out, g["out"], dt)
    assert d <= ORACLE_ATOL[dt], f"{dt}: max |oracle - reference| = {d}"
    frac = float(np.mean(as_f32(out, dt) != as_f32(g["out"], dt)))
    assert frac <= max_mismatch_frac, f"{dt}: {frac:.3%} elements differ from the reference"


@pytest.mark.parametrize("dt", DTS)
def test_decode_config1(oracle_mod, dt):
    c = C.make_decode_case(1, 8, 32, 600, 512, dt)
    g = golden(f"decode_c1_{dt}.npz")
    assert str(g["input_sha256"]) == C.decode_digest(c), "seeded inputs changed"
    out, _, _ = oracle_mod.run_decode_case(c)
    _check(out, g, dt, 1.0 if dt == "f32" else 0.05)


@pytest.mark.parametrize("dt", DTS)
def test_decode_edge_contexts(oracle_mod, dt):
    """Contexts 1, 2, 15, 16, 17, 31, 32, 33 and 600: block boundaries."""
    c = C.make_decode_case(11, 9, 0, 0, 128, dt, ctx_list=[1, 2, 15, 16, 17, 31, 32, 33, 600])
    g = golden(f"decode_edge_{dt}.npz")
    assert str(g["input_sha256"]) == C.decode_digest(c)
    out, _, _ = oracle_mod.run_decode_case(c)
    _check(out, g, dt, 1.0 if dt == "f32" else 0.05)


@pytest.mark.parametrize("dt", DTS)
@pytest.mark.parametrize("name,args", [
    ("prefill_small", (21, [1, 7, 33, 64, 16], [0, 5, 37, 100, 11], 48, 256)),
    ("prefill_noshare", (22, [20, 3, 48], [0, 16, 1], 0, 64)),
])
def test_prefill_small(oracle_mod, dt, name, args):
    c = C.make_prefill_case(*args, dt)
    g = golden(f"{name}_{dt}.npz")
    assert str(g["input_sha256"]) == C.prefill_digest(c)
    out, _, _ = oracle_mod.run_prefill_case(c)
    _check(out, g, dt, 1.0 if dt == "f32" else 0.05)


def test_decode_config3_full(oracle_mod):
    """BASELINE config 3 at full size (B=256, lognormal contexts), one layer."""
    c = C.make_decode_case(3, 256, 16, 8192, 0, "f16", lognormal_median=1024.0, pool_slack=1.1)
    g = golden("decode_c3_f16.npz")
    assert str(g["input_sha256"]) == C.decode_digest(c)
    assert int(g["sum_ctx"]) == int(c["ctx"].sum())
    out, _, _ = oracle_mod.run_decode_case(c)
    _check(out, g, "f16", 0.05)


def test_prefill_config4_full(oracle_mod):
    """BASELINE config 4 at full size (16 x 512-token chunks over a shared
    48-token prefix + private prior up to 4096); reference rows sampled."""
    c = C.make_c4_case()
    g = golden("prefill_c4_f16_rows.npz")
    assert str(g["input_sha256"]) == C.prefill_digest(c)
    out, _, _ = oracle_mod.run_prefill_case(c)
    d = max_abs_diff(out[g["rows"]], g["out"], "f16")
    assert d <= ORACLE_ATOL["f16"]


def test_append_and_cow_config2_bit_exact(oracle_mod):
    c = C.make_append_cow_case()
    with open(f"{GOLDEN}/append_cow_c2_f16.json") as f:
        g = json.load(f)
    assert g["input_sha256"] == C.append_cow_digest(c)
    kp, vp = c["k_pools"].copy(), c["v_pools"].copy()
    L = c["n_layers"]
    # the reference allocated each sequence's table from the seeded free list
    tables = g["tables"]
    pos = c["ctx"] - 1
    slots = np.array([tables[s][p // C.BS] * C.BS + p % C.BS for s, p in enumerate(pos)])
    for layer in range(L):
        assert oracle_mod.reshape_and_cache(kp[layer], vp[layer], c["k_new"][layer],
                                            c["v_new"][layer], slots, "f16") == 0
    assert C.digest(*kp, *vp) == g["pools_after_append_sha256"]
    assert oracle_mod.copy_blocks(kp, vp, np.array(g["pairs"], dtype=np.int32)) == 0
    assert C.digest(*kp, *vp) == g["pools_after_cow_sha256"]


def test_oracle_rejects_bad_block(oracle_mod):
    c = C.make_decode_case(5, 2, 20, 40, 16, "f32")
    tabs = C.pad_tables(c["tables"])
    tabs[0, 0] = 999  # outside the 16-block pool
    with pytest.raises(ValueError):
        oracle_mod.paged_attention(c["q"], c["k_pool"], c["v_pool"], tabs,
                                   np.arange(3, dtype=np.int32), (c["ctx"] - 1).astype(np.int32), "f32")


def test_e4m3_codec(oracle_mod):
    """The oracle's fp8 e4m3 codec: every finite code round-trips, the largest
    value is 448, ties round to the even mantissa, magnitudes saturate."""
    codes = np.arange(256, dtype=np.uint8)
    vals = oracle_mod.e4m3_decode(codes)
    fin = ~np.isnan(vals)
    assert fin.sum() == 254 and vals[fin].max() == 448.0 and vals[1] == 2.0 ** -9
    assert np.array_equal(oracle_mod.e4m3_decode(oracle_mod.e4m3_encode(vals[fin])), vals[fin])
    x = np.array([1.0625, 1.1875, 2.0 ** -10, 3 * 2.0 ** -10, 500.0, -1e9, -2.5], np.float32)
    assert oracle_mod.e4m3_decode(oracle_mod.e4m3_encode(x)).tolist() == \
        [1.0, 1.25, 0.0, 2.0 ** -8, 448.0, -448.0, -2.5]
    b, s = oracle_mod.fp8_quantize_rows(np.array([[0.0, 0.0], [1.0, -3.5]], np.float32))
    assert s.tolist() == [1.0, np.float32(3.5) / np.float32(448.0)] and b[1, 1] == 0xFE
