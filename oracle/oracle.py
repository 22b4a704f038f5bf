"""ctypes front end of the CPU oracle (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
this module, and only as the checker or the timed CPU baseline.  The product
(libpagedkv.so and the `pagedkv` package) never imports it.

The oracle restates the reference's paged-KV path on the CPU; see
pagedkv_oracle.c for the reference file:line of each function.  Inputs are
numpy arrays (bf16 carried as uint16 bit patterns).
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle_pagedkv.so")

DT_CODE = {"f32": 0, "f16": 1, "bf16": 2}
NP_DT = {"f32": np.float32, "f16": np.float16, "bf16": np.uint16}

_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", HERE, "OCC=gcc"], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        L.orc_reshape_and_cache.argtypes = [P, P, I64, I64, P, P, P, I, I, I, I, I, I]
        L.orc_reshape_and_cache.restype = I
        L.orc_copy_blocks.argtypes = [P, P, I64, I, I64, I, P, I]
        L.orc_copy_blocks.restype = I
        L.orc_paged_attention.argtypes = [P, P, P, P, P, I64, P, P, I, I, I, I, I, I, F, I, I]
        L.orc_paged_attention.restype = I
        L.orc_num_threads.argtypes = []
        L.orc_num_threads.restype = I
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.c_void_p)


def num_threads() -> int:
    return lib().orc_num_threads()


def reshape_and_cache(k_pool, v_pool, k, v, slots, dt: str) -> int:
    """In place: k_pool[slot] = k[t] for every token t with slot >= 0."""
    nb, bs, hkv, d = k_pool.shape
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    slots = np.ascontiguousarray(slots, dtype=np.int64)
    return lib().orc_reshape_and_cache(_p(k), _p(v), hkv * d, hkv * d, _p(k_pool), _p(v_pool),
                                       _p(slots), len(slots), nb, bs, hkv, d, DT_CODE[dt])


def copy_blocks(k_pools, v_pools, pairs) -> int:
    """In place over [L, NB, bs, Hkv, D] pools: block dst <- block src in every layer."""
    L, nb = k_pools.shape[:2]
    block_bytes = int(np.prod(k_pools.shape[2:])) * k_pools.itemsize
    pairs = np.ascontiguousarray(pairs, dtype=np.int32).reshape(-1, 2)
    return lib().orc_copy_blocks(_p(k_pools), _p(v_pools), nb * block_bytes, L, block_bytes, nb,
                                 _p(pairs), len(pairs))


def paged_attention(q, k_pool, v_pool, tables_padded, qsl, num_prior, dt: str,
                    scale: float = 0.125, threads: int = 0) -> np.ndarray:
    T, hq, d = q.shape
    nb, bs, hkv, _ = k_pool.shape
    out = np.zeros_like(q)
    tables_padded = np.ascontiguousarray(tables_padded, dtype=np.int32)
    qsl = np.ascontiguousarray(qsl, dtype=np.int32)
    num_prior = np.ascontiguousarray(num_prior, dtype=np.int32)
    rc = lib().orc_paged_attention(_p(out), _p(np.ascontiguousarray(q)), _p(k_pool), _p(v_pool),
                                   _p(tables_padded), tables_padded.shape[1], _p(qsl),
                                   _p(num_prior), len(num_prior), hq, hkv, d, bs, nb,
                                   float(scale), DT_CODE[dt], int(threads))
    if rc != 0:
        raise ValueError("oracle: block table entry outside the pool")
    return out


# ---- fp8 e4m3 KV (no reference counterpart: the reference's quant.py names
# fp8 KV as its next step).  Restated from the e4m3 format -- 1 sign bit, 4
# exponent bits (bias 7), 3 mantissa bits, no infinities, S.1111.111 = NaN,
# largest finite 448 -- and this library's row quantisation rule: scale =
# absmax(row) / 448 (1 for an all-zero row), byte = e4m3(x / scale) rounded
# to nearest with ties to the even mantissa, saturated at +-448.

def e4m3_decode(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b).astype(np.int64)
    s, e, m = (b >> 7) & 1, (b >> 3) & 15, b & 7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    val = np.where((e == 15) & (m == 7), np.nan, val)
    return np.where(s == 1, -val, val).astype(np.float32)


_E4M3_POS = e4m3_decode(np.arange(127))  # codes 0..126: the non-negative finite values, ascending


def e4m3_encode(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    a = np.minimum(np.abs(x), np.float32(448.0))
    hi = np.clip(np.searchsorted(_E4M3_POS, a, side="left"), 0, 126)
    lo = np.clip(hi - 1, 0, 126)
    dlo = a - _E4M3_POS[lo]
    dhi = _E4M3_POS[hi] - a
    code = np.where(dhi < dlo, hi, np.where(dlo < dhi, lo, np.where(hi % 2 == 0, hi, lo)))
    code = np.where(a == _E4M3_POS[hi], hi, code)
    return (code | (np.signbit(x).astype(np.int64) << 7)).astype(np.uint8)


def fp8_quantize_rows(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """x [..., D] (fp32 values of the source rows) -> (bytes [..., D], scale [...])."""
    x = np.asarray(x, dtype=np.float32)
    amax = np.abs(x).max(axis=-1)
    scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    return e4m3_encode(x / scale[..., None]), scale


def fp8_dequantize(b: np.ndarray, scale: np.ndarray) -> np.ndarray:
    return (e4m3_decode(b) * np.asarray(scale, dtype=np.float32)[..., None]).astype(np.float32)


def paged_attention_fp8(q32, k_bytes, v_bytes, k_scale, v_scale, tables_padded, qsl, num_prior,
                        scale: float = 0.125, threads: int = 0) -> np.ndarray:
    """Attention over fp8 pools: dequantised to fp32, then the fp32 oracle."""
    return paged_attention(np.ascontiguousarray(q32, dtype=np.float32),
                           np.ascontiguousarray(fp8_dequantize(k_bytes, k_scale)),
                           np.ascontiguousarray(fp8_dequantize(v_bytes, v_scale)),
                           tables_padded, qsl, num_prior, "f32", scale, threads)


# ---- whole-case runners (mirror the reference's append-then-attend order) ----

def run_decode_case(c, threads: int = 0):
    """Append each sequence's new token at position ctx-1, then attend over
    ctx tokens (PagedKVCache.append_and_fetch + Qwen2Model._attention)."""
    import cases as C  # tests/golden/cases.py (on sys.path in tests)

    k_pool, v_pool = c["k_pool"].copy(), c["v_pool"].copy()
    slots = C.decode_slots(c)
    assert reshape_and_cache(k_pool, v_pool, c["k_new"], c["v_new"], slots, c["dt"]) == 0
    B = len(c["ctx"])
    qsl = np.arange(B + 1, dtype=np.int32)
    out = paged_attention(c["q"], k_pool, v_pool, C.pad_tables(c["tables"]), qsl,
                          (c["ctx"] - 1).astype(np.int32), c["dt"], threads=threads)
    return out, k_pool, v_pool


def run_prefill_case(c, threads: int = 0):
    import cases as C

    k_pool, v_pool = c["k_pool"].copy(), c["v_pool"].copy()
    slots = C.prefill_slots(c)
    assert reshape_and_cache(k_pool, v_pool, c["k_new"], c["v_new"], slots, c["dt"]) == 0
    out = paged_attention(c["q"], k_pool, v_pool, C.pad_tables(c["tables"]), c["qsl"],
                          c["prior"].astype(np.int32), c["dt"], threads=threads)
    return out, k_pool, v_pool
