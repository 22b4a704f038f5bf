"""The C ABI surface of libpagedkv.so, checked without a GPU.

* the library loads and exports every function include/pagedkv.h declares;
* host-side argument validation answers with the documented negative codes
  before anything is launched (so these calls never reach the device);
* constants in the header agree with the Python binding.
"""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from pagedkv import _lib

HEADER = os.path.join(ROOT, "include", "pagedkv.h")


def header_functions():
    src = open(HEADER).read()
    return re.findall(r"^\s*(?:int|size_t|const char\s*\*)\s+(pkv_\w+)\s*\(", src, re.M)


def header_defines():
    src = open(HEADER).read()
    return {k: int(v) for k, v in re.findall(r"#define\s+(PKV_\w+)\s+\(?(-?\d+)\)?", src)}


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    names = header_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(L, n), f"{n} declared in pagedkv.h but not exported"
    assert sorted(names) == sorted(_lib.SIGNATURES), "binding and header disagree"


def test_header_constants_match_binding():
    d = header_defines()
    assert d["PKV_ABI_VERSION"] == _lib.load().pkv_abi_version()
    for name in ("F32", "F16", "BF16"):
        assert d[f"PKV_DTYPE_{name}"] == getattr(_lib, name)
    for name in ("NULL_POINTER", "BAD_SHAPE", "BAD_DTYPE", "WORKSPACE_TOO_SMALL", "MISALIGNED",
                 "UNSUPPORTED", "DRIVER"):
        assert d[f"PKV_ERR_{name}"] == getattr(_lib, f"ERR_{name}")
    for name in ("SLOT_OUT_OF_RANGE", "BLOCK_OUT_OF_RANGE", "CONTEXT_EXCEEDS_TABLE",
                 "PIPELINE_TIMEOUT", "BAD_QUERY_LAYOUT", "POSITION_OUT_OF_RANGE", "BAD_SCHEDULE"):
        assert d[f"PKV_FLAG_{name}"] == getattr(_lib, f"FLAG_{name}")


def test_status_strings():
    for code in (0, -1, -2, -3, -4, -5, -6, -7):
        s = _lib.status_string(code)
        assert s and "unknown" not in s
    assert "unknown" in _lib.status_string(-99)


FAKE = ctypes.c_void_p(0x1000)  # never dereferenced: validation fails first


def test_reshape_and_cache_validation():
    L = _lib.load()
    f = L.pkv_reshape_and_cache
    assert f(None, None, 128, 128, None, None, None, 0, 8, 16, 2, 64, 1, None, None) == 0  # no tokens
    assert f(None, FAKE, 128, 128, FAKE, FAKE, FAKE, 4, 8, 16, 2, 64, 1, None, None) == _lib.ERR_NULL_POINTER
    assert f(FAKE, FAKE, 128, 128, FAKE, FAKE, FAKE, 4, 8, 16, 2, 64, 7, None, None) == _lib.ERR_BAD_DTYPE
    assert f(FAKE, FAKE, 64, 128, FAKE, FAKE, FAKE, 4, 8, 16, 2, 64, 1, None, None) == _lib.ERR_BAD_SHAPE
    assert f(FAKE, FAKE, 128, 128, FAKE, FAKE, FAKE, -1, 8, 16, 2, 64, 1, None, None) == _lib.ERR_BAD_SHAPE


def test_copy_blocks_validation():
    L = _lib.load()
    f = L.pkv_copy_blocks
    assert f(None, None, 0, 24, None, 0, 8, 4096, None, None) == 0
    assert f(FAKE, None, 8 * 4096, 24, FAKE, 3, 8, 4096, None, None) == _lib.ERR_NULL_POINTER
    assert f(FAKE, FAKE, 100, 24, FAKE, 3, 8, 4096, None, None) == _lib.ERR_BAD_SHAPE
    assert f(FAKE, FAKE, 8 * 4096, 70000, FAKE, 3, 8, 4096, None, None) == _lib.ERR_UNSUPPORTED


def test_copy_blocks_peer_validation():
    f = _lib.load().pkv_copy_blocks_peer
    A = ctypes.c_void_p(0x10000)  # 16-byte aligned, never dereferenced
    ok = dict(dk=A, dv=A, dls=8 * 4096, dnb=8, sk=A, sv=A, sls=8 * 4096, snb=8, L=24, pairs=A,
              n=3, bb=4096, err=None, stream=None)

    def call(**kw):
        a = dict(ok)
        a.update(kw)
        return f(*a.values())

    assert call(n=0) == 0 and call(L=0) == 0
    assert call(sv=None) == _lib.ERR_NULL_POINTER
    assert call(pairs=None) == _lib.ERR_NULL_POINTER
    assert call(n=-1) == _lib.ERR_BAD_SHAPE
    assert call(dnb=0) == _lib.ERR_BAD_SHAPE
    assert call(sls=100) == _lib.ERR_BAD_SHAPE        # layers overlap
    assert call(L=70000) == _lib.ERR_UNSUPPORTED
    assert call(bb=4100, dls=8 * 4100, sls=8 * 4100) == _lib.ERR_MISALIGNED
    assert call(dk=ctypes.c_void_p(0x10008)) == _lib.ERR_MISALIGNED


def test_decode_schedule_validation():
    L = _lib.load()
    nbytes = L.pkv_decode_schedule_bytes(256, 512)
    assert nbytes >= 4 * (256 * 512 + 2 * 256 + 1)
    assert L.pkv_decode_schedule_bytes(-1, 4) == 0
    A = ctypes.c_void_p(0x10000)
    ok = dict(s=A, sb=nbytes, tabs=A, bts=512, mb=512, ctx=A, B=256, nb=4096, hq=14, hkv=2, d=64,
              bs=16, dt=1, fp8=0, err=None, stream=None)

    def call(**kw):
        a = dict(ok)
        a.update(kw)
        return L.pkv_decode_schedule(*a.values())

    assert call(s=None) == _lib.ERR_NULL_POINTER
    assert call(ctx=None) == _lib.ERR_NULL_POINTER
    assert call(s=ctypes.c_void_p(0x10004)) == _lib.ERR_MISALIGNED
    assert call(sb=nbytes - 4) == _lib.ERR_WORKSPACE_TOO_SMALL
    assert call(B=-1) == _lib.ERR_BAD_SHAPE
    assert call(hq=13) == _lib.ERR_BAD_SHAPE
    assert call(bts=100) == _lib.ERR_BAD_SHAPE
    assert call(dt=9) == _lib.ERR_BAD_DTYPE
    assert call(B=0) == _lib.OK
    # the scheduled decode entries check the schedule pointer before anything else
    d = dict(out=FAKE, out_stride=896, q=FAKE, q_stride=896, k_pool=FAKE, v_pool=FAKE,
             num_blocks=64, tables=FAKE, bt_stride=8, max_blocks=8, ctx=FAKE, n_seqs=4, hq=14,
             hkv=2, d=64, bs=16, scale=0.125, dtype=1, ws=FAKE, ws_bytes=1 << 30, err=None,
             stream=None)
    f = L.pkv_paged_decode_attention_scheduled
    assert f(*d.values(), None) == _lib.ERR_NULL_POINTER
    assert f(*d.values(), ctypes.c_void_p(0x10008)) == _lib.ERR_MISALIGNED


def test_ipc_validation():
    L = _lib.load()
    off = ctypes.c_uint64(0)
    h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    base = ctypes.c_void_p(0)
    assert L.pkv_ipc_export(None, h, ctypes.byref(off)) == _lib.ERR_NULL_POINTER
    assert L.pkv_ipc_export(FAKE, None, ctypes.byref(off)) == _lib.ERR_NULL_POINTER
    assert L.pkv_ipc_open(None, ctypes.byref(base)) == _lib.ERR_NULL_POINTER
    assert L.pkv_ipc_open(h, None) == _lib.ERR_NULL_POINTER
    assert L.pkv_ipc_close(None) == _lib.ERR_NULL_POINTER
    assert header_defines()["PKV_IPC_HANDLE_BYTES"] == _lib.IPC_HANDLE_BYTES


def _decode(**kw):
    a = dict(out=FAKE, out_stride=896, q=FAKE, q_stride=896, k_pool=FAKE, v_pool=FAKE,
             num_blocks=64, tables=FAKE, bt_stride=8, max_blocks=8, ctx=FAKE, n_seqs=4, hq=14,
             hkv=2, d=64, bs=16, scale=0.125, dtype=1, ws=FAKE, ws_bytes=1 << 30, err=None,
             stream=None)
    a.update(kw)
    return _lib.load().pkv_paged_decode_attention(*a.values())


def test_decode_validation():
    assert _decode(n_seqs=0) == 0
    assert _decode(q=None) == _lib.ERR_NULL_POINTER
    assert _decode(ctx=None) == _lib.ERR_NULL_POINTER
    assert _decode(dtype=3) == _lib.ERR_BAD_DTYPE
    assert _decode(hkv=3) == _lib.ERR_BAD_SHAPE          # 14 % 3 != 0
    assert _decode(d=512, q_stride=14 * 512, out_stride=14 * 512) == _lib.ERR_BAD_SHAPE
    assert _decode(bt_stride=4) == _lib.ERR_BAD_SHAPE     # stride < max_blocks
    assert _decode(q_stride=100) == _lib.ERR_BAD_SHAPE
    assert _decode(ws_bytes=16) == _lib.ERR_WORKSPACE_TOO_SMALL
    assert _decode(ws=None) == _lib.ERR_NULL_POINTER
    assert _decode(ws=ctypes.c_void_p(0x1010)) == _lib.ERR_MISALIGNED


def test_prefill_validation():
    f = _lib.load().pkv_paged_prefill_attention
    args = [FAKE, 896, FAKE, 896, FAKE, FAKE, 64, FAKE, 8, 8, FAKE, FAKE, 2, 10, 8, 14, 2, 64, 16,
            0.125, 1, None, None]
    bad = list(args)
    bad[10] = None  # query_start_loc
    assert f(*bad) == _lib.ERR_NULL_POINTER
    bad = list(args)
    bad[13] = -1  # n_tokens
    assert f(*bad) == _lib.ERR_BAD_SHAPE
    bad = list(args)
    bad[13] = 0
    assert f(*bad) == 0


def test_workspace_bytes():
    L = _lib.load()
    a = L.pkv_decode_workspace_bytes(256, 14, 64)
    b = L.pkv_decode_workspace_bytes(512, 14, 64)
    assert a > 0 and b >= a and a % 256 == 0
    assert L.pkv_decode_workspace_bytes(-1, 14, 64) == 0


def test_set_decode_impl_validation():
    L = _lib.load()
    assert L.pkv_set_decode_impl(5) == _lib.ERR_UNSUPPORTED
    assert L.pkv_set_decode_impl(_lib.DECODE_AUTO) == 0


def test_decode_append_validation():
    f = _lib.load().pkv_paged_decode_append_attention
    base = [FAKE, 896, FAKE, 896, FAKE, FAKE, 128, 128, FAKE, FAKE, 64, FAKE, 8, 8, FAKE, 4, 14, 2,
            64, 16, 0.125, 1, FAKE, 1 << 30, None, None]
    a = list(base)
    a[4] = None  # k_new
    assert f(*a) == _lib.ERR_NULL_POINTER
    a = list(base)
    a[6] = 64  # k_new row stride below n_kv_heads * head_dim
    assert f(*a) == _lib.ERR_BAD_SHAPE
    a = list(base)
    a[15] = 0  # no sequences: nothing to do
    assert f(*a) == 0


def test_rope_reshape_and_cache_validation():
    f = _lib.load().pkv_rope_reshape_and_cache
    # q_out, q_stride, qkv, qkv_stride, positions, cos, sin, max_pos, k_pool, v_pool, slots,
    # n_tokens, num_blocks, block_size, hq, hkv, d, dtype, err, stream
    base = [FAKE, 896, FAKE, 1152, FAKE, FAKE, FAKE, 4096, FAKE, FAKE, FAKE, 8, 64, 16, 14, 2, 64, 1,
            None, None]
    a = list(base)
    a[11] = 0  # no tokens: nothing to do
    assert f(*a) == 0
    a = list(base)
    a[4] = None  # positions
    assert f(*a) == _lib.ERR_NULL_POINTER
    a = list(base)
    a[3] = 1151  # qkv row shorter than (14 + 2 * 2) * 64
    assert f(*a) == _lib.ERR_BAD_SHAPE
    a = list(base)
    a[16] = 63  # odd head_dim
    assert f(*a) == _lib.ERR_BAD_SHAPE
    a = list(base)
    a[7] = 0  # no table rows
    assert f(*a) == _lib.ERR_BAD_SHAPE
    a = list(base)
    a[17] = 9
    assert f(*a) == _lib.ERR_BAD_DTYPE
