"""The allocation-free decode entry point, pkv_paged_decode_attention_noalloc.

It exists for callers that cannot allocate device memory where they run decode
attention (a thin FFI layer forwarding only the pointers it was handed, or a
process whose GPU memory belongs to another allocator) and therefore cannot
pass the split-K workspace pkv_paged_decode_attention needs.  It keeps that
scratch in a fixed 8 MiB device array inside the library instead.

These tests call it through the C ABI (ctypes, raw pointers) and check:
* two calls in a row each match the regular entry point (which gets its own
  workspace) and the CPU oracle within the fp16/bf16 tolerances the other
  parity tests use;
* a problem whose partials would not fit the fixed array is refused with
  PKV_ERR_SCRATCH_LIMIT before anything runs, leaving the output untouched.

This file is named so pytest collects it after every other test file.
"""

import numpy as np
import pytest
import torch

import cases as C
from conftest import PRODUCT_ATOL, max_abs_diff
from pagedkv import _lib, ops

pytestmark = pytest.mark.gpu

TORCH_DT = {"f16": torch.float16, "bf16": torch.bfloat16}


def _dev(a, dt=None):
    a = np.ascontiguousarray(a)
    if dt == "bf16":
        return torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()
    return torch.from_numpy(a).cuda()


def _host(t, dt):
    t = t.contiguous().cpu()
    return t.view(torch.int16).numpy().view(np.uint16) if dt == "bf16" else t.numpy()


def _call_noalloc(out, q, k_pool, v_pool, tables, ctx, err, scale=0.125):
    nb, bs, hkv, d = k_pool.shape
    B, hq, _ = q.shape
    return _lib.load().pkv_paged_decode_attention_noalloc(
        out.data_ptr(), hq * d, q.data_ptr(), hq * d, k_pool.data_ptr(), v_pool.data_ptr(), nb,
        tables.data_ptr(), tables.stride(0), tables.shape[1], ctx.data_ptr(), B, hq, hkv, d, bs,
        float(scale), ops.dtype_code(q.dtype), err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("name,dt,make", [
    ("config3", "f16", lambda: C.make_decode_case(3, 256, 16, 8192, 0, "f16",
                                                 lognormal_median=1024.0, pool_slack=1.1)),
    ("config1", "bf16", lambda: C.make_decode_case(1, 8, 32, 600, 512, "bf16")),
])
def test_noalloc_matches_regular_entry_point_on_two_calls(name, dt, make, oracle_mod):
    c = make()
    want, _, _ = oracle_mod.run_decode_case(c)
    kp, vp = _dev(c["k_pool"], dt), _dev(c["v_pool"], dt)
    ops.reshape_and_cache(_dev(c["k_new"], dt), _dev(c["v_new"], dt), kp, vp,
                          torch.from_numpy(C.decode_slots(c)).cuda())
    q = _dev(c["q"], dt)
    tables = _dev(C.pad_tables(c["tables"]))
    ctx = _dev(c["ctx"].astype(np.int32))
    err = ops.new_error_flags("cuda")
    ref = ops.paged_decode_attention(q, kp, vp, tables, ctx, 0.125, err=err)
    for call in range(2):
        out = torch.full_like(q, float("nan"))
        rc = _call_noalloc(out, q, kp, vp, tables, ctx, err)
        assert rc == _lib.OK, _lib.status_string(rc)
        torch.cuda.synchronize()
        d = max_abs_diff(_host(out, dt), _host(ref, dt), dt)
        assert d <= PRODUCT_ATOL[dt], f"{name} call {call}: max |noalloc - regular| = {d}"
        d = max_abs_diff(_host(out, dt), want, dt)
        assert d <= PRODUCT_ATOL[dt], f"{name} call {call}: max |noalloc - oracle| = {d}"
    assert int(err.item()) == 0


def test_noalloc_refuses_problems_beyond_its_scratch():
    # 32 query heads over 4 kv heads at head_dim 64: the split-K partials need
    # about 17 MB, more than the fixed 8 MiB array
    hq, hkv = 32, 4
    assert ops.decode_workspace_bytes(4, hq, 64) > _lib.NOALLOC_SCRATCH_BYTES
    kp = torch.randn(8, 16, hkv, 64, dtype=torch.float16, device="cuda")
    vp = torch.randn_like(kp)
    q = torch.randn(4, hq, 64, dtype=torch.float16, device="cuda")
    tables = torch.arange(8, dtype=torch.int32, device="cuda").view(4, 2)
    ctx = torch.full((4,), 20, dtype=torch.int32, device="cuda")
    out = torch.zeros_like(q)
    err = ops.new_error_flags("cuda")
    rc = _call_noalloc(out, q, kp, vp, tables, ctx, err)
    assert rc == _lib.ERR_SCRATCH_LIMIT
    assert "PKV_NOALLOC_SCRATCH_BYTES" in _lib.status_string(rc)
    torch.cuda.synchronize()
    assert int(out.abs().sum().item()) == 0 and int(err.item()) == 0
