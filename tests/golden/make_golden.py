"""Generate the golden vectors by running the REFERENCE's own Python path.

Run in a container that has the reference checked out (read-only is fine):

    REF_ROOT=/path/to/llm-inference-scheduler python tests/golden/make_golden.py

It imports `mini_engine` from REF_ROOT and drives exactly the calls the
reference engine makes on its hot path:

* `PagedKVCache.add_sequence` / `append_and_fetch` (block_manager.py:87-141):
  the scatter into the pool, the last-layer length update and the gather;
* `Qwen2Model._attention` (qwen2.py:98-128): GQA repeat_interleave, fp16/bf16
  score rounding, causal mask with the `num_prior` offset, fp32 softmax, cast
  of the probabilities back to the KV dtype, and the PV product;
* `BlockManager.allocate/incref/decref/copy_block` and
  `PagedKVCache.ensure_writable_tail` (block_manager.py:47-71, 99-109) for the
  copy-on-write fork of config 2;
* the reference's own unit scenarios from tests/test_block_manager.py:37-83.

Inputs come from tests/golden/cases.py (seeded numpy), so only digests of the
inputs and the reference's outputs are written here.  Nothing in the tests
imports the reference; the fixtures are the only thing that travels.
"""

from __future__ import annotations

import json
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases as C  # noqa: E402

REF_ROOT = os.environ.get("REF_ROOT", "/root/reference")
sys.path.insert(0, REF_ROOT)
from mini_engine.model.config import Qwen2Config  # noqa: E402
from mini_engine.model.qwen2 import Qwen2Model  # noqa: E402
from mini_engine.paged.block_manager import BlockManager, PagedKVCache  # noqa: E402

TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def t_of(a: np.ndarray, dt: str) -> torch.Tensor:
    if dt == "bf16":
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(np.ascontiguousarray(a))


def np_of(t: torch.Tensor, dt: str) -> np.ndarray:
    t = t.contiguous()
    if dt == "bf16":
        return t.view(torch.int16).numpy().view(np.uint16).copy()
    return t.numpy().copy()


def ref_model(dt: str) -> Qwen2Model:
    # _attention reads only the config and the scale; one tiny weight fixes dtype/device.
    return Qwen2Model(Qwen2Config(), {"model.embed_tokens.weight": torch.zeros(1, 896, dtype=TORCH_DT[dt])})


def ref_decode(c) -> np.ndarray:
    dt = c["dt"]
    mgr = BlockManager(c["num_blocks"], C.BS, 1, C.HKV, C.D, dtype=TORCH_DT[dt])
    mgr.k_pool[0].copy_(t_of(c["k_pool"], dt))
    mgr.v_pool[0].copy_(t_of(c["v_pool"], dt))
    kv = PagedKVCache(mgr)
    model = ref_model(dt)
    q, kn, vn = t_of(c["q"], dt), t_of(c["k_new"], dt), t_of(c["v_new"], dt)
    outs = []
    for s, table in enumerate(c["tables"]):
        kv.add_sequence(s, list(table), int(c["ctx"][s]) - 1)
        k_all, v_all, prior = kv.append_and_fetch(0, s, kn[s:s + 1], vn[s:s + 1])
        outs.append(model._attention(q[s:s + 1], k_all, v_all, prior).view(1, C.HQ, C.D))
    return np_of(torch.cat(outs), dt)


def ref_prefill(c, rows_per_seq: int | None = None):
    dt = c["dt"]
    mgr = BlockManager(c["num_blocks"], C.BS, 1, C.HKV, C.D, dtype=TORCH_DT[dt])
    mgr.k_pool[0].copy_(t_of(c["k_pool"], dt))
    mgr.v_pool[0].copy_(t_of(c["v_pool"], dt))
    kv = PagedKVCache(mgr)
    model = ref_model(dt)
    q, kn, vn = t_of(c["q"], dt), t_of(c["k_new"], dt), t_of(c["v_new"], dt)
    outs, rows = [], []
    for s, table in enumerate(c["tables"]):
        a, b = int(c["qsl"][s]), int(c["qsl"][s + 1])
        kv.add_sequence(s, list(table), int(c["prior"][s]))
        k_all, v_all, prior = kv.append_and_fetch(0, s, kn[a:b], vn[a:b])
        o = model._attention(q[a:b], k_all, v_all, prior).view(b - a, C.HQ, C.D)
        if rows_per_seq is not None:
            n = b - a
            pick = np.unique(np.concatenate([[0, n - 1], np.linspace(0, n - 1, rows_per_seq).round()]))
            pick = pick.astype(np.int64)
            o = o[torch.from_numpy(pick)]
            rows.append(pick + a)
        outs.append(o)
    out = np_of(torch.cat(outs), dt)
    return out, (np.concatenate(rows) if rows else None)


def ref_block_manager_scenarios() -> dict:
    """The reference's own unit scenarios (tests/test_block_manager.py:37-83),
    recorded as data so the product's BlockManager/PagedKVCache can replay them."""
    mgr = BlockManager(num_blocks=8, block_size=4, num_layers=2, num_kv_heads=1, head_dim=2)
    kv = PagedKVCache(mgr)
    table = [mgr.allocate() for _ in range(3)]
    kv.add_sequence(0, table, num_cached_tokens=0)
    k1 = torch.arange(10, dtype=torch.float32).reshape(5, 1, 2)
    r1 = [kv.append_and_fetch(layer, 0, k1, k1 * 10) for layer in range(2)]
    k2 = torch.arange(100, 106, dtype=torch.float32).reshape(3, 1, 2)
    r2 = [kv.append_and_fetch(layer, 0, k2, k2 * 10) for layer in range(2)]
    roundtrip = dict(
        table=table,
        step1=[dict(k=r[0].tolist(), v=r[1].tolist(), prior=r[2]) for r in r1],
        step2=[dict(k=r[0].tolist(), v=r[1].tolist(), prior=r[2]) for r in r2],
        seq_len=kv.seq_len(0),
        free_list=list(mgr.free_list),
    )

    mgr = BlockManager(num_blocks=8, block_size=4, num_layers=2, num_kv_heads=1, head_dim=2)
    kv = PagedKVCache(mgr)
    table = [mgr.allocate()]
    kv.add_sequence(0, table, 0)
    k = torch.ones(2, 1, 2)
    for layer in range(2):
        kv.append_and_fetch(layer, 0, k, k)
    for b in table:
        mgr.incref(b)
    kv.add_sequence(1, list(table), 2)
    kv.ensure_writable_tail(1)
    tables_after_cow = {str(s): list(t) for s, t in kv.block_tables.items()}
    k_new = torch.full((1, 1, 2), 7.0)
    for layer in range(2):
        kv.append_and_fetch(layer, 1, k_new, k_new)
    k0, _, _ = kv.append_and_fetch(0, 0, torch.zeros(0, 1, 2), torch.zeros(0, 1, 2))
    k1r, _, _ = kv.append_and_fetch(0, 1, torch.zeros(0, 1, 2), torch.zeros(0, 1, 2))
    cow = dict(
        tables_after_cow=tables_after_cow,
        ref_count=list(mgr.ref_count),
        free_list=list(mgr.free_list),
        k_seq0=k0.tolist(),
        k_seq1=k1r.tolist(),
        k_pool=[p.tolist() for p in mgr.k_pool],
        v_pool=[p.tolist() for p in mgr.v_pool],
    )
    return dict(roundtrip=roundtrip, cow=cow)


def ref_append_cow(c) -> dict:
    """Config 2 through the reference: append one token per sequence per
    layer, then fork sequences with a partial tail and let
    ensure_writable_tail copy it."""
    dt, L = c["dt"], c["n_layers"]
    mgr = BlockManager(c["num_blocks"], C.BS, L, C.HKV, C.D, dtype=TORCH_DT[dt])
    for layer in range(L):
        mgr.k_pool[layer].copy_(t_of(c["k_pools"][layer], dt))
        mgr.v_pool[layer].copy_(t_of(c["v_pools"][layer], dt))
    mgr.free_list = list(c["free_list"])
    kv = PagedKVCache(mgr)
    n = len(c["ctx"])
    tables = []
    for s in range(n):
        ctx = int(c["ctx"][s])
        table = [mgr.allocate() for _ in range((ctx + C.BS - 1) // C.BS)]
        tables.append(list(table))
        kv.add_sequence(s, table, ctx - 1)
    kn, vn = t_of(c["k_new"], dt), t_of(c["v_new"], dt)
    for s in range(n):
        for layer in range(L):
            kv.append_and_fetch(layer, s, kn[layer, s:s + 1], vn[layer, s:s + 1])
    after_append = C.digest(*[np_of(p, dt) for p in mgr.k_pool], *[np_of(p, dt) for p in mgr.v_pool])
    pairs = []
    for i, s in enumerate(c["forked"]):
        s = int(s)
        child = n + i
        for b in kv.block_tables[s]:
            mgr.incref(b)
        kv.add_sequence(child, list(kv.block_tables[s]), kv.seq_len(s))
        before = list(kv.block_tables[child])
        kv.ensure_writable_tail(child)
        after = kv.block_tables[child]
        diff = [(x, y) for x, y in zip(before, after) if x != y]
        assert len(diff) == 1
        pairs.append(list(diff[0]))
    after_cow = C.digest(*[np_of(p, dt) for p in mgr.k_pool], *[np_of(p, dt) for p in mgr.v_pool])
    return dict(
        input_sha256=C.append_cow_digest(c),
        tables=tables,
        pairs=pairs,
        child_tables={str(k): list(v) for k, v in kv.block_tables.items() if k >= n},
        ref_count=list(mgr.ref_count),
        free_list=list(mgr.free_list),
        pools_after_append_sha256=after_append,
        pools_after_cow_sha256=after_cow,
    )


def save_npz(name, **arrays):
    np.savez_compressed(os.path.join(HERE, name), **arrays)
    print(f"wrote {name}: {os.path.getsize(os.path.join(HERE, name)) / 1024:.1f} KiB")


def main():
    torch.set_num_threads(max(1, len(os.sched_getaffinity(0))))
    t0 = time.time()

    with open(os.path.join(HERE, "block_manager_ref.json"), "w") as f:
        json.dump(ref_block_manager_scenarios(), f)
    print("wrote block_manager_ref.json")

    for dt in ("f32", "f16", "bf16"):
        c = C.make_decode_case(1, 8, 32, 600, 512, dt)  # config 1 shape
        save_npz(f"decode_c1_{dt}.npz", out=ref_decode(c), input_sha256=C.decode_digest(c))
        c = C.make_decode_case(11, 9, 0, 0, 128, dt, ctx_list=[1, 2, 15, 16, 17, 31, 32, 33, 600])
        save_npz(f"decode_edge_{dt}.npz", out=ref_decode(c), input_sha256=C.decode_digest(c))
        c = C.make_prefill_case(21, [1, 7, 33, 64, 16], [0, 5, 37, 100, 11], 48, 256, dt)
        out, _ = ref_prefill(c)
        save_npz(f"prefill_small_{dt}.npz", out=out, input_sha256=C.prefill_digest(c))
        c = C.make_prefill_case(22, [20, 3, 48], [0, 16, 1], 0, 64, dt)  # no shared prefix
        out, _ = ref_prefill(c)
        save_npz(f"prefill_noshare_{dt}.npz", out=out, input_sha256=C.prefill_digest(c))

    # config 3 (full size, one layer): B=256, lognormal median 1024, sigma 0.5
    c = C.make_decode_case(3, 256, 16, 8192, 0, "f16", lognormal_median=1024.0, pool_slack=1.1)
    save_npz("decode_c3_f16.npz", out=ref_decode(c), input_sha256=C.decode_digest(c),
             sum_ctx=np.int64(c["ctx"].sum()))

    # config 4 (full size, one layer), outputs kept for a sample of query rows
    c = C.make_c4_case()
    out, rows = ref_prefill(c, rows_per_seq=8)
    save_npz("prefill_c4_f16_rows.npz", out=out, rows=rows, input_sha256=C.prefill_digest(c))

    c = C.make_append_cow_case()
    with open(os.path.join(HERE, "append_cow_c2_f16.json"), "w") as f:
        json.dump(ref_append_cow(c), f)
    print("wrote append_cow_c2_f16.json")
    print(f"done in {time.time() - t0:.1f} s")


if __name__ == "__main__":
    main()
