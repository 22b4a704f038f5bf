"""Multi-GPU host logic on CPU: two gloo ranks run what bench.py runs per rank.

The checks:
* the sequences are dealt to the ranks disjointly and completely (weak scaling:
  256 per rank; strong: 256 in total);
* each rank's pool and scattered block tables are private;
* the max-over-ranks timing and the sum-over-ranks bytes are right.

No collective touches the data path, so the gloo process group carries only
these scalars.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_ROOT


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out_dir, strong):
    import sys

    sys.path.insert(0, PKG_ROOT)
    from pagedkv import BlockManager, PagedKVCache
    from pagedkv import workloads as W

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ctx = W.shard_contexts(256, rank, world, strong=strong)
        idx = W.deal(256 if strong else 256 * world, rank, world)
        nb = int(np.ceil(1.1 * ((ctx + 15) // 16).sum()))
        tabs = W.make_tables(ctx, nb, seed=100 + rank)
        mgr = BlockManager(nb, 16, 24, 2, 64, device=None)
        kv = PagedKVCache(mgr)
        for i, c in enumerate(ctx):
            n = (int(c) + 15) // 16
            kv.add_sequence(i, tabs[i, :n].tolist(), int(c) - 1)
        a = kv.step_arrays([(i, 1) for i in range(len(ctx))])
        t = W.max_over_ranks(1.0 + rank)               # rank-dependent "time"
        b = W.sum_over_ranks(float(W.decode_bytes(ctx)))
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), ctx=ctx, idx=idx, slots=a["slots"],
                 tmax=t, bsum=b, mine=float(W.decode_bytes(ctx)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("strong", [False, True])
def test_two_gloo_ranks_shard_by_sequence(tmp_path, strong):
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), str(tmp_path), strong), nprocs=world,
             join=True)
    r = [np.load(tmp_path / f"r{k}.npz") for k in range(world)]
    import sys

    sys.path.insert(0, PKG_ROOT)
    from pagedkv import workloads as W

    total = 256 if strong else 256 * world
    all_ctx = W.config3_contexts(total)
    idx = np.concatenate([x["idx"] for x in r])
    assert sorted(idx.tolist()) == list(range(total))           # disjoint and complete
    for x in r:
        assert np.array_equal(x["ctx"], all_ctx[x["idx"]])
        assert float(x["tmax"]) == world                         # max over ranks
        assert float(x["bsum"]) == sum(float(y["mine"]) for y in r)
        assert len(set(x["slots"].tolist())) == len(x["slots"])  # private slots per rank
    if not strong:
        assert np.array_equal(r[0]["ctx"][:1], all_ctx[:1])
