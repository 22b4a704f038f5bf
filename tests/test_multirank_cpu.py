"""Multi-GPU host logic on CPU: two gloo ranks run what bench.py runs per rank.

The checks:
* the sequences are dealt to the ranks disjointly and completely (weak scaling:
  256 per rank; strong: 256 in total);
* each rank's pool and scattered block tables are private;
* the max-over-ranks timing, the sum-over-ranks bytes and the per-rank lists
  (gather over ranks) are right;
* each rank's share of the host cores (the bench pins a rank to it) is
  disjoint from the others' and together they cover the node's cores.

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
        g = W.gather_over_ranks(10.0 * rank + 0.5)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), ctx=ctx, idx=idx, slots=a["slots"],
                 tmax=t, bsum=b, mine=float(W.decode_bytes(ctx)), gathered=np.array(g))
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
        assert x["gathered"].tolist() == [10.0 * k + 0.5 for k in range(world)]
    if not strong:
        assert np.array_equal(r[0]["ctx"][:1], all_ctx[:1])


@pytest.mark.parametrize("n_cpus,world", [(32, 8), (30, 8), (7, 2), (3, 4), (1, 1), (16, 1)])
def test_rank_cpu_shares_are_disjoint_and_cover_the_node(n_cpus, world):
    import sys

    sys.path.insert(0, PKG_ROOT)
    from pagedkv import workloads as W

    cpus = list(range(100, 100 + n_cpus))[::-1]   # any order, any ids
    shares = [W.rank_cpus(cpus, r, world) for r in range(world)]
    assert all(shares), "every rank gets at least one core"
    if n_cpus >= world:
        flat = [c for s in shares for c in s]
        assert sorted(flat) == sorted(cpus)                   # cover, no overlap
        assert max(map(len, shares)) - min(map(len, shares)) <= 1
        for s in shares:                                      # contiguous slices
            assert s == list(range(s[0], s[0] + len(s)))
    else:
        assert all(len(s) == 1 for s in shares)


def test_local_cpu_share_keeps_ranks_near_their_gpu():
    """Two NUMA nodes of 16 cores, four GPUs each: every rank's cores are on
    its GPU's node, the ranks of a node split it disjointly; a GPU reporting
    no allowed core falls back to a share of all allowed cores; a
    restricted affinity is respected."""
    import sys

    sys.path.insert(0, PKG_ROOT)
    from pagedkv import workloads as W

    node0, node1 = list(range(0, 16)), list(range(16, 32))
    gpu_cpus = [node0] * 4 + [node1] * 4
    allowed = list(range(32))
    shares = [W.local_cpu_share(allowed, gpu_cpus, r) for r in range(8)]
    for r, s in enumerate(shares):
        assert s and set(s) <= set(gpu_cpus[r])
    assert sorted(c for s in shares[:4] for c in s) == node0
    assert sorted(c for s in shares[4:] for c in s) == node1
    # one GPU, whole node
    assert W.local_cpu_share(allowed, [node1], 0) == node1
    # the driver reports nothing (or nothing allowed): plain share of the allowed cores
    assert W.local_cpu_share(allowed, [None, None], 1) == W.rank_cpus(allowed, 1, 2)
    assert W.local_cpu_share(list(range(8)), [node1], 0) == list(range(8))
    # affinity restricted to part of a node
    assert W.local_cpu_share(list(range(4, 12)), [node0, node0], 0) == [4, 5, 6, 7]
