"""KV block migration between ranks (pagedkv.migration).

CPU (gloo, two ranks): the host protocol with the device copy replaced by
copies between shared-memory CPU pools, standing in for the IPC mappings.
The fake is test scaffolding: it overrides only the export / open / copy /
sync methods.  The checks:
* push and pull both move the right blocks into freshly allocated ones;
* a destination that cannot allocate raises OutOfBlocks on both ranks and
  keeps nothing;
* a failed copy raises on both ranks and frees the destination's blocks;
* a fresh destination block that a queued copy-on-write pair still reads is
  not handed to the source before that pair is launched (and, in push mode,
  before the destination's stream has drained);
* migrate_sequence registers the sequence on the destination with its
  length and a table of ceil(len / 16) blocks.

GPU (marked gpu): two processes share real pools through CUDA IPC.
* With two GPUs, the ranks sit on cuda:0 and cuda:1 and the copy crosses
  NVLink.
* On one GPU, both processes use cuda:0: the same IPC mapping and kernel, with
  no peer link.
* The copied blocks (fp16 K/V, then fp8 bytes and scales) must equal the
  source's bit for bit, and untouched blocks must stay untouched.
"""

from __future__ import annotations

import os
import socket
import sys

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


def _fake_peer_pools_cls():
    sys.path.insert(0, PKG_ROOT)
    from pagedkv import migration

    class SharedPeerPools(migration.PeerPools):
        """Peer pools are shared-memory CPU tensors; a pool address is its rank."""

        pools: dict = {}
        fail_copy = False

        def _export(self):
            d = dict(self.meta)
            d["handles"] = [self.rank]
            return d

        def _local_ref(self):
            return self._ref_from([self.rank] * 4, self.mgr.num_blocks)

        def _open(self, meta):
            return self._ref_from([meta["handles"][0]] * 4, meta["num_blocks"])

        def close(self):
            dist.barrier(group=self.host_group)

        def _sync(self):
            self.syncs = getattr(self, "syncs", 0) + 1

        def _send(self, values, peer):
            # the destination's reply with fresh ids: record what was still
            # queued and whether its stream had been drained
            if self.rank == 1 and len(values) > 1 and values[0] == 0:
                self.replies = getattr(self, "replies", []) + [
                    (len(self.mgr.pending_copies), getattr(self, "syncs", 0))]
            super()._send(values, peer)

        def _launch_copy(self, dst, src, pairs):
            if self.fail_copy:
                raise RuntimeError("injected copy failure")
            sp, dp = self.pools[src.k], self.pools[dst.k]
            for s, d in pairs:
                for a, b in zip(sp, dp):
                    b[:, d] = a[:, s]

    return SharedPeerPools


def _cpu_rank(rank, world, port, pools, out_dir):
    sys.path.insert(0, PKG_ROOT)
    from pagedkv import BlockManager, PagedKVCache
    from pagedkv.block_manager import OutOfBlocks
    from pagedkv.migration import migrate_blocks, migrate_sequence

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    res = {}
    try:
        Fake = _fake_peer_pools_cls()
        Fake.pools = pools
        nb = pools[rank][0].shape[1]
        mgr = BlockManager(nb, 16, 2, 2, 64, device=None)
        for b in range(nb):          # the source's blocks are all in use
            if rank == 0:
                mgr.allocate()
        for mode in ("push", "pull"):
            peers = Fake(mgr, mode=mode)
            src_blocks = [5, 2, 7] if mode == "push" else [1, 6]
            ids = migrate_blocks(peers, 0, 1, src_blocks if rank == 0 else None)
            res[f"{mode}_ids"] = np.array(ids)
            res[f"{mode}_src"] = np.array(src_blocks)
            peers.close()
        peers = Fake(mgr)
        # destination too small: 7 free blocks left on rank 1, ask for 8
        free_before = mgr.num_free
        try:
            migrate_blocks(peers, 0, 1, list(range(8)) if rank == 0 else None)
            res["oob"] = np.array(0)
        except OutOfBlocks:
            res["oob"] = np.array(1)
        res["free_kept"] = np.array(int(mgr.num_free == free_before))
        # a failed copy on the launching side (push: the source; pull: the
        # destination): both ranks raise, the destination keeps nothing
        Fake.fail_copy = True
        for mode in ("push", "pull"):
            fpeers = Fake(mgr, mode=mode)
            free_before = mgr.num_free
            try:
                migrate_blocks(fpeers, 0, 1, [3] if rank == 0 else None)
                res[f"fail_{mode}"] = np.array(0)
            except RuntimeError:
                res[f"fail_{mode}"] = np.array(1)
            res[f"fail_freed_{mode}"] = np.array(int(mgr.num_free == free_before))
            fpeers.close()
        Fake.fail_copy = False
        # the destination recycles a block that a queued copy-on-write pair
        # still reads: the pair must be launched (and, for push, the stream
        # drained) before the fresh ids reach the source
        for mode in ("push", "pull"):
            rpeers = Fake(mgr, mode=mode)
            if rank == 1:
                a = mgr.allocate()
                mgr.incref(a)
                d = mgr.copy_block(a)   # queued (a, d)
                mgr.decref(a)
                mgr.decref(a)           # a is free again, first in the LIFO list
            ids = migrate_blocks(rpeers, 0, 1, [2] if rank == 0 else None)
            if rank == 1:
                pend, syncs = rpeers.replies[-1]
                res[f"recycled_{mode}"] = np.array([int(ids[0] == a), pend, int(syncs > 0)])
                res[f"recycled_ids_{mode}"] = np.array(ids)
                mgr.decref(d)
                mgr.decref(ids[0])
            rpeers.close()
        # a whole sequence: 37 tokens in a 4-block table -> 3 blocks move
        cache = PagedKVCache(mgr)
        if rank == 0:
            cache.add_sequence(42, [9, 4, 8, 0], 37)
        length, table = migrate_sequence(peers, cache, 42, 0, 1)
        res["seq_len"] = np.array(length)
        res["seq_table"] = np.array(table)
        if rank == 1:
            res["seq_registered"] = np.array(
                [cache.seq_len(42), int(cache.block_tables[42] == table)])
        peers.close()
    finally:
        dist.destroy_process_group()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), **res)


def test_migration_protocol_two_gloo_ranks(tmp_path):
    nb0, nb1 = 10, 12
    g = torch.Generator().manual_seed(0)
    pools = {}
    for r, nb in ((0, nb0), (1, nb1)):
        pools[r] = [torch.randn((2, nb, 16, 2, 64), generator=g).half().share_memory_()
                    for _ in range(2)]
    before = {r: [p.clone() for p in pools[r]] for r in pools}
    mp.spawn(_cpu_rank, args=(2, _free_port(), pools, str(tmp_path)), nprocs=2, join=True)
    r0, r1 = (np.load(tmp_path / f"r{k}.npz") for k in range(2))
    # LIFO allocator on rank 1: fresh blocks 0, 1, 2 then 3, 4
    assert r1["push_ids"].tolist() == [0, 1, 2] == r0["push_ids"].tolist()
    assert r1["pull_ids"].tolist() == [3, 4] == r0["pull_ids"].tolist()
    for mode in ("push", "pull"):
        for s, d in zip(r0[f"{mode}_src"], r1[f"{mode}_ids"]):
            for a, b in zip(before[0], pools[1]):
                assert torch.equal(a[:, s], b[:, d]), (mode, s, d)
    touched = set(r1["push_ids"].tolist()) | set(r1["pull_ids"].tolist()) | set(r1["seq_table"].tolist())
    touched |= set(r1["recycled_ids_push"].tolist()) | set(r1["recycled_ids_pull"].tolist())
    for d in range(nb1):
        if d not in touched:
            for a, b in zip(before[1], pools[1]):
                assert torch.equal(a[:, d], b[:, d]), d
    assert r0["oob"] == 1 and r1["oob"] == 1 and r1["free_kept"] == 1
    # recycled block: nothing queued at the reply; push drained the stream
    assert r1["recycled_push"].tolist() == [1, 0, 1]
    assert r1["recycled_pull"].tolist()[:2] == [1, 0]
    for mode in ("push", "pull"):
        assert r0[f"fail_{mode}"] == 1 and r1[f"fail_{mode}"] == 1, mode
        assert r1[f"fail_freed_{mode}"] == 1, mode
    assert r0["seq_len"] == r1["seq_len"] == 37
    assert len(r1["seq_table"]) == 3 and r0["seq_table"].tolist() == r1["seq_table"].tolist()
    assert r1["seq_registered"].tolist() == [37, 1]
    for s, d in zip([9, 4, 8], r1["seq_table"]):
        for a, b in zip(before[0], pools[1]):
            assert torch.equal(a[:, s], b[:, d])


# ---------------------------------------------------------------- GPU (IPC)

def _gpu_rank(rank, world, port, n_dev, out_dir):
    sys.path.insert(0, PKG_ROOT)
    from pagedkv import BlockManager, ops
    from pagedkv.migration import PeerPools, migrate_blocks

    dev = torch.device("cuda", rank % n_dev)
    torch.cuda.set_device(dev)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    res = {}
    try:
        for kind in ("f16", "fp8"):
            nb = 40 + 8 * rank
            dt = torch.float16 if kind == "f16" else torch.float8_e4m3fn
            mgr = BlockManager(nb, 16, 3, 2, 64, device=dev, dtype=dt)
            g = torch.Generator(device=dev).manual_seed(100 + rank)
            if kind == "f16":
                mgr.k_cache.normal_(generator=g)
                mgr.v_cache.normal_(generator=g)
            else:
                mgr.k_cache.random_(0, 256, generator=g)
                mgr.v_cache.random_(0, 256, generator=g)
                mgr.k_scale_cache.uniform_(0.5, 2.0, generator=g)
                mgr.v_scale_cache.uniform_(0.5, 2.0, generator=g)
            if rank == 0:
                for _ in range(nb):
                    mgr.allocate()
            pools = [mgr.k_cache, mgr.v_cache] + ([mgr.k_scale_cache, mgr.v_scale_cache]
                                                  if kind == "fp8" else [])
            before = [p.cpu() for p in pools]
            ids = {}
            for mode, src_blocks in (("push", [3, 17, 30, 11]), ("pull", [0, 39, 25])):
                peers = PeerPools(mgr, mode=mode)
                ids[mode] = migrate_blocks(peers, 0, 1, src_blocks if rank == 0 else None)
                peers.close()
            torch.cuda.synchronize()
            after = [p.cpu() for p in pools]
            for i, (b, a) in enumerate(zip(before, after)):
                np.save(os.path.join(out_dir, f"{kind}_r{rank}_p{i}_before.npy"),
                        b.view(torch.uint8).numpy())
                np.save(os.path.join(out_dir, f"{kind}_r{rank}_p{i}_after.npy"),
                        a.view(torch.uint8).numpy())
            res[f"{kind}_push"] = np.array(ids["push"])
            res[f"{kind}_pull"] = np.array(ids["pull"])
            ops.check_flags(mgr.err, "migration")
    finally:
        dist.destroy_process_group()
    np.savez(os.path.join(out_dir, f"r{rank}.npz"), **res)


@pytest.mark.gpu
def test_migration_ipc_bit_exact(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    n_dev = min(2, torch.cuda.device_count())
    mp.spawn(_gpu_rank, args=(2, _free_port(), n_dev, str(tmp_path)), nprocs=2, join=True)
    r1 = np.load(tmp_path / "r1.npz")
    src = {"push": [3, 17, 30, 11], "pull": [0, 39, 25]}
    for kind, n_pools in (("f16", 2), ("fp8", 4)):
        moved = {}
        for mode in ("push", "pull"):
            for s, d in zip(src[mode], r1[f"{kind}_{mode}"].tolist()):
                moved[d] = s
        for i in range(n_pools):
            s_before = np.load(tmp_path / f"{kind}_r0_p{i}_before.npy")
            s_after = np.load(tmp_path / f"{kind}_r0_p{i}_after.npy")
            d_before = np.load(tmp_path / f"{kind}_r1_p{i}_before.npy")
            d_after = np.load(tmp_path / f"{kind}_r1_p{i}_after.npy")
            assert np.array_equal(s_before, s_after), "the source pool changed"
            for d in range(d_after.shape[1]):
                want = s_before[:, moved[d]] if d in moved else d_before[:, d]
                assert np.array_equal(d_after[:, d], want), (kind, i, d)
