"""Synthetic workloads of the BASELINE configurations and their per-GPU
sharding (host-side helpers used by bench.py and the multi-rank tests).

Work is partitioned by sequence: every GPU owns an independent block pool and
a disjoint set of sequences, so no collective touches the data path.  The
only cross-rank operations are a barrier and a max-reduction of timings.
"""

from __future__ import annotations

import numpy as np

BLOCK_SIZE = 16
N_Q_HEADS, N_KV_HEADS, HEAD_DIM, N_LAYERS = 14, 2, 64, 24  # Qwen2.5-0.5B (config.py:13-23)


def config3_contexts(n_seqs: int, seed: int = 3, median: float = 1024.0, sigma: float = 0.5,
                     lo: int = 16, hi: int = 8192) -> np.ndarray:
    """Config 3 context lengths: clip(round(exp(N(ln median, sigma^2))), lo, hi).

    The first draw of the seeded PCG64 stream, so the first 256 values are
    the same for any n_seqs >= 256.
    """
    rng = np.random.default_rng(seed)
    z = rng.standard_normal(n_seqs)
    return np.clip(np.round(np.exp(np.log(median) + sigma * z)), lo, hi).astype(np.int64)


def deal(n_total: int, rank: int, world: int) -> np.ndarray:
    """Round-robin dealing of sequence indices to ranks (sequence -> GPU)."""
    return np.arange(rank, n_total, world, dtype=np.int64)


def shard_contexts(per_gpu_batch: int, rank: int, world: int, strong: bool = False,
                   seed: int = 3) -> np.ndarray:
    """Contexts of this rank's sequences.

    weak (default): the job is per_gpu_batch * world sequences, each GPU gets
    per_gpu_batch of them (per-GPU work fixed as N grows; N=1 is config 3).
    strong: the job is per_gpu_batch sequences dealt over the world.
    """
    total = per_gpu_batch if strong else per_gpu_batch * world
    ctx = config3_contexts(total, seed=seed)
    return ctx[deal(total, rank, world)]


def decode_bytes(ctx: np.ndarray, n_q_heads: int = N_Q_HEADS, n_kv_heads: int = N_KV_HEADS,
                 head_dim: int = HEAD_DIM, esize: int = 2, block_size: int = BLOCK_SIZE) -> int:
    """Algorithmic bytes of one paged-decode launch: every context token's K
    and V rows once, q read + out written once, the used block-table entries
    and the context lengths.  Split-K partials are not counted."""
    ctx = np.asarray(ctx, dtype=np.int64)
    kv = int(ctx.sum()) * n_kv_heads * head_dim * 2 * esize
    qo = len(ctx) * n_q_heads * head_dim * esize * 2
    tables = int(((ctx + block_size - 1) // block_size).sum()) * 4
    return kv + qo + tables + len(ctx) * 4


def append_bytes(n_tokens: int, n_kv_heads: int = N_KV_HEADS, head_dim: int = HEAD_DIM,
                 esize: int = 2) -> int:
    """Algorithmic bytes of one reshape_and_cache launch: K and V rows read and
    written once, plus the int64 slot of each token."""
    return n_tokens * (n_kv_heads * head_dim * esize * 2 * 2 + 8)


def make_tables(ctx: np.ndarray, num_blocks: int, seed: int, block_size: int = BLOCK_SIZE):
    """Scattered, disjoint block tables: consecutive slices of a seeded
    permutation of the pool (config 3: "block tables scattered randomly")."""
    rng = np.random.default_rng(seed)
    nblk = (np.asarray(ctx) + block_size - 1) // block_size
    perm = rng.permutation(num_blocks).astype(np.int32)
    width = int(nblk.max()) if len(nblk) else 1
    tab = np.zeros((len(ctx), max(1, width)), dtype=np.int32)
    o = 0
    for i, n in enumerate(nblk):
        tab[i, :n] = perm[o:o + n]
        o += n
    return tab


def max_over_ranks(value: float, group=None) -> float:
    """Max of a float over all ranks of the default process group (identity
    when torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def sum_over_ranks(value: float, group=None) -> float:
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return float(t.item())


def gather_over_ranks(value: float, group=None) -> list[float]:
    """[value of rank 0, value of rank 1, ...] over the default process group
    ([value] when torch.distributed is not initialised)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return [float(value)]
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    out = [torch.empty_like(t) for _ in range(dist.get_world_size(group))]
    dist.all_gather(out, t, group=group)
    return [float(x.item()) for x in out]


def rank_cpus(cpus, local_rank: int, local_world: int) -> list[int]:
    """This rank's share of the host cores: the sorted core list cut into
    local_world contiguous, disjoint slices (the last ones one core shorter
    when the count does not divide), so that the ranks of one node do not
    contend for the same cores when they enqueue work.  Every rank gets at
    least one core; with fewer cores than ranks, ranks share them round-robin."""
    cpus = sorted(int(c) for c in cpus)
    if not cpus:
        return []
    if local_world <= 1:
        return cpus
    if len(cpus) < local_world:
        return [cpus[local_rank % len(cpus)]]
    base, extra = divmod(len(cpus), local_world)
    start = local_rank * base + min(local_rank, extra)
    return cpus[start:start + base + (1 if local_rank < extra else 0)]


def local_cpu_share(allowed, gpu_cpus, local_rank: int) -> list[int]:
    """This rank's host cores, near its GPU: the allowed cores that the driver
    reports as local to the rank's GPU (gpu_cpus[r]: the cores of local rank
    r's GPU, or None), split disjointly (rank_cpus) among the local ranks
    whose GPUs report the same allowed set.  Pinned host buffers that the
    rank allocates afterwards then sit in its GPU's NUMA node.  A rank whose
    GPU reports no allowed core gets its rank_cpus share of all allowed
    cores."""
    allowed = sorted(set(int(c) for c in allowed))
    local = [sorted(set(s or ()) & set(allowed)) for s in gpu_cpus]
    mine = local[local_rank]
    if not mine:
        return rank_cpus(allowed, local_rank, len(gpu_cpus))
    peers = [r for r, s in enumerate(local) if s == mine]
    return rank_cpus(mine, peers.index(local_rank), len(peers))


def config4_layout(seed: int = 4, n_seqs: int = 16, chunk: int = 512, prior_hi: int = 4096,
                   shared: int = 48):
    """Config 4: n_seqs chunks of `chunk` queries over a `shared`-token radix
    prefix (same physical blocks in every table) plus a private prior ~ U[0, prior_hi]."""
    rng = np.random.default_rng(seed + 1000)
    priv = rng.integers(0, prior_hi + 1, size=n_seqs).astype(np.int64)
    prior = shared + priv
    return prior, np.full(n_seqs, chunk, dtype=np.int64)


def prefill_flops(prior: np.ndarray, chunk: np.ndarray, n_q_heads: int = N_Q_HEADS,
                  head_dim: int = HEAD_DIM) -> int:
    """Algorithmic FLOPs of one chunked-prefill launch: QK^T and PV over the
    visible (query, key) pairs only, 2 * 2 * head_dim per pair and head.
    Query i of a chunk sees prior + i + 1 keys."""
    pairs = sum(int(c) * int(p) + int(c) * (int(c) + 1) // 2 for p, c in zip(prior, chunk))
    return 4 * head_dim * n_q_heads * pairs


def prefill_tables(prior: np.ndarray, chunk: np.ndarray, shared: int, num_blocks: int, seed: int,
                   block_size: int = BLOCK_SIZE):
    """Tables whose first shared // 16 blocks are common to all sequences
    (a radix-cache hit) followed by private blocks from a seeded permutation."""
    rng = np.random.default_rng(seed)
    n_shared = shared // block_size
    perm = rng.permutation(num_blocks).astype(np.int32)
    need = (prior + chunk + block_size - 1) // block_size
    tab = np.zeros((len(prior), int(need.max())), dtype=np.int32)
    o = n_shared
    for i, n in enumerate(need):
        tab[i, :n_shared] = perm[:n_shared]
        tab[i, n_shared:n] = perm[o:o + n - n_shared]
        o += n - n_shared
    return tab
