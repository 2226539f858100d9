"""Expert-parallel groups of GpuBatch objects: one process per GPU, the MoE experts partitioned over the ranks.

The data path is the library's own: every rank maps every other rank's exchange region (CUDA IPC) and its kernels
push MoE rows and results through peer memory.  torch.distributed only carries the 64-byte region handles here (any
backend: gloo on CPU hosts, NCCL on GPU nodes) and the barriers around the timed region.
"""
from __future__ import annotations

from .configs import shard


def sequences(total: int, rank: int, world: int) -> range:
    """Global ids of the sequences rank `rank` decodes (contiguous, rank-major): attention is data-parallel."""
    return shard(total, rank, world)


def experts(n_experts: int, rank: int, world: int) -> range:
    """Experts rank `rank` computes for every rank's tokens (contiguous, n_experts / world each)."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    return shard(n_experts, rank, world)


def contiguous_placement(n_experts: int, world: int) -> list:
    """owner[e] with experts in contiguous blocks of n_experts / world (the batch's default placement)."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    return [e // (n_experts // world) for e in range(n_experts)]


def interleaved_placement(n_experts: int, world: int) -> list:
    """owner[e] = e mod world: neighbouring expert ids on different ranks."""
    if n_experts % world:
        raise ValueError(f"{n_experts} experts do not split over {world} ranks")
    return [e % world for e in range(n_experts)]


def balanced_placement(loads, world: int) -> list:
    """owner[e] that evens out the ranks' summed `loads` (e.g. the pairs routed to each expert over earlier steps)
    with n_experts / world experts per rank: experts in decreasing load (lower id first on ties), each to the rank
    with the least load so far among those with room left (lower rank first on ties)."""
    loads = [float(x) for x in loads]
    n = len(loads)
    if n % world:
        raise ValueError(f"{n} experts do not split over {world} ranks")
    per = n // world
    owner = [0] * n
    total = [0.0] * world
    count = [0] * world
    for e in sorted(range(n), key=lambda i: (-loads[i], i)):
        r = min((q for q in range(world) if count[q] < per), key=lambda q: (total[q], q))
        owner[e] = r
        total[r] += loads[e]
        count[r] += 1
    return owner


def owned(owner, rank: int) -> list:
    """Experts of `rank` under the placement owner[e], ascending (the order of its grouped GEMMs)."""
    return [e for e, r in enumerate(owner) if r == rank]


def connect_group(batch, group=None):
    """All-gathers the exchange-region handle of every rank's batch, in rank order, and connects this rank's batch to
    all of them.  Every rank of the group must call it (it is a collective)."""
    import torch.distributed as dist

    if batch.world == 1:
        batch.connect()
        return
    handles = [None] * batch.world
    dist.all_gather_object(handles, batch.exchange_handle(), group=group)
    batch.connect(handles)
