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
