"""Host side of the expert-parallel batched decode on CPU: the partition of sequences and experts over ranks and the
exchange of region handles among world_size 2 gloo processes (the GPU data path is tested in test_gpu_ep.py)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from lastro_b200 import ep
from lastro_b200 import configs as CFG


def test_partitions_cover_everything_once():
    for total in (1, 7, 64, 65):
        for world in (1, 2, 4, 8):
            got = [list(ep.sequences(total, r, world)) for r in range(world)]
            assert sum(got, []) == list(range(total))
            assert max(map(len, got)) - min(map(len, got)) <= 1
    for world in (1, 2, 4, 8):
        got = [list(ep.experts(40, r, world)) for r in range(world)]
        assert sum(got, []) == list(range(40)) and all(len(g) == 40 // world for g in got)
    with pytest.raises(ValueError):
        ep.experts(40, 0, 3)


def test_expert_placements():
    for world in (1, 2, 4, 8):
        assert ep.contiguous_placement(40, world) == [e // (40 // world) for e in range(40)]
        assert [ep.owned(ep.contiguous_placement(40, world), r) for r in range(world)] == \
            [list(ep.experts(40, r, world)) for r in range(world)]
        assert ep.interleaved_placement(40, world) == [e % world for e in range(40)]
    with pytest.raises(ValueError):
        ep.interleaved_placement(40, 3)
    # balanced: E/world experts per rank, the heaviest loads spread, deterministic on ties
    zipf = [(e + 1) ** -0.8 for e in range(40)]
    for world in (2, 4, 8):
        owner = ep.balanced_placement(zipf, world)
        per = [ep.owned(owner, r) for r in range(world)]
        assert sorted(sum(per, [])) == list(range(40)) and all(len(p) == 40 // world for p in per)
        sums = [sum(zipf[e] for e in p) for p in per]
        cont = [sum(zipf[e] for e in ep.owned(ep.contiguous_placement(40, world), r)) for r in range(world)]
        assert max(sums) - min(sums) < 0.25 * (max(cont) - min(cont)) and max(sums) < max(cont)
        assert owner[:world] == list(range(world))  # the world heaviest experts on distinct ranks, in rank order
    assert ep.balanced_placement([1.0] * 8, 2) == [0, 1, 0, 1, 0, 1, 0, 1]
    with pytest.raises(ValueError):
        ep.balanced_placement([1.0] * 7, 2)


class FakeBatch:
    """Stands in for GpuBatch: a handle that names the rank, and a record of what connect() received."""

    def __init__(self, rank, world):
        self.rank, self.world, self.got = rank, world, None

    def exchange_handle(self):
        return bytes([self.rank]) * 64

    def connect(self, handles=None):
        self.got = handles


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    b = FakeBatch(rank, world)
    ep.connect_group(b)
    out.put((rank, [h[0] for h in b.got], len(b.got[0])))
    dist.barrier()
    dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_connect_group_gathers_handles_in_rank_order_over_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    world, port = 2, _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, order, size in res:
        assert order == [0, 1] and size == 64


def test_world_one_connects_without_a_process_group():
    b = FakeBatch(0, 1)
    ep.connect_group(b)
    assert b.got is None
    assert list(ep.sequences(CFG.C5_BATCH["batch"], 0, 1)) == list(range(64))
