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


def _placement(kind, n_experts, world):
    if kind == "contiguous":
        return ep.contiguous_placement(n_experts, world)
    if kind == "interleaved":
        return ep.interleaved_placement(n_experts, world)
    import numpy as np
    owner = ep.balanced_placement([(e + 1) ** -0.8 for e in range(n_experts)], world)
    return [int(x) for x in np.random.default_rng(5).permutation(owner)]


EP_SEQS, EP_STEPS = 5, 4


def _ep_tokens(g, step, vocab):
    return (7 * g + 3 * step + 1) % vocab


def _ep_worker(rank, world, port, out, cfg_name, kind):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import oracle as O
    from ep_oracle import EPRank
    from helpers import reference_tiny_weights

    def gather(obj):
        got = [None] * world
        dist.all_gather_object(got, obj)
        return got

    cfg = getattr(CFG, cfg_name)
    om = O.Model(cfg, weights=reference_tiny_weights(cfg))
    pool = O.Pool(2)
    mine = list(ep.sequences(EP_SEQS, rank, world))
    sessions = [O.Session(om, pool, 32) for _ in mine]
    r = EPRank(om, pool, rank, world, _placement(kind, cfg["experts"], world), gather, CFG.zipf_router_bias(cfg))
    res = []
    for step in range(EP_STEPS):
        logits, routes = r.step(sessions, [_ep_tokens(g, step, cfg["vocab"]) for g in mine])
        res.append((logits, routes))
    out.put((rank, mine, res))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("cfg_name,world,kind", [("TINY", 2, "contiguous"), ("TINY", 2, "interleaved"),
                                                  ("TINY_768", 2, "balanced"), ("TINY", 4, "interleaved"),
                                                  ("TINY_768", 4, "contiguous")])
def test_expert_parallel_exchange_equals_the_single_rank_oracle(cfg_name, world, kind):
    """The expert-parallel data flow of the batched step (rank-major sequences, the placement table, pairs grouped
    by (local expert, sender, pair), results returned and combined in routing order) restated on the CPU oracle
    (oracle/ep_oracle.py) and run as gloo ranks: every sequence's logits and routes equal its own single-rank oracle
    session bit for bit, with the Zipf router bias so that the experts' loads differ."""
    import numpy as np

    import oracle as O
    from helpers import reference_tiny_weights

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, q, cfg_name, kind)) for r in range(world)]
    for p in procs:
        p.start()
    got = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    cfg = getattr(CFG, cfg_name)
    om = O.Model(cfg, weights=reference_tiny_weights(cfg))
    om.set_router_bias(CFG.zipf_router_bias(cfg))
    pool = O.Pool(2)
    ref = {g: O.Session(om, pool, 32) for g in range(EP_SEQS)}
    want = {g: [ref[g].step(_ep_tokens(g, step, cfg["vocab"]))[:2] for step in range(EP_STEPS)] for g in range(EP_SEQS)}
    seen = []
    for rank, mine, res in got:
        seen += mine
        for step, (logits, routes) in enumerate(res):
            for i, g in enumerate(mine):
                lo, io = want[g][step]
                assert np.array_equal(logits[i].view(np.uint32), lo.view(np.uint32)), f"rank {rank} seq {g} step {step}"
                assert np.array_equal(routes[i], io), f"rank {rank} seq {g} step {step}"
    assert sorted(seen) == list(range(EP_SEQS))
