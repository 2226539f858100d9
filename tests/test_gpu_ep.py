"""Expert-parallel batched decode over 2, 4 and 8 GPUs (one process per GPU) against the same batch on one GPU.

Every output element of the batched step depends only on its own token's column (GEMM columns, attention, routing,
combine), the expert partition keeps each expert's pairs in global token order (sequences are rank-major), and the
ranks' exchange goes through peer memory: so the logits, routes and next ids of every sequence must be bitwise equal
to the single-GPU run.  Skipped where the box has fewer GPUs than ranks (run under a multi-GPU allocation).
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

NSEQ, STEPS, MAX_LEN = 8, 5, 32


def _placement(kind, n_experts, world):
    from lastro_b200 import ep

    if kind == "contiguous":
        return ep.contiguous_placement(n_experts, world)
    if kind == "interleaved":
        return ep.interleaved_placement(n_experts, world)
    # balanced over a Zipf-like load, then experts shuffled between ranks' slots: an arbitrary placement
    owner = ep.balanced_placement([(e + 1) ** -0.8 for e in range(n_experts)], world)
    rng = np.random.default_rng(5)
    return [int(x) for x in rng.permutation(owner)]


def _run(rank, world, port, out_dir, kind="contiguous"):
    import torch
    import torch.distributed as dist

    import lastro_b200 as LB
    import synth_np as S
    from lastro_b200 import configs as CFG
    from lastro_b200 import ep

    if world > 1:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    c = CFG.C5_BATCH
    cfg = c["model"]
    ctx = LB.Context(rank)
    m = LB.GpuModel(ctx, cfg, 8, kv_dtype="bf16")
    m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
    mine = list(ep.sequences(NSEQ, rank, world))
    b = LB.GpuBatch(m, len(mine), MAX_LEN, rank, world)
    ep.connect_group(b)
    if kind != "contiguous":
        b.set_expert_placement(_placement(kind, cfg["experts"], world))
    b.set_router_bias(CFG.zipf_router_bias(cfg))
    prompts = {g: S.tokens(STEPS, 700 + g, cfg["vocab"]) for g in mine}
    res = {"next": [], "logits": [], "routes": []}
    for t in range(STEPS):
        nxt, lg, rt = b.step(list(range(len(mine))), [int(prompts[g][t]) for g in mine], want_logits=True,
                             want_routes=True)
        res["next"].append(nxt)
        res["logits"].append(lg)
        res["routes"].append(rt)
    ids = b.decode(list(range(len(mine))), res["next"][-1], 3)
    np.savez(os.path.join(out_dir, f"w{world}_r{rank}.npz"), seqs=np.array(mine), next=np.array(res["next"]),
             logits=np.array(res["logits"]), routes=np.array(res["routes"]), decode=ids)
    if world > 1:
        dist.barrier()
    b.close()
    m.close()
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


def _gather(out_dir, world):
    parts = [np.load(os.path.join(out_dir, f"w{world}_r{r}.npz")) for r in range(world)]
    cat = {k: np.concatenate([p[k] for p in parts], axis=1 if k != "seqs" else 0) for k in ("next", "logits", "routes",
                                                                                               "decode")}
    assert np.concatenate([p["seqs"] for p in parts]).tolist() == list(range(NSEQ))
    return cat


@pytest.mark.parametrize("world,kind", [(2, "contiguous"), (2, "interleaved"), (2, "shuffled"), (4, "contiguous"),
                                        (4, "shuffled"), (8, "contiguous"), (8, "shuffled")])
def test_expert_parallel_equals_single_gpu_bitwise(world, kind, tmp_path):
    """Every placement of the experts over the ranks gives the single-GPU results bitwise."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < world:
        pytest.skip(f"{torch.cuda.device_count()} GPU(s) here, the test needs {world}")
    mpc = mp.get_context("spawn")
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    for w in (1, world):
        procs = [mpc.Process(target=_run, args=(r, w, port, str(tmp_path), kind)) for r in range(w)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=600)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    one, many = _gather(str(tmp_path), 1), _gather(str(tmp_path), world)
    assert np.array_equal(one["routes"], many["routes"])
    assert np.array_equal(one["logits"], many["logits"])
    assert np.array_equal(one["next"], many["next"]) and np.array_equal(one["decode"], many["decode"])
