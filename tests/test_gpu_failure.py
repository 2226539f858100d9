"""Failure detection on the GPU without a GPU fault (the reference's poison policy, gpu_model.rs:249-267).

An expert-parallel group of two ranks on one GPU: rank 1 is a child process that creates its batch, exchanges handles
and connects, then never steps.  Rank 0's step waits for rank 1's dispatch flag, which nothing sets; with a 50 ms wait
limit the wait gives up, records its code in the batch's error word, and every later wait of the step returns at once
(it finds the word set), so the step ends within a fraction of a second: LASTRO_E_CUDA, then LASTRO_E_POISONED on the
next call.  Rank 1 launches nothing, so no two kernels wait on each other; rank 0 closes its mapping of rank 1's
region before rank 1 exits.  Afterwards a fresh batch on the same GPU decodes like the CPU oracle.
"""
import multiprocessing as mp
import queue
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_SEQS, MAX_LEN = 2, 32


def _idle_rank(to_child, from_child):
    import lastro_b200 as LB
    from lastro_b200 import configs as CFG

    ctx = LB.Context(0)
    m = LB.GpuModel(ctx, CFG.TINY, 8, kv_dtype="bf16")
    m.fill_synthetic(1, 0.02, 0.0)
    b = LB.GpuBatch(m, MAX_SEQS, MAX_LEN, rank=1, world=2)
    from_child.put(b.exchange_handle())
    h0 = to_child.get(timeout=300)
    b.connect([h0, b.exchange_handle()])
    from_child.put("connected")
    to_child.get(timeout=600)  # "done": rank 0 has closed its mapping of this rank's region
    b.close()
    m.close()
    ctx.close()


def test_a_rank_that_never_steps_makes_the_step_give_up_and_poison(gpu_ctx, pool):
    import lastro_b200 as LB
    import oracle as O
    from helpers import reference_tiny_weights, rel_l2
    from lastro_b200 import configs as CFG

    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    spawn = mp.get_context("spawn")
    to_child, from_child = spawn.Queue(), spawn.Queue()
    child = spawn.Process(target=_idle_rank, args=(to_child, from_child), daemon=True)
    child.start()
    try:
        m = LB.GpuModel(gpu_ctx, cfg, 8, kv_dtype="bf16")
        m.load_weights(w)
        b = LB.GpuBatch(m, MAX_SEQS, MAX_LEN, rank=0, world=2)
        try:
            h1 = from_child.get(timeout=300)
            to_child.put(b.exchange_handle())
            b.connect([b.exchange_handle(), h1])
            assert from_child.get(timeout=300) == "connected"
            b.set_wait_limit(0.05)
            t0 = time.time()
            with pytest.raises(LB.LastroError) as e:
                b.step([0], [3])
            took = time.time() - t0
            assert e.value.code == LB.E_CUDA, str(e.value)
            assert "gave up" in str(e.value)
            # one limit per step, not one per layer and exchange
            assert took < 5.0, f"the step took {took:.2f} s to give up"
            with pytest.raises(LB.LastroError) as e:
                b.step([0], [3])
            assert e.value.code == LB.E_POISONED
        finally:
            b.close()
            m.close()
    finally:
        to_child.put("done")
        child.join(120)
        if child.is_alive():
            child.kill()
    assert child.exitcode == 0

    # the GPU and this context still work: a fresh single-rank batch decodes like the oracle
    m = LB.GpuModel(gpu_ctx, cfg, 8, kv_dtype="bf16")
    m.load_weights(w)
    b = LB.GpuBatch(m, 2, MAX_LEN)
    b.connect()
    om = O.Model(cfg, weights=w)
    s = O.Session(om, pool, MAX_LEN, kv_bf16=True)
    for tok in (3, 11, 7):
        nxt, lg, rt = b.step([0], [tok], want_logits=True, want_routes=True)
        lo, io, _ = s.step(tok)
        assert rel_l2(lg[0], lo) < 1e-4
        assert np.array_equal(rt[0], io)
    s.close()
    om.close()
    b.close()
    m.close()


def test_wait_limit_is_refused_outside_its_range(gpu_ctx):
    import lastro_b200 as LB
    from lastro_b200 import configs as CFG

    m = LB.GpuModel(gpu_ctx, CFG.TINY, 8, kv_dtype="bf16")
    m.fill_synthetic(1, 0.02, 0.0)
    b = LB.GpuBatch(m, 2, MAX_LEN)
    b.connect()
    for bad in (0.0, 1e-4, 1e4):
        with pytest.raises(LB.LastroError) as e:
            b.set_wait_limit(bad)
        assert e.value.code == LB.E_ARG
    b.set_wait_limit(2.0)
    nxt, _, _ = b.step([0], [5])
    assert 0 <= int(nxt[0]) < CFG.TINY["vocab"]
    b.close()
    m.close()
