"""Batched decode (GpuBatch, one rank) on the GPU through the C ABI, against the CPU oracle.

A batched step has the reference's multi-position contract: every sequence's results equal its own single-sequence
step up to summation order (cpu.rs:234-238).  So each sequence of the batch is checked against its own oracle Session
(model.rs:134-245), with sequences of different lengths stepped in changing subsets and orders, the router bias of the
C5 workload on and off.  The batched GEMMs run on tensor cores with every activation split into two bf16 terms, so the
products are f32-accurate to ~2^-17 relative, against the 2^-24 of the batch-1 kernels: the logits gate is 1e-4
(rel-L2), routing identical.
"""
import numpy as np
import pytest

import lastro_b200 as LB
import oracle as O
import synth_np as S
from helpers import first_route_difference, reference_tiny_weights, rel_l2
from lastro_b200 import configs as CFG

pytestmark = pytest.mark.gpu

GATE = 1e-4


def batch_for(ctx, cfg, w, max_seqs, max_len, kv="f32", gemm=2, attn_tc=None):
    m = LB.GpuModel(ctx, cfg, 8, kv_dtype=kv)
    m.load_weights(w)
    b = LB.GpuBatch(m, max_seqs, max_len)
    b.connect()
    b.set_options(gemm=gemm, attn_tc=attn_tc)
    return m, b


@pytest.mark.parametrize("gemm", [2, 1, 0], ids=["tcgen05-ws", "tcgen05", "mma.sync"])
@pytest.mark.parametrize("kv", ["f32", "bf16", "bf16-cuda-core-attention"])
@pytest.mark.parametrize("biased", [False, True], ids=["plain", "zipf-bias"])
@pytest.mark.parametrize("base", ["tiny", "tiny768"])
def test_batch_matches_oracle_per_sequence(gpu_ctx, pool, kv, gemm, biased, base):
    cfg = CFG.TINY if base == "tiny" else CFG.TINY_768
    w = reference_tiny_weights(cfg)
    nseq, max_len = 5, 200  # 200 positions: two 128-position attention splits, the second partial
    attn_tc = None
    if kv == "bf16-cuda-core-attention":
        kv, attn_tc = "bf16", False
    m, b = batch_for(gpu_ctx, cfg, w, nseq, max_len, kv, gemm, attn_tc)
    om = O.Model(cfg, weights=w)
    bias = CFG.zipf_router_bias(cfg, std=0.5) if biased else None
    if biased:
        b.set_router_bias(bias)
        om.set_router_bias(bias)
    sessions = [O.Session(om, pool, max_len, kv_bf16=kv == "bf16") for _ in range(nseq)]
    lengths = [150, 9, 33, 1, 130]  # sequence q decodes lengths[q] tokens (past one 128-position split for 2 of them)
    prompts = [S.tokens(n, 100 + q, cfg["vocab"]) for q, n in enumerate(lengths)]
    rng = np.random.default_rng(5)
    for t in range(max(lengths)):
        active = [q for q in range(nseq) if t < lengths[q]]
        rng.shuffle(active)  # the batch order is free
        toks = [int(prompts[q][t]) for q in active]
        nxt, lg, rt = b.step(active, toks, want_logits=True, want_routes=True)
        for i, q in enumerate(active):
            lo, io, _ = sessions[q].step(toks[i])
            assert rel_l2(lg[i], lo) < GATE, f"seq {q} position {t}: {rel_l2(lg[i], lo):.2e}"
            assert np.array_equal(rt[i], io), f"seq {q} position {t}: routing"
            assert nxt[i] == O.argmax_last(lg[i])
    for q in range(nseq):
        assert b.position(q) == lengths[q]
    for s in sessions:
        s.close()
    om.close()
    m.close()


def test_batch_decode_equals_steps_and_graphs_equal_direct(gpu_ctx):
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    seqs = [3, 0, 2]
    first = [5, 11, 17]
    runs = []
    for mode in ("decode", "steps", "direct"):
        m, b = batch_for(gpu_ctx, cfg, w, 4, 64)
        if mode == "direct":
            b.set_options(graphs=False)
        if mode == "decode":
            ids = b.decode(seqs, first, 20)
        else:
            ids, tok = [], first
            for _ in range(20):
                nxt, _, _ = b.step(seqs, tok)
                ids.append(nxt)
                tok = nxt
            ids = np.array(ids)
        runs.append(ids)
        m.close()
    assert np.array_equal(runs[0], runs[1]) and np.array_equal(runs[1], runs[2])


def test_batch_trace_covers_the_step_and_changes_nothing(gpu_ctx):
    """lastro_batch_trace: the batched step graph replayed with every CTA stamping the global timer.  Every kernel kind
    of the step shows up, the kinds' exposed times add up to the step, the router's milestones are in order, and the
    traced steps decode like the product graph (bf16 KV: tensor-core attention; tcgen05 GEMMs)."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    seqs, first = [2, 0, 1], [5, 11, 17]
    m1, a = batch_for(gpu_ctx, cfg, w, 3, 64, kv="bf16")
    m2, b = batch_for(gpu_ctx, cfg, w, 3, 64, kv="bf16")
    tr = a.trace(seqs, first, 3)
    ids_b = b.decode(seqs, first, 3)
    for k in ("norm", "qkv", "rope_kv", "attention", "oproj", "router", "gate_up", "down", "combine", "lm_head",
              "argmax"):
        assert tr["exposed"][k] > 0.0 and tr["span"][k] > 0.0, k
    total = sum(tr["exposed"].values())
    assert abs(total - tr["step_ms"]) <= 0.02 * tr["step_ms"] + 1e-3, (total, tr["step_ms"])
    L = cfg["layers"]
    raw = a.trace_raw(1 + 8 * (L - 1) + 4).astype(np.int64)  # the last layer's router
    raw = raw[raw[:, 0] > 0]
    assert len(raw) == len(seqs)
    for r in raw:  # start <= release <= RMSNorm <= logits <= top-k <= rows sent <= ids sent <= exit
        seq = [r[0], r[1], r[8], r[3], r[6], r[7], r[4], r[2]]
        assert all(x > 0 for x in seq) and seq == sorted(seq), seq
    tok = ids_b[-1].tolist()
    na, la, _ = a.step(seqs, tok, want_logits=True)
    nb, lb, _ = b.step(seqs, tok, want_logits=True)
    assert np.array_equal(na, nb) and np.array_equal(la, lb)  # the stamps change no result
    m1.close()
    m2.close()


def test_batch_3b_shape_with_zipf_bias_matches_oracle(gpu_ctx, pool):
    """The C5 model (Granite-3B shape) with its Zipf router bias: 8 sequences, 6 positions each, against the oracle.
    Routing is identical except where the oracle's router scores of the two experts differ by less than 1e-4 (the
    north star's allowance); such a sequence is compared up to that point only, and at most one may diverge."""
    c = CFG.C5_BATCH
    cfg = c["model"]
    nseq, steps = 8, 6
    m = LB.GpuModel(gpu_ctx, cfg, 8, kv_dtype="f32")
    m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
    b = LB.GpuBatch(m, nseq, 16)
    b.connect()
    bias = CFG.zipf_router_bias(cfg)
    b.set_router_bias(bias)
    om = O.Model(cfg, synthetic_seed=c["weight_seed"], std=CFG.WEIGHT_STD, norm_std=0.0, threads=8)
    om.set_router_bias(bias)
    sessions = [O.Session(om, pool, 16) for _ in range(nseq)]
    prompts = [S.tokens(steps, 300 + q, cfg["vocab"]) for q in range(nseq)]
    diverged = set()
    for t in range(steps):
        toks = [int(p[t]) for p in prompts]
        nxt, lg, rt = b.step(list(range(nseq)), toks, want_logits=True, want_routes=True)
        for q in range(nseq):
            lo, io, _ = sessions[q].step(toks[q])
            if q in diverged:
                continue
            d = first_route_difference(rt[q], io, sessions[q].router_logits())
            if d is not None:
                assert d[2] < 1e-4, f"seq {q} position {t}: layer {d[0]} slot {d[1]} routed differently, gap {d[2]:.2e}"
                diverged.add(q)
                continue
            assert rel_l2(lg[q], lo) < GATE, f"seq {q} position {t}: {rel_l2(lg[q], lo):.2e}"
    assert len(diverged) <= 1, diverged
    for s in sessions:
        s.close()
    om.close()
    m.close()


def test_batch_refusals_leave_it_usable(gpu_ctx):
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    m = LB.GpuModel(gpu_ctx, cfg, 8, kv_dtype="f32")
    m.load_weights(w)
    b = LB.GpuBatch(m, 3, 4)
    with pytest.raises(LB.LastroError) as e:
        b.step([0], [1])  # not connected
    assert e.value.code == LB.E_STATE
    b.connect()
    E = cfg["experts"]
    for owner in ([0] * (E - 1), [1] + [0] * (E - 1), [-1] * E):  # wrong count, ranks outside the group
        with pytest.raises(LB.LastroError) as e:
            b.set_expert_placement(owner)
        assert e.value.code == LB.E_ARG
    b.set_expert_placement([0] * E)
    for seqs, toks in (([0, 0], [1, 2]), ([3], [1]), ([0], [cfg["vocab"]]), ([], [])):
        with pytest.raises(LB.LastroError) as e:
            b.step(seqs, toks)
        assert e.value.code == LB.E_ARG
    for _ in range(4):
        b.step([1], [2])
    with pytest.raises(LB.LastroError) as e:
        b.step([1], [2])
    assert e.value.code == LB.E_FULL
    b.reset(1)
    nxt, _, _ = b.step([1, 2], [2, 2])
    assert nxt[0] == nxt[1]  # same token at position 0 of two sequences
    m.close()
