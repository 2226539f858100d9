"""Whole-model decode (GpuModel) on the GPU through the C ABI, checked against the CPU oracle and the goldens.

Restates rust/moe-rt/tests/model.rs:136-157 and 252-281 (GPU model vs CPU model, rel-L2 < 1e-5 over more than one
attention slice, routing identical, reset reproduces) and bin/m1b-gulosa.rs (greedy ids identical except where the
reference's top1-top2 gap < 1e-3).
"""
import os

import numpy as np
import pytest

import lastro_b200 as LB
import oracle as O
import synth_np as S
from helpers import first_route_difference, reference_tiny_weights, rel_l2, values
from lastro_b200 import configs as CFG

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TIE_GAP = 1e-3  # bin/m1b-gulosa.rs:20


def gpu_model(ctx, cfg, weights, max_len, kv="f32", fused=False, attn_tc=None):
    m = LB.GpuModel(ctx, cfg, max_len, kv_dtype=kv)
    m.load_weights(weights)
    m.set_options(fused=fused)
    if attn_tc is not None:
        m.set_attention(attn_tc)
    assert m.fused == fused
    return m


def toks_like_reference(n, vocab, seed=77):
    """tests/model.rs:260: ((v + 1) * 16) as usize % vocab"""
    return [int((float(v) + 1.0) * 16.0) % vocab for v in values(n, seed)]


# f32 KV: the reference's gate (tests/model.rs:268) on the logits; the routing weights are a softmax of router
# logits whose f32 sums run in another order on each side (the fused step reduces one share per CTA), which moves
# them by up to a few 1e-5.  bf16 KV rounds every cached K/V element (2^-9 relative), which moves logits by ~1e-3
# and the routing weights by ~1e-3 while the routing itself stays identical.
@pytest.mark.parametrize("fused", [True, False], ids=["fused", "chain"])
@pytest.mark.parametrize("kv,gate,wtol", [("f32", 1e-5, 5e-5), ("bf16", 2e-3, 5e-3)])
def test_model_matches_oracle_over_more_than_one_page(gpu_ctx, pool, kv, gate, wtol, fused):
    """tests/model.rs:252-281 on the reference's tiny model (70 positions: two KV pages, two attention tiles), for the
    fused step kernel and for the per-layer kernel chain."""
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    steps = 70
    m = gpu_model(gpu_ctx, cfg, w, 128, kv, fused)
    om = O.Model(cfg, weights=w)
    s = O.Session(om, pool, 128)
    toks = toks_like_reference(steps, cfg["vocab"])
    for t, tok in enumerate(toks):
        lg, nxt, ids, rw = m.step(tok)
        lo, io, wo = s.step(tok)
        assert lg.shape == (cfg["vocab"],)
        assert rel_l2(lg, lo) < gate, f"position {t}: {rel_l2(lg, lo):.2e}"
        assert np.array_equal(ids, io), f"position {t}: routing"
        np.testing.assert_allclose(rw, wo, atol=wtol)
        assert nxt == O.argmax_last(lg)
    # after reset the same sequence gives the same logits (the stale cache is masked by the length)
    m.reset()
    s.reset()
    for tok in toks[:3]:
        lg, _, _, _ = m.step(tok)
        lo, _, _ = s.step(tok)
        assert rel_l2(lg, lo) < gate
    m.close()


@pytest.mark.parametrize("fused", [True, False], ids=["fused", "chain"])
def test_model_768_hidden_matches_oracle(gpu_ctx, pool, fused):
    """tests/model.rs:127-157: H = 768 = 3 x 256 (the 3B shape in miniature), 12 heads / 4 KV heads."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    m = gpu_model(gpu_ctx, cfg, w, 64, "f32", fused)
    om = O.Model(cfg, weights=w)
    s = O.Session(om, pool, 64)
    for t in range(12):
        tok = (t * 11 + 5) % cfg["vocab"]
        lg, _, ids, _ = m.step(tok)
        lo, io, _ = s.step(tok)
        assert rel_l2(lg, lo) < 1e-5, f"position {t}"
        assert np.array_equal(ids, io)
    m.close()


def test_tiny_golden_greedy_and_teacher_forced(gpu_ctx):
    """The transformers golden (tests/golden/tiny_model.npz): greedy ids and logits at every position."""
    import json
    g = np.load(os.path.join(GOLDEN, "tiny_model.npz"))
    meta = json.loads(str(g["meta"]))
    cfg = CFG.TINY
    w = S.as_bits(S.model_weights(cfg, meta["seed"], 0.0, stds=meta["stds"]))
    m = gpu_model(gpu_ctx, cfg, w, 128)
    out = m.generate(g["prompt"], len(g["generated"]))
    for i, (a, b) in enumerate(zip(out, g["generated"])):
        assert a == b or g["gaps"][i] < TIE_GAP, f"step {i}: {a} vs {b}"
    m.reset()
    seq = np.concatenate([g["prompt"], g["generated"][:-1]])
    for t, tok in enumerate(seq):
        lg, _, ids, _ = m.step(int(tok))
        assert rel_l2(lg, g["logits"][t]) < 1e-4, f"position {t}"
        assert np.array_equal(ids, g["route_idx"][:, t, :]), f"position {t}"
    m.close()


def test_graph_pdl_and_direct_launches_agree_bitwise(gpu_ctx):
    """The kernel chain is bitwise the same with and without graphs / PDL; the fused step is bitwise the same with
    and without a graph, and within the f32 gate of the chain (different summation orders)."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    m = gpu_model(gpu_ctx, cfg, w, 64, "bf16")
    toks = toks_like_reference(20, cfg["vocab"], seed=5)
    runs = []
    for graphs, pdl in ((True, True), (False, True), (False, False), (True, False)):
        m.set_options(graphs, pdl, fused=False)
        m.reset()
        runs.append(np.stack([m.step(t)[0] for t in toks]))
    for r in runs[1:]:
        assert np.array_equal(r, runs[0])
    fused = []
    for graphs in (True, False):
        m.set_options(graphs, True, fused=True)
        assert m.fused
        m.reset()
        fused.append(np.stack([m.step(t)[0] for t in toks]))
    assert np.array_equal(fused[0], fused[1])
    for t in range(len(toks)):
        assert rel_l2(fused[0][t], runs[0][t]) < 1e-5, f"position {t}"
    m.close()


@pytest.mark.parametrize("kv,n", [("f32", 5000), ("bf16", 9600)])
def test_fused_long_context_stages_kv_in_chunks(gpu_ctx, pool, kv, n):
    """A context longer than one staged K/V chunk per attention unit (74 splits x kv_cap rows on the tiny model):
    the fused kernel loads the remaining chunks inside the attention phase.  Prefill by greedy steps on both sides,
    then logits compared with the oracle (f32 KV) or the kernel chain (bf16 KV, the oracle keeps f32 K/V)."""
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    m = gpu_model(gpu_ctx, cfg, w, n + 8, kv, True)
    toks = toks_like_reference(n, cfg["vocab"], seed=11)
    m.generate(toks, 1)
    if kv == "f32":
        om = O.Model(cfg, weights=w)
        s = O.Session(om, pool, n + 8)
        for t in toks:
            s.step(t)
        for tok in (3, 17, 29):
            lg, _, ids, _ = m.step(tok)
            lo, io, _ = s.step(tok)
            assert rel_l2(lg, lo) < 1e-4, f"{rel_l2(lg, lo):.2e}"
            assert np.array_equal(ids, io)
        s.close()
        om.close()
    else:
        ref = gpu_model(gpu_ctx, cfg, w, n + 8, kv, False)
        ref.generate(toks, 1)
        for tok in (3, 17, 29):
            lg, _, ids, _ = m.step(tok)
            lr, _, ir, _ = ref.step(tok)
            assert rel_l2(lg, lr) < 1e-4, f"{rel_l2(lg, lr):.2e}"
            assert np.array_equal(ids, ir)
        ref.close()
    m.close()


def test_generate_and_decode_match_step_by_step(gpu_ctx):
    cfg = CFG.TINY
    w = S.as_bits(S.model_weights(cfg, 10, 0.0, stds=S.TINY_STD))
    m = gpu_model(gpu_ctx, cfg, w, 128, "bf16")
    prompt = S.tokens(10, 3, cfg["vocab"])
    ids = m.generate(prompt, 30)
    m.reset()
    for t in prompt[:-1]:
        m.step(int(t))
    _, nxt, _, _ = m.step(int(prompt[-1]))
    seq = [nxt]
    for _ in range(29):
        _, nxt, _, _ = m.step(seq[-1])
        seq.append(nxt)
    assert ids.tolist() == seq
    assert m.pos == len(prompt) + 29
    m.close()


def test_errors_refused_before_launch_and_model_stays_usable(gpu_ctx):
    """gpu_model.rs:252-257: bad token / full KV are refused and the model stays usable."""
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    m = LB.GpuModel(gpu_ctx, cfg, 4, kv_dtype="bf16")
    with pytest.raises(LB.LastroError) as e:
        m.step(1)
    assert e.value.code == LB.E_STATE  # weights not loaded yet
    m.load_weights(w)
    with pytest.raises(LB.LastroError) as e:
        m.step(cfg["vocab"])
    assert e.value.code == LB.E_ARG
    for t in range(4):
        m.step(t)
    with pytest.raises(LB.LastroError) as e:
        m.step(0)
    assert e.value.code == LB.E_FULL
    m.reset()
    lg, _, _, _ = m.step(3)
    assert np.isfinite(lg).all()
    m.close()


@pytest.mark.parametrize("fused", [False, True], ids=["chain", "fused"])
def test_c2_1b_greedy_matches_transformers_golden(gpu_ctx, fused):
    """BASELINE config 1 at full size: 128-token prompt, 128 greedy ids vs transformers."""
    g = np.load(os.path.join(GOLDEN, "c2_greedy.npz"))
    c = CFG.C2_1B
    cfg = c["model"]
    m = LB.GpuModel(gpu_ctx, cfg, 320, kv_dtype="bf16")
    m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
    m.set_options(fused=fused)
    assert m.fused == fused
    out = m.generate(g["prompt"], len(g["generated"]))
    for i, (a, b) in enumerate(zip(out, g["generated"])):
        assert a == b or g["gaps"][i] < TIE_GAP, f"step {i}: {a} vs {b}"
    m.close()


@pytest.mark.parametrize("kv,gate", [("f32", 1e-4), ("bf16", 5e-3)])
def test_c2_1b_logits_match_transformers_golden_every_step(gpu_ctx, kv, gate):
    """BASELINE config 1 at full size, logits rather than ids: after the 128-token prompt, every one of the 128 greedy
    steps (fed the golden's own ids) has the golden's top-16 logits (transformers GraniteMoeForCausalLM in fp32 on
    the same bf16 weights) at rel-L2 < gate, and the same argmax except at top1-top2 gaps < 1e-3."""
    g = np.load(os.path.join(GOLDEN, "c2_greedy.npz"))
    c = CFG.C2_1B
    cfg = c["model"]
    m = LB.GpuModel(gpu_ctx, cfg, 320, kv_dtype=kv)
    m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
    for tok in g["prompt"][:-1]:
        m.step(int(tok), want_logits=False, want_routes=False)
    prev, worst = int(g["prompt"][-1]), 0.0
    for i, want in enumerate(g["generated"]):
        lg, nxt, _, _ = m.step(prev, want_routes=False)
        err = rel_l2(lg[g["top_idx"][i]], g["top_val"][i])
        assert err < gate, f"step {i}: top-16 logits rel-L2 {err:.2e}"
        assert nxt == want or g["gaps"][i] < TIE_GAP, f"step {i}: {nxt} vs {want}"
        worst = max(worst, err)
        prev = int(want)
    print(f"C2 {kv} KV: worst top-16 logits rel-L2 {worst:.2e} over {len(g['generated'])} steps")
    m.close()


@pytest.mark.parametrize("fused", [False, True], ids=["chain", "fused"])
def test_c3_3b_logits_match_oracle_at_full_size(gpu_ctx, pool, fused):
    """BASELINE config 2 shape (Granite-3B, 32 layers, E 40): device-filled weights are bit-identical to the
    oracle's, so logits and routing can be compared at full size for a short sequence."""
    c = CFG.C3_3B
    cfg = c["model"]
    m = LB.GpuModel(gpu_ctx, cfg, 64, kv_dtype="f32")
    m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.1)
    m.set_options(fused=fused)
    assert m.fused == fused  # the 3B shape fits the fused step kernel
    om = O.Model(cfg, synthetic_seed=c["weight_seed"], std=CFG.WEIGHT_STD, norm_std=0.1, threads=os.cpu_count() or 8)
    s = O.Session(om, pool, 64)
    toks = S.tokens(6, c["prompt_seed"], cfg["vocab"])
    for t, tok in enumerate(toks):
        lg, _, ids, _ = m.step(int(tok))
        lo, io, _ = s.step(int(tok))
        d = first_route_difference(ids, io, s.router_logits())
        assert d is None or d[2] < 1e-4, f"position {t}: layer {d[0]} slot {d[1]} routes differ at gap {d[2]:.2e}"
        if d is not None and set(ids[d[0]].tolist()) != set(io[d[0]].tolist()):
            break  # a router tie legitimately changed the experts: the runs diverge from here
        assert rel_l2(lg, lo) < 1e-4, f"position {t}: {rel_l2(lg, lo):.2e}"
    s.close()
    om.close()
    m.close()


def test_profile_direct_launches_report_every_kernel(gpu_ctx):
    """lastro_model_profile: direct launches with an event between kernels, after a synthetic context."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    m = gpu_model(gpu_ctx, cfg, w, 400, "bf16", False)
    m.fill_kv_synthetic(300)
    prof = m.profile(3)
    assert m.pos == 303
    for k in ("qkv_rope", "attention", "oproj", "head") + (("moe",) if m.moe else ("gate_up", "down")):
        assert prof[k] > 0.0, k
    assert (prof["gate_up"] == 0.0) == m.moe
    assert prof["router"] == 0.0  # folded into oproj
    assert prof["fused_step"] == 0.0
    m.set_options(fused=True)
    assert m.fused
    prof = m.profile(2)
    assert m.pos == 305
    assert prof["fused_step"] > 0.0
    assert all(v == 0.0 for k, v in prof.items() if k != "fused_step")
    lg, _, _, _ = m.step(5)
    assert np.isfinite(lg).all()
    m.close()


@pytest.mark.parametrize("attn_tc,mma,splits", [(True, False, 16), (False, False, 16), (False, True, 16),
                                                 (False, True, 8)],
                         ids=["batched-tensor-core-kernel", "split-kernel-cuda-cores", "split-kernel-mma-16",
                              "split-kernel-mma-8"])
def test_bf16_kv_attention_kernels_match_oracle(gpu_ctx, pool, attn_tc, mma, splits):
    """The chain with bf16 KV on each attention form (the batched step's tensor-core kernel with TMA page loads; the
    split kernel on CUDA cores, the default, or on tensor cores) against the oracle storing bf16-rounded K/V
    (Session(kv_bf16=True)): 150 positions, three KV pages, so the context splits hold 0, 1 or 2 pages and every
    offset of a split's rows within the 16-row groups of the tensor-core form."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    m = gpu_model(gpu_ctx, cfg, w, 256, "bf16", False, attn_tc)
    if not attn_tc:
        m.set_tuning(splits, 0, attn_mma=mma)
    om = O.Model(cfg, weights=w)
    s = O.Session(om, pool, 256, kv_bf16=True)
    for t, tok in enumerate(toks_like_reference(150, cfg["vocab"])):
        lg, nxt, ids, _ = m.step(tok)
        lo, io, _ = s.step(tok)
        assert rel_l2(lg, lo) < 1e-4, f"position {t}: {rel_l2(lg, lo):.2e}"
        assert np.array_equal(ids, io), f"position {t}: routing"
    s.close()
    om.close()
    m.close()


def test_trace_in_graph_timeline_covers_the_step(gpu_ctx):
    """lastro_model_trace: the step graph replayed with every CTA stamping the global timer.  Every kernel kind of the
    chain shows up, the kinds' exposed times add up to the step, and the traced steps decode like the product graph."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    a = gpu_model(gpu_ctx, cfg, w, 400, "bf16", False)
    b = gpu_model(gpu_ctx, cfg, w, 400, "bf16", False)
    for m in (a, b):
        m.fill_kv_synthetic(300)
    tr = a.trace(3)
    b.decode(3)
    assert a.pos == b.pos == 303
    for k in ("qkv_rope", "attention", "oproj", "head") + (("moe",) if a.moe else ("gate_up", "down")):
        assert tr["exposed"][k] > 0.0 and tr["span"][k] > 0.0, k
    assert tr["exposed"]["router"] == 0.0 and tr["exposed"]["fused_step"] == 0.0
    total = sum(tr["exposed"].values())
    assert abs(total - tr["step_ms"]) <= 0.02 * tr["step_ms"] + 1e-3, (total, tr["step_ms"])
    la, na, _, _ = a.step(7)
    lb, nb, _, _ = b.step(7)
    assert na == nb and np.array_equal(la, lb)  # the stamps change no result
    a.close()
    b.close()


def test_generate_until_stops_after_the_end_of_text(gpu_ctx):
    """geracao_regra.rs:181-245 in normal use: the loop emits the end-of-text token and stops without feeding it.
    The end-of-text id is taken from a fixed-length run (the token whose first appearance comes last), so the stop
    falls inside a later chunk; the ids equal the fixed-length run's prefix, the position is the reference's, and the
    next step continues exactly like a model stepped token by token."""
    cfg = CFG.TINY
    w = S.as_bits(S.model_weights(cfg, 10, 0.0, stds=S.TINY_STD))
    m = gpu_model(gpu_ctx, cfg, w, 128, "bf16")
    prompt = S.tokens(10, 3, cfg["vocab"])
    free = m.generate(prompt, 48).tolist()
    first = {}
    for i, t in enumerate(free):
        first.setdefault(t, i)
    eos, stop = max(first.items(), key=lambda kv: kv[1])
    assert stop > 0
    m.reset()
    out = m.generate_until(prompt, 48, eos)
    assert out.tolist() == free[:stop + 1]
    assert m.pos == len(prompt) + stop
    lg, nxt, _, _ = m.step(int(out[-1]))
    ref = gpu_model(gpu_ctx, cfg, w, 128, "bf16")
    for t in list(prompt) + out.tolist()[:-1]:
        ref.step(int(t), want_logits=False, want_routes=False)
    lr, nr, _, _ = ref.step(int(out[-1]))
    assert nxt == nr and np.array_equal(lg, lr)
    # eos < 0: never stops (the fixed-length proof mode)
    m.reset()
    assert m.generate_until(prompt, 48, -1).tolist() == free
    assert m.pos == len(prompt) + 47
    with pytest.raises(LB.LastroError) as e:
        m.generate_until(prompt, 48, cfg["vocab"])
    assert e.value.code == LB.E_ARG
    ref.close()
    m.close()


@pytest.mark.parametrize("which", ["tiny", "tiny768", "tiny_q8", "c3"])
def test_one_launch_moe_equals_the_gate_up_and_down_kernels_bitwise(gpu_ctx, which):
    """The MoE block as one persistent launch (routing, gate_up and down streamed through one ring, a grid barrier
    between them) computes every dot in the same order as the gate_up + down kernels: logits and routes bitwise
    equal over 20 positions, bf16 and Q8_0 weights, up to the 3B shape."""
    if which == "c3":
        c = CFG.C3_3B
        cfg = c["model"]
        models = []
        for _ in range(2):
            m = LB.GpuModel(gpu_ctx, cfg, 64, kv_dtype="bf16")
            m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
            models.append(m)
    else:
        cfg = {"tiny": CFG.TINY, "tiny768": CFG.TINY_768, "tiny_q8": dict(CFG.TINY, weight_dtype="q8_0")}[which]
        w = S.model_weights_q8(cfg, 12) if which == "tiny_q8" else reference_tiny_weights(cfg)
        models = [gpu_model(gpu_ctx, cfg, w, 64, "bf16") for _ in range(2)]
    a, b = models
    assert not a.moe  # the two kernels are the default
    a.set_moe(True)
    assert a.moe and not b.moe
    for t in range(20):
        tok = (t * 7 + 3) % cfg["vocab"]
        la, na, ia, wa = a.step(tok)
        lb, nb, ib, wb = b.step(tok)
        assert np.array_equal(la, lb) and na == nb and np.array_equal(ia, ib) and np.array_equal(wa, wb), f"position {t}"
    a.close()
    b.close()


@pytest.mark.parametrize("splits,merge,smem", [(16, 0, 0), (8, 0, 0), (16, 1, 0), (8, 1, 0), (8, 2, 0), (8, 2, 1),
                                               (16, 2, 0)],
                         ids=["16-last-cta", "8-last-cta", "16-oproj", "8-oproj", "8-cluster", "8-cluster-oproj-smem",
                              "16-cluster"])
def test_attention_split_and_merge_variants_match_oracle(gpu_ctx, pool, splits, merge, smem):
    """Every tuning of the CUDA-core attention (8 or 16 context splits; the splits merged by the last CTA of a KV head,
    by the output projection, or by a thread-block cluster in distributed shared memory) and of the output projection
    (weights in registers or staged in shared memory) against the oracle over 150 positions (three K/V pages), f32 KV,
    at the f32 model gate."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    m = gpu_model(gpu_ctx, cfg, w, 256, "f32")
    m.set_tuning(splits, merge, bool(smem), prefetch_down=True)
    om = O.Model(cfg, weights=w)
    s = O.Session(om, pool, 256)
    worst = 0.0
    for t, tok in enumerate(toks_like_reference(150, cfg["vocab"])):
        lg, _, ids, _ = m.step(tok)
        lo, io, _ = s.step(tok)
        worst = max(worst, rel_l2(lg, lo))
        assert rel_l2(lg, lo) < 1e-5, f"position {t}: {rel_l2(lg, lo):.2e}"
        assert np.array_equal(ids, io), f"position {t}: routing"
    s.close()
    om.close()
    m.close()


@pytest.mark.parametrize("mma", [False, True], ids=["cuda-cores", "tensor-cores"])
@pytest.mark.parametrize("splits,merge", [(16, 0), (8, 0), (16, 1), (8, 2)],
                         ids=["16-last-cta", "8-last-cta", "16-oproj", "8-cluster"])
def test_bf16_kv_staged_by_swizzled_boxes_is_bitwise_the_bulk_copy_staging(gpu_ctx, splits, merge, mma):
    """bf16 K/V staged as 8-row TMA boxes with the 128-byte swizzle against one bulk copy per page run (the default):
    the same rows in the same order, so logits and routes are bitwise equal, over 150 positions (three 64-position
    pages; split boundaries at every offset within a box, the new row inside a staged box or starting one); the
    cluster merge runs the bulk-copy form only (both sides)."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    a = gpu_model(gpu_ctx, cfg, w, 256, "bf16")
    b = gpu_model(gpu_ctx, cfg, w, 256, "bf16")
    a.set_tuning(splits, merge, attn_tma=merge != 2, attn_mma=mma and merge != 2)
    b.set_tuning(splits, merge, attn_mma=mma and merge != 2)
    for t, tok in enumerate(toks_like_reference(150, cfg["vocab"])):
        la, na, ia, _ = a.step(tok)
        lb, nb, ib, _ = b.step(tok)
        assert np.array_equal(la, lb) and na == nb and np.array_equal(ia, ib), f"position {t}"
    a.close()
    b.close()


def gate_up_misses(m, layers):
    """CTAs of the traced step's gate_up launches that re-staged their rows after a misprediction (milestone 6)."""
    m.trace(1)  # one traced decode step: launches qkv, attention, oproj, gate_up, down per layer, then head
    return sum(int((m.trace_raw(5 * l + 3)[:, 3 + 6] > 0).sum()) for l in range(layers))


@pytest.mark.parametrize("mode", ["l2", "stage", "attn"])
@pytest.mark.parametrize("which", ["tiny", "tiny768", "c3-2layer"])
def test_speculative_expert_fetch_is_bitwise_the_plain_chain(gpu_ctx, which, mode):
    """The experts predicted from the layer's input fetched before the routing is known -- hinted into L2 by the
    output projection or staged into the gate_up CTAs' shared memory -- against no speculation (the default): the routing and the rows computed do not depend on the prediction, so logits and routes are bitwise
    equal (staging: CTAs whose prediction missed re-stage, counted from the timeline)."""
    if which == "tiny":
        cfg, w, n = CFG.TINY, reference_tiny_weights(CFG.TINY), 60
    elif which == "tiny768":
        cfg, w, n = CFG.TINY_768, reference_tiny_weights(CFG.TINY_768), 120
    else:
        cfg, w, n = dict(CFG.C3_3B["model"], layers=2), None, 40
    models = []
    for spec in (True, False):
        m = LB.GpuModel(gpu_ctx, cfg, 256, kv_dtype="bf16")
        if w is None:
            m.fill_synthetic(CFG.C3_3B["weight_seed"], CFG.WEIGHT_STD, 0.0)
        else:
            m.load_weights(w)
        m.set_tuning(16, 0, speculation=mode if spec else False)
        models.append(m)
    a, b = models
    toks = toks_like_reference(n, cfg["vocab"])
    for t, tok in enumerate(toks):
        la, na, ia, _ = a.step(tok)
        lb, nb, ib, _ = b.step(tok)
        assert np.array_equal(la, lb) and na == nb and np.array_equal(ia, ib), f"position {t}"
    misses = gate_up_misses(a, cfg["layers"])
    assert gate_up_misses(b, cfg["layers"]) == 0
    if mode != "stage":
        assert misses == 0
    print(f"{which} {mode}: gate_up CTAs re-staged after a misprediction in one traced step: {misses}")
    a.close()
    b.close()


@pytest.mark.parametrize("which", ["tiny768", "c3-2layer"])
def test_down_taking_the_published_routing_is_bitwise_its_own_reduction(gpu_ctx, which):
    """The down kernel taking the routing gate_up's first CTA publishes (the default; a per-layer flag stamped with the
    step counter) against every down CTA reducing the router shares itself: the same routing, bitwise the same logits
    and routes, also across a reset (the counter keeps rising, so no flag of an earlier step is taken)."""
    if which == "tiny768":
        cfg, w = CFG.TINY_768, reference_tiny_weights(CFG.TINY_768)
    else:
        cfg, w = dict(CFG.C3_3B["model"], layers=2), None
    models = []
    for own in (False, True):
        m = LB.GpuModel(gpu_ctx, cfg, 128, kv_dtype="bf16")
        if w is None:
            m.fill_synthetic(CFG.C3_3B["weight_seed"], CFG.WEIGHT_STD, 0.0)
        else:
            m.load_weights(w)
        m.set_tuning(16, 0, down_routes=own)
        models.append(m)
    a, b = models
    for rnd in range(2):
        for t, tok in enumerate(toks_like_reference(40, cfg["vocab"])):
            la, na, ia, _ = a.step(tok)
            lb, nb, ib, _ = b.step(tok)
            assert np.array_equal(la, lb) and na == nb and np.array_equal(ia, ib), f"round {rnd} position {t}"
        a.reset()
        b.reset()
    a.close()
    b.close()


def test_output_projection_weights_in_shared_memory_is_bitwise_the_register_form(gpu_ctx):
    """oproj_smem_kernel (weights staged by one bulk copy, 256 threads) against oproj_kernel (weights in registers,
    512 threads): the same dot order, so logits and routes are bitwise equal; bf16 and Q8_0 weights."""
    for cfg, w in ((CFG.TINY_768, reference_tiny_weights(CFG.TINY_768)),
                   (dict(CFG.TINY, weight_dtype="q8_0"), S.model_weights_q8(dict(CFG.TINY, weight_dtype="q8_0"), 12))):
        a = gpu_model(gpu_ctx, cfg, w, 64, "bf16")
        b = gpu_model(gpu_ctx, cfg, w, 64, "bf16")
        b.set_tuning(16, 0, True)
        for t in range(12):
            tok = (t * 5 + 2) % cfg["vocab"]
            la, na, ia, _ = a.step(tok)
            lb, nb, ib, _ = b.step(tok)
            assert np.array_equal(la, lb) and na == nb and np.array_equal(ia, ib), f"position {t}"
        a.close()
        b.close()
