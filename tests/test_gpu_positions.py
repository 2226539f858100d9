"""The multi-position step (lastro_model_step_positions) against the token-by-token step and the CPU oracle.

Restates rust/moe-rt/tests/motor_passo_gpu.rs:100-150: the tokens [3, 17, 5, 17, 3, 29, 5, 8, 17, 3, 5, 29, 8, 17] in
blocks of 8, 3, 1 and 2 positions give, at every position, the logits of the token-by-token path of the same engine
and of the CPU reference, and the same K/V rows (cuda_backend.rs:264-274: per-position results equal the single-position
path up to summation order).  The multi-position step runs the batched path's tensor-core GEMMs, whose activations
are split into bf16 hi + lo (a relative residue below 2^-17), while the token-by-token chain runs f32 GEMVs on CUDA
cores: the gates below allow that summation-order difference and nothing more.
"""
import numpy as np
import pytest

import lastro_b200 as LB
import oracle as O
from helpers import reference_tiny_weights, rel_l2
from lastro_b200 import configs as CFG

pytestmark = pytest.mark.gpu

TOKENS = [3, 17, 5, 17, 3, 29, 5, 8, 17, 3, 5, 29, 8, 17]  # motor_passo_gpu.rs:103
BLOCKS = [8, 3, 1, 2]                                       # motor_passo_gpu.rs:101


def model(ctx, cfg, w, max_len, kv):
    m = LB.GpuModel(ctx, cfg, max_len, kv_dtype=kv)
    m.load_weights(w)
    return m


@pytest.mark.parametrize("kv,gate_step,gate_cpu,gate_kv", [("f32", 1e-5, 1e-4, 1e-5), ("bf16", 2e-3, 2e-3, 5e-3)])
def test_blocks_of_8_3_1_2_match_token_by_token_and_the_cpu(gpu_ctx, pool, kv, gate_step, gate_cpu, gate_kv):
    """motor_passo_gpu.rs:108-150 on the reference's tiny model with attention weights 0.3 (tiny_model_attn)."""
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg, attn=0.3)
    a = model(gpu_ctx, cfg, w, 32, kv)
    b = model(gpu_ctx, cfg, w, 32, kv)
    om = O.Model(cfg, weights=w)
    s = O.Session(om, pool, 32, kv_bf16=(kv == "bf16"))
    step_logits, i = [], 0
    for n in BLOCKS:
        lg, nxt = a.step_positions(TOKENS[i:i + n])
        assert lg.shape == (n, cfg["vocab"]) and nxt.tolist() == [O.argmax_last(x) for x in lg]
        step_logits += list(lg)
        i += n
    assert a.pos == len(TOKENS)
    for t, tok in enumerate(TOKENS):
        lt, _, _, _ = b.step(tok)
        lo, _, _ = s.step(tok)
        assert rel_l2(step_logits[t], lt) <= gate_step, f"position {t}: step vs token by token {rel_l2(step_logits[t], lt):.2e}"
        assert rel_l2(step_logits[t], lo) <= gate_cpu, f"position {t}: step vs cpu {rel_l2(step_logits[t], lo):.2e}"
    for layer in range(cfg["layers"]):
        ka, va = a.read_kv(layer, 0, len(TOKENS))
        kb, vb = b.read_kv(layer, 0, len(TOKENS))
        assert rel_l2(ka, kb) <= gate_kv and rel_l2(va, vb) <= gate_kv, f"layer {layer}"
    # the model continues from the step like from token-by-token steps
    la, na, _, _ = a.step(7)
    lb, nb, _, _ = b.step(7)
    assert rel_l2(la, lb) <= gate_step and na == nb
    s.close()
    om.close()
    a.close()
    b.close()


@pytest.mark.parametrize("n", [1, 8, 32])
def test_steps_of_1_8_and_32_positions_on_the_768_model(gpu_ctx, n):
    """Every position of 64 prompt ids fed n at a time equals the token-by-token chain (f32 KV), across the 64-position
    page boundary; the greedy continuation after the prompt is the same."""
    cfg = CFG.TINY_768
    w = reference_tiny_weights(cfg)
    prompt = [(11 * t + 5) % cfg["vocab"] for t in range(64)]
    a = model(gpu_ctx, cfg, w, 96, "f32")
    b = model(gpu_ctx, cfg, w, 96, "f32")
    got = []
    for i in range(0, len(prompt), n):
        lg, _ = a.step_positions(prompt[i:i + n])
        got += list(lg)
    worst = 0.0
    for t, tok in enumerate(prompt):
        lt, _, _, _ = b.step(tok)
        worst = max(worst, rel_l2(got[t], lt))
    assert worst <= 1e-5, f"worst position rel-L2 {worst:.2e}"
    a.decode(8)
    b.decode(8)
    assert a.pos == b.pos == 72
    la, _, _, _ = a.step(9)
    lb, _, _, _ = b.step(9)
    assert rel_l2(la, lb) <= 1e-5
    a.close()
    b.close()


def test_c3_prefill_by_32_position_steps_matches_token_by_token(gpu_ctx):
    """The C3 model (3B shape, bf16 KV, bench settings): 96 prompt ids in steps of 32 against the token-by-token chain,
    then 16 greedy steps of each.  At the first positions a token attends mostly to its own bf16 K/V row, so a 1-ulp
    f32 difference between the two paths can flip a stored rounding and grow through the layers (the same effect the
    bf16 real-prefill test in test_gpu_headline.py measures against the oracle): the gate is 2e-2, and the ids equal."""
    c = CFG.C3_3B
    cfg = c["model"]
    prompt = CFG.synthetic_tokens(96, c["prompt_seed"], cfg["vocab"])
    models = []
    for _ in range(2):
        m = LB.GpuModel(gpu_ctx, cfg, 128, kv_dtype="bf16")
        m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
        models.append(m)
    a, b = models
    got = []
    for i in range(0, 96, 32):
        lg, _ = a.step_positions(prompt[i:i + 32])
        got += list(lg)
    worst = 0.0
    for t, tok in enumerate(prompt):
        lt, _, _, _ = b.step(int(tok))
        worst = max(worst, rel_l2(got[t], lt))
    assert worst <= 2e-2, f"worst position rel-L2 {worst:.2e}"
    ta, tb = O.argmax_last(got[-1]), O.argmax_last(lt)
    assert ta == tb
    worst_g = 0.0
    for _ in range(16):
        la, ta, _, _ = a.step(ta)
        lb, tb, _, _ = b.step(tb)
        assert ta == tb
        worst_g = max(worst_g, rel_l2(la, lb))
    assert worst_g <= 2e-2
    print(f"C3 prefill by 32: worst position rel-L2 {worst:.2e}, greedy continuation {worst_g:.2e}")
    a.close()
    b.close()


def test_refusals_leave_the_model_usable(gpu_ctx):
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    m = model(gpu_ctx, cfg, w, 40, "bf16")
    for bad, code in (([], LB.E_ARG), ([1] * 33, LB.E_ARG), ([cfg["vocab"]], LB.E_ARG)):
        with pytest.raises(LB.LastroError) as e:
            m.step_positions(bad)
        assert e.value.code == code
    m.step_positions([1] * 32)
    with pytest.raises(LB.LastroError) as e:
        m.step_positions([2] * 9)
    assert e.value.code == LB.E_FULL
    lg, nxt = m.step_positions([3] * 8)
    assert np.isfinite(lg).all() and m.pos == 40
    m.close()
