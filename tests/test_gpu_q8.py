"""Q8_0 weights on the GPU (the C4 configuration) through the C ABI, against the CPU oracle's dequantised path.

The oracle itself is pinned by tests/test_q8.py (generator vs numpy, model vs transformers on the dequantised
weights).  Here the library's Q8_0 kernels are checked against it: the MoE block (router, gate_up, down) at the f32
block gate of the bf16 tests, the whole model (q/k/v, o-projection, router fold, experts) at the gates below, and the
device fill against the oracle's tensors bit for bit.

Gates.  The C4 weights (int8 ~U[-127,127] times an fp16 scale ~U(1e-4, 4e-3)) have a standard deviation near 0.17,
eight times the 0.02 of the bf16 models, and a model with such weights is chaotic: scaling one layer-0 norm weight
vector by (1 + 2e-7), the size of one f32 rounding, moves the oracle's own logits by up to 7.8e-6 / 2.3e-5 (tiny /
tiny768, f32 KV, 70 positions) and 1.9e-3 within 8 positions on the 3B-shaped C4 model, against 5e-7 on the bf16 C3
model.  With bf16 KV every such difference can flip a stored element's rounding, and the same perturbation grows to
1.4e-3 on tiny768 and 1.1e-1 (85% of routes kept) by position 7 on the C4 model (tests/test_q8.py::
test_q8_models_amplify_rounding pins the tiny figures).  So: the MoE block, which is not recurrent, keeps the 1e-5 f32
gate; the tiny models are compared over 70 positions at 1e-4 with f32 KV and over the first 16 positions at 5e-3 with
bf16 KV (against the oracle storing bf16-rounded K/V as the paged cache does); the C4 model itself with f32 KV at
1e-2.  bf16 KV storage is the same code for both weight types and is checked tightly on the bf16 models.  The north
star's bar for Q8_0 is 5e-2 on the MoE block and identical greedy tokens.
"""
import json
import os

import numpy as np
import pytest

import lastro_b200 as LB
import oracle as O
import synth_np as S
from helpers import rel_l2
from lastro_b200 import configs as CFG

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
TIE_GAP = 1e-3


def q8_model(ctx, cfg, max_len, kv, seed=12):
    m = LB.GpuModel(ctx, cfg, max_len, kv_dtype=kv)
    w = S.model_weights_q8(cfg, seed)
    m.load_weights(w)
    return m, w


@pytest.mark.parametrize("E,H,I,k", [(4, 256, 128, 2), (32, 1024, 512, 8), (40, 1536, 512, 8)])
def test_q8_block_matches_oracle(gpu_ctx, pool, E, H, I, k):
    """The Q8_0 MoE block (router, gate_up with SwiGLU, down with the weighted combine) against the oracle's
    dequantised block (cpu.rs:115-150 on weight = scale x value) for 6 tokens: routing identical, y within 1e-5."""
    router, gu, dn = S.q8_0(E, H, 11), S.q8_0(E * 2 * I, H, 12), S.q8_0(E * H, I, 13)
    layer = LB.GpuLayer(gpu_ctx, router, gu.reshape(E, 2 * I, -1), dn.reshape(E, H, -1), k)
    for t in range(6):
        x = S.values_f32(H, 40 + t, 1.0)
        y, ids, w, lg = layer.forward(x)
        yo, io, wo, lo = O.block_forward_w(pool, O.W_Q8_0, router, gu, dn, E, H, I, k, x)
        np.testing.assert_allclose(lg, lo, rtol=1e-5, atol=1e-5)
        assert ids.tolist() == io.tolist(), f"token {t}"
        np.testing.assert_allclose(w, wo, atol=2e-6)
        assert rel_l2(y, yo) < 1e-5, f"token {t}: {rel_l2(y, yo):.2e}"
    layer.close()


@pytest.mark.parametrize("kv,gate", [("f32", 1e-4), ("bf16", 5e-3)])
@pytest.mark.parametrize("base", ["tiny", "tiny768"])
def test_q8_model_matches_oracle(gpu_ctx, pool, kv, gate, base):
    cfg = dict(CFG.TINY if base == "tiny" else CFG.TINY_768, weight_dtype="q8_0")
    m, w = q8_model(gpu_ctx, cfg, 96, kv)
    om = O.Model(cfg, weights=w)
    s = O.Session(om, pool, 96, kv_bf16=kv == "bf16")
    toks = S.tokens(70 if kv == "f32" else 16, 5, cfg["vocab"])
    for t, tok in enumerate(toks):
        lg, nxt, ids, _ = m.step(int(tok))
        lo, io, _ = s.step(int(tok))
        assert rel_l2(lg, lo) < gate, f"position {t}: {rel_l2(lg, lo):.2e}"
        assert np.array_equal(ids, io), f"position {t}: routing"
        assert nxt == O.argmax_last(lg)
    s.close()
    om.close()
    m.close()


def test_q8_tiny_golden_greedy_and_teacher_forced(gpu_ctx):
    """tests/golden/tiny_q8.npz (transformers on the dequantised weights)."""
    g = np.load(os.path.join(GOLDEN, "tiny_q8.npz"))
    meta = json.loads(str(g["meta"]))
    cfg = meta["cfg"]
    m, _ = q8_model(gpu_ctx, cfg, 128, "f32", meta["seed"])
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


def test_q8_device_fill_equals_oracle_tensors(gpu_ctx):
    """fill_synthetic on the device and the upload of the oracle's synthetic tensors give bitwise-equal logits."""
    cfg = dict(CFG.TINY_768, weight_dtype="q8_0")
    a = LB.GpuModel(gpu_ctx, cfg, 32, kv_dtype="bf16")
    a.fill_synthetic(9, 0.3, 0.1)
    om = O.Model(cfg, synthetic_seed=9, std=0.3, norm_std=0.1, threads=4)
    H, I, E, V = cfg["hidden"], cfg["inter"], cfg["experts"], cfg["vocab"]
    qd, kvd = cfg["heads"] * 64, cfg["kv_heads"] * 64
    nb = lambda c: c // 32 * 34  # noqa: E731
    b = LB.GpuModel(gpu_ctx, cfg, 32, kv_dtype="bf16")
    b.load_tensor("model.embed_tokens.weight", om.tensor(-1, O.T_EMBED, V * H).reshape(V, H))
    b.load_tensor("model.norm.weight", om.tensor(-1, O.T_NORM, H, np.float32))
    shapes = {O.T_Q: (qd, nb(H)), O.T_K: (kvd, nb(H)), O.T_V: (kvd, nb(H)), O.T_O: (H, nb(qd)), O.T_ROUTER: (E, nb(H)),
              O.T_GATE_UP: (E, 2 * I, nb(H)), O.T_DOWN: (E, H, nb(I))}
    names = dict(zip((O.T_LN_ATTN, O.T_LN_MOE, O.T_Q, O.T_K, O.T_V, O.T_O, O.T_ROUTER, O.T_GATE_UP, O.T_DOWN),
                     LB.TENSOR_NAMES))
    for l in range(cfg["layers"]):
        for kind, name in names.items():
            if kind in shapes:
                arr = om.tensor(l, kind, int(np.prod(shapes[kind])), np.uint8).reshape(shapes[kind])
            else:
                arr = om.tensor(l, kind, H, np.float32)
            b.load_tensor(f"model.layers.{l}.{name}", arr)
    for tok in (3, 17, 5, 29):
        la, _, ia, _ = a.step(tok)
        lb, _, ib, _ = b.step(tok)
        assert np.array_equal(la, lb) and np.array_equal(ia, ib)
    a.close()
    b.close()
    om.close()


def test_c4_3b_q8_matches_oracle_at_full_size(gpu_ctx, pool):
    """The C4 model (Granite-3B shape, every linear Q8_0, device-filled weights bit-identical to the oracle's) against
    the oracle's dequantised path, f32 KV, over its first 6 positions: position 0 (no KV history: 32 layers of f32
    rounding only) within 1e-3, the next ones within 1e-2 while the chaos of these weights (module notes) is still
    below that; greedy ids identical except at top1-top2 gaps below 1e-2.  Longer sequences are compared on the
    tiny Q8_0 models, whose floor stays low for 70 positions."""
    c = CFG.C4_3B_Q8
    cfg = c["model"]
    m = LB.GpuModel(gpu_ctx, cfg, 64, kv_dtype="f32")
    m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.1)
    om = O.Model(cfg, synthetic_seed=c["weight_seed"], std=CFG.WEIGHT_STD, norm_std=0.1, threads=os.cpu_count() or 8)
    s = O.Session(om, pool, 64)
    for t, tok in enumerate(S.tokens(6, c["prompt_seed"], cfg["vocab"])):
        lg, nxt, ids, _ = m.step(int(tok))
        lo, io, _ = s.step(int(tok))
        assert rel_l2(lg, lo) < (1e-3 if t == 0 else 1e-2), f"position {t}: {rel_l2(lg, lo):.2e}"
        assert (ids == io).mean() > 0.98, f"position {t}"
        top2 = np.sort(lo)[-2:]
        assert nxt == O.argmax_last(lo) or top2[1] - top2[0] < 1e-2, f"position {t}: greedy id"
    s.close()
    om.close()
    m.close()


def test_c4_3b_q8_64_greedy_steps_state_synchronised(gpu_ctx):
    """bench.py's C4 model (every linear Q8_0, norm weights 1.0, a synthetic 512-position context filled identically on
    both sides) for 64 greedy steps.  These weights are chaotic (module notes): two free-running trajectories part
    after a few positions whatever the kernels do, so each step is compared from the same state -- after every step
    the K/V rows the GPU wrote replace the oracle's.  The cache is f32 here: within ONE step this model turns a bf16
    rounding flip of a stored K/V element (2^-9) into logits ~1e-1 apart (measured: 0.15 at the second step with bf16
    KV), so bf16 storage of the Q8_0 path is compared on the tiny models above.  Per step: the greedy id the oracle's
    except at top1-top2 gaps < 1e-2, layer 0's routing identical except at router gaps < 1e-4, and >= 95 % of all
    (layer, slot) ids equal.  Logits: within 5e-2 (the north star's Q8_0 bar) at every step whose 32 layers all route
    as the oracle does.  A deeper layer's router already sees an input that differs by the rounding the layers before
    it amplified, and a flip there (or a layer-0 flip at a gap < 1e-4) swaps one of the 8 experts of that layer's
    output: the step then follows another valid trajectory, and its logits are only held to 2.5e-1 (garbage sits
    near 1.4).  Measured: flip-free steps
    within 2.9e-3; 5 of 64 steps with a first flip at layers 13-25 (oracle k-th/(k+1)-th gaps 3e-4..1.5e-2), the
    largest logits deviation among them 6.6e-2.  A change of the attention's online-softmax grouping alone moves
    which steps flip (an earlier grouping: flip-free within 1.9e-2, flips at steps 28 and 53)."""
    c = CFG.C4_3B_Q8
    cfg = c["model"]
    n_ctx, steps = c["context"], 64
    threads = os.cpu_count() or 8
    m = LB.GpuModel(gpu_ctx, cfg, n_ctx + steps + 8, kv_dtype="f32")
    m.fill_synthetic(c["weight_seed"], CFG.WEIGHT_STD, 0.0)
    m.fill_kv_synthetic(n_ctx, c["prompt_seed"], 0.5)
    om = O.Model(cfg, synthetic_seed=c["weight_seed"], std=CFG.WEIGHT_STD, norm_std=0.0, threads=threads)
    pool = O.Pool(threads)
    s = O.Session(om, pool, n_ctx + steps + 8)
    s.fill_kv(n_ctx, c["prompt_seed"], 0.5)
    k0, v0 = m.read_kv(0, 0, n_ctx)
    assert np.array_equal(k0, s.kv(0)[0]) and np.array_equal(v0, s.kv(0)[1])
    tok = int(CFG.synthetic_tokens(1, c["prompt_seed"], cfg["vocab"])[0])
    worst, worst_flip, flips, same = 0.0, 0.0, [], []
    for t in range(steps):
        lg, nxt, ids, _ = m.step(tok)
        lo, io, _ = s.step(tok)
        rl = s.router_logits()
        err = rel_l2(lg, lo)
        flipped = [layer for layer in range(cfg["layers"]) if set(ids[layer].tolist()) != set(io[layer].tolist())]
        if flipped:
            assert err < 2.5e-1, f"step {t}: logits rel-L2 {err:.2e} after a route flip at layer {flipped[0]}"
            flips.append((t, flipped[0]))
            worst_flip = max(worst_flip, err)
        else:
            assert err < 5e-2, f"step {t}: logits rel-L2 {err:.2e} with every layer routed as the oracle"
            worst = max(worst, err)
        if not np.array_equal(ids[0], io[0]):
            j = int(np.argmax(ids[0] != io[0]))
            gap = abs(float(rl[0, io[0, j]]) - float(rl[0, ids[0, j]]))
            assert gap < 1e-4, f"step {t}: layer 0 slot {j} routes differ at router gap {gap:.2e}"
        same.append(float((ids == io).mean()))
        top2 = np.sort(lo)[-2:]
        assert nxt == O.argmax_last(lo) or top2[1] - top2[0] < 1e-2, f"step {t}: greedy {nxt}"
        pos = m.pos - 1
        for layer in range(cfg["layers"]):
            k, v = m.read_kv(layer, pos, 1)
            s.write_kv(layer, pos, k, v)
        tok = O.argmax_last(lo)
    print(f"C4 64 steps: worst logits rel-L2 {worst:.2e} (flip-free steps), {len(flips)} steps with a route flip "
          f"(step, first layer) {flips} (worst {worst_flip:.2e}), routes equal {np.mean(same):.4f} (min {min(same):.4f})")
    assert np.mean(same) >= 0.95 and len(flips) <= steps // 4
    s.close()
    pool.close()
    om.close()
    m.close()
