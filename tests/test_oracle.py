"""Pin the CPU oracle against the reference's own known-answer tests (no GPU).

Each test restates a test of brenoperucchi/lastro-rust (file:line given) against the C oracle, so the oracle is
checked on the same cases before it is used to check the CUDA library.
"""
import numpy as np
import pytest

import oracle as O
import synth_np as S


from helpers import reference_tiny_weights, values, values_py  # noqa: E402
from lastro_b200 import configs as CFG  # noqa: E402


def bf(v):
    return O.f32_to_bf16(np.asarray(v, dtype=np.float32))


def test_router_top_k_order_and_lowest_index_tie_break():
    """tests/block.rs:13-23"""
    ids, w = O.routing(np.array([0.5, 2.0, -1.0, 2.0, 1.0], np.float32), 3)
    assert ids.tolist() == [1, 3, 4]
    ex = np.exp(np.array([2.0, 2.0, 1.0], np.float32))
    np.testing.assert_allclose(w, ex / ex.sum(), atol=1e-6)
    assert abs(w.sum() - 1.0) < 1e-6


def test_swiglu_known_answer():
    """tests/block.rs:121-129"""
    a = O.swiglu(np.array([0.0, 1.0, -2.0, 3.0, 4.0, 5.0], np.float32))
    silu = lambda g: g / (1.0 + np.exp(-g))
    np.testing.assert_allclose(a, [silu(0.0) * 3.0, silu(1.0) * 4.0, silu(-2.0) * 5.0], atol=1e-6)


def test_rmsnorm_known_answer():
    """tests/model.rs:49-54"""
    y = O.rmsnorm(np.array([3.0, 4.0], np.float32), np.array([1.0, 2.0], np.float32), 0.0)
    r = np.sqrt(12.5)
    assert abs(y[0] - 3.0 / r) < 1e-6 and abs(y[1] - 8.0 / r) < 1e-6


def test_rope_position_zero_is_identity_and_matches_f64():
    """tests/model.rs:26-47 (tiny config: head_dim 64, theta 1e4)"""
    d = 64
    x = values(2 * d, 5)
    assert np.array_equal(O.rope(x, d, O.rope_cos_sin(10000.0, d, 0)), x)
    pos, half = 7, d // 2
    y = O.rope(x, d, O.rope_cos_sin(10000.0, d, pos))
    for head in range(2):
        for j in range(half):
            a = pos * (1.0 / 10000.0 ** ((2 * j) / d))
            x1, x2 = float(x[head * d + j]), float(x[head * d + j + half])
            assert abs(y[head * d + j] - (x1 * np.cos(a) - x2 * np.sin(a))) < 1e-5
            assert abs(y[head * d + j + half] - (x2 * np.cos(a) + x1 * np.sin(a))) < 1e-5


@pytest.mark.parametrize("n", [0, 1, 7, 31, 32, 33, 64, 100, 1024, 1029])
def test_dot_matches_f64_with_and_without_remainder_of_32(n):
    """tests/block.rs:39-48; the SIMD and portable paths must also agree bit for bit."""
    w = bf(values(n, 3 + n))
    x = values(n, 9)
    want = float(np.dot(O.bf16_to_f32(w).astype(np.float64), x.astype(np.float64)))
    got = O.dot(w, x)
    assert abs(got - want) <= 1e-5 * (1.0 + abs(want))
    assert got == O.dot(w, x, portable=True)


@pytest.mark.parametrize("rows,cols,threads", [(7, 13, 3), (3, 64, 8), (64, 1024, 4), (1, 5, 1)])
def test_gemv_matches_f64(rows, cols, threads):
    """tests/block.rs:25-37"""
    w = bf(values(rows * cols, 11 + rows))
    x = values(cols, 7)
    p = O.Pool(threads)
    y = O.gemv(p, w, rows, cols, x)
    p.close()
    want = O.bf16_to_f32(w).astype(np.float64).reshape(rows, cols) @ x.astype(np.float64)
    assert np.all(np.abs(y - want) <= 1e-5 * (1.0 + np.abs(want)))


def naive_block(router, gu, dn, x, k):
    """tests/block.rs:204-219: the block in f64 (routing from f64 logits rounded to f32)."""
    E, H = router.shape
    I = dn.shape[2]
    f = lambda b: O.bf16_to_f32(b).astype(np.float64)
    logits = (f(router) @ x.astype(np.float64)).astype(np.float32)
    ids, w = O.routing(logits, k)
    y = np.zeros(H)
    for e, g in zip(ids, w):
        hh = f(gu[e]) @ x.astype(np.float64)
        a = hh[:I] / (1.0 + np.exp(-hh[:I])) * hh[I:]
        y += float(g) * (f(dn[e]) @ a)
    return y, ids


def rel_l2(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.sqrt(((got - want) ** 2).sum() / (want ** 2).sum()))


def synthetic_layer(e, h, i):
    """tests/block.rs:182-202 weights (router values(.,1), gate_up values(.,2)*0.1, down values(.,3)*0.1)."""
    router = bf(values(e * h, 1)).reshape(e, h)
    gu = bf(values(e * 2 * i * h, 2) * np.float32(0.1)).reshape(e, 2 * i, h)
    dn = bf(values(e * h * i, 3) * np.float32(0.1)).reshape(e, h, i)
    return router, gu, dn


def test_block_on_cpu_matches_naive_f64(pool):
    """tests/block.rs:227-239"""
    router, gu, dn = synthetic_layer(6, 24, 10)
    for t in range(4):
        x = values(24, 100 + t)
        y, ids, w, _ = O.block_forward(pool, router, gu, dn, 6, 24, 10, 2, x)
        want, wids = naive_block(router, gu, dn, x, 2)
        assert ids.tolist() == wids.tolist()
        assert rel_l2(y, want) < 1e-5


# ---- route.rs:130-269: eight logit families, E = 32 and 40, and the mutants that must be caught ----------------------

def lcg_logits(state):
    """route.rs:145-149: signed logits in [-8, 8)."""
    state[0] = (state[0] * 6364136223846793005 + 1442695040888963407) & 0xFFFFFFFFFFFFFFFF
    v = (state[0] >> 32) & 0xFFFFFFFF
    v = v - (1 << 32) if v >= (1 << 31) else v
    return np.float32(np.float32(v) / np.float32(1 << 31) * np.float32(8.0))


FAMILIES = ["distinct", "ties", "negative", "spread", "all_equal_-1e30", "all_equal_-2e30", "two_max", "tie_at_cut"]


def family_logits(kind, e, state):
    v = np.array([lcg_logits(state) for _ in range(e)], dtype=np.float32)
    if kind == "ties":
        v = np.floor(v * 2.0) / 2.0
    elif kind == "negative":
        v = v - 10.0
    elif kind == "spread":
        v = v * 12.0
    elif kind == "all_equal_-1e30":
        v[:] = -1.0e30
    elif kind == "all_equal_-2e30":
        v[:] = -2.0e30
    elif kind == "two_max":
        v = v - 20.0
        v[e - 1] = 5.0
        v[3] = 5.0
    elif kind == "tie_at_cut":
        v = v - 20.0
        for r, i in enumerate([0, 1, 2, 3, 4, 6, 7]):
            v[i] = 10.0 - r
        for i in (5, 9, 20):
            v[i] = 1.0
    return v.astype(np.float32)


def reference_topk(v, k, highest_index_first=False):
    """Routing::from_logits by sorting (block.rs:82-84); the mutant breaks ties by the highest index instead."""
    key = (lambda i: (-float(v[i]), -i)) if highest_index_first else (lambda i: (-float(v[i]), i))
    return sorted(range(len(v)), key=key)[:k]


def route_cases(n_per=20):
    state = [7]
    for kind in FAMILIES:
        for e in (32, 40):
            for _ in range(n_per):
                yield kind, e, family_logits(kind, e, state)


def test_oracle_routing_matches_sort_on_all_logit_families():
    for kind, e, v in route_cases():
        ids, w = O.routing(v, 8)
        assert ids.tolist() == reference_topk(v, 8), (kind, e)
        top = v[ids[0]]
        ex = np.exp((v[ids] - top).astype(np.float32))
        np.testing.assert_allclose(w, ex / ex.sum(), rtol=1e-6, atol=1e-7)


def test_tie_break_mutant_is_caught_only_on_tie_families():
    """route.rs:250-259 control: a highest-index tie-break differs from the oracle exactly on the families with ties."""
    bad = {k: 0 for k in FAMILIES}
    for kind, e, v in route_cases():
        ids, _ = O.routing(v, 8)
        if ids.tolist() != reference_topk(v, 8, highest_index_first=True):
            bad[kind] += 1
    has_ties = {"ties", "all_equal_-1e30", "all_equal_-2e30", "two_max", "tie_at_cut"}
    for kind, n in bad.items():
        assert (n > 0) == (kind in has_ties), (kind, bad)


def test_argmax_keeps_the_last_maximum():
    """bin/m1b-gulosa.rs:22-24 (Iterator::max_by keeps the last of equal maxima)"""
    assert O.argmax_last(np.array([1.0, 3.0, 2.0, 3.0, 0.5], np.float32)) == 3
    assert O.argmax_last(np.array([-0.0, 0.0], np.float32)) == 1
    assert O.argmax_last(np.array([0.0, -0.0], np.float32)) == 0  # total_cmp: +0 > -0


def test_synthetic_generator_matches_numpy_restatement():
    for seed in (0, 1, 2**40 + 7):
        assert np.array_equal(O.synth_bf16(50_000, seed, 0.02), S.values_bf16(50_000, seed, 0.02))
        assert np.array_equal(O.synth_f32(5000, seed, 0.1, 1.0), S.values_f32(5000, seed, 0.1, 1.0))
        assert np.array_equal(O.synth_tokens(100, seed, 49155), S.tokens(100, seed, 49155))
        for layer, kind in ((-1, 0), (0, 9), (31, 10)):
            assert O.tensor_seed(seed, layer, kind) == S.tensor_seed(seed, layer, kind)
    v = S.values_f32(1 << 20, 3, 0.02)
    assert abs(float(v.std()) - 0.02) < 2e-4 and abs(float(v.mean())) < 1e-4


def test_reference_test_data_generator_c_matches_python():
    for seed in (1, 2, 3, 11, 77, 300):
        assert np.array_equal(values(1000, seed), values_py(1000, seed))


def test_session_kv_bf16_stores_rounded_rows_of_the_f32_session(pool):
    """kv_bf16 sessions keep the K/V rows an f32 session computes, rounded to bf16 (RNE), as the paged bf16 cache
    stores them; the first position's rows are computed before any rounding can feed back, so they match exactly."""
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    m = O.Model(cfg, weights=w)
    a, b = O.Session(m, pool, 8), O.Session(m, pool, 8, kv_bf16=True)
    for tok in (3, 9, 1):
        a.step(tok)
        b.step(tok)
    for layer in range(cfg["layers"]):
        for fa, fb in zip(a.kv(layer), b.kv(layer)):
            assert not (fb.view(np.uint32) & 0xFFFF).any()  # bf16-representable
            want = S.bf16_to_f32(O.f32_to_bf16(fa[0]))
            assert np.array_equal(fb[0], want)
    for o in (a, b, m):
        o.close()
