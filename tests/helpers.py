"""Shared test helpers: the reference's deterministic test data and comparison metrics."""
import numpy as np

import oracle as O


def values_py(n, seed):
    """rust/moe-rt/tests/common/mod.rs:28-38: xorshift values in [-1, 1) (exact in f32), in Python."""
    s = seed | 1
    out = np.empty(n, dtype=np.float32)
    M = (1 << 64) - 1
    for i in range(n):
        s ^= (s << 13) & M
        s ^= s >> 7
        s ^= (s << 17) & M
        out[i] = (s >> 40) / float(1 << 23) * 2.0 - 1.0
    return out


def values(n, seed):
    """The same values from the oracle's C restatement (checked against values_py in test_oracle)."""
    return O.ref_values(n, seed)


def bf(v):
    return O.f32_to_bf16(np.asarray(v, dtype=np.float32))


def rel_l2(got, want):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    return float(np.sqrt(((got - want) ** 2).sum() / max((want ** 2).sum(), 1e-300)))


def synthetic_layer(e, h, i):
    """tests/block.rs:182-202: router values(.,1), gate_up values(.,2)*0.1, down values(.,3)*0.1 (bf16 bits)."""
    router = bf(values(e * h, 1)).reshape(e, h)
    gu = bf(values(e * 2 * i * h, 2) * np.float32(0.1)).reshape(e, 2 * i, h)
    dn = bf(values(e * h * i, 3) * np.float32(0.1)).reshape(e, h, i)
    return router, gu, dn


def naive_block(router, gu, dn, x, k):
    """tests/block.rs:204-219: the block in f64."""
    I = dn.shape[2]
    f = lambda b: O.bf16_to_f32(b).astype(np.float64)
    logits = (f(router) @ x.astype(np.float64)).astype(np.float32)
    ids, w = O.routing(logits, k)
    y = np.zeros(router.shape[1])
    for e, g in zip(ids, w):
        hh = f(gu[e]) @ x.astype(np.float64)
        a = hh[:I] / (1.0 + np.exp(-hh[:I])) * hh[I:]
        y += float(g) * (f(dn[e]) @ a)
    return y, ids


def reference_tiny_weights(cfg, attn=0.1):
    """tests/common/mod.rs:94-131 tiny_model_attn: seed 10, each tensor values(n, ++seed) * scale, norms 1 + x."""
    H, I, E, V, d = cfg["hidden"], cfg["inter"], cfg["experts"], cfg["vocab"], cfg["head_dim"]
    qd, kvd = cfg["heads"] * d, cfg["kv_heads"] * d
    seed = [10]

    def w(n, scale):
        seed[0] += 1
        return bf(values(n, seed[0]) * np.float32(scale))

    def norm(b):
        return (O.bf16_to_f32(b) + np.float32(1.0)).astype(np.float32)

    def norm_f32(b):
        # bf16::from_f32(1.0 + x) widened back to f32 (model.rs:95-97)
        return O.bf16_to_f32(O.f32_to_bf16(norm(b)))

    out = dict(embed=w(V * H, 1.0).reshape(V, H), norm=norm_f32(w(H, 0.1)), layers=[])
    for _ in range(cfg["layers"]):
        lw = dict(ln_attn=norm_f32(w(H, 0.1)), ln_moe=norm_f32(w(H, 0.1)),
                  q=w(qd * H, attn).reshape(qd, H), k=w(kvd * H, attn).reshape(kvd, H),
                  v=w(kvd * H, attn).reshape(kvd, H), o=w(H * qd, attn).reshape(H, qd),
                  router=w(E * H, 0.5).reshape(E, H), gate_up=w(E * 2 * I * H, 0.1).reshape(E, 2 * I, H),
                  down=w(E * H * I, 0.1).reshape(E, H, I))
        out["layers"].append(lw)
    return out


def exact_logit_router(logits, H):
    """Router rows whose GEMV against x = [1, 1, 1, 0, ...] reproduces `logits` exactly: each f32 value is split
    into three bf16 terms (8 + 8 + 8 mantissa bits) summed in order."""
    v = np.asarray(logits, np.float32)
    b0 = O.f32_to_bf16(v)
    r1 = (v - O.bf16_to_f32(b0)).astype(np.float32)
    b1 = O.f32_to_bf16(r1)
    r2 = (r1 - O.bf16_to_f32(b1)).astype(np.float32)
    b2 = O.f32_to_bf16(r2)
    assert np.array_equal((O.bf16_to_f32(b0) + O.bf16_to_f32(b1)) + O.bf16_to_f32(b2), v)
    w = np.zeros((v.size, H), np.uint16)
    w[:, 0], w[:, 1], w[:, 2] = b0, b1, b2
    x = np.zeros(H, np.float32)
    x[:3] = 1.0
    return w, x


def first_route_difference(ids, ids_ref, logits_ref, tol=1e-4):
    """Compares per-layer routes ([layers, k] ids) against the reference's and its router logits [layers, experts].

    Returns None when every layer routes the same, else (layer, slot, gap) of the first difference, where gap is the
    reference's logit difference between the expert it chose at that slot and the one chosen instead -- a difference
    the north star allows when the gap is below 1e-4 (the two sides then round differently across the tie), after
    which the sequence's later layers and positions legitimately diverge.
    """
    for l in range(ids.shape[0]):
        if np.array_equal(ids[l], ids_ref[l]):
            continue
        j = int(np.argmax(ids[l] != ids_ref[l]))
        gap = abs(float(logits_ref[l, ids_ref[l, j]]) - float(logits_ref[l, ids[l, j]]))
        return l, j, gap
    return None
