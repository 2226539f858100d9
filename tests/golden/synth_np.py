"""Independent numpy implementation of the synthetic generator (test infrastructure).

The same integer formula is implemented three times: in the CPU oracle
(``oracle/lastro_oracle.c``), in the library's device fill kernel
(``lastro-rust_b200/csrc/synth.cu``) and here.  The fixtures in this folder are
generated from this file, so a drift in either C implementation shows up as a
fixture mismatch.

value(seed, i) = (c0 + c1 + c2 + c3 - 131070) * (std / 37837.2265)
where c0..c3 are the four 16-bit chunks of mix64(seed + (i + 1) * GOLDEN); the
sum of four discrete uniforms is an Irwin-Hall(4) stand-in for N(0, std).
"""
import numpy as np

GOLDEN = np.uint64(0x9E3779B97F4A7C15)
M1 = np.uint64(0xBF58476D1CE4E5B9)
M2 = np.uint64(0x94D049BB133111EB)


def mix64(z):
    z = np.asarray(z, dtype=np.uint64)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * M1
        z = (z ^ (z >> np.uint64(27))) * M2
    return z ^ (z >> np.uint64(31))


def tensor_seed(base: int, layer: int, kind: int) -> int:
    with np.errstate(over="ignore"):
        v = np.uint64(base) * GOLDEN + np.uint64(((layer + 1) & 0xFFFFFFFF) << 8) + np.uint64(kind + 1)
    return int(mix64(v))


def scale(std: float) -> np.float32:
    return np.float32(std) / np.float32(37837.2265)


def values_f32(n: int, seed: int, std: float, mean: float = 0.0, chunk: int = 1 << 24) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    sc = scale(std)
    for s in range(0, n, chunk):
        idx = np.arange(s, min(n, s + chunk), dtype=np.uint64)
        with np.errstate(over="ignore"):
            h = mix64(np.uint64(seed) + (idx + np.uint64(1)) * GOLDEN)
        m = np.uint64(0xFFFF)
        tot = ((h & m) + ((h >> np.uint64(16)) & m) + ((h >> np.uint64(32)) & m) + (h >> np.uint64(48))).astype(np.int64)
        v = (tot - 131070).astype(np.float32) * sc
        if mean != 0.0:
            v = v + np.float32(mean)
        out[s:s + v.size] = v
    return out


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)
    return u.astype(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def values_bf16(n: int, seed: int, std: float, mean: float = 0.0) -> np.ndarray:
    return f32_to_bf16(values_f32(n, seed, std, mean))


def tokens(n: int, seed: int, vocab: int) -> np.ndarray:
    idx = np.arange(n, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = mix64(np.uint64(seed) + (idx + np.uint64(1)) * GOLDEN)
    return (h % np.uint64(vocab)).astype(np.int32)


# ---- whole-model weights (canonical layouts of rust/moe-rt/src/model.rs:99-132) ---------------------------------------
T_EMBED, T_NORM, T_LN_ATTN, T_LN_MOE, T_Q, T_K, T_V, T_O, T_ROUTER, T_GATE_UP, T_DOWN = range(11)

# per-tensor std of the tiny golden model: large enough that greedy decoding is not degenerate
TINY_STD = dict(embed=0.3, norm=0.1, attn=0.25, router=0.5, experts=0.8)


def bf16_f32(n, seed, std, mean=0.0):
    return bf16_to_f32(values_bf16(n, seed, std, mean))


def model_weights(cfg, seed, std, *, stds=None):
    """f32 arrays holding bf16 values; norms are 1 + noise (bf16) as checkpoints store them."""
    stds = stds or dict(embed=std, norm=0.0, attn=std, router=std, experts=std)
    H, I, E, V = cfg["hidden"], cfg["inter"], cfg["experts"], cfg["vocab"]
    qd, kvd = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    ts = tensor_seed
    w = dict(embed=bf16_f32(V * H, ts(seed, -1, T_EMBED), stds["embed"]).reshape(V, H),
             norm=bf16_f32(H, ts(seed, -1, T_NORM), stds["norm"], 1.0), layers=[])
    for l in range(cfg["layers"]):
        w["layers"].append(dict(
            ln_attn=bf16_f32(H, ts(seed, l, T_LN_ATTN), stds["norm"], 1.0),
            ln_moe=bf16_f32(H, ts(seed, l, T_LN_MOE), stds["norm"], 1.0),
            q=bf16_f32(qd * H, ts(seed, l, T_Q), stds["attn"]).reshape(qd, H),
            k=bf16_f32(kvd * H, ts(seed, l, T_K), stds["attn"]).reshape(kvd, H),
            v=bf16_f32(kvd * H, ts(seed, l, T_V), stds["attn"]).reshape(kvd, H),
            o=bf16_f32(H * qd, ts(seed, l, T_O), stds["attn"]).reshape(H, qd),
            router=bf16_f32(E * H, ts(seed, l, T_ROUTER), stds["router"]).reshape(E, H),
            gate_up=bf16_f32(E * 2 * I * H, ts(seed, l, T_GATE_UP), stds["experts"]).reshape(E, 2 * I, H),
            down=bf16_f32(E * H * I, ts(seed, l, T_DOWN), stds["experts"]).reshape(E, H, I)))
    return w


# ---- Q8_0: blocks of 32 int8 values with one fp16 scale, 34 bytes (scale, then values) ---------
def q8_0(rows: int, cols: int, seed: int) -> np.ndarray:
    """Synthetic Q8_0 matrix [rows, cols] as uint8 [rows, cols/32 * 34]: value of element i uniform in [-127, 127]
    from mix64(seed + (i + 1) * GOLDEN) % 255 - 127; scale of block b = fp16(1e-4 + u * 3.9e-3), u = 24 hash bits of
    mix64((seed ^ 0xA5..A5) + (b + 1) * GOLDEN) / 2^24 (f32 arithmetic, round to nearest even)."""
    nb = cols // 32
    idx = np.arange(rows * cols, dtype=np.uint64)
    with np.errstate(over="ignore"):
        h = mix64(np.uint64(seed) + (idx + np.uint64(1)) * GOLDEN)
        vals = ((h % np.uint64(255)).astype(np.int64) - 127).astype(np.int8).reshape(rows, nb, 32)
        bidx = np.arange(rows * nb, dtype=np.uint64)
        hb = mix64((np.uint64(seed) ^ np.uint64(0xA5A5A5A5A5A5A5A5)) + (bidx + np.uint64(1)) * GOLDEN)
    u = (hb >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)
    d = (np.float32(1e-4) + u * np.float32(3.9e-3)).astype(np.float16).reshape(rows, nb, 1)
    out = np.empty((rows, nb, 34), dtype=np.uint8)
    out[:, :, :2] = d.view(np.uint8)
    out[:, :, 2:] = vals.view(np.uint8)
    return out.reshape(rows, nb * 34)


def q8_dequant(q: np.ndarray) -> np.ndarray:
    """Q8_0 [..., nb*34] -> f32 [..., nb*32]: scale * value (exact in f32)."""
    shp = q.shape[:-1]
    b = np.ascontiguousarray(q).reshape(-1, 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    v = b[:, 2:].view(np.int8).astype(np.float32)
    return (d * v).reshape(*shp, -1)


def model_weights_q8(cfg, seed, *, embed_std=0.3, norm_std=0.1):
    """Q8_0 linear weights (uint8 blocks, the form the oracle and the library take), bf16 embedding (uint16 bits),
    f32 norms holding bf16 values; the same tensor seeds as model_weights."""
    H, I, E, V = cfg["hidden"], cfg["inter"], cfg["experts"], cfg["vocab"]
    qd, kvd = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    ts = tensor_seed
    w = dict(embed=values_bf16(V * H, ts(seed, -1, T_EMBED), embed_std).reshape(V, H),
             norm=bf16_f32(H, ts(seed, -1, T_NORM), norm_std, 1.0), layers=[])
    for l in range(cfg["layers"]):
        w["layers"].append(dict(
            ln_attn=bf16_f32(H, ts(seed, l, T_LN_ATTN), norm_std, 1.0),
            ln_moe=bf16_f32(H, ts(seed, l, T_LN_MOE), norm_std, 1.0),
            q=q8_0(qd, H, ts(seed, l, T_Q)), k=q8_0(kvd, H, ts(seed, l, T_K)), v=q8_0(kvd, H, ts(seed, l, T_V)),
            o=q8_0(H, qd, ts(seed, l, T_O)), router=q8_0(E, H, ts(seed, l, T_ROUTER)),
            gate_up=q8_0(E * 2 * I, H, ts(seed, l, T_GATE_UP)).reshape(E, 2 * I, -1),
            down=q8_0(E * H, I, ts(seed, l, T_DOWN)).reshape(E, H, -1)))
    return w


def dequant_model(wq):
    """The Q8_0 model of model_weights_q8 as f32 arrays (the dequantised path, for transformers)."""
    def conv(key, a):
        return a.astype(np.float32) if key.startswith("ln") else q8_dequant(a)
    return dict(embed=bf16_to_f32(wq["embed"]), norm=wq["norm"].astype(np.float32),
                layers=[{k: conv(k, v) for k, v in lw.items()} for lw in wq["layers"]])


def as_bits(w):
    """The same weights as bf16 bit arrays (uint16) with f32 norms, the form the oracle and the library take."""
    def conv(key, a):
        return a.astype(np.float32) if key.startswith("ln") or key == "norm" else f32_to_bf16(a)
    return dict(embed=f32_to_bf16(w["embed"]), norm=w["norm"].astype(np.float32),
                layers=[{k: conv(k, v) for k, v in lw.items()} for lw in w["layers"]])
