"""Model shapes and workloads of the Granite-MoE decode path.

The shapes are those of IBM Granite 3.0 1B-A400M / 3B-A800M (the models the
reference runtime serves, rust/moe-rt/src/model.rs:14-61 reads them from
config.json).  Weights are random-init (no checkpoints here): every tensor is
drawn from the library's synthetic generator with the seeds below, std 0.02
(transformers' initializer_range), RMSNorm weights 1.0 (transformers' init).
"""
import math

import numpy as np

# Granite muP multipliers (model.rs:1-7; values of the 1B/3B Granite 3.0 configs)
GRANITE_MUP = dict(embedding_multiplier=12.0, residual_multiplier=0.22, attention_multiplier=0.015625,
                   logits_scaling=6.0, eps=1e-6)

# Tiny synthetic Granite of the reference's own tests (rust/moe-rt/tests/common/mod.rs:79-87)
TINY = dict(hidden=256, inter=128, layers=2, heads=4, kv_heads=2, head_dim=64, vocab=33, experts=4, k=2,
            rope_theta=10000.0, eps=1e-6, embedding_multiplier=2.0, residual_multiplier=0.5,
            attention_multiplier=0.125, logits_scaling=4.0)

# The reference's H = 768 test model (tests/model.rs:127-134): the 3B shape in miniature
TINY_768 = dict(TINY, hidden=768, heads=12, kv_heads=4)

GRANITE_1B = dict(hidden=1024, inter=512, layers=24, heads=16, kv_heads=8, head_dim=64, vocab=49155, experts=32, k=8,
                  rope_theta=10000.0, **GRANITE_MUP)

GRANITE_3B = dict(hidden=1536, inter=512, layers=32, heads=24, kv_heads=8, head_dim=64, vocab=49155, experts=40, k=8,
                  rope_theta=10000.0, **GRANITE_MUP)

WEIGHT_STD = 0.02

# Workloads (BASELINE configs[0..4])
C1_BLOCK = dict(name="c1-block-1b", experts=32, hidden=1024, inter=512, k=8, weight_seed=0, x_seed=0xC1, tokens=8)
C2_1B = dict(name="c2-1b-greedy", model=GRANITE_1B, weight_seed=1, prompt_seed=1, prompt_len=128, new_tokens=128)
C3_3B = dict(name="c3-3b-ctx2048", model=GRANITE_3B, weight_seed=2, prompt_seed=2, context=2048, new_tokens=256)
GRANITE_3B_Q8 = dict(GRANITE_3B, weight_dtype="q8_0")
C4_3B_Q8 = dict(name="c4-3b-q8_0-ctx512", model=GRANITE_3B_Q8, weight_seed=4, prompt_seed=4, context=512,
                new_tokens=256)
C5_BATCH = dict(name="c5-3b-bs64-ctx1024", model=GRANITE_3B, weight_seed=3, prompt_seed=3, batch=64, context=1024,
                new_tokens=128, zipf_s=0.8)


def dims(cfg: dict) -> dict:
    d = dict(cfg)
    d["qd"] = cfg["heads"] * cfg["head_dim"]
    d["kvd"] = cfg["kv_heads"] * cfg["head_dim"]
    return d


def weight_bytes(cfg: dict) -> float:
    """HBM bytes per linear weight: 2 (bf16) or 34/32 (Q8_0: 32 int8 values and one fp16 scale per block)."""
    return 34 / 32 if cfg.get("weight_dtype", "bf16") == "q8_0" else 2


def bytes_per_token(cfg: dict, context: float, kv_bytes: int = 2) -> dict:
    """Algorithmic HBM bytes one batch-1 decode step reads (bf16 or Q8_0 linear weights, bf16 embedding).

    literal = active-expert weights + KV read; full = literal + router + attention
    projections + lm_head (the tied embedding) + norms.
    """
    H, I, L, E, k, V = cfg["hidden"], cfg["inter"], cfg["layers"], cfg["experts"], cfg["k"], cfg["vocab"]
    qd, kvd = cfg["heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    wb = weight_bytes(cfg)
    experts = L * k * 3 * I * H * wb
    kv = L * 2 * kvd * kv_bytes * context
    router = L * E * H * wb
    attn = L * (qd * H + 2 * kvd * H + H * qd) * wb
    head = V * H * 2
    norms = (2 * L + 1) * H * 4
    literal = experts + kv
    return dict(experts=experts, kv=kv, router=router, attn=attn, head=head, norms=norms, literal=literal,
                full=literal + router + attn + head + norms)


_GOLDEN = 0x9E3779B97F4A7C15
_MASK = (1 << 64) - 1


def _mix64(z: int) -> int:
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _MASK
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _MASK
    return z ^ (z >> 31)


def synthetic_tokens(n: int, seed: int, vocab: int) -> list:
    """Uniform random token ids: mix64(seed + (i + 1) * golden) % vocab (the generator of the synthetic weights)."""
    return [_mix64((seed + (i + 1) * _GOLDEN) & _MASK) % vocab for i in range(n)]


def zipf_router_bias(cfg: dict, s: float = 0.8, beta: float = 0.8, std: float = WEIGHT_STD) -> np.ndarray:
    """Router logit bias [layers, experts] that skews expert load towards Zipf(s) (the C5 workload).

    bias_e = beta * sigma * ln(p_e), p_e = (e + 1)^-s / sum, sigma = std * sqrt(hidden) the spread of the random router's
    logits.  With top-k routing an expert is chosen at most once per token, so the largest shares are capped; beta = 0.8
    minimises the L1 distance of the top-8 load shares to Zipf(0.8) for 40 experts (expert 0 gets ~10% of the
    token-expert pairs, experts 0-4 ~36%, against 16% and 43% for the uncapped distribution).
    """
    E = cfg["experts"]
    p = np.arange(1, E + 1, dtype=np.float64) ** -s
    p /= p.sum()
    b = beta * std * math.sqrt(cfg["hidden"]) * np.log(p)
    return np.tile(b.astype(np.float32), (cfg["layers"], 1))


def shard(total: int, rank: int, world: int) -> range:
    """Contiguous share of `total` items (sequences or experts) owned by `rank` of `world` (earlier ranks get the
    remainder first)."""
    base, extra = divmod(total, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (rank < extra))
