"""ctypes wrapper of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle (``lastro_oracle.c``) restates the reference's CPU decode path
(``rust/moe-rt/src/{cpu.rs,block.rs,model.rs,pool.rs}`` of brenoperucchi/lastro-rust).
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this module, always as the checker or as the timed CPU baseline; the product
library never calls it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblastro_oracle.so")

_lib = None


def build() -> str:
    """Compile liblastro_oracle.so in place (gcc, a few seconds)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = _declare(C.CDLL(LIB_PATH))
    return _lib


class Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden", "inter", "layers", "heads", "kv_heads", "head_dim", "vocab",
                                         "experts", "k")] + \
               [(n, C.c_float) for n in ("rope_theta", "eps", "embedding_multiplier", "residual_multiplier",
                                         "attention_multiplier", "logits_scaling")] + \
               [("weight_dtype", C.c_int32)]


W_BF16, W_Q8_0 = 0, 1


class LayerWeights(C.Structure):
    _fields_ = [("ln_attn", C.c_void_p), ("ln_moe", C.c_void_p), ("q", C.c_void_p), ("k", C.c_void_p),
                ("v", C.c_void_p), ("o", C.c_void_p), ("router", C.c_void_p), ("gate_up", C.c_void_p),
                ("down", C.c_void_p)]


T_EMBED, T_NORM, T_LN_ATTN, T_LN_MOE, T_Q, T_K, T_V, T_O, T_ROUTER, T_GATE_UP, T_DOWN = range(11)

_P = C.c_void_p
_I = C.c_int32
_F = C.c_float
_U64 = C.c_uint64
_SZ = C.c_size_t


def _declare(L):
    sig = {
        "lo_mix64": (_U64, [_U64]),
        "lo_tensor_seed": (_U64, [_U64, _I, _I]),
        "lo_synth_value": (_F, [_U64, _U64, _F]),
        "lo_synth_scale": (_F, [_F]),
        "lo_synth_bf16": (None, [_P, _SZ, _U64, _F, _F, C.c_int]),
        "lo_synth_f32": (None, [_P, _SZ, _U64, _F, _F, C.c_int]),
        "lo_synth_tokens": (None, [_P, _SZ, _U64, _I]),
        "lo_ref_values": (None, [_P, _SZ, _U64]),
        "lo_f32_to_bf16": (C.c_uint16, [_F]),
        "lo_bf16_to_f32": (_F, [C.c_uint16]),
        "lo_pool_create": (_P, [C.c_int]),
        "lo_pool_destroy": (None, [_P]),
        "lo_pool_threads": (C.c_int, [_P]),
        "lo_dot": (_F, [_P, _P, _SZ]),
        "lo_dot_portable": (_F, [_P, _P, _SZ]),
        "lo_dot_q8": (_F, [_P, _P, _SZ]),
        "lo_dot_q8_portable": (_F, [_P, _P, _SZ]),
        "lo_f32_to_f16": (C.c_uint16, [_F]),
        "lo_f16_to_f32": (_F, [C.c_uint16]),
        "lo_synth_q8_0": (None, [_P, _SZ, _SZ, _U64, _I]),
        "lo_gemv_w": (None, [_P, _I, _P, _I, _I, _P, _P]),
        "lo_block_forward_w": (None, [_P, _I, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
        "lo_gemv": (None, [_P, _P, _I, _I, _P, _P]),
        "lo_swiglu": (None, [_P, _I, _P]),
        "lo_routing": (None, [_P, _I, _I, _P, _P]),
        "lo_experts": (None, [_P, _P, _I, _P, _P, _P, _I, _I, _P]),
        "lo_block_forward": (None, [_P, _P, _P, _P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
        "lo_rmsnorm": (None, [_P, _P, _I, _F, _P]),
        "lo_rope_cos_sin": (None, [_F, _I, _I, _P]),
        "lo_rope": (None, [_P, _I, _I, _P]),
        "lo_argmax_last": (_I, [_P, _I]),
        "lo_total_cmp": (C.c_int, [_F, _F]),
        "lo_model_create": (_P, [C.POINTER(Config), _P, _P, C.POINTER(LayerWeights)]),
        "lo_model_create_synthetic": (_P, [C.POINTER(Config), _U64, _F, _F, C.c_int]),
        "lo_model_destroy": (None, [_P]),
        "lo_model_set_router_bias": (None, [_P, _P]),
        "lo_model_tensor": (_P, [_P, _I, _I]),
        "lo_session_create": (_P, [_P, _P, _I]),
        "lo_session_destroy": (None, [_P]),
        "lo_session_reset": (None, [_P]),
        "lo_session_set_kv_bf16": (None, [_P, C.c_int32]),
        "lo_session_router_logits": (_P, [_P]),
        "lo_session_pos": (_I, [_P]),
        "lo_session_step": (C.c_int, [_P, _I, _P, _P, _P]),
        "lo_session_fill_kv": (C.c_int, [_P, _I, _U64, _F]),
        "lo_session_step_begin": (C.c_int, [_P, _I]),
        "lo_session_layer_attention": (None, [_P, _I, _P]),
        "lo_session_layer_moe": (None, [_P, _I, _P]),
        "lo_session_residual": (None, [_P, _P]),
        "lo_session_step_end": (None, [_P, _P]),
        "lo_session_k": (_P, [_P, _I]),
        "lo_session_v": (_P, [_P, _I]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    return L


def _ptr(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "arrays passed to the oracle must be C-contiguous"
    return a.ctypes.data_as(C.c_void_p)


# ---- synthetic data (the same formula as the device fill kernel) ----------------------------------------------------

def tensor_seed(base: int, layer: int, kind: int) -> int:
    return int(lib().lo_tensor_seed(base, layer, kind))


def synth_bf16(n: int, seed: int, std: float, mean: float = 0.0, threads: int = 8) -> np.ndarray:
    out = np.empty(n, dtype=np.uint16)
    lib().lo_synth_bf16(_ptr(out), n, seed, std, mean, threads)
    return out


def synth_f32(n: int, seed: int, std: float, mean: float = 0.0, threads: int = 8) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    lib().lo_synth_f32(_ptr(out), n, seed, std, mean, threads)
    return out


def synth_tokens(n: int, seed: int, vocab: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int32)
    lib().lo_synth_tokens(_ptr(out), n, seed, vocab)
    return out


def ref_values(n: int, seed: int) -> np.ndarray:
    """The reference's test data generator (tests/common/mod.rs:28-38)."""
    out = np.empty(n, dtype=np.float32)
    lib().lo_ref_values(_ptr(out), n, seed)
    return out


def bf16_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (finite inputs)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


# ---- thin object wrappers --------------------------------------------------------------------------------------------

class Pool:
    def __init__(self, threads: int):
        self.h = lib().lo_pool_create(threads)
        self.threads = threads

    def close(self):
        if self.h:
            lib().lo_pool_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


def synth_q8_0(rows: int, cols: int, seed: int, threads: int = 8) -> np.ndarray:
    """Synthetic Q8_0 matrix [rows, cols] as uint8 [rows, cols/32 * 34] (blocks: fp16 scale, 32 int8 values)."""
    out = np.empty((rows, cols // 32 * 34), dtype=np.uint8)
    lib().lo_synth_q8_0(_ptr(out), rows, cols, seed, threads)
    return out


def q8_dequant(q: np.ndarray) -> np.ndarray:
    """Q8_0 blocks [..., nb*34] -> f32 [..., nb*32], scale * value."""
    shp = q.shape[:-1]
    b = q.reshape(-1, 34)
    d = b[:, :2].copy().view(np.float16).astype(np.float32)
    v = b[:, 2:].view(np.int8).astype(np.float32)
    return (d * v).reshape(*shp, -1)


def dot_q8(row: np.ndarray, x: np.ndarray, portable: bool = False) -> float:
    f = lib().lo_dot_q8_portable if portable else lib().lo_dot_q8
    return float(f(_ptr(row), _ptr(x), x.size))


def f32_to_f16(v: float) -> int:
    return int(lib().lo_f32_to_f16(v))


def f16_to_f32(h: int) -> float:
    return float(lib().lo_f16_to_f32(h))


def dot(w: np.ndarray, x: np.ndarray, portable: bool = False) -> float:
    f = lib().lo_dot_portable if portable else lib().lo_dot
    return float(f(_ptr(w), _ptr(x), min(w.size, x.size)))


def gemv(pool: Pool, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    y = np.empty(rows, dtype=np.float32)
    lib().lo_gemv(pool.h, _ptr(w), rows, cols, _ptr(x), _ptr(y))
    return y


def swiglu(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.float32)
    a = np.empty(h.size // 2, dtype=np.float32)
    lib().lo_swiglu(_ptr(h), h.size // 2, _ptr(a))
    return a


def routing(logits: np.ndarray, k: int):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    ids = np.empty(k, dtype=np.int32)
    w = np.empty(k, dtype=np.float32)
    lib().lo_routing(_ptr(logits), logits.size, k, _ptr(ids), _ptr(w))
    return ids, w


def block_forward(pool: Pool, router, gate_up, down, experts: int, hidden: int, inter: int, k: int, x: np.ndarray):
    """HostLayer::forward_cpu (block.rs:56-62). Weights are bf16 bit arrays."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(hidden, dtype=np.float32)
    ids = np.empty(k, dtype=np.int32)
    w = np.empty(k, dtype=np.float32)
    logits = np.empty(experts, dtype=np.float32)
    lib().lo_block_forward(pool.h, _ptr(router), _ptr(gate_up), _ptr(down), experts, hidden, inter, k, _ptr(x),
                           _ptr(y), _ptr(ids), _ptr(w), _ptr(logits))
    return y, ids, w, logits


def block_forward_w(pool: Pool, dtype: int, router, gate_up, down, experts: int, hidden: int, inter: int, k: int,
                    x: np.ndarray):
    """block_forward for either weight type (W_BF16: uint16 bits; W_Q8_0: uint8 34-byte blocks along each row)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(hidden, dtype=np.float32)
    ids = np.empty(k, dtype=np.int32)
    w = np.empty(k, dtype=np.float32)
    logits = np.empty(experts, dtype=np.float32)
    router, gate_up, down = (np.ascontiguousarray(a) for a in (router, gate_up, down))
    lib().lo_block_forward_w(pool.h, dtype, _ptr(router), _ptr(gate_up), _ptr(down), experts, hidden, inter, k,
                             _ptr(x), _ptr(y), _ptr(ids), _ptr(w), _ptr(logits))
    return y, ids, w, logits


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    out = np.empty_like(x)
    lib().lo_rmsnorm(_ptr(x), _ptr(w), x.size, eps, _ptr(out))
    return out


def rope_cos_sin(theta: float, head_dim: int, pos: int) -> np.ndarray:
    cs = np.empty(head_dim, dtype=np.float32)
    lib().lo_rope_cos_sin(theta, head_dim, pos, _ptr(cs))
    return cs


def rope(x: np.ndarray, d: int, cs: np.ndarray) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True)
    lib().lo_rope(_ptr(y), y.size, d, _ptr(np.ascontiguousarray(cs, dtype=np.float32)))
    return y


def argmax_last(v: np.ndarray) -> int:
    v = np.ascontiguousarray(v, dtype=np.float32)
    return int(lib().lo_argmax_last(_ptr(v), v.size))


def make_config(d: dict) -> Config:
    vals = {f: d[f] for f, _ in Config._fields_ if f != "weight_dtype"}
    return Config(**vals, weight_dtype=W_Q8_0 if d.get("weight_dtype", "bf16") == "q8_0" else W_BF16)


class Model:
    """Whole-model oracle (model.rs HostModel + CpuSession)."""

    def __init__(self, cfg: dict, *, synthetic_seed: int | None = None, std: float = 0.02, norm_std: float = 0.0,
                 threads: int = 8, weights: dict | None = None):
        self.cfg = dict(cfg)
        self._c = make_config(cfg)
        self._keep = []
        if synthetic_seed is not None:
            self.h = lib().lo_model_create_synthetic(C.byref(self._c), synthetic_seed, std, norm_std, threads)
        else:
            assert weights is not None
            L = cfg["layers"]
            arr = (LayerWeights * L)()
            for l in range(L):
                lw = weights["layers"][l]
                vals = {}
                for name in ("ln_attn", "ln_moe", "q", "k", "v", "o", "router", "gate_up", "down"):
                    a = np.ascontiguousarray(lw[name])
                    self._keep.append(a)
                    vals[name] = a.ctypes.data
                arr[l] = LayerWeights(**vals)
            emb = np.ascontiguousarray(weights["embed"])
            norm = np.ascontiguousarray(weights["norm"], dtype=np.float32)
            self._keep += [emb, norm, arr]
            self.h = lib().lo_model_create(C.byref(self._c), _ptr(emb), _ptr(norm), arr)

    def set_router_bias(self, bias):
        """[layers, experts] f32 added to the router logits before every layer's routing (None removes it)."""
        if bias is None:
            lib().lo_model_set_router_bias(self.h, None)
            return
        b = np.ascontiguousarray(bias, dtype=np.float32)
        assert b.shape == (self.cfg["layers"], self.cfg["experts"])
        lib().lo_model_set_router_bias(self.h, _ptr(b))

    def tensor(self, layer: int, kind: int, count: int, dtype=np.uint16) -> np.ndarray:
        p = lib().lo_model_tensor(self.h, layer, kind)
        buf = (C.c_char * (count * np.dtype(dtype).itemsize)).from_address(p)
        return np.frombuffer(buf, dtype=dtype, count=count).copy()

    def close(self):
        if getattr(self, "h", None):
            lib().lo_model_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()


class Session:
    def __init__(self, model: Model, pool: Pool, max_len: int, kv_bf16: bool = False):
        """kv_bf16: K/V rows are rounded to bf16 when stored (a paged bf16 KV cache); f32 otherwise."""
        self.model = model
        self.pool = pool
        self.h = lib().lo_session_create(model.h, pool.h, max_len)
        lib().lo_session_set_kv_bf16(self.h, int(kv_bf16))
        c = model.cfg
        self.logits = np.empty(c["vocab"], dtype=np.float32)
        self.ids = np.empty(c["layers"] * c["k"], dtype=np.int32)
        self.w = np.empty(c["layers"] * c["k"], dtype=np.float32)

    def step(self, token: int):
        rc = lib().lo_session_step(self.h, int(token), _ptr(self.logits), _ptr(self.ids), _ptr(self.w))
        if rc != 0:
            raise ValueError("oracle step refused (KV full or token out of range)")
        c = self.model.cfg
        return self.logits.copy(), self.ids.reshape(c["layers"], c["k"]).copy(), self.w.reshape(c["layers"], c["k"]).copy()

    # CpuSession::step in phases, for a caller that runs every layer's MoE block itself (oracle/ep.py): begin, then
    # per layer in order layer_attention (returns the block's input xn) and layer_moe (x += resid * y), then end.
    def step_begin(self, token: int):
        if lib().lo_session_step_begin(self.h, int(token)) != 0:
            raise ValueError("oracle step refused (KV full or token out of range)")

    def layer_attention(self, layer: int) -> np.ndarray:
        xn = np.empty(self.model.cfg["hidden"], dtype=np.float32)
        lib().lo_session_layer_attention(self.h, layer, _ptr(xn))
        return xn

    def residual(self) -> np.ndarray:
        """The residual stream of the step in progress (between phases: the next layer's input)."""
        x = np.empty(self.model.cfg["hidden"], dtype=np.float32)
        lib().lo_session_residual(self.h, _ptr(x))
        return x

    def layer_moe(self, layer: int, y: np.ndarray):
        y = np.ascontiguousarray(y, dtype=np.float32)
        lib().lo_session_layer_moe(self.h, layer, _ptr(y))

    def step_end(self) -> np.ndarray:
        lib().lo_session_step_end(self.h, _ptr(self.logits))
        return self.logits.copy()

    def router_logits(self) -> np.ndarray:
        """[layers, experts] router logits of the last step (bias included)."""
        c = self.model.cfg
        n = c["layers"] * c["experts"]
        buf = (C.c_float * n).from_address(lib().lo_session_router_logits(self.h))
        return np.frombuffer(buf, dtype=np.float32, count=n).reshape(c["layers"], c["experts"]).copy()

    def fill_kv(self, n: int, seed: int, std: float):
        if lib().lo_session_fill_kv(self.h, n, seed, std) != 0:
            raise ValueError("fill_kv beyond max_len")

    def reset(self):
        lib().lo_session_reset(self.h)

    @property
    def pos(self) -> int:
        return int(lib().lo_session_pos(self.h))

    def kv(self, layer: int):
        c = self.model.cfg
        kvd = c["kv_heads"] * c["head_dim"]
        n = self.pos * kvd
        out = []
        for f in (lib().lo_session_k, lib().lo_session_v):
            p = f(self.h, layer)
            buf = (C.c_float * max(n, 1)).from_address(p)
            out.append(np.frombuffer(buf, dtype=np.float32, count=n).reshape(self.pos, kvd).copy())
        return out

    def write_kv(self, layer: int, pos: int, k: np.ndarray, v: np.ndarray):
        """Overwrite the cached K and V rows of position pos (< self.pos) of one layer (state-synchronised tests)."""
        c = self.model.cfg
        kvd = c["kv_heads"] * c["head_dim"]
        assert 0 <= pos < self.pos and k.size == kvd and v.size == kvd
        for f, row in ((lib().lo_session_k, k), (lib().lo_session_v, v)):
            src = np.ascontiguousarray(row, dtype=np.float32)
            C.memmove(f(self.h, layer) + pos * kvd * 4, src.ctypes.data, kvd * 4)

    def close(self):
        if getattr(self, "h", None):
            lib().lo_session_destroy(self.h)
            self.h = None

    def __del__(self):
        self.close()
