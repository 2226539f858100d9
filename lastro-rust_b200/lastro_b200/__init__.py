"""Python binding of liblastro_b200.so (ctypes over the C ABI in include/lastro_b200.h).

Mirrors the reference's operator API (rust/moe-rt/src/gpu.rs ``GpuLayer`` and gpu_model.rs ``GpuModel``) so
that tests and benchmarks read like the reference's own.  There is no fallback: if the CUDA library is missing or
no GPU is present, constructing a context raises.
"""
from __future__ import annotations

import ctypes as C
import sys
import os
import subprocess
import weakref

import numpy as np

from . import configs  # noqa: F401

PKG_DIR = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(PKG_DIR, "liblastro_b200.so")
HEADER = os.path.join(PKG_DIR, "..", "include", "lastro_b200.h")

OK, E_ARG, E_CUDA, E_POISONED, E_FULL, E_NOMEM, E_UNSUPPORTED, E_STATE, E_IO = range(9)
TRACE_WORDS = 11  # LASTRO_TRACE_WORDS: start, release, exit, 8 milestones per CTA
DTYPE_BF16, DTYPE_F32, DTYPE_Q8_0 = 1, 2, 3

_lib = None


class LastroError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def build(quiet: bool = True) -> str:
    """Compile liblastro_b200.so in place (nvcc, sm_100a)."""
    subprocess.run(["make", "-s" if quiet else "-j2", "-C", PKG_DIR], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)
    return LIB_PATH


class ModelDesc(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("hidden", "inter", "layers", "heads", "kv_heads", "head_dim", "vocab",
                                         "experts", "k")] + \
               [(n, C.c_float) for n in ("rope_theta", "eps", "embedding_multiplier", "residual_multiplier",
                                         "attention_multiplier", "logits_scaling")] + \
               [("weight_dtype", C.c_int32), ("kv_dtype", C.c_int32)]


EXPORTS = {
    "lastro_version": (C.c_char_p, []),
    "lastro_ctx_create": (C.c_int, [C.c_int32, C.c_void_p, C.POINTER(C.c_void_p)]),
    "lastro_ctx_destroy": (None, [C.c_void_p]),
    "lastro_ctx_synchronize": (C.c_int, [C.c_void_p]),
    "lastro_last_error": (C.c_char_p, [C.c_void_p]),
    "lastro_layer_create": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                      C.c_void_p, C.POINTER(C.c_void_p)]),
    "lastro_layer_create_q8_0": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                           C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    "lastro_layer_forward": (C.c_int, [C.c_void_p] + [C.c_void_p] * 5),
    "lastro_layer_add_into": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_void_p]),
    "lastro_layer_destroy": (None, [C.c_void_p]),
    "lastro_moe_block_forward_noalloc": (C.c_int, [C.c_void_p] * 4 + [C.c_int32] * 4 + [C.c_void_p] * 4),
    "lastro_moe_block_noalloc_status": (C.c_int, [C.c_void_p, C.c_void_p]),
    "lastro_model_create": (C.c_int, [C.c_void_p, C.POINTER(ModelDesc), C.c_int32, C.POINTER(C.c_void_p)]),
    "lastro_model_load_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int32, C.POINTER(C.c_int64), C.c_int32,
                                           C.c_void_p]),
    "lastro_model_fill_synthetic": (C.c_int, [C.c_void_p, C.c_uint64, C.c_float, C.c_float]),
    "lastro_model_fill_kv_synthetic": (C.c_int, [C.c_void_p, C.c_int32, C.c_uint64, C.c_float]),
    "lastro_model_read_kv": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "lastro_model_step": (C.c_int, [C.c_void_p, C.c_int32] + [C.c_void_p] * 4),
    "lastro_model_step_positions": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p]),
    "lastro_model_generate": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_void_p]),
    "lastro_model_generate_until": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_void_p,
                                              C.POINTER(C.c_int32)]),
    "lastro_model_decode": (C.c_int, [C.c_void_p, C.c_int32]),
    "lastro_model_reset": (C.c_int, [C.c_void_p]),
    "lastro_model_position": (C.c_int, [C.c_void_p, C.POINTER(C.c_int32)]),
    "lastro_model_profile": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32]),
    "lastro_model_trace": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32,
                                     C.c_void_p]),
    "lastro_model_set_options": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32]),
    "lastro_model_fused": (C.c_int, [C.c_void_p]),
    "lastro_model_set_moe": (C.c_int, [C.c_void_p, C.c_int32]),
    "lastro_model_moe": (C.c_int, [C.c_void_p]),
    "lastro_model_set_tuning": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32]),
    "lastro_model_trace_raw": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32]),
    "lastro_model_set_attention": (C.c_int, [C.c_void_p, C.c_int32]),
    "lastro_model_destroy": (None, [C.c_void_p]),
    "lastro_checkpoint_open": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_int32]),
    "lastro_checkpoint_close": (None, [C.c_void_p]),
    "lastro_checkpoint_count": (C.c_int, [C.c_void_p]),
    "lastro_checkpoint_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_char_p, C.c_int32, C.c_void_p, C.c_int32,
                                           C.POINTER(C.c_int32)]),
    "lastro_checkpoint_read_bf16": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_int64, C.c_char_p, C.c_int32]),
    "lastro_config_from_json": (C.c_int, [C.c_char_p, C.c_void_p, C.c_char_p, C.c_int32]),
    "lastro_checkpoint_config": (C.c_int, [C.c_void_p, C.c_void_p, C.c_char_p, C.c_int32]),
    "lastro_model_load_checkpoint": (C.c_int, [C.c_void_p, C.c_void_p]),
    "lastro_tokenizer_load": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p), C.c_char_p, C.c_int32]),
    "lastro_tokenizer_from_json": (C.c_int, [C.c_char_p, C.c_size_t, C.POINTER(C.c_void_p), C.c_char_p, C.c_int32]),
    "lastro_tokenizer_destroy": (None, [C.c_void_p]),
    "lastro_tokenizer_vocab_size": (C.c_int32, [C.c_void_p]),
    "lastro_tokenizer_encode": (C.c_int, [C.c_void_p, C.c_char_p, C.c_size_t, C.c_void_p, C.c_int32,
                                          C.POINTER(C.c_int32)]),
    "lastro_tokenizer_decode_bytes": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_char_p, C.c_size_t,
                                                C.POINTER(C.c_size_t)]),
    "lastro_tokenizer_decode": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32, C.c_char_p, C.c_size_t,
                                          C.POINTER(C.c_size_t)]),
    "lastro_tokenizer_pretokenize": (C.c_int, [C.c_char_p, C.c_size_t, C.c_void_p, C.c_int32, C.POINTER(C.c_int32)]),
    "lastro_chat_render": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int32, C.c_int32, C.c_char_p, C.c_char_p,
                                     C.c_size_t, C.POINTER(C.c_size_t)]),
    "lastro_format_date": (C.c_int, [C.c_int32, C.c_int32, C.c_int32, C.c_char_p, C.c_int32]),
    "lastro_batch_create": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.POINTER(C.c_void_p)]),
    "lastro_batch_exchange_handle": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32]),
    "lastro_batch_connect": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32]),
    "lastro_batch_set_router_bias": (C.c_int, [C.c_void_p, C.c_void_p]),
    "lastro_batch_set_expert_placement": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int32]),
    "lastro_batch_step": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p,
                                    C.c_void_p]),
    "lastro_batch_decode": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p]),
    "lastro_batch_fill_kv_synthetic": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_uint64, C.c_float]),
    "lastro_batch_reset": (C.c_int, [C.c_void_p, C.c_int32]),
    "lastro_batch_position": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(C.c_int32)]),
    "lastro_batch_set_options": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int32]),
    "lastro_batch_profile": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p,
                                       C.c_int32]),
    "lastro_batch_set_wait_limit": (C.c_int, [C.c_void_p, C.c_uint64]),
    "lastro_batch_trace": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p, C.c_int32, C.c_void_p, C.c_void_p,
                                     C.c_void_p, C.c_int32, C.c_void_p]),
    "lastro_batch_trace_raw": (C.c_int, [C.c_void_p, C.c_int32, C.c_void_p, C.c_int32]),
    "lastro_batch_destroy": (None, [C.c_void_p]),
}

HANDLE_BYTES = 64  # cudaIpcMemHandle_t


def lib():
    """Load the in-tree CUDA library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: run `make -C lastro-rust_b200` (or __graft_entry__.build())")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in EXPORTS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


class Context:
    """One device and one stream (the reference's Arc<Stream>)."""

    def __init__(self, device: int = 0, stream: int | None = None):
        h = C.c_void_p()
        rc = lib().lastro_ctx_create(device, stream, C.byref(h))
        if rc != OK:
            raise LastroError(rc, f"lastro_ctx_create(device={device}) failed: no usable CUDA device")
        self.h = h
        # objects created on this context; they are destroyed before it (the C ABI requires that order)
        self._children = weakref.WeakSet()

    def check(self, rc: int):
        if rc != OK:
            raise LastroError(rc, lib().lastro_last_error(self.h).decode())

    def synchronize(self):
        self.check(lib().lastro_ctx_synchronize(self.h))

    def close(self):
        if getattr(self, "h", None):
            for child in list(self._children):
                child.close()
            lib().lastro_ctx_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        # at interpreter exit (module globals already cleared) the process's CUDA context goes with the process
        if getattr(self, "h", None) and not _finalizing():
            self.close()


class GpuLayer:
    """MoE block with every expert resident (gpu.rs GpuLayer).

    bf16 weights as uint16 bit arrays router [E,H], gate_up [E,2I,H], down [E,H,I]; or Q8_0 weights as uint8 arrays
    whose last axis holds each row's 34-byte blocks (router [E, H/32*34], gate_up [E, 2I, H/32*34], down
    [E, H, I/32*34])."""

    def __init__(self, ctx: Context, router: np.ndarray, gate_up: np.ndarray, down: np.ndarray, k: int):
        q8 = router.dtype == np.uint8
        E = router.shape[0]
        H = router.shape[1] // 34 * 32 if q8 else router.shape[1]
        I = gate_up.shape[1] // 2
        want_gu = (E, 2 * I, H // 32 * 34 if q8 else H)
        want_dn = (E, H, I // 32 * 34 if q8 else I)
        assert gate_up.shape == want_gu and down.shape == want_dn, (gate_up.shape, down.shape)
        self.ctx, self.E, self.H, self.I, self.k, self.q8 = ctx, E, H, I, k, q8
        h = C.c_void_p()
        r, g, d = (np.ascontiguousarray(a, dtype=np.uint8 if q8 else np.uint16) for a in (router, gate_up, down))
        create = lib().lastro_layer_create_q8_0 if q8 else lib().lastro_layer_create
        ctx.check(create(ctx.h, E, H, I, k, _p(r), _p(g), _p(d), C.byref(h)))
        self.h = h
        ctx._children.add(self)

    def forward(self, x: np.ndarray):
        """(y, ids, weights, logits) for one token, host in/out (GpuLayer::forward)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty(self.H, np.float32)
        ids = np.empty(self.k, np.int32)
        w = np.empty(self.k, np.float32)
        lg = np.empty(self.E, np.float32)
        self.ctx.check(lib().lastro_layer_forward(self.h, _p(x), _p(y), _p(ids), _p(w), _p(lg)))
        return y, ids, w, lg

    def add_into(self, xn_ptr: int, h_ptr: int, resid: float, ids_ptr: int | None = None, w_ptr: int | None = None):
        self.ctx.check(lib().lastro_layer_add_into(self.h, xn_ptr, h_ptr, resid, ids_ptr, w_ptr))

    def close(self):
        if getattr(self, "h", None):
            lib().lastro_layer_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        # at interpreter exit (module globals already cleared) the process's CUDA context goes with the process
        if getattr(self, "h", None) and not _finalizing():
            self.close()


def moe_block_forward_noalloc(x: int, router: int, gate_up: int, down: int, experts: int, hidden: int, inter: int,
                              k: int, y: int, ids: int, weights: int, stream: int | None = None) -> int:
    """Allocation-free MoE block on device pointers (lastro_moe_block_forward_noalloc); returns the status code."""
    return lib().lastro_moe_block_forward_noalloc(x, router, gate_up, down, experts, hidden, inter, k, y, ids, weights,
                                                  stream)


def moe_block_noalloc_status(status: int, stream: int | None = None) -> int:
    """Enqueue a copy of the allocation-free block's error word into caller memory at `status`
    (lastro_moe_block_noalloc_status); returns the status code of the call itself."""
    return lib().lastro_moe_block_noalloc_status(status, stream)


DESC_KEYS = ("hidden", "inter", "layers", "heads", "kv_heads", "head_dim", "vocab", "experts", "k", "rope_theta",
             "eps", "embedding_multiplier", "residual_multiplier", "attention_multiplier", "logits_scaling")


def _desc_dict(d: "ModelDesc") -> dict:
    return {k: getattr(d, k) for k in DESC_KEYS}


def config_from_json(text: str) -> dict:
    """Config::from_json (model.rs:34-61) through the C ABI: the model config dict, or LastroError with the reason."""
    d = ModelDesc()
    err = C.create_string_buffer(512)
    rc = lib().lastro_config_from_json(text.encode(), C.byref(d), err, len(err))
    if rc != OK:
        raise LastroError(rc, err.value.decode())
    return _desc_dict(d)


class Checkpoint:
    """A safetensors checkpoint directory (weights.rs Checkpoint): index on open, tensors read on request.  Host-only."""

    def __init__(self, path: str):
        h = C.c_void_p()
        err = C.create_string_buffer(512)
        rc = lib().lastro_checkpoint_open(os.fsencode(path), C.byref(h), err, len(err))
        if rc != OK:
            raise LastroError(rc, err.value.decode())
        self.h, self.path = h, path

    def __len__(self):
        return lib().lastro_checkpoint_count(self.h)

    def info(self, name: str):
        """(dtype, shape) of one tensor, or None when absent."""
        dt = C.create_string_buffer(32)
        shape = (C.c_int64 * 8)()
        nd = C.c_int32()
        if lib().lastro_checkpoint_tensor(self.h, name.encode(), dt, len(dt), shape, 8, C.byref(nd)) != OK:
            return None
        return dt.value.decode(), tuple(shape[i] for i in range(min(nd.value, 8)))

    def bf16(self, name: str) -> np.ndarray:
        """Checkpoint::bf16: the tensor's bf16 bits (uint16) with its shape."""
        inf = self.info(name)
        shape = inf[1] if inf else ()
        n = int(np.prod(shape)) if inf and all(d >= 0 for d in shape) and np.prod([float(d) for d in shape]) < 2**40 else 0
        out = np.empty(max(n, 1), np.uint16)
        err = C.create_string_buffer(512)
        rc = lib().lastro_checkpoint_read_bf16(self.h, name.encode(), _p(out), n, err, len(err))
        if rc != OK:
            raise LastroError(rc, err.value.decode())
        return out[:n].reshape(shape)

    def config(self) -> dict:
        d = ModelDesc()
        err = C.create_string_buffer(512)
        rc = lib().lastro_checkpoint_config(self.h, C.byref(d), err, len(err))
        if rc != OK:
            raise LastroError(rc, err.value.decode())
        return _desc_dict(d)

    def close(self):
        if getattr(self, "h", None):
            lib().lastro_checkpoint_close(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        # at interpreter exit (module globals already cleared) the process's CUDA context goes with the process
        if getattr(self, "h", None) and not _finalizing():
            self.close()


class Tokenizer:
    """Byte-level BPE tokenizer of a Granite 3.1 tokenizer.json (tokenizador.rs Tokenizador).  Host-only."""

    def __init__(self, path: str | None = None, *, json_text: str | bytes | None = None):
        h = C.c_void_p()
        err = C.create_string_buffer(512)
        if path is not None:
            rc = lib().lastro_tokenizer_load(os.fsencode(path), C.byref(h), err, len(err))
        else:
            raw = json_text.encode() if isinstance(json_text, str) else bytes(json_text)
            rc = lib().lastro_tokenizer_from_json(raw, len(raw), C.byref(h), err, len(err))
        if rc != OK:
            raise LastroError(rc, err.value.decode())
        self.h = h

    @property
    def vocab_size(self) -> int:
        return lib().lastro_tokenizer_vocab_size(self.h)

    def encode(self, text: str) -> list[int]:
        """codifica: text -> ids (no BOS), as `tokenizers` encodes it."""
        raw = text.encode("utf-8")
        n = C.c_int32()
        lib().lastro_tokenizer_encode(self.h, raw, len(raw), None, 0, C.byref(n))
        out = np.empty(max(n.value, 1), np.int32)
        rc = lib().lastro_tokenizer_encode(self.h, raw, len(raw), _p(out), out.size, C.byref(n))
        if rc != OK:
            raise LastroError(rc, "encode")
        return out[:n.value].tolist()

    def _decode(self, fn, ids) -> bytes:
        a = np.ascontiguousarray(np.asarray(ids, np.int32).reshape(-1))
        n = C.c_size_t()
        rc = fn(self.h, _p(a), a.size, None, 0, C.byref(n))
        if rc != OK and n.value == 0 and a.size:
            raise LastroError(rc, "decode: an id outside the vocabulary")
        buf = C.create_string_buffer(max(n.value, 1))
        rc = fn(self.h, _p(a), a.size, buf, len(buf), C.byref(n))
        if rc != OK:
            raise LastroError(rc, "decode: an id outside the vocabulary")
        return buf.raw[:n.value]

    def decode_bytes(self, ids) -> bytes:
        """decodifica_bytes: the exact bytes (added tokens as their literal text)."""
        return self._decode(lib().lastro_tokenizer_decode_bytes, ids)

    def decode(self, ids) -> str:
        """decodifica: UTF-8 text, invalid sequences replaced by U+FFFD, no space clean-up."""
        return self._decode(lib().lastro_tokenizer_decode, ids).decode("utf-8")

    def close(self):
        if getattr(self, "h", None):
            lib().lastro_tokenizer_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        # at interpreter exit (module globals already cleared) the process's CUDA context goes with the process
        if getattr(self, "h", None) and not _finalizing():
            self.close()


def pretokenize(text: str) -> list[str]:
    """pre_tokeniza: the GPT-2 regex pieces of text."""
    raw = text.encode("utf-8")
    n = C.c_int32()
    lib().lastro_tokenizer_pretokenize(raw, len(raw), None, 0, C.byref(n))
    ends = np.empty(max(n.value, 1), np.int32)
    rc = lib().lastro_tokenizer_pretokenize(raw, len(raw), _p(ends), ends.size, C.byref(n))
    if rc != OK:
        raise LastroError(rc, "pretokenize")
    out, start = [], 0
    for e in ends[:n.value].tolist():
        out.append(raw[start:e].decode("utf-8"))
        start = e
    return out


ROLES = {"system": 0, "user": 1, "assistant": 2}


def render_chat(messages: list[dict], add_generation_prompt: bool, date: str) -> str:
    """renderiza_chat: the Granite 3.1 chat template for [{"role": system|user|assistant, "content": str}, ...]."""
    n = len(messages)
    if n == 0:
        raise LastroError(E_ARG, "an empty message list")
    roles = np.array([ROLES[m["role"]] for m in messages], np.int32)
    raws = [m["content"].encode("utf-8") for m in messages]
    bufs = [C.create_string_buffer(r, max(len(r), 1)) for r in raws]
    ptrs = (C.c_char_p * n)(*[C.cast(b, C.c_char_p) for b in bufs])
    lens = (C.c_size_t * n)(*[len(r) for r in raws])
    out_n = C.c_size_t()
    lib().lastro_chat_render(_p(roles), ptrs, lens, n, int(add_generation_prompt), date.encode(), None, 0,
                             C.byref(out_n))
    out = C.create_string_buffer(max(out_n.value, 1))
    rc = lib().lastro_chat_render(_p(roles), ptrs, lens, n, int(add_generation_prompt), date.encode(), out, len(out),
                                  C.byref(out_n))
    if rc != OK:
        raise LastroError(rc, "render_chat")
    return out.raw[:out_n.value].decode("utf-8")


def chat(model, tokenizer, messages: list[dict], max_new_tokens: int, *, date: str | None = None, eos: int = 0):
    """The reference's text loop (tokenizador.rs renderiza_chat + codifica, geracao_regra.rs greedy generation that
    stops at the first EOS, decodifica): renders the Granite chat template with the generation prompt, encodes it,
    generates on the device from the model's current position, and decodes the new ids without the EOS.
    Returns (text, ids)."""
    if date is None:
        import datetime
        d = datetime.date.today()
        date = format_date(d.year, d.month, d.day)
    prompt = tokenizer.encode(render_chat(messages, True, date))
    ids = model.generate_until(prompt, max_new_tokens, eos)
    body = ids[:-1] if ids.size and ids[-1] == eos else ids
    return tokenizer.decode(body), ids


def format_date(year: int, month: int, day: int) -> str:
    """formata_data: strftime("%B %d, %Y") in English."""
    out = C.create_string_buffer(48)
    rc = lib().lastro_format_date(year, month, day, out, len(out))
    if rc != OK:
        raise LastroError(rc, f"invalid date {year}-{month}-{day}")
    return out.value.decode()


TENSOR_NAMES = ("input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
                "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                "block_sparse_moe.router.layer.weight", "block_sparse_moe.input_linear.weight",
                "block_sparse_moe.output_linear.weight")
LAYER_KEYS = ("ln_attn", "ln_moe", "q", "k", "v", "o", "router", "gate_up", "down")


class GpuModel:
    """Whole model resident on one GPU (gpu_model.rs GpuModel), batch-1 decode."""

    def __init__(self, ctx: Context, cfg: dict, max_len: int, kv_dtype: str = "bf16"):
        self.ctx, self.cfg, self.max_len, self.kv_dtype = ctx, dict(cfg), max_len, kv_dtype
        wd = DTYPE_Q8_0 if cfg.get("weight_dtype", "bf16") == "q8_0" else DTYPE_BF16
        d = ModelDesc(**{f: cfg[f] for f, _ in ModelDesc._fields_[:15]}, weight_dtype=wd,
                      kv_dtype=DTYPE_F32 if kv_dtype == "f32" else DTYPE_BF16)
        h = C.c_void_p()
        ctx.check(lib().lastro_model_create(ctx.h, C.byref(d), max_len, C.byref(h)))
        self.h = h
        ctx._children.add(self)
        self._batches = weakref.WeakSet()  # destroyed before the model
        self._logits = np.empty(cfg["vocab"], np.float32)
        self._ids = np.empty(cfg["layers"] * cfg["k"], np.int32)
        self._w = np.empty(cfg["layers"] * cfg["k"], np.float32)
        self._next = np.empty(1, np.int32)

    def load_tensor(self, name: str, arr: np.ndarray):
        """bf16 tensors as uint16 bit arrays, norms as float32 (or bf16 bits), Q8_0 tensors as uint8 arrays whose last
        axis holds each row's 34-byte blocks (fp16 scale, then 32 int8 values): n blocks stand for n * 32 columns."""
        arr = np.ascontiguousarray(arr)
        dims = list(arr.shape)
        if arr.dtype == np.float32:
            dtype = DTYPE_F32
        elif arr.dtype == np.uint8:
            dtype = DTYPE_Q8_0
            assert dims[-1] % 34 == 0, f"{name}: Q8_0 rows are whole 34-byte blocks"
            dims[-1] = dims[-1] // 34 * 32
        else:
            assert arr.dtype == np.uint16, f"{name}: bf16 tensors are passed as uint16 bit arrays"
            dtype = DTYPE_BF16
        shape = (C.c_int64 * len(dims))(*dims)
        self.ctx.check(lib().lastro_model_load_tensor(self.h, name.encode(), dtype, shape, len(dims), _p(arr)))

    def load_weights(self, w: dict):
        """w: embed [V,H] u16, norm [H] f32, layers[l] dict with LAYER_KEYS (u16 bf16 bits / f32 norms)."""
        self.load_tensor("model.embed_tokens.weight", w["embed"])
        self.load_tensor("model.norm.weight", w["norm"])
        for l, lw in enumerate(w["layers"]):
            for key, name in zip(LAYER_KEYS, TENSOR_NAMES):
                self.load_tensor(f"model.layers.{l}.{name}", lw[key])

    def load_checkpoint(self, ck: "Checkpoint"):
        """HostModel::load + GpuModel::upload from a safetensors checkpoint (every tensor checked before it is read)."""
        self.ctx.check(lib().lastro_model_load_checkpoint(self.h, ck.h))

    def fill_synthetic(self, seed: int, std: float = 0.02, norm_std: float = 0.0):
        self.ctx.check(lib().lastro_model_fill_synthetic(self.h, seed, std, norm_std))

    def fill_kv_synthetic(self, n: int, seed: int = 7, std: float = 0.5):
        """A context of n positions with synthetic K/V (no model steps), element for element the CPU oracle's
        Session.fill_kv(n, seed, std): for benchmarks, profiling and parity at long contexts."""
        self.ctx.check(lib().lastro_model_fill_kv_synthetic(self.h, n, seed, std))

    def read_kv(self, layer: int, pos0: int, n: int):
        """K and V rows of positions [pos0, pos0 + n) of one layer as f32 [n, kv_heads * head_dim]."""
        kvd = self.cfg["kv_heads"] * self.cfg["head_dim"]
        k = np.empty((n, kvd), np.float32)
        v = np.empty((n, kvd), np.float32)
        self.ctx.check(lib().lastro_model_read_kv(self.h, layer, pos0, n, _p(k), _p(v)))
        return k, v

    def step(self, token: int, want_logits: bool = True, want_routes: bool = True):
        """(logits, next_token, route_ids [L,k], route_w [L,k]) (GpuModel::step)."""
        self.ctx.check(lib().lastro_model_step(self.h, int(token), _p(self._logits) if want_logits else None,
                                               _p(self._next), _p(self._ids) if want_routes else None,
                                               _p(self._w) if want_routes else None))
        c = self.cfg
        return (self._logits.copy() if want_logits else None, int(self._next[0]),
                self._ids.reshape(c["layers"], c["k"]).copy() if want_routes else None,
                self._w.reshape(c["layers"], c["k"]).copy() if want_routes else None)

    def step_positions(self, tokens, want_logits: bool = True):
        """Multi-position step: (logits [n, V] or None, next ids [n]) for n = len(tokens) <= 32 consecutive positions."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        n = t.size
        lg = np.empty((n, self.cfg["vocab"]), np.float32) if want_logits else None
        nxt = np.empty(n, np.int32)
        self.ctx.check(lib().lastro_model_step_positions(self.h, n, _p(t), _p(lg), _p(nxt)))
        return lg, nxt

    def prefill(self, prompt, chunk: int = 32):
        """Feed a prompt through multi-position steps of up to `chunk` positions; returns the last greedy id."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        nxt = None
        for i in range(0, p.size, chunk):
            _, nxt = self.step_positions(p[i:i + chunk], want_logits=False)
        return int(nxt[-1])

    def generate(self, prompt, n_new: int) -> np.ndarray:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(max(n_new, 1), np.int32)
        self.ctx.check(lib().lastro_model_generate(self.h, _p(p), p.size, n_new, _p(out)))
        return out[:n_new]

    def generate_until(self, prompt, n_new: int, eos: int = 0) -> np.ndarray:
        """Greedy generation that stops after the first `eos` (included), geracao_regra.rs's normal use."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(n_new, np.int32)
        n = C.c_int32()
        self.ctx.check(lib().lastro_model_generate_until(self.h, _p(p), p.size, n_new, eos, _p(out), C.byref(n)))
        return out[:n.value]

    def decode(self, n: int):
        self.ctx.check(lib().lastro_model_decode(self.h, n))

    def reset(self):
        self.ctx.check(lib().lastro_model_reset(self.h))

    @property
    def pos(self) -> int:
        v = C.c_int32()
        self.ctx.check(lib().lastro_model_position(self.h, C.byref(v)))
        return v.value

    KERNELS = ("qkv_rope", "attention", "oproj", "router", "gate_up", "down", "head", "fused_step", "moe")

    def profile(self, steps: int) -> dict:
        """Per-kernel device ms per step (summed over layers), measured with events between direct launches."""
        out = np.zeros(len(self.KERNELS), np.float32)
        self.ctx.check(lib().lastro_model_profile(self.h, steps, _p(out), out.size))
        return dict(zip(self.KERNELS, out.tolist()))

    def trace(self, steps: int) -> dict:
        """In-graph timeline of `steps` graph-replayed steps: {"exposed": {kind: ms}, "span": {..}, "wait": {..},
        "step_ms": ms}; exposed times are each kind's share of the step's critical path (they sum to the step); wait
        is the hand-off latency from the previous launch's last exit to the first release from griddepcontrol.wait."""
        ex, sp, wt = (np.zeros(len(self.KERNELS), np.float32) for _ in range(3))
        st = np.zeros(1, np.float32)
        self.ctx.check(lib().lastro_model_trace(self.h, steps, _p(ex), _p(sp), _p(wt), ex.size, _p(st)))
        kinds = self.KERNELS
        return {"exposed": dict(zip(kinds, ex.tolist())), "span": dict(zip(kinds, sp.tolist())),
                "wait": dict(zip(kinds, wt.tolist())), "step_ms": float(st[0])}

    def set_options(self, graphs: bool = True, pdl: bool = True, fused: bool = False):
        self.ctx.check(lib().lastro_model_set_options(self.h, int(graphs), int(pdl), int(fused)))

    def set_moe(self, one_launch: bool = True):
        """The MoE block as one persistent launch per layer (default where it fits) or the gate_up + down kernels."""
        self.ctx.check(lib().lastro_model_set_moe(self.h, int(one_launch)))

    def trace_raw(self, launch: int) -> np.ndarray:
        """Stamps of one launch of the last traced step: [1024 CTAs, 11] global-timer ns (start, release, exit, then
        the kernel's 8 milestones; 0 where not stamped)."""
        out = np.zeros((1024, TRACE_WORDS), np.uint64)
        self.ctx.check(lib().lastro_model_trace_raw(self.h, launch, _p(out), out.size))
        return out

    def set_tuning(self, attn_splits: int = 16, attn_merge: int = 0, oproj_smem: bool = False,
                   prefetch_down: bool = False, attn_tma: bool = False, speculation: str | bool = False,
                   attn_mma: bool = False, down_routes: bool = False):
        """Batch-1 attention: context splits (8, 16, or 0 for the size-based choice) and how they are merged (0 the
        attention's last CTA, 1 the output projection, 2 a thread-block cluster per KV head); the output projection's
        weights in shared memory (256-thread CTAs) or registers; gate_up hinting the down rows into L2; bf16 K/V
        staged by swizzled 8-row TMA boxes (attn_tma) or by bulk copies per page run; the experts predicted from
        the layer's input fetched before the routing is known (speculation: "l2" hinted into L2 by the output
        projection, "stage" streamed into the gate_up CTAs' shared memory, "attn" hinted into L2 by the attention
        kernel's CTAs, False off: the default); bf16 K/V
        attention on tensor cores (attn_mma); every down CTA reducing the router shares itself (down_routes) instead
        of taking the routing gate_up publishes."""
        assert speculation in ("l2", "stage", "attn", False)
        flags = (1 if oproj_smem else 0) | (2 if prefetch_down else 0) | (4 if attn_tma else 0) | \
            {"l2": 8, "stage": 16, "attn": 128, False: 0}[speculation] | (32 if attn_mma else 0) | (64 if down_routes else 0)
        self.ctx.check(lib().lastro_model_set_tuning(self.h, attn_splits, int(attn_merge), flags))

    @property
    def moe(self) -> bool:
        return bool(lib().lastro_model_moe(self.h))

    def set_attention(self, tensor_cores: bool = True):
        """bf16 KV: attention on tensor cores or the CUDA-core split kernel (the default: faster at batch 1)."""
        self.ctx.check(lib().lastro_model_set_attention(self.h, int(tensor_cores)))

    @property
    def fused(self) -> bool:
        """True when decode steps run as the single fused step kernel."""
        return bool(lib().lastro_model_fused(self.h))

    def close(self):
        if getattr(self, "h", None):
            for b in list(getattr(self, "_batches", ())):
                b.close()
            lib().lastro_model_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        # at interpreter exit (module globals already cleared) the process's CUDA context goes with the process
        if getattr(self, "h", None) and not _finalizing():
            self.close()


class GpuBatch:
    """Batched decode of many independent sequences on a GpuModel's weights, the MoE experts partitioned over the
    `world` ranks of an expert-parallel group (one process per GPU).  world 1: call connect() with no handles.
    world > 1: every rank passes exchange_handle() to the others (e.g. torch.distributed.all_gather_object) and calls
    connect(handles in rank order); the ranks then step the same number of times."""

    def __init__(self, model: GpuModel, max_seqs: int, max_len: int, rank: int = 0, world: int = 1):
        self.model, self.ctx, self.cfg = model, model.ctx, model.cfg
        self.max_seqs, self.max_len, self.rank, self.world = max_seqs, max_len, rank, world
        self.kv_dtype = model.kv_dtype
        h = C.c_void_p()
        self.ctx.check(lib().lastro_batch_create(model.h, max_seqs, max_len, rank, world, C.byref(h)))
        self.h = h
        model._batches.add(self)
        self.ctx._children.add(self)

    def exchange_handle(self) -> bytes:
        buf = (C.c_char * HANDLE_BYTES)()
        self.ctx.check(lib().lastro_batch_exchange_handle(self.h, buf, HANDLE_BYTES))
        return bytes(buf)

    def connect(self, handles=None):
        if handles is None:
            self.ctx.check(lib().lastro_batch_connect(self.h, None, HANDLE_BYTES))
            return
        assert len(handles) == self.world and all(len(x) == HANDLE_BYTES for x in handles)
        buf = (C.c_char * (HANDLE_BYTES * self.world)).from_buffer_copy(b"".join(handles))
        self.ctx.check(lib().lastro_batch_connect(self.h, buf, HANDLE_BYTES))

    def set_router_bias(self, bias):
        if bias is None:
            self.ctx.check(lib().lastro_batch_set_router_bias(self.h, None))
            return
        b = np.ascontiguousarray(bias, dtype=np.float32)
        assert b.shape == (self.cfg["layers"], self.cfg["experts"])
        self.ctx.check(lib().lastro_batch_set_router_bias(self.h, _p(b)))

    def set_expert_placement(self, owner):
        """owner[e]: the rank that computes expert e (E/world experts per rank; the same on every rank)."""
        o = np.ascontiguousarray(owner, dtype=np.int32)
        self.ctx.check(lib().lastro_batch_set_expert_placement(self.h, _p(o), o.size))

    def step(self, seq_ids, tokens, want_logits: bool = False, want_routes: bool = False):
        """(next [n], logits [n, V] or None, route ids [n, layers, k] or None) for one token of each sequence."""
        sq = np.ascontiguousarray(seq_ids, dtype=np.int32)
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        n, c = sq.size, self.cfg
        nxt = np.empty(n, np.int32)
        lg = np.empty((n, c["vocab"]), np.float32) if want_logits else None
        rt = np.empty((n, c["layers"], c["k"]), np.int32) if want_routes else None
        self.ctx.check(lib().lastro_batch_step(self.h, n, _p(sq), _p(tk), _p(nxt), _p(lg), _p(rt)))
        return nxt, lg, rt

    def decode(self, seq_ids, tokens, steps: int, want_ids: bool = True):
        """`steps` greedy steps on the device (each step's ids fed back); ids [steps, n]."""
        sq = np.ascontiguousarray(seq_ids, dtype=np.int32)
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty((max(steps, 1), sq.size), np.int32) if want_ids else None
        self.ctx.check(lib().lastro_batch_decode(self.h, sq.size, _p(sq), _p(tk), steps, _p(out)))
        return out[:steps] if want_ids else None

    def fill_kv_synthetic(self, seq: int, n: int, seed: int = 7, std: float = 0.5):
        self.ctx.check(lib().lastro_batch_fill_kv_synthetic(self.h, seq, n, seed, std))

    def reset(self, seq: int):
        self.ctx.check(lib().lastro_batch_reset(self.h, seq))

    def position(self, seq: int) -> int:
        v = C.c_int32()
        self.ctx.check(lib().lastro_batch_position(self.h, seq, C.byref(v)))
        return v.value

    def set_options(self, graphs: bool = True, gemm: int = 2, attn_tc: bool | None = None):
        """gemm: 2 tcgen05 warp-specialised (TMA weight tiles), 1 tcgen05 with all threads loading, 0 mma.sync;
        attn_tc: attention on tensor cores (default where available: bf16 KV) or CUDA cores."""
        if attn_tc is None:
            attn_tc = self.kv_dtype == "bf16"
        self.ctx.check(lib().lastro_batch_set_options(self.h, int(graphs), int(gemm), int(attn_tc)))

    def set_wait_limit(self, seconds: float):
        """Bound of every wait on another rank's exchange flag (default 10 s)."""
        self.ctx.check(lib().lastro_batch_set_wait_limit(self.h, int(seconds * 1e9)))

    KERNELS = ("norm", "qkv", "rope_kv", "attention", "oproj", "router", "group", "gate_up", "down", "combine",
               "lm_head", "argmax")

    def profile(self, seq_ids, tokens, steps: int) -> dict:
        """Mean device ms per step of each kernel kind (summed over layers), direct launches timed with events."""
        sq = np.ascontiguousarray(seq_ids, dtype=np.int32)
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(len(self.KERNELS), np.float32)
        self.ctx.check(lib().lastro_batch_profile(self.h, sq.size, _p(sq), _p(tk), steps, _p(out), out.size))
        return dict(zip(self.KERNELS, out.tolist()))

    def trace(self, seq_ids, tokens, steps: int) -> dict:
        """In-graph timeline of `steps` graph-replayed steps: {"exposed": {kind: ms}, "span": {..}, "wait": {..},
        "step_ms": ms} per step (exposed: each kind's share of the step's critical path; the positions advance)."""
        sq = np.ascontiguousarray(seq_ids, dtype=np.int32)
        tk = np.ascontiguousarray(tokens, dtype=np.int32)
        ex, sp, wt = (np.zeros(len(self.KERNELS), np.float32) for _ in range(3))
        st = np.zeros(1, np.float32)
        self.ctx.check(lib().lastro_batch_trace(self.h, sq.size, _p(sq), _p(tk), steps, _p(ex), _p(sp), _p(wt), ex.size,
                                                _p(st)))
        kinds = self.KERNELS
        return {"exposed": dict(zip(kinds, ex.tolist())), "span": dict(zip(kinds, sp.tolist())),
                "wait": dict(zip(kinds, wt.tolist())), "step_ms": float(st[0])}

    def trace_raw(self, launch: int) -> np.ndarray:
        """[1024, TRACE_WORDS] stamps of one launch of the last traced step (0 the layer-0 norm, then 8 per layer:
        qkv, rope_kv, attention, oproj, router, gate_up, down, combine; then lm_head, argmax)."""
        out = np.zeros((1024, TRACE_WORDS), np.uint64)
        self.ctx.check(lib().lastro_batch_trace_raw(self.h, launch, _p(out), out.size))
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().lastro_batch_destroy(self.h)
            self.h = None

    def __del__(self, _finalizing=sys.is_finalizing):
        # at interpreter exit (module globals already cleared) the process's CUDA context goes with the process
        if getattr(self, "h", None) and not _finalizing():
            self.close()
