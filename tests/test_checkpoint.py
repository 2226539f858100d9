"""safetensors checkpoints and config.json through the C ABI (host-only: no GPU needed, except the last test).

Restates rust/moe-rt/tests/block.rs:132-180 (the reader reads BF16, refuses another dtype, an absent tensor and
offsets past the end of the file; malformed headers are refused without a crash; a shape whose byte count overflows
fails on read) and model.rs:34-61 (Config::from_json's refusals), and loads a whole model from a checkpoint.
"""
import json
import os
import struct

import numpy as np
import pytest

import lastro_b200 as LB
from helpers import bf, reference_tiny_weights, values
from lastro_b200 import configs as CFG

U64_MAX = (1 << 64) - 1


def write_safetensors(path, tensors, metadata=None):
    """tensors: [(name, dtype, shape, raw bytes)] in order; data laid out back to back."""
    head, blobs, off = {}, [], 0
    if metadata is not None:
        head["__metadata__"] = metadata
    for name, dtype, shape, raw in tensors:
        head[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(head).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def write_head(path, entry):
    h = json.dumps({"a": entry}).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + bytes(16))


def test_reader_reads_bf16_and_refuses_wrong_dtype_absent_tensor_and_bad_offsets(tmp_path):
    """tests/block.rs:132-150"""
    v = bf(values(6, 3))
    p = tmp_path / "m.safetensors"
    write_safetensors(p, [("a", "BF16", [2, 3], v.tobytes()), ("b", "F32", [1], bytes(4))], {"format": "pt"})
    ck = LB.Checkpoint(str(tmp_path))
    assert len(ck) == 2
    assert ck.info("a") == ("BF16", (2, 3))
    got = ck.bf16("a")
    assert got.shape == (2, 3) and np.array_equal(got.ravel(), v)
    with pytest.raises(LB.LastroError, match="F32"):
        ck.bf16("b")
    with pytest.raises(LB.LastroError, match="absent"):
        ck.bf16("c")
    ck.close()
    raw = p.read_bytes()
    p.write_bytes(raw[:-6])  # offsets past the end of the file
    with pytest.raises(LB.LastroError, match="outside the file") as e:
        LB.Checkpoint(str(tmp_path))
    assert e.value.code == LB.E_ARG


@pytest.mark.parametrize("entry", [
    {"dtype": "BF16", "shape": [2], "data_offsets": [0]},
    {"dtype": "BF16", "shape": [2], "data_offsets": []},
    {"dtype": "BF16", "shape": [2], "data_offsets": [0, 4, 8]},
    {"dtype": "BF16", "shape": [2], "data_offsets": ["0", 4]},
    {"dtype": "BF16", "shape": [2], "data_offsets": [U64_MAX, U64_MAX]},
    {"dtype": "BF16", "shape": [2], "data_offsets": [U64_MAX - 4, U64_MAX]},
    {"dtype": "BF16", "shape": [2], "data_offsets": [4, 0]},
    {"shape": [2], "data_offsets": [0, 4]},
    {"dtype": "BF16", "data_offsets": [0, 4]},
    {"dtype": "BF16", "shape": [-2], "data_offsets": [0, 4]},
    {"dtype": "BF16", "shape": [2]},
    5,
], ids=lambda e: json.dumps(e)[:40])
def test_reader_refuses_malformed_headers_without_crashing(tmp_path, entry):
    """tests/block.rs:152-171: every malformed entry is an error (here: a LastroError with a message), not a crash."""
    write_head(tmp_path / "m.safetensors", entry)
    with pytest.raises(LB.LastroError) as e:
        LB.Checkpoint(str(tmp_path))
    assert e.value.code == LB.E_ARG and "safetensors" in str(e.value)


def test_shape_whose_byte_count_overflows_fails_on_read(tmp_path):
    """tests/block.rs:172-178"""
    write_head(tmp_path / "m.safetensors", {"dtype": "BF16", "shape": [U64_MAX, 4], "data_offsets": [0, 4]})
    ck = LB.Checkpoint(str(tmp_path))
    with pytest.raises(LB.LastroError, match="size does not match"):
        ck.bf16("a")
    ck.close()


def test_directory_without_safetensors_and_oversized_or_garbled_header(tmp_path):
    with pytest.raises(LB.LastroError, match="no \\*.safetensors"):
        LB.Checkpoint(str(tmp_path))
    with pytest.raises(LB.LastroError) as e:
        LB.Checkpoint(str(tmp_path / "missing"))
    assert e.value.code == LB.E_IO
    p = tmp_path / "m.safetensors"
    p.write_bytes(struct.pack("<Q", (100 << 20) + 1) + bytes(8))
    with pytest.raises(LB.LastroError, match="header of"):
        LB.Checkpoint(str(tmp_path))
    p.write_bytes(struct.pack("<Q", 5) + b"{\"a\":")
    with pytest.raises(LB.LastroError, match="safetensors"):
        LB.Checkpoint(str(tmp_path))


def test_tensors_spread_over_several_files_are_indexed_together(tmp_path):
    a, b = bf(values(8, 1)), bf(values(4, 2))
    write_safetensors(tmp_path / "model-00001-of-00002.safetensors", [("x", "BF16", [8], a.tobytes())])
    write_safetensors(tmp_path / "model-00002-of-00002.safetensors", [("y", "BF16", [2, 2], b.tobytes())])
    ck = LB.Checkpoint(str(tmp_path))
    assert len(ck) == 2
    assert np.array_equal(ck.bf16("x"), a) and np.array_equal(ck.bf16("y").ravel(), b)
    ck.close()


def granite_config(**over):
    """A Granite-3.0-3B-A800M-shaped config.json (the fields Config::from_json reads)."""
    c = {"model_type": "granitemoe", "hidden_size": 1536, "intermediate_size": 512, "num_hidden_layers": 32,
         "num_attention_heads": 24, "num_key_value_heads": 8, "vocab_size": 49155, "num_local_experts": 40,
         "num_experts_per_tok": 8, "rope_theta": 10000.0, "rms_norm_eps": 1e-6, "embedding_multiplier": 12.0,
         "residual_multiplier": 0.22, "attention_multiplier": 0.015625, "logits_scaling": 6.0,
         "rope_scaling": None, "attention_bias": False, "tie_word_embeddings": True}
    c.update(over)
    return c


def test_config_from_json_reads_the_granite_fields():
    d = LB.config_from_json(json.dumps(granite_config()))
    want = CFG.GRANITE_3B
    for k in ("hidden", "inter", "layers", "heads", "kv_heads", "head_dim", "vocab", "experts", "k"):
        assert d[k] == want[k], k
    for k in ("rope_theta", "eps", "embedding_multiplier", "residual_multiplier", "attention_multiplier",
              "logits_scaling"):
        assert d[k] == pytest.approx(want[k], rel=1e-7), k
    assert LB.config_from_json(json.dumps(granite_config(head_dim=128)))["head_dim"] == 128


@pytest.mark.parametrize("over,code,msg", [
    ({"model_type": "granite"}, "E_UNSUPPORTED", "granitemoe"),
    ({"rope_scaling": {"type": "linear", "factor": 2.0}}, "E_UNSUPPORTED", "rope_scaling"),
    ({"attention_bias": True}, "E_UNSUPPORTED", "attention_bias"),
    ({"tie_word_embeddings": False}, "E_UNSUPPORTED", "untied"),
    ({"vocab_size": None}, "E_ARG", "vocab_size"),
    ({"rms_norm_eps": "1e-6"}, "E_ARG", "rms_norm_eps"),
])
def test_config_from_json_refuses_what_the_reference_refuses(over, code, msg):
    """model.rs:37-42 and the missing-field errors of model.rs:35-36"""
    with pytest.raises(LB.LastroError, match=msg) as e:
        LB.config_from_json(json.dumps(granite_config(**over)))
    assert e.value.code == getattr(LB, code)
    with pytest.raises(LB.LastroError):
        LB.config_from_json("{not json")


def write_model_checkpoint(d, cfg, w, config_over=None, drop=None, reshape=None):
    """The tiny reference model as a Granite checkpoint: two safetensors files and config.json."""
    tensors = [("model.embed_tokens.weight", w["embed"]), ("model.norm.weight", bf(w["norm"]))]
    names = ("input_layernorm.weight", "post_attention_layernorm.weight", "self_attn.q_proj.weight",
             "self_attn.k_proj.weight", "self_attn.v_proj.weight", "self_attn.o_proj.weight",
             "block_sparse_moe.router.layer.weight", "block_sparse_moe.input_linear.weight",
             "block_sparse_moe.output_linear.weight")
    keys = ("ln_attn", "ln_moe", "q", "k", "v", "o", "router", "gate_up", "down")
    for l, lw in enumerate(w["layers"]):
        for n, k in zip(names, keys):
            a = lw[k]
            tensors.append((f"model.layers.{l}.{n}", bf(a) if a.dtype == np.float32 else a))
    out = []
    for name, a in tensors:
        if name == drop:
            continue
        shape = list(a.shape) if reshape is None or name != reshape[0] else reshape[1]
        out.append((name, "BF16", shape, np.ascontiguousarray(a).tobytes()))
    half = len(out) // 2
    write_safetensors(os.path.join(d, "model-00001-of-00002.safetensors"), out[:half])
    write_safetensors(os.path.join(d, "model-00002-of-00002.safetensors"), out[half:])
    c = granite_config(hidden_size=cfg["hidden"], intermediate_size=cfg["inter"], num_hidden_layers=cfg["layers"],
                       num_attention_heads=cfg["heads"], num_key_value_heads=cfg["kv_heads"], vocab_size=cfg["vocab"],
                       num_local_experts=cfg["experts"], num_experts_per_tok=cfg["k"], rope_theta=cfg["rope_theta"],
                       rms_norm_eps=cfg["eps"], embedding_multiplier=cfg["embedding_multiplier"],
                       residual_multiplier=cfg["residual_multiplier"],
                       attention_multiplier=cfg["attention_multiplier"], logits_scaling=cfg["logits_scaling"])
    c.update(config_over or {})
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(c, f)


def test_checkpoint_config_and_tensors_of_a_whole_model(tmp_path):
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    write_model_checkpoint(str(tmp_path), cfg, w)
    ck = LB.Checkpoint(str(tmp_path))
    d = ck.config()
    for k in ("hidden", "inter", "layers", "heads", "kv_heads", "head_dim", "vocab", "experts", "k"):
        assert d[k] == cfg[k]
    assert len(ck) == 2 + 9 * cfg["layers"]
    assert np.array_equal(ck.bf16("model.layers.1.block_sparse_moe.input_linear.weight"), w["layers"][1]["gate_up"])
    ck.close()


@pytest.mark.gpu
def test_model_loaded_from_a_checkpoint_decodes_like_the_loaded_weights(gpu_ctx, tmp_path):
    """HostModel::load + GpuModel::upload: the model built from the checkpoint (config.json + safetensors) steps
    bitwise like the same weights passed tensor by tensor; an absent tensor or a wrong shape is refused before any
    step, naming the tensor."""
    cfg = CFG.TINY
    w = reference_tiny_weights(cfg)
    write_model_checkpoint(str(tmp_path), cfg, w)
    ck = LB.Checkpoint(str(tmp_path))
    c = dict(cfg, **ck.config())
    a = LB.GpuModel(gpu_ctx, c, 32, kv_dtype="bf16")
    a.load_checkpoint(ck)
    b = LB.GpuModel(gpu_ctx, cfg, 32, kv_dtype="bf16")
    b.load_weights(w)
    for tok in (3, 17, 29, 5):
        la, na, ia, _ = a.step(tok)
        lb, nb, ib, _ = b.step(tok)
        assert na == nb and np.array_equal(la, lb) and np.array_equal(ia, ib)
    ck.close()
    for sub, kw, msg in (("drop", dict(drop="model.layers.1.self_attn.o_proj.weight"), "absent"),
                         ("shape", dict(reshape=("model.layers.0.self_attn.k_proj.weight",
                                                 [cfg["hidden"], cfg["kv_heads"] * cfg["head_dim"]])), "shape")):
        dd = tmp_path / sub
        dd.mkdir()
        write_model_checkpoint(str(dd), cfg, w, **kw)
        bad = LB.Checkpoint(str(dd))
        m = LB.GpuModel(gpu_ctx, cfg, 32, kv_dtype="bf16")
        with pytest.raises(LB.LastroError, match=msg) as e:
            m.load_checkpoint(bad)
        assert e.value.code == LB.E_ARG
        m.close()
        bad.close()
    a.close()
    b.close()
