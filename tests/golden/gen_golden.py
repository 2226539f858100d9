#!/usr/bin/env python3
"""Generate the golden fixtures of this folder with transformers' GraniteMoe.

This is the reference's own oracle method (tools/ref_moe_block.py and
tools/ref_greedy.py of brenoperucchi/lastro-rust run GraniteMoeForCausalLM on CPU
in fp32 from bf16 weights), applied to random-init weights drawn from
``synth_np`` (the checkpoints the reference used are not available here).

Fixtures:
  block_c1.npz   one Granite-1B-shaped MoE block: x, y,
                 router logits, top-8 ids and weights for 8 tokens
  tiny_model.npz the reference's tiny test Granite (tests/common/mod.rs:79-87)
                 with larger weights: prompt, greedy ids, teacher-forced logits
                 and routing at every position
  c2_greedy.npz  the Granite-1B-shaped model of BASELINE config 1: 128-token
                 prompt, 128 greedy ids, top1-top2 gaps, top-16 logits per step
  tiny_q8.npz    the tiny test Granite with every linear weight Q8_0 (BASELINE
                 config C4's format), run dequantised in fp32: prompt, greedy
                 ids, teacher-forced logits and routing at every position

Run from the repository root:  python tests/golden/gen_golden.py [--skip-c2] [--only NAME]
"""
import argparse
import json
import os
import sys

import numpy as np
import torch
import transformers

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
sys.path.insert(0, os.path.join(HERE, "..", "..", "lastro-rust_b200"))
import synth_np as S  # noqa: E402
from lastro_b200 import configs as CFG  # noqa: E402

T_EMBED, T_NORM, T_LN_ATTN, T_LN_MOE, T_Q, T_K, T_V, T_O, T_ROUTER, T_GATE_UP, T_DOWN = range(11)
TINY_STD = S.TINY_STD
bf16_f32 = S.bf16_f32
model_weights = S.model_weights


def hf_config(cfg):
    c = transformers.GraniteMoeConfig(
        vocab_size=cfg["vocab"], hidden_size=cfg["hidden"], intermediate_size=cfg["inter"],
        num_hidden_layers=cfg["layers"], num_attention_heads=cfg["heads"], num_key_value_heads=cfg["kv_heads"],
        num_local_experts=cfg["experts"], num_experts_per_tok=cfg["k"], max_position_embeddings=4096,
        rms_norm_eps=cfg["eps"], embedding_multiplier=cfg["embedding_multiplier"],
        residual_multiplier=cfg["residual_multiplier"], attention_multiplier=cfg["attention_multiplier"],
        logits_scaling=cfg["logits_scaling"], tie_word_embeddings=True, attention_bias=False,
        rope_parameters={"rope_type": "default", "rope_theta": cfg["rope_theta"]},
        pad_token_id=None, bos_token_id=None, eos_token_id=None)
    c._attn_implementation = "eager"
    return c


def hf_model(cfg, w):
    torch.manual_seed(0)
    m = transformers.GraniteMoeForCausalLM(hf_config(cfg)).eval()
    t = torch.from_numpy
    with torch.no_grad():
        m.model.embed_tokens.weight.copy_(t(w["embed"]))
        m.model.norm.weight.copy_(t(w["norm"]))
        for l, lw in enumerate(w["layers"]):
            L = m.model.layers[l]
            L.input_layernorm.weight.copy_(t(lw["ln_attn"]))
            L.post_attention_layernorm.weight.copy_(t(lw["ln_moe"]))
            L.self_attn.q_proj.weight.copy_(t(lw["q"]))
            L.self_attn.k_proj.weight.copy_(t(lw["k"]))
            L.self_attn.v_proj.weight.copy_(t(lw["v"]))
            L.self_attn.o_proj.weight.copy_(t(lw["o"]))
            L.block_sparse_moe.router.layer.weight.copy_(t(lw["router"]))
            L.block_sparse_moe.input_linear.weight.copy_(t(lw["gate_up"]))
            L.block_sparse_moe.output_linear.weight.copy_(t(lw["down"]))
    m.tie_weights()
    assert m.lm_head.weight.data_ptr() == m.model.embed_tokens.weight.data_ptr()
    return m


def router_capture(model, layers):
    """Router logits per layer via a hook on router.layer; top-k + softmax as GraniteMoeTopKGating does."""
    got = {}

    def hook(L):
        def f(_m, _i, out):
            got.setdefault(L, []).append(out.detach().float().reshape(-1, out.shape[-1]).clone())
        return f

    hs = [model.model.layers[L].block_sparse_moe.router.layer.register_forward_hook(hook(L)) for L in layers]
    return got, hs


def topk_softmax(logits, k):
    v, i = logits.topk(k, dim=-1)
    return i.numpy().astype(np.int32), torch.softmax(v, dim=-1).numpy().astype(np.float32)


def gen_block_c1(out):
    c = CFG.C1_BLOCK
    E, H, I, k, T = c["experts"], c["hidden"], c["inter"], c["k"], c["tokens"]
    seed = c["weight_seed"]
    router = bf16_f32(E * H, S.tensor_seed(seed, 0, T_ROUTER), CFG.WEIGHT_STD).reshape(E, H)
    gu = bf16_f32(E * 2 * I * H, S.tensor_seed(seed, 0, T_GATE_UP), CFG.WEIGHT_STD).reshape(E, 2 * I, H)
    dn = bf16_f32(E * H * I, S.tensor_seed(seed, 0, T_DOWN), CFG.WEIGHT_STD).reshape(E, H, I)
    x = S.values_f32(T * H, c["x_seed"], 1.0).reshape(T, H)
    hc = transformers.GraniteMoeConfig(hidden_size=H, intermediate_size=I, num_local_experts=E, num_experts_per_tok=k)
    blk = transformers.models.granitemoe.modeling_granitemoe.GraniteMoeMoE(hc).eval()
    with torch.no_grad():
        blk.router.layer.weight.copy_(torch.from_numpy(router))
        blk.input_linear.weight.copy_(torch.from_numpy(gu))
        blk.output_linear.weight.copy_(torch.from_numpy(dn))
        logits = blk.router.layer(torch.from_numpy(x)).float()
        y = blk(torch.from_numpy(x)[None])[0].numpy()
    idx, w = topk_softmax(logits, k)
    np.savez_compressed(os.path.join(out, "block_c1.npz"), x=x, y=y, idx=idx, w=w, logits=logits.numpy(),
                        meta=json.dumps(dict(c, std=CFG.WEIGHT_STD, torch=torch.__version__,
                                             transformers=transformers.__version__)))
    print("block_c1:", y.shape, idx[0].tolist())


def greedy(model, ids, n):
    with torch.inference_mode():
        out = model.generate(torch.tensor([ids]), attention_mask=torch.ones(1, len(ids), dtype=torch.long),
                             max_new_tokens=n, do_sample=False, output_scores=True, return_dict_in_generate=True,
                             eos_token_id=None, pad_token_id=0)
    gen = out.sequences[0, len(ids):].tolist()
    scores = torch.stack([s[0].float() for s in out.scores])
    return gen, scores


def gen_tiny(out):
    cfg, seed = CFG.TINY, 10
    w = model_weights(cfg, seed, 0.0, stds=TINY_STD)
    m = hf_model(cfg, w)
    prompt = S.tokens(24, 77, cfg["vocab"]).tolist()
    gen, scores = greedy(m, prompt, 48)
    seq = prompt + gen[:-1]
    got, hs = router_capture(m, range(cfg["layers"]))
    with torch.inference_mode():
        logits = m(torch.tensor([seq]), use_cache=False).logits[0].float()
    for h in hs:
        h.remove()
    idx = np.stack([topk_softmax(got[L][0], cfg["k"])[0] for L in range(cfg["layers"])])
    rw = np.stack([topk_softmax(got[L][0], cfg["k"])[1] for L in range(cfg["layers"])])
    top2 = scores.topk(2, dim=-1).values
    np.savez_compressed(os.path.join(out, "tiny_model.npz"), prompt=np.array(prompt, np.int32),
                        generated=np.array(gen, np.int32), logits=logits.numpy(), route_idx=idx, route_w=rw,
                        gaps=(top2[:, 0] - top2[:, 1]).numpy(),
                        meta=json.dumps(dict(cfg=cfg, seed=seed, stds=TINY_STD, torch=torch.__version__,
                                             transformers=transformers.__version__)))
    print("tiny:", prompt, gen)


def gen_tiny_q8(out):
    cfg, seed = dict(CFG.TINY, weight_dtype="q8_0"), 12
    wq = S.model_weights_q8(cfg, seed)
    m = hf_model(cfg, S.dequant_model(wq))
    prompt = S.tokens(20, 78, cfg["vocab"]).tolist()
    gen, scores = greedy(m, prompt, 32)
    seq = prompt + gen[:-1]
    got, hs = router_capture(m, range(cfg["layers"]))
    with torch.inference_mode():
        logits = m(torch.tensor([seq]), use_cache=False).logits[0].float()
    for h in hs:
        h.remove()
    idx = np.stack([topk_softmax(got[L][0], cfg["k"])[0] for L in range(cfg["layers"])])
    top2 = scores.topk(2, dim=-1).values
    np.savez_compressed(os.path.join(out, "tiny_q8.npz"), prompt=np.array(prompt, np.int32),
                        generated=np.array(gen, np.int32), logits=logits.numpy(), route_idx=idx,
                        gaps=(top2[:, 0] - top2[:, 1]).numpy(),
                        meta=json.dumps(dict(cfg=cfg, seed=seed, torch=torch.__version__,
                                             transformers=transformers.__version__)))
    print("tiny_q8:", prompt, gen)


def gen_c2(out, new_tokens):
    c = CFG.C2_1B
    cfg = c["model"]
    torch.set_num_threads(os.cpu_count() or 8)
    w = model_weights(cfg, c["weight_seed"], CFG.WEIGHT_STD)
    m = hf_model(cfg, w)
    del w
    prompt = S.tokens(c["prompt_len"], c["prompt_seed"], cfg["vocab"]).tolist()
    gen, scores = greedy(m, prompt, new_tokens)
    tv, ti = scores.topk(16, dim=-1)
    np.savez_compressed(os.path.join(out, "c2_greedy.npz"), prompt=np.array(prompt, np.int32),
                        generated=np.array(gen, np.int32), gaps=(tv[:, 0] - tv[:, 1]).numpy(),
                        top_val=tv.numpy(), top_idx=ti.numpy().astype(np.int32),
                        meta=json.dumps(dict(c, std=CFG.WEIGHT_STD, torch=torch.__version__,
                                             transformers=transformers.__version__)))
    print("c2:", gen[:16], "min gap", float((tv[:, 0] - tv[:, 1]).min()))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--skip-c2", action="store_true")
    ap.add_argument("--c2-tokens", type=int, default=128)
    ap.add_argument("--only", choices=("block_c1", "tiny", "tiny_q8", "c2"), help="regenerate one fixture")
    a = ap.parse_args()
    torch.set_num_threads(os.cpu_count() or 8)
    jobs = dict(block_c1=lambda: gen_block_c1(HERE), tiny=lambda: gen_tiny(HERE), tiny_q8=lambda: gen_tiny_q8(HERE),
                c2=lambda: gen_c2(HERE, a.c2_tokens))
    for name, job in jobs.items():
        if (a.only and name != a.only) or (name == "c2" and a.skip_c2 and not a.only):
            continue
        job()


if __name__ == "__main__":
    main()
