"""Text in, text out on the device: the Granite chat template, the tokenizer and greedy generation with the EOS stop
(tokenizador.rs with geracao_regra.rs:25-48), against the CPU oracle fed the same ids.

The model has the tiny shapes with the vocabulary of the synthetic tokenizer (tests/golden/bpe_tokenizer.json), random
weights; the oracle runs the same synthetic weights (both generators are seeded identically), f32 KV."""
import os

import numpy as np
import pytest

import lastro_b200 as LB
import oracle as O
from lastro_b200 import configs as CFG

pytestmark = pytest.mark.gpu

TOK_JSON = os.path.join(os.path.dirname(__file__), "golden", "bpe_tokenizer.json")


def test_chat_round_trip_matches_the_oracle(gpu_ctx, pool):
    tok = LB.Tokenizer(TOK_JSON)
    cfg = dict(CFG.TINY_768, vocab=tok.vocab_size)
    m = LB.GpuModel(gpu_ctx, cfg, 512, kv_dtype="f32")
    m.fill_synthetic(21, CFG.WEIGHT_STD, 0.0)
    om = O.Model(cfg, synthetic_seed=21, std=CFG.WEIGHT_STD, norm_std=0.0, threads=8)
    s = O.Session(om, pool, 512)
    messages = [{"role": "user", "content": "Quem é você? Answer in one line, please: it's a test."}]
    text, ids = LB.chat(m, tok, messages, 24, date="November 07, 2026")
    prompt = tok.encode(LB.render_chat(messages, True, "November 07, 2026"))
    sfx = tok.encode("<|start_of_role|>assistant<|end_of_role|>")
    assert prompt[-len(sfx):] == sfx
    # the oracle: the prompt, then greedy ids (last maximum) until the EOS or 24 new ids
    for t in prompt[:-1]:
        s.step(int(t))
    lo, _, _ = s.step(int(prompt[-1]))
    want = []
    for _ in range(24):
        nxt = O.argmax_last(lo)
        want.append(nxt)
        if nxt == 0:
            break
        lo, _, _ = s.step(nxt)
    assert ids.tolist() == want
    body = want[:-1] if want and want[-1] == 0 else want
    assert text == tok.decode(body)
    print(f"chat: {len(prompt)} prompt ids, {len(want)} generated, text {text[:40]!r}")
    s.close()
    om.close()
    m.close()
    tok.close()
