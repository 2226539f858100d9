"""Fixtures of the tokenizer tests (tests/test_tokenizer.py).

1. bpe_tokenizer.json: a byte-level BPE tokenizer in the Granite 3.1 tokenizer.json configuration (no normalizer;
   ByteLevel pre-tokenizer with add_prefix_space false and use_regex true; BPE without dropout, unk token or byte
   fallback; ByteLevel decoder; special added tokens, <|end_of_text|> = 0), trained with the Hugging Face `tokenizers`
   library on a seeded synthetic corpus.  The Granite vocabulary itself is not available offline; the reference
   (rust/moe-rt/src/tokenizador.rs) is checked against `tokenizers`, and so is the restatement here, on this file.
   Like Granite's, its alphabet lacks the symbols of bytes 0xC0, 0xC1, 0xF1 and 0xF5..0xFF.
2. tokenizer_cases.json:
   - "encode": texts and the ids `tokenizers` gives them with bpe_tokenizer.json: the reference's edge-case texts
     (category "borda" of qual-runs/A2-LOTE-20261103/5a-referencia/casos.json) and synthetic ones;
   - "chat": the reference's chat-template cases of the same file (messages, add_generation_prompt, date and the text
     transformers' apply_chat_template rendered with the Granite 3.1 template);
   - "cut": id prefixes that split a character, with the bytes decoded lossily by Python (U+FFFD per maximal
     invalid subsequence).

Run with `tokenizers` installed and the reference checkout's root in LASTRO_REFERENCE (the cases file sits at
qual-runs/A2-LOTE-20261103/5a-referencia/casos.json under it): python tests/golden/gen_tokenizer_golden.py
"""
import json
import os
import random

from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

HERE = os.path.dirname(os.path.abspath(__file__))
CASES = os.path.join(os.environ.get("LASTRO_REFERENCE", "reference"), "qual-runs", "A2-LOTE-20261103", "5a-referencia",
                     "casos.json")

SPECIAL = ["<|end_of_text|>", "<fim_prefix>", "<fim_middle>", "<fim_suffix>", "<fim_pad>", "<filename>",
           "<|start_of_role|>", "<|end_of_role|>", "<|tool_call|>", "<|ab|>", "<|ab|>c"]
MISSING_BYTES = [0xC0, 0xC1, 0xF1] + list(range(0xF5, 0x100))


def byte_symbols():
    out, n = {}, 0
    for b in range(256):
        if 33 <= b <= 126 or 161 <= b <= 172 or 174 <= b <= 255:
            out[b] = chr(b)
        else:
            out[b] = chr(256 + n)
            n += 1
    return out


def corpus(seed=5, n_lines=6000):
    rng = random.Random(seed)
    syl = ["ta", "ke", "ri", "mo", "lu", "sa", "ne", "po", "di", "ga", "ex", "pert", "rou", "ter", "lay", "er", "to",
           "ken", "str", "ing", "tion", "al", "ed", "ly", "the", "and", "of", "in", "que", "ção", "ões", "mem", "ória"]
    scripts = ["日本語のテキスト", "中文字符", "Привет мир", "Γειά σου", "مرحبا بالعالم", "שלום עולם", "नमस्ते दुनिया",
               "สวัสดี", "안녕하세요", "😀🚀✨", "Ⅻ ⓐⓑ", "١٢٣ ٤٥", "೧೨೩", "café naïve façade", "ação coração"]
    contr = ["'s", "'t", "'re", "'ve", "'ll", "'d", "'m"]
    code = ["def f(x):\n    return x * 2\n", "for (int i = 0; i < n; ++i) { a[i] += b[i]; }", "{\"k\": [1, 2.5, null]}",
            "if x != y and not z: pass", "SELECT * FROM t WHERE id = 42;", "grep -E '^[a-z]+$' file.txt | wc -l"]
    lines = []
    for _ in range(n_lines):
        parts = []
        for _ in range(rng.randint(3, 14)):
            r = rng.random()
            if r < 0.55:
                w = "".join(rng.choice(syl) for _ in range(rng.randint(1, 4)))
                if rng.random() < 0.2:
                    w = w.capitalize()
                if rng.random() < 0.1:
                    w += rng.choice(contr)
                parts.append(w)
            elif r < 0.65:
                parts.append(str(rng.randint(0, 10 ** rng.randint(1, 7))))
            elif r < 0.75:
                parts.append(rng.choice([",", ".", "!", "?", ";", ":", "--", "(", ")", "\"", "...", "%", "$"]))
            elif r < 0.85:
                parts.append(rng.choice(scripts))
            else:
                parts.append(rng.choice(code))
        sep = rng.choice([" ", " ", " ", "  ", "\t", "\n", " \n"])
        lines.append(sep.join(parts))
    return lines


def synthetic_texts(seed=7):
    rng = random.Random(seed)
    texts = ["", " ", "   ", "\n", "a", "'s", "x's", "it's don't we're they've I'll she'd I'm", "  leading", "trailing  ",
             "a  \n\n  b", "\t\ttab", "1234567890 12.5e-3", "<|end_of_text|>", "<|end_of_text|><|end_of_text|>",
             "x<|start_of_role|>user<|end_of_role|>y", "<|ab|>c<|ab|>d<|ab|", "<|ab|>cc", "tool<|tool_call|>[1]",
             "é́ é", "\U0001F600 \U0001F680x", "ⅠⅡ Ⓐ", "٠١٢ ०१",
             "�", "\U00040000\U0005ABCD", "　 x y\u0085z", "!!'s ?'re 's't"]
    pool = [chr(c) for c in list(range(0x20, 0x7F)) + [0xE9, 0xE7, 0x3B1, 0x416, 0x5D0, 0x627, 0x915, 0x93E, 0xE01,
                                                          0x4E2D, 0x65E5, 0xAC00, 0x1F600, 0x2160, 0x24B6, 0x660,
                                                          0x3000, 0xA0, 0x9, 0xA, 0xD, 0x27]]
    for _ in range(200):
        texts.append("".join(rng.choice(pool) for _ in range(rng.randint(1, 40))))
    return texts


def main():
    alphabet = [s for b, s in byte_symbols().items() if b not in MISSING_BYTES]
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=4096, min_frequency=2, special_tokens=SPECIAL, initial_alphabet=alphabet,
                                  show_progress=False)
    tok.train_from_iterator(corpus(), trainer=trainer)
    path = os.path.join(HERE, "bpe_tokenizer.json")
    tok.save(path)
    with open(path) as f:
        spec = json.load(f)
    assert spec["normalizer"] is None and spec["model"]["byte_fallback"] is False

    ref = json.load(open(CASES))
    edge = [c["texto"] for c in ref["casos"] if c["categoria"] == "borda"]
    texts = edge + synthetic_texts()
    encode = [{"text": t, "ids": tok.encode(t, add_special_tokens=False).ids} for t in texts]
    chat = [{"name": c["nome"], "messages": c["mensagens"], "add_generation_prompt": c["add_generation_prompt"],
             "date": c["data"], "rendered": c["renderizado"]} for c in ref["casos"] if c["tipo"] == "chat"]
    cut = []
    for t in ["ação 日本 😀 ok", "naïve 😀😀 ẞ", "\U0001F680 \U0001F600x"]:
        ids = tok.encode(t, add_special_tokens=False).ids
        for k in range(1, len(ids) + 1):
            raw = b"".join(bytes(bytearray(byte_value(tok.id_to_token(i)))) for i in ids[:k])
            cut.append({"ids": ids[:k], "text": raw.decode("utf-8", errors="replace")})
    with open(os.path.join(HERE, "tokenizer_cases.json"), "w") as f:
        json.dump({"tokenizers": __import__("tokenizers").__version__, "encode": encode, "chat": chat, "cut": cut}, f,
                  ensure_ascii=False, indent=0)
    print(f"{len(encode)} encode cases, {len(chat)} chat cases, {len(cut)} cut prefixes; vocab {tok.get_vocab_size()}")


_INV = {s: b for b, s in byte_symbols().items()}


def byte_value(token):
    return [_INV[ch] for ch in token]


if __name__ == "__main__":
    main()
