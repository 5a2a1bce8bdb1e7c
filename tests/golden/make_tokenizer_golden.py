"""Generates the tokenizer fixtures in tests/golden/tokenizer/ (run in a container
that has the Python `tokenizers` package; the fixtures are committed).

The reference builds its tokenizer with the HF `tokenizers` crate
(packages/rust/crates/oxbitnet/src/tokenizer.rs:20-92, crate 0.21.4 in
packages/rust/Cargo.lock): a BPE model over the GGUF vocabulary and merges with
unk token "<unk>", a ByteLevel pre-tokenizer and decoder with
add_prefix_space = false, trim_offsets = true, use_regex = false. The Python
`tokenizers` package wraps the same Rust library, so this script builds exactly
that pipeline and records what it produces.

No real vocabulary is available offline, so a small byte-level BPE is trained
here on a seeded synthetic corpus (ASCII words, punctuation, digits, accented
Latin, CJK and emoji), and the LLaMA 3 chat specials are appended to its
vocabulary the way a GGUF token list carries them.
"""
import json
import os
import random

from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tokenizer")
SPECIALS = ["<|begin_of_text|>", "<|end_of_text|>", "<|start_header_id|>",
            "<|end_header_id|>", "<|eot_id|>"]


def corpus(seed=7, n=4000):
    rng = random.Random(seed)
    syll = ["ta", "ne", "ri", "ko", "mu", "sa", "lo", "vi", "en", "th", "er", "in", "an", "qu",
            "st", "ing", "ion", "the", "and"]
    extra = ["é", "ü", "ñ", "ç", "日本", "語", "😀", "🚀", "—", "…", "€"]
    punct = [".", ",", "!", "?", ":", ";", "'s", "'t", "(", ")", "\n", "\n\n", "  ", "\t"]
    out = []
    for _ in range(n):
        words = []
        for _ in range(rng.randint(3, 12)):
            w = "".join(rng.choice(syll) for _ in range(rng.randint(1, 3)))
            if rng.random() < 0.1:
                w += rng.choice(extra)
            if rng.random() < 0.15:
                w = w.capitalize()
            if rng.random() < 0.1:
                w = str(rng.randint(0, 2025))
            words.append(w)
            if rng.random() < 0.2:
                words.append(rng.choice(punct))
        out.append(" ".join(words))
    return out


def reference_tokenizer(vocab: dict, merges: list) -> Tokenizer:
    bpe = models.BPE(vocab=vocab, merges=merges, unk_token="<unk>")
    tok = Tokenizer(bpe)
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, trim_offsets=True,
                                                 use_regex=False)
    tok.decoder = decoders.ByteLevel(add_prefix_space=False, trim_offsets=True, use_regex=False)
    return tok


def main():
    os.makedirs(HERE, exist_ok=True)
    trainer_tok = Tokenizer(models.BPE(unk_token="<unk>"))
    trainer_tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False)
    trainer = trainers.BpeTrainer(vocab_size=700, special_tokens=["<unk>"],
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  show_progress=False)
    trainer_tok.train_from_iterator(corpus(), trainer)
    model = json.loads(trainer_tok.to_str())["model"]
    vocab = model["vocab"]
    merges = [tuple(m) if isinstance(m, list) else tuple(m.split(" ", 1)) for m in model["merges"]]
    tokens = [None] * len(vocab)
    for t, i in vocab.items():
        tokens[i] = t
    assert all(t is not None for t in tokens)
    tokens += SPECIALS
    full_vocab = {t: i for i, t in enumerate(tokens)}
    tok = reference_tokenizer(full_vocab, merges)

    rng = random.Random(11)
    texts = ["", "a", "Hello, world!", "the quick brown fox", "  leading spaces",
             "trailing space ", "line one\nline two\n\nline four", "tabs\tand\tmore",
             "numbers 12345 and 2025", "café naïve façade", "日本語のテキスト", "emoji 😀🚀!",
             "mixed: ta-ne-ri ing ion the and", "<|eot_id|> is plain text here",
             "<unk>", " nbsp​zero-width", "x" * 200, "ß∂ƒ©˙∆˚¬…æ"]
    texts += [s[:rng.randint(1, 120)] for s in rng.sample(corpus(seed=99, n=300), 40)]
    cases = []
    for t in texts:
        ids = tok.encode(t, add_special_tokens=False).ids
        cases.append({"text": t, "ids": ids, "decoded": tok.decode(ids, skip_special_tokens=True)})
    decode_one = [tok.decode([i], skip_special_tokens=True) for i in range(len(tokens))]
    with open(os.path.join(HERE, "vocab.json"), "w") as f:
        json.dump({"tokens": tokens, "merges": [f"{a} {b}" for a, b in merges],
                   "bos": tokens.index("<|begin_of_text|>"),
                   "eos": tokens.index("<|end_of_text|>")}, f, ensure_ascii=False)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump({"generator": "tokenizers " + __import__("tokenizers").__version__,
                   "cases": cases, "decode_one": decode_one}, f, ensure_ascii=False, indent=0)
    print(len(tokens), "tokens,", len(merges), "merges,", len(cases), "cases")


if __name__ == "__main__":
    main()
