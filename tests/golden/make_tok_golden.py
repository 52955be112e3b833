"""Generate tests/golden/qwen2_tok.json: golden vectors for the Qwen2
tokenizer (hako_b200/host/hakm_bpe.c, hakm_pretok.c).

The oracle is the HF `tokenizers` library (0.22.2 here) configured as Qwen2's
own tokenizer.json configures it: pre_tokenizer = Sequence[Split(<the Qwen2
pattern>, behavior "isolated"), ByteLevel(add_prefix_space false, use_regex
false)], model = BPE without unk or dropout. The Qwen2 vocabulary itself is
not available offline, so a small vocabulary is trained here with the same
pipeline on seeded synthetic text (words, numbers, punctuation runs,
contractions, whitespace runs, non-Latin letters and digits), and written as
an MLF2 tokenizer blob (include/mlf2.h:89-102 of mithraeums/hako: u32
n_tokens, u32 n_merges, {u8 type, u32 len, bytes} per token, {u32 len, "A B"}
per merge in rank order).

The fixture holds the blob (base64), the pretokenizer's piece ends (byte
offsets) and the token ids the oracle gives for a set of texts: seeded
synthetic texts and the edge cases (empty, whitespace-only, newline runs,
long letter and digit runs, every contraction in both cases).

    python tests/golden/make_tok_golden.py     # rewrites qwen2_tok.json
"""
from __future__ import annotations

import base64
import json
import os
import random
import struct

QWEN2_PATTERN = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}"
                 r"| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+")
SPECIAL = ["<|endoftext|>", "<|im_start|>", "<|im_end|>"]
HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "qwen2_tok.json")

SYLLABLES = ["th", "e", "qu", "ick", "br", "own", "fo", "x", "ju", "mp", "s", "ov", "er", "la", "zy", "do", "g",
             "in", "g", "an", "d", "ti", "on", "re", "st", "ar", "al", "ly", "pre", "ment"]
FOREIGN = ["été", "Straße", "naïve", "中文", "日本語", "привет", "Ελλάδα", "مرحبا", "१२३", "٣٤", "Ⅻ", "ǅemal",
           "ﬁne", "ſtill", "😀", "é", " ", "　"]
PUNCT = [".", ",", "!", "?", "...", "!!!", "--", "(", ")", "\"", ":", ";", "#", "$", "%", "&", "*", "@", "/", "'"]
SPACES = [" ", " ", " ", " ", "  ", "   ", "\t", "\n", "\n\n", "\r\n", " \n", "\n ", " \t "]
CONTRACTIONS = ["'s", "'t", "'re", "'ve", "'m", "'ll", "'d", "'S", "'T", "'RE", "'Ve", "'M", "'LL", "'D"]


def word(rng: random.Random) -> str:
    r = rng.random()
    if r < 0.62:
        w = "".join(rng.choice(SYLLABLES) for _ in range(rng.randint(1, 4)))
        return w.capitalize() if rng.random() < 0.2 else (w.upper() if rng.random() < 0.05 else w)
    if r < 0.76:
        return str(rng.randint(0, 10 ** rng.randint(1, 7)))
    if r < 0.86:
        return rng.choice(FOREIGN)
    if r < 0.96:
        return rng.choice(PUNCT) * rng.randint(1, 2)
    return rng.choice(SYLLABLES) + rng.choice(CONTRACTIONS)


def text(rng: random.Random, n_words: int) -> str:
    out = []
    for _ in range(n_words):
        out.append(word(rng))
        out.append(rng.choice(SPACES) if rng.random() < 0.85 else "")
    return "".join(out)


def edge_cases() -> list[str]:
    return ["", " ", "   ", "\n", "\n\n\n", "\r\n\r\n", " \n \n ", "\t", "a", "a ", " a", "a  b", "a   b  ",
            "hello world", "Hello, world!!! 12345 and 3.14159", "don't I'M we'LL they've she'd you're It's",
            "'s's'ss", "x'", "'", "''", "aſ", "ab'ſc", "a-b_c", "#include <stdio.h>\nint main() {}\n",
            "    indented\n\tcode();\n", "  trailing  ", "¡Hola! ¿Qué tal?", "2024-12-02T10:00:00Z",
            "9" * 300, "z" * 3000, "ab" * 700 + " " + "!?" * 300, "中文 text 混合 123", "emoji 😀😀 ok",
            "é (decomposed)", "non breaking space", "ideographic　space"]


def build_vocab(corpus: list[str], vocab_size: int):
    from tokenizers import Regex, Tokenizer, models, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(QWEN2_PATTERN), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    trainer = trainers.BpeTrainer(vocab_size=vocab_size, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  special_tokens=SPECIAL, show_progress=False)
    tok.train_from_iterator(corpus, trainer)
    return tok


def mlf2_blob(tok) -> tuple[bytes, int]:
    model = json.loads(tok.to_str())["model"]
    vocab = sorted(model["vocab"].items(), key=lambda kv: kv[1])
    assert [i for _, i in vocab] == list(range(len(vocab)))
    merges = [m if isinstance(m, str) else " ".join(m) for m in model["merges"]]
    out = [struct.pack("<II", len(vocab), len(merges))]
    for s, _ in vocab:
        b = s.encode("utf-8")
        out.append(struct.pack("<BI", 3 if s in SPECIAL else 1, len(b)) + b)
    for m in merges:
        b = m.encode("utf-8")
        out.append(struct.pack("<I", len(b)) + b)
    return b"".join(out), model["vocab"]["<|endoftext|>"]


def piece_ends(pre, s: str) -> list[int]:
    ends, pos = [], 0
    for piece, _ in pre.pre_tokenize_str(s):
        pos += len(piece.encode("utf-8"))
        ends.append(pos)
    return ends


def main() -> None:
    import tokenizers
    from tokenizers import Regex, pre_tokenizers
    rng = random.Random(20241202)
    corpus = [text(rng, rng.randint(20, 120)) for _ in range(3000)]
    tok = build_vocab(corpus, 1200)
    blob, eos = mlf2_blob(tok)
    split = pre_tokenizers.Split(Regex(QWEN2_PATTERN), behavior="isolated", invert=False)
    trng = random.Random(7)
    texts = edge_cases() + [text(trng, trng.randint(1, 60)) for _ in range(120)]
    cases = [{"text": s, "ends": piece_ends(split, s), "ids": tok.encode(s, add_special_tokens=False).ids}
             for s in texts]
    fixture = {
        "generator": "tests/golden/make_tok_golden.py",
        "oracle": "HF tokenizers %s, Qwen2 pre_tokenizer + ByteLevel + BPE" % tokenizers.__version__,
        "pattern": QWEN2_PATTERN,
        "eos_id": eos,
        "n_tokens": tok.get_vocab_size(),
        "blob_b64": base64.b64encode(blob).decode(),
        "cases": cases,
    }
    with open(OUT, "w") as f:
        json.dump(fixture, f, ensure_ascii=True, separators=(",", ":"))
    print(f"{OUT}: {len(cases)} cases, vocab {fixture['n_tokens']}, blob {len(blob)} bytes")


if __name__ == "__main__":
    main()
