"""Generate tests/golden/tokenizer_synth.json: a small byte-level BPE
tokenizer.json in the layout textsift's loader reads (model.type "BPE",
model.vocab, model.merges as [a, b] pairs, added_tokens), trained on a
seeded synthetic corpus.  The real model's tokenizer.json is not available
here, so the tokenizer tests use this one with oracle/tokenizer.py as the
reference.

The corpus mixes the scripts and character classes the pretokenizer pattern
distinguishes: Latin (lower, upper, title case, accents, contractions),
Greek, Cyrillic, CJK, Arabic, Devanagari with combining marks, digits,
punctuation and symbols, emoji (astral code points), and whitespace runs with
CR/LF, tabs and no-break spaces.

Usage: python tests/golden/gen_tokenizer_fixture.py
"""
import collections
import json
import os
import random
import sys

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", ".."))
from oracle.tokenizer import bytes_to_unicode, pretokenizer_pattern  # noqa: E402

import regex  # noqa: E402

N_MERGES = 1200
SPECIALS = ["<|endoftext|>", "<|startoftext|>", "<|pad|>", "<|pad|>!"]


def corpus(seed=2026, n_words=6000):
    r = random.Random(seed)
    latin = "etaoinshrdlucmfwypvbgkjqxz"
    pieces = []
    for _ in range(n_words):
        k = r.random()
        if k < 0.45:
            w = "".join(r.choice(latin[:12] if r.random() < 0.7 else latin) for _ in range(r.randint(1, 9)))
            form = r.random()
            w = w.capitalize() if form < 0.2 else (w.upper() if form < 0.27 else w)
            if r.random() < 0.06:
                w += r.choice(["'s", "'t", "'re", "'ve", "'m", "'ll", "'d", "'S", "'LL", "'Re"])
        elif k < 0.52:
            w = "".join(r.choice("éèàüößçñ" + latin[:6]) for _ in range(r.randint(2, 7)))
        elif k < 0.58:
            w = "".join(r.choice("αβγδεζηθικλμνξοπρστυφχψω") for _ in range(r.randint(2, 8)))
        elif k < 0.64:
            w = "".join(r.choice("абвгдежзийклмнопрстуфхцчшщ") for _ in range(r.randint(2, 8)))
            w = w.capitalize() if r.random() < 0.3 else w
        elif k < 0.69:
            w = "".join(r.choice("的一是不了人我在有他这中大来上国个到说") for _ in range(r.randint(1, 4)))
        elif k < 0.72:
            w = "".join(r.choice("ابتثجحخدذرزسشصضطظعغفقكلمنهوي") for _ in range(r.randint(2, 6)))
        elif k < 0.75:
            w = "".join(r.choice("कखगघचछजझटठडढतथदधनपफबभमयरलवसह") + r.choice(["", "ा", "ि", "ी", "ु", "्", "ं"])
                        for _ in range(r.randint(1, 4)))
        elif k < 0.84:
            w = str(r.randint(0, 10 ** r.randint(1, 7)))
        elif k < 0.92:
            w = "".join(r.choice("!\"#$%&()*+,-./:;<=>?@[\\]^_`{|}~") for _ in range(r.randint(1, 3)))
        elif k < 0.95:
            w = r.choice(["😀", "🚀", "👍🏽", "🎉", "💡", "𝔘𝔫𝔦", "🇩🇪"])
        else:
            w = r.choice(["\r\n", "\n", "\n\n", "\t", "  ", " ", " \n", "\r\n\r\n"])
        pieces.append(w)
        pieces.append(r.choice([" ", " ", " ", " ", "", "\n", ", ", ". "]))
    return "".join(pieces)


def train(text, n_merges):
    b2c = bytes_to_unicode()
    pre = regex.compile(pretokenizer_pattern())
    words = collections.Counter()
    for m in pre.finditer(text):
        words[tuple(chr(b2c[b]) for b in m.group(0).encode("utf-8"))] += 1
    vocab = {chr(b2c[b]): i for i, b in enumerate(range(256))}
    merges = []
    words = dict(words)
    for _ in range(n_merges):
        pairs = collections.Counter()
        for w, c in words.items():
            for a, b in zip(w, w[1:]):
                pairs[(a, b)] += c
        if not pairs:
            break
        (a, b), _ = max(pairs.items(), key=lambda kv: (kv[1], kv[0]))
        merges.append([a, b])
        vocab.setdefault(a + b, len(vocab))
        new = {}
        for w, c in words.items():
            out, i = [], 0
            while i < len(w):
                if i + 1 < len(w) and w[i] == a and w[i + 1] == b:
                    out.append(a + b)
                    i += 2
                else:
                    out.append(w[i])
                    i += 1
            t = tuple(out)
            new[t] = new.get(t, 0) + c
        words = new
    return vocab, merges


def main():
    vocab, merges = train(corpus(), N_MERGES)
    base = len(vocab)
    added = [{"id": base + i, "content": s, "special": True} for i, s in enumerate(SPECIALS)]
    doc = {"model": {"type": "BPE", "vocab": vocab, "merges": merges}, "added_tokens": added}
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tokenizer_synth.json")
    with open(out, "w", encoding="utf-8") as f:
        json.dump(doc, f, ensure_ascii=False, separators=(",", ":"))
    print(f"vocab {len(vocab)} + {len(added)} specials, {len(merges)} merges -> {out}")


if __name__ == "__main__":
    main()
