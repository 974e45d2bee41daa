"""The library's host tokenizer (C ABI ts_tok_*, textsift_b200.tokenizer)
against the restatement of textsift's Tokenizer (oracle/tokenizer.py,
packages/textsift/src/browser/model/tokenizer.ts) on a synthetic BPE
tokenizer.json (tests/golden/gen_tokenizer_fixture.py): token ids and
tokenToCharOffset (UTF-16 code units) must be identical.

The real model's tokenizer.json is not available here; the fixture is
trained on a corpus covering the scripts and character classes the
pretokenizer pattern distinguishes, and the texts below probe each of its
alternatives and their boundaries.  CPU only (no GPU is involved).
"""
import os
import random

import numpy as np
import pytest

from conftest import ROOT

FIXTURE = os.path.join(ROOT, "tests", "golden", "tokenizer_synth.json")

# characters by the class boundaries the pattern cares about
POOL = {
    "lower": "abcdefghijklmnopqrstuvwxyzßàéöçñαβγабвг",
    "upper": "ABCDEFGHIJKLMNOPQRSTUVWXYZÀÉÖÇÑΑΒΓАБВГ",
    "title": "ǅǈǋǲᾈᾉ",              # Lt
    "modifier": "ʰʲˈˌ々ー",           # Lm
    "other_letter": "的一是中文ابتकखगאבגあいう",  # Lo
    "mark": "́̈ःा्ִ⃝",  # Mn, Mc, Me
    "digit": "0123456789٠١٢३४५⅓²",   # Nd, No, Nl-ish
    "punct": "!\"#$%&()*+,-./:;<=>?@[\\]^_`{|}~«»¿¡—…€™",
    "space": " \t  　  ﻿\u000b\u000c",  # JavaScript \s beyond ' '
    "crlf": "\r\n",
    "not_js_space": "\u0085\u001c\u001f​",  # \s in Python, not in JavaScript
    "emoji": "😀🚀👍🏽🎉💡𝔘🇩🇪‍",
    "apos": "'",
}
CONTRACTIONS = ["'s", "'t", "'re", "'ve", "'m", "'ll", "'d", "'S", "'T", "'RE", "'Ve", "'lL", "'D", "'x"]
SPECIALS = ["<|endoftext|>", "<|startoftext|>", "<|pad|>", "<|pad|>!", "<|pad", "|>"]


def random_text(r, n):
    out = []
    keys = list(POOL)
    while len(out) < n:
        k = r.random()
        if k < 0.06:
            out.append(r.choice(CONTRACTIONS))
        elif k < 0.09:
            out.append(r.choice(SPECIALS))
        elif k < 0.15:
            out.append(r.choice(["word", "Word", "WORD", "wORD", " the", "  ", "\r\n", "\n\n", " \n ", "12345678"]))
        else:
            cls = r.choice(keys)
            out.append("".join(r.choice(POOL[cls]) for _ in range(r.randint(1, 4))))
    return "".join(out)


EDGE = [
    "", " ", "  ", "\n", "\r\n", " \r\n", "\r\n ", "a", "A", "Aa", "aA", "AAAA", "ǅa", "ʰa", "́a", "á",
    "́", "12", "1234", "1234567", "١٢٣٤", "..", " ..", " ./\n/", "!\r\n/", "a  b", "a   ", "   a", "\t\ta",
    "don't", "DON'T", "it'S", "they'RE", "I'll", "x'", "'s", "''s", "a'sb", "<|endoftext|>", "a<|endoftext|>b",
    "<|pad|>!", "<|pad|>", "<|pad", "<|pad|><|pad|>!!", "😀", "a😀b", "👍🏽", " 🇩🇪 ", " a", "a ",
    "\u0085a", "a\u001cb", " ", "x y", "﻿a", "中文字", "中A", "Hello, World!", "e.g. 3.14 and 2,000",
    "https://example.com/path?q=1", "a\r\n\r\n\r\nb", "   \n   \n   x",
]


@pytest.fixture(scope="module")
def toks(cuda_lib):
    from oracle.tokenizer import Tokenizer as Ref
    from textsift_b200.tokenizer import Tokenizer
    data = open(FIXTURE, "rb").read()
    return Tokenizer(data), Ref(data)


def same(lib_tok, ref, text):
    e = lib_tok.encode(text)
    ids, offs = ref.encode(text)
    assert e.token_ids.tolist() == ids, repr(text)
    assert e.token_to_char_offset.tolist() == offs, repr(text)
    assert e.attention_mask.tolist() == [1] * len(ids)
    # byte offsets index the UTF-8 input and tile it
    b = text.encode("utf-8")
    assert e.byte_offsets[0] == 0 if ids else True
    assert e.byte_offsets[-1] == (len(b) if ids else 0)
    assert np.all(np.diff(e.byte_offsets.astype(np.int64)) >= 0)


def test_edge_cases(toks):
    lib_tok, ref = toks
    for text in EDGE:
        same(lib_tok, ref, text)


@pytest.mark.parametrize("seed", range(6))
def test_random_texts(toks, seed):
    lib_tok, ref = toks
    r = random.Random(1000 + seed)
    for _ in range(150):
        same(lib_tok, ref, random_text(r, r.randint(0, 60)))


def test_batch_matches_single(toks):
    lib_tok, ref = toks
    r = random.Random(77)
    texts = [random_text(r, r.randint(0, 80)) for _ in range(300)] + [""]
    got = lib_tok.encode_batch(texts, threads=4)
    for text, (ids, st, en) in zip(texts, got):
        rids, roffs = ref.encode(text)
        assert ids.tolist() == rids
        assert st.tolist() == roffs[:-1]
        if rids:
            assert en[-1] == roffs[-1]


def test_decode_round_trip(toks):
    lib_tok, ref = toks
    r = random.Random(5)
    for _ in range(100):
        text = random_text(r, r.randint(0, 40))
        ids = lib_tok.encode(text).token_ids
        assert lib_tok.decode(ids) == text == ref.decode(ids.tolist())


def test_vocab_size_and_errors(toks, cuda_lib):
    import ctypes
    from textsift_b200 import TextsiftCudaError
    from textsift_b200.tokenizer import Tokenizer
    lib_tok, ref = toks
    assert lib_tok.vocab_size() == max(ref.vocab.values()) + 1
    with pytest.raises(ValueError, match="BPE"):
        Tokenizer(b'{"model": {"type": "WordPiece", "vocab": {}, "merges": []}}')
    with pytest.raises(ValueError, match="tokenizer.json"):
        Tokenizer(b'{"model": {"type": "BPE", "vocab": {"a": 0}, "merges": [')
    n = ctypes.c_size_t()
    bad = b"ab\xff\xfe"
    assert cuda_lib.ts_tok_encode(lib_tok._h, bad, len(bad), None, None, None, 0, ctypes.byref(n)) != 0
    from textsift_b200 import abi
    assert "UTF-8" in abi.last_error()
    with pytest.raises(TextsiftCudaError):
        ids = np.empty(1, np.int32)
        abi.check(cuda_lib.ts_tok_encode(lib_tok._h, b"hello world", 11, ids.ctypes.data, None, None, 1,
                                         ctypes.byref(n)))
