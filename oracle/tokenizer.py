"""Test oracle: a restatement of textsift's o200k-style BPE tokenizer
(packages/textsift/src/browser/model/tokenizer.ts) in Python.  Test
infrastructure only: the library's tokenizer (textsift_b200/csrc/
tokenizer.cu, C ABI ts_tok_*) is checked against it; nothing in the product
imports this file.

The reference runs in JavaScript on UTF-16 strings; this restatement works on
Python strings (code points) and reports offsets in UTF-16 code units, as
`tokenToCharOffset` does.  The pretokenizer pattern is the reference's
(tokenizer.ts:510-525) with the inline case-insensitive contraction group
expanded the same way (tokenizer.ts:528-545), and with JavaScript's `\\s`
spelled out, since Python's differs (it also matches U+001C-U+001F, U+0085).
Unicode letter/mark/number classes are those of the `regex` module, which
may be a different Unicode version from the JavaScript engine the reference
runs in: parity is exact for every code point whose class the two agree on.
"""
import json

import regex

# ECMAScript \s (WhiteSpace + LineTerminator)
_JS_S = "\\t\\n\\x0b\\x0c\\r \\xa0\\u1680\\u2000-\\u200a\\u2028\\u2029\\u202f\\u205f\\u3000\\ufeff"
S = "[" + _JS_S + "]"
NOT_S = "[^" + _JS_S + "]"


def _contractions():
    # tokenizer.ts:528-545: every ASCII case variant of each base, in order
    def cases(s):
        if not s:
            return [""]
        c, tail = s[0], cases(s[1:])
        variants = [c] if c.lower() == c.upper() else [c.lower(), c.upper()]
        return [v + t for v in variants for t in tail]
    alts = [v for base in ["'s", "'t", "'re", "'ve", "'m", "'ll", "'d"] for v in cases(base)]
    return "(?:" + "|".join(alts) + ")?"


def pretokenizer_pattern():
    """tokenizer.ts:510-525 with \\s as JavaScript defines it."""
    c = _contractions()
    not_crlf_l_n = "[^\\r\\n\\p{L}\\p{N}]"
    up = "[\\p{Lu}\\p{Lt}\\p{Lm}\\p{Lo}\\p{M}]"
    lo = "[\\p{Ll}\\p{Lm}\\p{Lo}\\p{M}]"
    return (not_crlf_l_n + "?" + up + "*" + lo + "+" + c +
            "|" + not_crlf_l_n + "?" + up + "+" + lo + "*" + c +
            "|\\p{N}{1,3}" +
            "| ?[^" + _JS_S + "\\p{L}\\p{N}]+[\\r\\n/]*" +
            "|" + S + "*[\\r\\n]+" +
            "|" + S + "+(?!" + NOT_S + ")" +
            "|" + S + "+")


def bytes_to_unicode():
    """GPT-2's byte -> printable code point map (tokenizer.ts:488-507)."""
    bs = list(range(ord("!"), ord("~") + 1)) + list(range(ord("¡"), ord("¬") + 1)) + list(range(ord("®"), ord("ÿ") + 1))
    cs = list(bs)
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    out = [0] * 256
    for b, c in zip(bs, cs):
        out[b] = c
    return out


def _u16len(s):
    return sum(2 if ord(ch) > 0xFFFF else 1 for ch in s)


class Tokenizer:
    """Tokenizer.fromBundle / encode / decode (tokenizer.ts:134-334)."""

    def __init__(self, tokenizer_json):
        j = json.loads(tokenizer_json)
        if j.get("model", {}).get("type") != "BPE":
            raise ValueError("tokenizer.json model.type must be BPE")
        self.vocab = dict(j["model"]["vocab"])
        for t in j.get("added_tokens", []):
            self.vocab[t["content"]] = t["id"]
        self.id_to_token = {i: t for t, i in self.vocab.items()}
        self.ranks = {}
        for i, m in enumerate(j["model"]["merges"]):
            a, b = (m.split(" ", 1) if isinstance(m, str) else m)
            self.ranks[(a, b)] = i  # Map.set: a repeated pair keeps its last rank (tokenizer.ts:183-188)
        self.b2c = bytes_to_unicode()
        self.c2b = {c: b for b, c in enumerate(self.b2c)}
        self.special = {t["content"]: t["id"] for t in j.get("added_tokens", []) if t.get("special")}
        # tokenizer.ts:190-204: the regex-escaped literals sorted (stably) by
        # descending length in UTF-16 units; the first that matches at a position wins
        meta = set(".*+?^${}()|[]\\")
        self.special_order = sorted(self.special, key=lambda t: -(_u16len(t) + sum(ch in meta for ch in t)))
        self.pre = regex.compile(pretokenizer_pattern())
        self.cache = {}

    # tokenizer.ts:340-362
    def _split_special(self, text):
        if not self.special:
            return [(text, 0, False)]
        out, cursor, i = [], 0, 0
        while i < len(text):
            hit = next((s for s in self.special_order if text.startswith(s, i)), None)
            if hit is None:
                i += 1
                continue
            if i > cursor:
                out.append((text[cursor:i], cursor, False))
            out.append((hit, i, True))
            cursor = i = i + len(hit)
        if cursor < len(text):
            out.append((text[cursor:], cursor, False))
        return out

    # tokenizer.ts:364-397 (Split with Isolated behaviour: matches and gaps)
    def _pretokenize(self, text, base):
        out, cursor = [], 0
        for m in self.pre.finditer(text):
            if m.end() == m.start():
                continue
            if m.start() > cursor:
                out.append((text[cursor:m.start()], base + cursor))
            out.append((m.group(0), base + m.start()))
            cursor = m.end()
        if cursor < len(text):
            out.append((text[cursor:], base + cursor))
        return out

    # tokenizer.ts:413-458
    def _bpe(self, mapped):
        if not mapped:
            return []
        if mapped in self.cache:
            return self.cache[mapped]
        sym = list(mapped)
        while len(sym) > 1:
            best, best_rank = -1, None
            for i in range(len(sym) - 1):
                r = self.ranks.get((sym[i], sym[i + 1]))
                if r is not None and (best_rank is None or r < best_rank):
                    best, best_rank = i, r
            if best < 0:
                break
            a, b = sym[best], sym[best + 1]
            merged, i = [], 0
            while i < len(sym):
                if i < len(sym) - 1 and sym[i] == a and sym[i + 1] == b:
                    merged.append(a + b)
                    i += 2
                else:
                    merged.append(sym[i])
                    i += 1
            sym = merged
        ids = [self.vocab[s] for s in sym]
        self.cache[mapped] = ids
        return ids

    # tokenizer.ts:467-478 (byte positions of each UTF-16 unit) + 460-504
    def _distribute(self, piece, ids, start_u16):
        units = []  # byte offset at each UTF-16 code unit of the piece
        byte = 0
        for ch in piece:
            n = len(ch.encode("utf-8"))
            units.append(byte)
            if ord(ch) > 0xFFFF:
                units.append(byte)
            byte += n
        units.append(byte)
        n_units = len(units) - 1
        bounds = [0]
        bc = 0
        for i in ids:
            bc += len(self.id_to_token[i])
            bounds.append(bc)
        if bc != byte:
            bounds = [min(b, byte) for b in bounds]
        offs, u = [], 0
        for target in bounds:
            while u < n_units and units[u] < target:
                u += 1
            offs.append(u)
        return [(start_u16 + offs[i], start_u16 + offs[i + 1]) for i in range(len(ids))]

    def encode(self, text):
        """(token ids, tokenToCharOffset) with offsets in UTF-16 code units."""
        ids, starts, ends = [], [], []
        for piece, cp_start, special in self._split_special(text):
            u16_base = _u16len(text[:cp_start])
            if special:
                ids.append(self.special[piece])
                starts.append(u16_base)
                ends.append(u16_base + _u16len(piece))
                continue
            for pt, pstart in self._pretokenize(piece, 0):
                mapped = "".join(chr(self.b2c[b]) for b in pt.encode("utf-8"))
                tids = self._bpe(mapped)
                base = u16_base + _u16len(piece[:pstart])
                for tid, (s, e) in zip(tids, self._distribute(pt, tids, base)):
                    ids.append(tid)
                    starts.append(s)
                    ends.append(e)
        offsets = starts + [ends[-1] if ids else 0]
        return ids, offsets

    def decode(self, ids):
        out = bytearray()
        for i in ids:
            tok = self.id_to_token.get(i)
            if tok is None:
                continue
            if tok in self.special:
                out += tok.encode("utf-8")
                continue
            for ch in tok:
                b = self.c2b.get(ord(ch))
                out += ch.encode("utf-8") if b is None else bytes([b])
        return out.decode("utf-8", errors="replace")
