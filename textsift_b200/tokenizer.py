"""Python face of the library's host tokenizer (C ABI ts_tok_*): the
counterpart of textsift's Tokenizer (packages/textsift/src/browser/model/
tokenizer.ts) with the same `encode` result (token ids, attention mask,
tokenToCharOffset in UTF-16 code units) plus a multi-threaded batch encode.
"""
import ctypes
from dataclasses import dataclass
from typing import List, Sequence, Tuple, Union

import numpy as np

from . import abi


@dataclass
class EncodeResult:
    """Tokenizer.encode's result (tokenizer.ts:34-55)."""
    token_ids: np.ndarray            # int32 [n]
    attention_mask: np.ndarray       # uint8 [n], all ones
    token_to_char_offset: np.ndarray  # uint32 [n + 1], UTF-16 code units
    byte_offsets: np.ndarray         # uint32 [n + 1], UTF-8 bytes of the input
    decoded_mismatch: bool = False


class Tokenizer:
    """o200k-style byte-level BPE from a tokenizer.json (Tokenizer.fromBundle)."""

    def __init__(self, tokenizer_json: Union[bytes, str]):
        data = tokenizer_json.encode("utf-8") if isinstance(tokenizer_json, str) else bytes(tokenizer_json)
        err = ctypes.create_string_buffer(1024)
        self._lib = abi.lib()
        self._h = self._lib.ts_tok_create(data, len(data), err, 1024)
        if not self._h:
            raise ValueError(err.value.decode("utf-8", "replace"))

    @classmethod
    def from_file(cls, path: str) -> "Tokenizer":
        with open(path, "rb") as f:
            return cls(f.read())

    def vocab_size(self) -> int:
        return int(self._lib.ts_tok_vocab_size(self._h))

    def encode(self, text: str) -> EncodeResult:
        b = text.encode("utf-8")
        n = ctypes.c_size_t()
        abi.check(self._lib.ts_tok_encode(self._h, b, len(b), None, None, None, 0, ctypes.byref(n)))
        ids = np.empty(n.value, np.int32)
        co = np.empty(n.value + 1, np.uint32)
        bo = np.empty(n.value + 1, np.uint32)
        abi.check(self._lib.ts_tok_encode(self._h, b, len(b), ids.ctypes.data, co.ctypes.data, bo.ctypes.data,
                                          n.value, ctypes.byref(n)))
        return EncodeResult(ids, np.ones(n.value, np.uint8), co, bo)

    def encode_batch(self, texts: Sequence[str], threads: int = 0) -> List[Tuple[np.ndarray, np.ndarray, np.ndarray]]:
        """[(ids, starts, ends)] per text; starts/ends in UTF-16 code units."""
        enc = [t.encode("utf-8") for t in texts]
        k = len(enc)
        ptrs = (ctypes.c_char_p * max(1, k))(*enc)
        lens = (ctypes.c_size_t * max(1, k))(*[len(e) for e in enc])
        begin = np.zeros(k + 1, np.uint64)
        # every token covers at least one byte of its text: one call with room
        # for as many tokens as there are bytes tokenizes each text once
        cap = max(1, sum(len(e) for e in enc))
        ids = np.empty(cap, np.int32)
        st = np.empty(cap, np.uint32)
        en = np.empty(cap, np.uint32)
        abi.check(self._lib.ts_tok_encode_batch(self._h, ptrs, lens, k, threads, ids.ctypes.data, st.ctypes.data,
                                                en.ctypes.data, cap, begin.ctypes.data))
        return [(ids[begin[i]:begin[i + 1]], st[begin[i]:begin[i + 1]], en[begin[i]:begin[i + 1]]) for i in range(k)]

    def decode(self, ids) -> str:
        a = np.ascontiguousarray(ids, np.int32)
        n = ctypes.c_size_t()
        abi.check(self._lib.ts_tok_decode(self._h, a.ctypes.data, a.size, None, 0, ctypes.byref(n)))
        buf = ctypes.create_string_buffer(max(1, n.value))
        abi.check(self._lib.ts_tok_decode(self._h, a.ctypes.data, a.size, buf, n.value, ctypes.byref(n)))
        return buf.raw[:n.value].decode("utf-8", "replace")

    def close(self) -> None:
        if getattr(self, "_h", None):
            self._lib.ts_tok_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()
