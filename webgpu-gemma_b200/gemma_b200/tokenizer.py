"""The reference's tokenizer (src/tokenizer.ts) through the C-ABI: libgemma_b200.so's
gg_tokenizer_* functions (csrc/gg_tokenizer.cpp), the greedy longest-match encoder with the
reference's UTF-16 code-unit semantics. Host only: it needs the library, not a GPU.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import gguf

FUNC_TOKEN_NAMES = ["<start_function_declaration>", "<end_function_declaration>", "<start_function_call>",
                    "<end_function_call>", "<start_function_response>", "<end_function_response>", "<escape>"]


class Tokenizer:
    def __init__(self, vocab: list[str]):
        from . import native
        self._lib = native.load()
        self.vocab = vocab
        raw = [t.encode("utf-8", "surrogatepass") for t in vocab]
        arr = (ctypes.c_char_p * len(raw))(*raw)
        lens = (ctypes.c_size_t * len(raw))(*[len(b) for b in raw])
        h = ctypes.c_void_p()
        rc = self._lib.gg_tokenizer_create(arr, lens, len(raw), ctypes.byref(h))
        if rc != 0:
            raise native.GemmaB200Error(f"gg_tokenizer_create failed ({rc})")
        self._h = h
        # funcTokens (tokenizer.ts:59-68): the function-call tokens the vocabulary has
        self.func_tokens = {n: i for n in FUNC_TOKEN_NAMES if (i := self.token_id(n)) >= 0}

    @classmethod
    def from_gguf(cls, parsed: "gguf.GGUFParsed") -> "Tokenizer":
        """extractFromGGUF (tokenizer.ts:26-41)."""
        kv = parsed.kv.get("tokenizer.ggml.tokens")
        if kv is None or kv.type != "array":
            raise ValueError("No tokenizer found in GGUF metadata")
        return cls([v.value for v in kv.value])

    def token_id(self, text: str) -> int:
        out = ctypes.c_int32()
        self._lib.gg_tokenizer_token_id(self._h, text.encode("utf-8"), ctypes.byref(out))
        return out.value

    def encode(self, text: str) -> list[int]:
        b = text.encode("utf-8", "surrogatepass")
        n = ctypes.c_int()
        cap = len(b) + 2  # at most one id per UTF-16 unit, plus <bos> and the leading '▁'
        ids = np.empty(cap, np.int32)
        rc = self._lib.gg_tokenizer_encode(self._h, b, len(b), ids.ctypes.data_as(ctypes.c_void_p), cap,
                                           ctypes.byref(n))
        if rc != 0 or n.value > cap:
            raise RuntimeError(f"gg_tokenizer_encode failed ({rc})")
        return ids[:n.value].tolist()

    def decode_tokens(self, ids) -> str:
        a = np.ascontiguousarray(np.asarray(list(ids), dtype=np.int32))
        ln = ctypes.c_size_t()
        self._lib.gg_tokenizer_decode(self._h, a.ctypes.data_as(ctypes.c_void_p), a.size, None, 0, ctypes.byref(ln))
        buf = ctypes.create_string_buffer(ln.value)
        self._lib.gg_tokenizer_decode(self._h, a.ctypes.data_as(ctypes.c_void_p), a.size, buf, ln.value,
                                      ctypes.byref(ln))
        return buf.raw[:ln.value].decode("utf-8")

    def decode_token(self, tid: int) -> str:
        return self.decode_tokens([tid])

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            self._lib.gg_tokenizer_destroy(self._h)
            self._h = ctypes.c_void_p()

    __del__ = close
