"""Greedy longest-match tokenizer, restated from the reference (src/tokenizer.ts:1-142).

Same special ids (1 <eos>, 2 <bos>, 105 <start_of_turn>, 106 <end_of_turn>), the same
function-call tokens when the vocabulary has them, the same '▁' space marker and the same
longest-prefix-first search; unknown characters are skipped (tokenizer.ts:96-97).
"""
from __future__ import annotations

import re

from . import gguf

SPECIAL_TOKENS = {"<start_of_turn>": 105, "<end_of_turn>": 106, "<eos>": 1, "<bos>": 2}
FUNC_TOKEN_NAMES = ["<start_function_declaration>", "<end_function_declaration>", "<start_function_call>",
                    "<end_function_call>", "<start_function_response>", "<end_function_response>", "<escape>"]


class Tokenizer:
    def __init__(self, vocab: list[str]):
        self.vocab = vocab
        self.token_by_text: dict[str, int] = {}
        self.max_token_len = 0
        for i, t in enumerate(vocab):  # buildTokenIndex (tokenizer.ts:43-57): first id wins
            if t:
                self.token_by_text.setdefault(t, i)
                self.max_token_len = max(self.max_token_len, len(t))
        self.special_tokens = dict(SPECIAL_TOKENS)
        self.func_tokens: dict[str, int] = {}
        for name in FUNC_TOKEN_NAMES:  # initFunctionTokens (tokenizer.ts:59-68)
            if name in self.token_by_text:
                self.func_tokens[name] = self.token_by_text[name]
                self.special_tokens[name] = self.token_by_text[name]
        names = sorted(self.special_tokens, key=len, reverse=True)
        self._special_re = re.compile("|".join(re.escape(n) for n in names))

    @classmethod
    def from_gguf(cls, parsed: "gguf.GGUFParsed") -> "Tokenizer":
        """extractFromGGUF (tokenizer.ts:26-41)."""
        kv = parsed.kv.get("tokenizer.ggml.tokens")
        if kv is None or kv.type != "array":
            raise ValueError("No tokenizer found in GGUF metadata")
        return cls([v.value for v in kv.value])

    def _encode_segment(self, text: str, add_prefix: bool = True) -> list[int]:
        out: list[int] = []
        rem = text.replace(" ", "▁")
        if add_prefix:
            rem = "▁" + rem
        while rem:
            best_len, best_id = 0, -1
            for ln in range(min(len(rem), self.max_token_len), 0, -1):
                tid = self.token_by_text.get(rem[:ln])
                if tid is not None:
                    best_len, best_id = ln, tid
                    break
            if best_len == 0:
                rem = rem[1:]
            else:
                out.append(best_id)
                rem = rem[best_len:]
        return out

    def encode(self, text: str) -> list[int]:
        """encode (tokenizer.ts:106-126): BOS, then segments split on special tokens."""
        toks = [2]
        last, after_special = 0, False
        for mt in self._special_re.finditer(text):
            before = text[last:mt.start()]
            if before:
                toks += self._encode_segment(before, not after_special)
            toks.append(self.special_tokens[mt.group(0)])
            last, after_special = mt.end(), True
        rem = text[last:]
        if rem:
            toks += self._encode_segment(rem, not after_special)
        return toks

    def decode_token(self, tid: int) -> str:
        if 0 <= tid < len(self.vocab) and self.vocab[tid]:
            return self.vocab[tid].replace("▁", " ")
        return f"<unk:{tid}>"

    def decode_tokens(self, ids) -> str:
        return "".join(self.decode_token(int(t)) for t in ids)
