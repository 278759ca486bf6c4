"""Greedy longest-match tokenizer, restated from the reference (src/tokenizer.ts:1-142).

TEST INFRASTRUCTURE ONLY: the checker for the C++ tokenizer of libgemma_b200.so
(gg_tokenizer_*, webgpu-gemma_b200/csrc/gg_tokenizer.cpp). Nothing in the product imports it.

The reference runs on JavaScript strings, so every length, prefix and skip here is counted in
UTF-16 code units, as there: text and vocabulary are held as UTF-16-LE bytes and sliced two
bytes per unit. Same special ids (1 <eos>, 2 <bos>, 105 <start_of_turn>, 106 <end_of_turn>),
the same function-call tokens when the vocabulary has them (tokenizer.ts:59-68), the same '▁'
space marker and the same longest-prefix-first search; unknown code units are skipped
(tokenizer.ts:96-97).
"""
from __future__ import annotations

SPECIAL_TOKENS = {"<start_of_turn>": 105, "<end_of_turn>": 106, "<eos>": 1, "<bos>": 2}
FUNC_TOKEN_NAMES = ["<start_function_declaration>", "<end_function_declaration>", "<start_function_call>",
                    "<end_function_call>", "<start_function_response>", "<end_function_response>", "<escape>"]


def u16(s: str) -> bytes:
    return s.encode("utf-16-le", "surrogatepass")


def from_u16(b: bytes) -> str:
    return b.decode("utf-16-le", "surrogatepass")


SPACE = u16("▁")


class RefTokenizer:
    def __init__(self, vocab: list[str]):
        self.vocab = vocab
        self.token_by_text: dict[bytes, int] = {}
        self.max_token_len = 0  # code units
        for i, t in enumerate(vocab):  # buildTokenIndex (tokenizer.ts:43-57): first id wins
            if t:
                k = u16(t)
                self.token_by_text.setdefault(k, i)
                self.max_token_len = max(self.max_token_len, len(k) // 2)
        self.special_tokens: dict[str, int] = dict(SPECIAL_TOKENS)
        self.func_tokens: dict[str, int] = {}
        for name in FUNC_TOKEN_NAMES:  # initFunctionTokens (tokenizer.ts:59-68)
            if u16(name) in self.token_by_text:
                self.func_tokens[name] = self.token_by_text[u16(name)]
                self.special_tokens[name] = self.token_by_text[u16(name)]
        # the alternation regex tries names longest first (stable sort, tokenizer.ts:70-75)
        self._special = sorted(self.special_tokens, key=lambda n: len(u16(n)), reverse=True)

    def _encode_segment(self, text: bytes, add_prefix: bool = True) -> list[int]:
        """encodeSegment (tokenizer.ts:77-104) on UTF-16-LE bytes."""
        out: list[int] = []
        rem = b"".join(SPACE if text[i:i + 2] == b" \x00" else text[i:i + 2] for i in range(0, len(text), 2))
        if add_prefix:
            rem = SPACE + rem
        while rem:
            best_len, best_id = 0, -1
            for ln in range(min(len(rem) // 2, self.max_token_len), 0, -1):
                tid = self.token_by_text.get(rem[:2 * ln])
                if tid is not None:
                    best_len, best_id = ln, tid
                    break
            if best_len == 0:
                rem = rem[2:]
            else:
                out.append(best_id)
                rem = rem[2 * best_len:]
        return out

    def encode(self, text: str) -> list[int]:
        """encode (tokenizer.ts:106-126): BOS, then segments split on special tokens."""
        t = u16(text)
        toks = [2]
        last, after_special, i = 0, False, 0
        names = [(u16(n), self.special_tokens[n]) for n in self._special]
        while i < len(t):
            hit = next(((nb, tid) for nb, tid in names if t.startswith(nb, i)), None)
            if hit is None:
                i += 2
                continue
            if i > last:
                toks += self._encode_segment(t[last:i], not after_special)
            toks.append(hit[1])
            i += len(hit[0])
            last, after_special = i, True
        if last < len(t):
            toks += self._encode_segment(t[last:], not after_special)
        return toks

    def decode_token(self, tid: int) -> str:
        """decodeToken (tokenizer.ts:128-133)."""
        if 0 <= tid < len(self.vocab) and self.vocab[tid]:
            return self.vocab[tid].replace("▁", " ")
        return f"<unk:{tid}>"
