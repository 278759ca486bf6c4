"""Tokenizer (src/tokenizer.ts) and chat template (src/conversation.ts).

The tokenizer is the C++ one in libgemma_b200.so (gg_tokenizer_*; host code, no GPU); the
checker is the Python restatement in oracle/tokenizer_ref.py, which follows the reference's
UTF-16 code-unit semantics.
"""
import random

import pytest

from gemma_b200.conversation import build_chat_prompt
from gemma_b200.synth import make_vocab
from gemma_b200.tokenizer import Tokenizer
from oracle.tokenizer_ref import RefTokenizer


def vocab():
    v = make_vocab(4096)
    v[300] = "▁hello"
    v[301] = "▁world"
    v[302] = "hel"
    v[303] = "é"
    v[304] = "▁über"
    v[305] = "😀"           # one code point, two UTF-16 units
    v[306] = "a😀"          # three UTF-16 units
    v[307] = "<end_function_call>"
    v[308] = "<escape>"
    v[309] = "▁▁▁▁"
    v[310] = "日本"
    v[311] = "hello"        # duplicate text later in the vocabulary: the first id wins
    v[312] = "hello"
    return v


@pytest.fixture(scope="module")
def toks():
    v = vocab()
    return Tokenizer(v), RefTokenizer(v)


def test_encode_decode(toks):
    t, _ = toks
    ids = t.encode("hello world")
    assert ids[0] == 2  # BOS
    assert ids[1:] == [300, 301]
    assert t.decode_tokens(ids[1:]) == " hello world"
    # special tokens split segments; no '▁' prefix right after a special token
    ids = t.encode("<start_of_turn>user\nhello<end_of_turn>")
    assert ids[1] == 105 and ids[-1] == 106
    assert ids[-2] == 311
    assert t.decode_token(999999) == "<unk:999999>"
    assert t.decode_token(-1) == "<unk:-1>"


def test_unknown_chars_are_skipped(toks):
    t, _ = toks
    assert t.encode("ß") == [2, t.token_id("▁")]  # '▁' then the unknown char is dropped


def test_function_tokens(toks):
    t, r = toks
    assert t.func_tokens == {"<end_function_call>": 307, "<escape>": 308} == r.func_tokens
    ids = t.encode("call<end_function_call>x<escape>")
    assert 307 in ids and 308 in ids
    assert ids == r.encode("call<end_function_call>x<escape>")


def test_utf16_semantics(toks):
    """Astral characters are two code units, as in JavaScript: '😀' is one token, and an unknown
    one is skipped a unit at a time, leaving no id."""
    t, r = toks
    for s in ["😀", "a😀b", "🙂", "x🙂y😀", "日本語 über é", "    spaces  "]:
        assert t.encode(s) == r.encode(s), s
    assert t.encode("😀")[-1] == 305
    assert t.encode("a😀") == [2, t.token_id("▁"), 306]
    assert t.encode("🙂") == [2, t.token_id("▁")]


def test_matches_restatement_on_random_text(toks):
    t, r = toks
    rng = random.Random(0)
    alphabet = list("helowrd ") + ["▁", "é", "ü", "日", "本", "😀", "🙂", "\n", "<", ">"] + \
        ["<start_of_turn>", "<end_of_turn>", "<eos>", "<bos>", "<escape>", "<end_function_call>", "hello", "world"]
    for _ in range(300):
        s = "".join(rng.choice(alphabet) for _ in range(rng.randint(0, 40)))
        assert t.encode(s) == r.encode(s), repr(s)
        ids = t.encode(s)
        assert t.decode_tokens(ids) == "".join(r.decode_token(i) for i in ids)


def test_long_prompt(toks):
    t, r = toks
    s = ("hello world über 日本 " * 500) + "<end_of_turn>"
    assert t.encode(s) == r.encode(s)


def test_chat_prompt():
    h = [{"role": "user", "text": "Hi"}, {"role": "model", "text": "Yo"}, {"role": "user", "text": "?"}]
    assert build_chat_prompt(h) == ("<start_of_turn>user\nHi<end_of_turn>\n<start_of_turn>model\nYo<end_of_turn>\n"
                                    "<start_of_turn>user\n?<end_of_turn>\n<start_of_turn>model\n")
    tools = '[{"name":"f","description":"d","parameters":{"type":"object","properties":{"a":{"description":"x","type":"string"}},"required":["a"]}}]'
    p = build_chat_prompt([{"role": "user", "text": "u"}], tools)
    assert p.startswith("<start_of_turn>developer\nYou are a model that can do function calling")
    assert "<start_function_declaration>declaration:f{description:<escape>d<escape>,parameters:{properties:{a:{description:<escape>x<escape>,type:<escape>string<escape>}},required:[<escape>a<escape>],type:<escape>object<escape>}}<end_function_declaration>" in p
    assert build_chat_prompt([{"role": "user", "text": "u"}], "not json") == "<start_of_turn>user\nu<end_of_turn>\n<start_of_turn>model\n"
