"""Tokenizer (src/tokenizer.ts) and chat template (src/conversation.ts) restatements."""
from gemma_b200.conversation import build_chat_prompt
from gemma_b200.synth import make_vocab
from gemma_b200.tokenizer import Tokenizer


def tok():
    v = make_vocab(4096)
    v[300] = "▁hello"
    v[301] = "▁world"
    v[302] = "hel"
    return Tokenizer(v)


def test_encode_decode():
    t = tok()
    ids = t.encode("hello world")
    assert ids[0] == 2  # BOS
    assert ids[1:] == [300, 301]
    assert t.decode_tokens(ids[1:]) == " hello world"
    # special tokens split segments; no '▁' prefix right after a special token
    ids = t.encode("<start_of_turn>user\nhello<end_of_turn>")
    assert ids[1] == 105 and ids[-1] == 106
    assert t.decode_token(999999) == "<unk:999999>"


def test_unknown_chars_are_skipped():
    t = tok()
    assert t.encode("é") == [2, t.token_by_text["▁"]]  # '▁' then the unknown char is dropped


def test_chat_prompt():
    h = [{"role": "user", "text": "Hi"}, {"role": "model", "text": "Yo"}, {"role": "user", "text": "?"}]
    assert build_chat_prompt(h) == ("<start_of_turn>user\nHi<end_of_turn>\n<start_of_turn>model\nYo<end_of_turn>\n"
                                    "<start_of_turn>user\n?<end_of_turn>\n<start_of_turn>model\n")
    tools = '[{"name":"f","description":"d","parameters":{"type":"object","properties":{"a":{"description":"x","type":"string"}},"required":["a"]}}]'
    p = build_chat_prompt([{"role": "user", "text": "u"}], tools)
    assert p.startswith("<start_of_turn>developer\nYou are a model that can do function calling")
    assert "<start_function_declaration>declaration:f{description:<escape>d<escape>,parameters:{properties:{a:{description:<escape>x<escape>,type:<escape>string<escape>}},required:[<escape>a<escape>],type:<escape>object<escape>}}<end_function_declaration>" in p
    assert build_chat_prompt([{"role": "user", "text": "u"}], "not json") == "<start_of_turn>user\nu<end_of_turn>\n<start_of_turn>model\n"
