"""The host mirror of the reference's generate loop (src/engine.ts:957-1031) on the CPU.

`GemmaEngine.generate` decides which ids are prefilled where, when the KV cache is reset, at
which positions tokens are decoded, when the loop stops and what the conversation history
keeps. Those decisions are host logic; here they run against a scripted stand-in for the
native engine that records every call, with the real tokenizer (the library's host-only
C++ code) and chat template. The GPU side of the same calls is covered by the gpu tests.
"""
import pytest

from gemma_b200.config import default_config
from gemma_b200.conversation import build_chat_prompt
from gemma_b200.engine import GemmaEngine, STOP_IDS
from gemma_b200.synth import make_vocab
from gemma_b200.tokenizer import Tokenizer

HELLO, WORLD, END_FUNC = 300, 301, 307
END_OF_TURN = 106


class ScriptedNative:
    """Stands in for NativeEngine: returns scripted tokens and records the calls."""

    def __init__(self, tokens, ctx):
        self.tokens = list(tokens)
        self.ctx = ctx
        self.calls = []

    def _next(self):
        return self.tokens.pop(0)

    def seen_reset(self, seq=0):
        self.calls.append(("seen_reset", seq))

    def reset_kv(self, seq=0):
        self.calls.append(("reset_kv", seq))

    def prefill(self, ids, start_pos, seq=0):
        assert start_pos >= 0 and start_pos + len(ids) <= self.ctx
        self.calls.append(("prefill", list(ids), start_pos))

    def sample_last(self, seq=0, temperature=0.0, top_p=0.9, rep=1.0, uniform=0.0):
        self.calls.append(("sample_last", temperature, top_p, rep, uniform))
        return self._next()

    def step(self, token, pos, seq=0, temperature=0.0, top_p=0.9, rep=1.0, uniform=0.0):
        assert 0 <= pos < self.ctx - 1
        self.calls.append(("step", token, pos, temperature, top_p, rep, uniform))
        return self._next()

    def close(self):
        self.calls.append(("close",))

    def of(self, kind):
        return [c for c in self.calls if c[0] == kind]


@pytest.fixture(scope="module")
def tokenizer():
    v = make_vocab(4096)
    v[HELLO] = "▁hello"
    v[WORLD] = "▁world"
    v[END_FUNC] = "<end_function_call>"
    return Tokenizer(v)


def make_engine(tokenizer, tokens, ctx=2048, draws=None):
    """A GemmaEngine wired to the scripted native engine (no model file, no GPU)."""
    eng = GemmaEngine.__new__(GemmaEngine)
    eng.config = default_config()
    eng.config.context_length = ctx
    eng._on_progress = None
    it = iter(draws if draws is not None else [0.5] * 10000)
    eng._random = lambda: next(it)
    eng.conversation_history = []
    eng.kv_position = 0
    eng.tokenizer = tokenizer
    eng._mm = None
    eng._native = ScriptedNative(tokens, ctx)
    return eng


def test_first_turn_prefill_positions_and_stop(tokenizer):
    eng = make_engine(tokenizer, [HELLO, WORLD, END_OF_TURN])
    eng.add_user_message("hello world")
    out = list(eng.generate(temperature=0.0, top_p=0.9, rep_penalty=1.0))
    prompt = tokenizer.encode(build_chat_prompt([{"role": "user", "text": "hello world"}], "[]"))
    nat = eng.native
    assert nat.of("prefill") == [("prefill", prompt, 0)]
    n = len(prompt)
    # the stop id is decoded (a KV write) but neither yielded nor kept
    assert [(c[1], c[2]) for c in nat.of("step")] == [(HELLO, n), (WORLD, n + 1)]
    assert out == [tokenizer.decode_token(HELLO), tokenizer.decode_token(WORLD)]
    assert eng.kv_position == n + 2
    assert eng.conversation_history[-1] == {"role": "model", "text": tokenizer.decode_tokens([HELLO, WORLD])}
    # the repetition-penalty set starts from this turn's prompt (engine.ts:989)
    assert nat.calls.index(("seen_reset", 0)) < nat.calls.index(nat.of("prefill")[0])


def test_second_turn_appends_suffix_after_cached_prefix(tokenizer):
    eng = make_engine(tokenizer, [HELLO, END_OF_TURN, WORLD, END_OF_TURN])
    eng.add_user_message("hello")
    list(eng.generate())
    pos1 = eng.kv_position
    eng.add_user_message("world")
    list(eng.generate())
    suffix = "<end_of_turn>\n<start_of_turn>user\nworld<end_of_turn>\n<start_of_turn>model\n"
    ids = tokenizer.encode(suffix)[1:]  # without <bos>
    pf = eng.native.of("prefill")
    assert pf[1] == ("prefill", ids, pos1)
    assert eng.native.of("reset_kv") == []
    assert eng.native.of("step")[-1][2] == pos1 + len(ids)
    assert eng.kv_position == pos1 + len(ids) + 1
    assert [h["role"] for h in eng.conversation_history] == ["user", "model", "user", "model"]


def test_first_token_stop_is_yielded_once(tokenizer):
    eng = make_engine(tokenizer, [END_OF_TURN])
    eng.add_user_message("hello")
    out = list(eng.generate())
    assert out == [tokenizer.decode_token(END_OF_TURN)]  # yielded before the loop, as the reference does
    assert eng.native.of("step") == []
    n = len(eng.native.of("prefill")[0][1])
    assert eng.kv_position == n
    assert eng.conversation_history[-1]["text"] == tokenizer.decode_tokens([END_OF_TURN])


@pytest.mark.parametrize("stop", sorted(STOP_IDS))
def test_every_stop_id_ends_the_turn(tokenizer, stop):
    eng = make_engine(tokenizer, [HELLO, stop, WORLD])
    eng.add_user_message("hello")
    out = list(eng.generate())
    assert out == [tokenizer.decode_token(HELLO)]
    assert len(eng.native.tokens) == 1  # WORLD never requested


def test_end_function_call_is_kept_but_not_yielded(tokenizer):
    assert tokenizer.func_tokens["<end_function_call>"] == END_FUNC
    eng = make_engine(tokenizer, [HELLO, END_FUNC, WORLD])
    eng.add_user_message("hello")
    out = list(eng.generate())
    assert out == [tokenizer.decode_token(HELLO)]
    assert eng.conversation_history[-1]["text"] == tokenizer.decode_tokens([HELLO, END_FUNC])
    assert len(eng.native.tokens) == 1


def test_max_tokens_counts_the_first_token(tokenizer):
    eng = make_engine(tokenizer, [HELLO] * 10)
    eng.add_user_message("hello")
    out = list(eng.generate(max_tokens=3))
    assert len(out) == 3
    assert len(eng.native.of("step")) == 2


def test_context_limit_stops_before_the_last_position(tokenizer):
    ctx = 48
    eng = make_engine(tokenizer, [HELLO] * 100, ctx=ctx)
    eng.add_user_message("hello")
    list(eng.generate())
    n = len(eng.native.of("prefill")[0][1])
    steps = eng.native.of("step")
    assert [c[2] for c in steps] == list(range(n, ctx - 1))  # positions n .. ctx-2
    assert eng.kv_position == ctx - 1


def test_context_overflow_resets_to_the_last_user_message(tokenizer):
    ctx = 64
    eng = make_engine(tokenizer, [HELLO, END_OF_TURN] * 3, ctx=ctx)
    eng.add_user_message("hello")
    list(eng.generate())
    eng.kv_position = ctx - 12  # as if earlier turns had filled the cache
    eng.add_user_message("world world world")
    list(eng.generate())
    fresh = tokenizer.encode(build_chat_prompt([{"role": "user", "text": "world world world"}], "[]"))
    nat = eng.native
    assert nat.of("reset_kv") == [("reset_kv", 0)]
    assert nat.of("prefill")[-1] == ("prefill", fresh, 0)
    assert [h["role"] for h in eng.conversation_history] == ["user", "model"]
    assert eng.conversation_history[0]["text"] == "world world world"
    assert eng.kv_position == len(fresh) + 1


def test_sampling_options_and_injected_draws_reach_every_call(tokenizer):
    draws = [0.11, 0.22, 0.33, 0.44]
    eng = make_engine(tokenizer, [HELLO, WORLD, END_OF_TURN], draws=draws)
    eng.add_user_message("hello")
    list(eng.generate(temperature=0.8, top_p=0.7, rep_penalty=1.3))
    nat = eng.native
    assert nat.of("sample_last") == [("sample_last", 0.8, 0.7, 1.3, 0.11)]
    assert [c[3:] for c in nat.of("step")] == [(0.8, 0.7, 1.3, 0.22), (0.8, 0.7, 1.3, 0.33)]


def test_defaults_match_the_reference(tokenizer):
    eng = make_engine(tokenizer, [END_OF_TURN])
    eng.add_user_message("hello")
    list(eng.generate())
    assert eng.native.of("sample_last")[0][1:4] == (0.7, 0.9, 1.2)  # engine.ts:959-961


def test_abort_signal_stops_before_the_next_step(tokenizer):
    class Signal:
        aborted = False

    sig = Signal()
    eng = make_engine(tokenizer, [HELLO] * 10)
    eng.add_user_message("hello")
    out = []
    for s in eng.generate(signal=sig):
        out.append(s)
        if len(out) == 2:
            sig.aborted = True
    assert len(out) == 2
    assert len(eng.native.of("step")) == 1


def test_reset_conversation_and_dispose(tokenizer):
    eng = make_engine(tokenizer, [HELLO, END_OF_TURN])
    eng.add_user_message("hello")
    list(eng.generate())
    eng.reset_conversation()
    assert eng.conversation_history == [] and eng.kv_position == 0
    assert eng.native.of("reset_kv") == [("reset_kv", 0)]
    nat = eng.native
    eng.dispose()
    assert nat.of("close") == [("close",)]
    eng.dispose()  # a second dispose is harmless
    with pytest.raises(RuntimeError):
        next(eng.generate())
