"""The user-facing path on the GPU: create_gemma_engine -> add_user_message -> generate.

A synthetic tiny model is written as a GGUF file and loaded the way a user loads one (GGUF
parse, weight upload and repack, tokenizer from the file's vocabulary, chat template); two
greedy turns are generated and compared token for token with the CPU oracle run on the same
prompt ids at the same positions (the second turn appends its suffix after the cached prefix,
as the reference's generate does, src/engine.ts:966-975).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _until_stop(ids, end_func):
    """The tokens generate yields for a greedy id sequence: the first always, then up to a stop."""
    out = [ids[0]]
    if ids[0] in (0, 1, 106) or ids[0] == end_func:
        return out
    for t in ids[1:]:
        if t in (0, 1, 106) or t == end_func:
            break
        out.append(t)
    return out


def test_generate_two_greedy_turns_match_the_oracle(tmp_path, monkeypatch, oracle_mod):
    from gemma_b200 import synth
    from gemma_b200.conversation import build_chat_prompt
    from gemma_b200.engine import create_gemma_engine
    from oracle.oracle import OracleModel

    monkeypatch.setenv("GEMMA_B200_CACHE", str(tmp_path))
    progress = []
    eng = create_gemma_engine("synthetic:tiny", on_progress=progress.append)
    assert progress and progress[-1]["loaded"] == progress[-1]["total"]
    tok = eng.tokenizer
    end_func = tok.func_tokens.get("<end_function_call>")
    orc = OracleModel.from_tensors(eng.config, synth.make_tensors(synth.SHAPES["tiny"], 7))

    m = 6
    eng.add_user_message("hello world")
    out1 = list(eng.generate(temperature=0.0, top_p=0.9, rep_penalty=1.0, max_tokens=m))
    prompt1 = tok.encode(build_chat_prompt([{"role": "user", "text": "hello world"}], "[]"))
    ref1 = orc.greedy(prompt1, m)
    want1 = _until_stop(ref1, end_func)
    assert out1 == [tok.decode_token(t) for t in want1]
    if len(want1) < m:
        pytest.skip("the synthetic model stopped early in turn 1; the second turn needs a full first turn")
    assert eng.kv_position == len(prompt1) + m - 1

    eng.add_user_message("again")
    out2 = list(eng.generate(temperature=0.0, top_p=0.9, rep_penalty=1.0, max_tokens=m))
    suffix = "<end_of_turn>\n<start_of_turn>user\nagain<end_of_turn>\n<start_of_turn>model\n"
    ids2 = tok.encode(suffix)[1:]
    ref2 = orc.greedy(ids2, m, start_pos=len(prompt1) + m - 1)
    assert out2 == [tok.decode_token(t) for t in _until_stop(ref2, end_func)]
    assert [h["role"] for h in eng.conversation_history] == ["user", "model", "user", "model"]

    eng.reset_conversation()
    assert eng.kv_position == 0
    eng.dispose()
