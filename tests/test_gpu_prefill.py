"""Batched prefill (tensor-core GEMMs, gg_prefill default) against the serial per-token path.

The serial path (GG_FLAG_SERIAL_PREFILL) runs the reference's order, one token per launch,
and is itself pinned to the oracle by test_gpu_parity.py. The batched path must leave the
same KV cache and hidden state (relative L2 within 1e-4), the same first-token logits (within
the 2e-3 bound of the north star; measured ~1e-5) and the same greedy continuation, for a
prompt in one chunk, a prompt over several 512-token chunks, and a second turn appended at
start_pos > 0.
"""
import numpy as np
import pytest

from conftest import rel_l2, synthetic

pytestmark = pytest.mark.gpu

STATE_TOL = 1e-4
LOGIT_TOL = 2e-3


def _engines(shape, seed):
    from gemma_b200.native import GG_FLAG_SERIAL_PREFILL, engine_from_tensors
    cfg, tens = synthetic(shape, seed)
    return cfg, engine_from_tensors(cfg, tens), engine_from_tensors(cfg, tens, flags=GG_FLAG_SERIAL_PREFILL)


def _compare(cfg, a, b, start, n, ngen):
    assert rel_l2(a.hidden(), b.hidden()) < STATE_TOL
    for layer in range(cfg.num_layers):
        for p in sorted({start, start + n // 2, start + n - 1}):
            for which in (0, 1):
                assert rel_l2(a.kv_row(layer, p, which), b.kv_row(layer, p, which)) < STATE_TOL, (layer, p, which)
    ta, tb = a.sample_last(0), b.sample_last(0)
    assert rel_l2(a.logits(), b.logits()) < LOGIT_TOL
    assert ta == tb
    ga = [ta] + list(a.decode(ta, start + n, ngen))
    gb = [tb] + list(b.decode(tb, start + n, ngen))
    assert ga == gb
    return ga


@pytest.mark.parametrize("shape,seed,plen", [("tiny", 7, 37), ("small", 3, 130), ("mid", 5, 64)])
def test_batched_prefill_matches_serial(shape, seed, plen):
    from gemma_b200 import synth
    cfg, a, b = _engines(shape, seed)
    prompt = synth.make_prompt(seed, plen, cfg.vocab_size)
    a.prefill(prompt, 0)
    b.prefill(prompt, 0)
    _compare(cfg, a, b, 0, plen, 6)
    a.close()
    b.close()


def test_batched_prefill_several_chunks_and_second_turn():
    from gemma_b200 import synth
    cfg, a, b = _engines("mid", 9)  # context 1024
    p1 = synth.make_prompt(9, 700, cfg.vocab_size)  # chunks of 512 + 188
    a.prefill(p1, 0)
    b.prefill(p1, 0)
    g = _compare(cfg, a, b, 0, len(p1), 4)
    # second turn: the last sampled token and 90 new ids appended after the cached prefix
    start = len(p1) + 4
    p2 = [g[-1]] + list(synth.make_prompt(10, 89, cfg.vocab_size))
    a.prefill(p2, start)
    b.prefill(p2, start)
    _compare(cfg, a, b, start, len(p2), 4)
    a.close()
    b.close()


def test_batched_prefill_single_token_and_odd_lengths():
    from gemma_b200 import synth
    cfg, a, b = _engines("small", 4)
    for n in (1, 2, 63, 65, 129):
        a.reset_kv(0)
        b.reset_kv(0)
        prompt = synth.make_prompt(100 + n, n, cfg.vocab_size)
        a.prefill(prompt, 0)
        b.prefill(prompt, 0)
        _compare(cfg, a, b, 0, n, 2)
    a.close()
    b.close()
