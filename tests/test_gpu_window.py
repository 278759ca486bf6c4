"""Sliding-window attention (gg_config.sliding_window > 0, Gemma 3 as specified) against the
oracle with the same window, on every path: serial prefill + decode kernel, batched prefill,
and batched decode.

The reference attends the whole prefix on every layer; the window is opt-in. The test model
uses a window of 16 positions, a local RoPE base of 1e4 and swa_period 2 (layers alternate
windowed and global), with prompts longer than the window, so the masked ranges, the first
partial split and the per-layer RoPE tables are all exercised. Tolerances as in
test_gpu_parity.py: logits within 2e-3 relative L2, identical greedy tokens.
"""
import dataclasses

import numpy as np
import pytest

from conftest import rel_l2, synthetic

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def _windowed(shape, seed, window=16):
    cfg, tens = synthetic(shape, seed)
    cfg = dataclasses.replace(cfg, sliding_window=window, rope_theta_swa=10000.0, swa_period=2)
    return cfg, tens


@pytest.mark.parametrize("serial", [True, False])
@pytest.mark.parametrize("shape,seed,plen", [("small", 3, 41), ("mid", 5, 70)])
def test_window_decode_matches_oracle(shape, seed, plen, serial, oracle_mod):
    from gemma_b200 import synth
    from gemma_b200.native import GG_FLAG_SERIAL_PREFILL, engine_from_tensors
    from oracle.oracle import OracleModel
    cfg, tens = _windowed(shape, seed)
    eng = engine_from_tensors(cfg, tens, flags=GG_FLAG_SERIAL_PREFILL if serial else 0)
    orc = OracleModel.from_tensors(cfg, tens)
    prompt = synth.make_prompt(seed, plen, cfg.vocab_size)
    eng.prefill(prompt, 0)
    for i, t in enumerate(prompt):
        orc.forward(int(t), i)
    tok = eng.sample_last(0)
    assert rel_l2(eng.logits(), orc.logits()) < LOGIT_TOL
    assert tok == oracle_mod.argmax(orc.logits())
    pos = plen
    for _ in range(12):
        t_g = eng.step(tok, pos)
        orc.forward(tok, pos)
        lc = orc.logits()
        assert rel_l2(eng.logits(), lc) < LOGIT_TOL
        assert t_g == oracle_mod.argmax(lc)
        tok, pos = t_g, pos + 1
    eng.close()


def test_window_batched_decode_matches_steps():
    from gemma_b200 import synth
    from gemma_b200.native import engine_from_tensors
    cfg, tens = _windowed("small", 7)
    n, steps = 3, 8
    prompts = [list(synth.make_prompt(70 + i, 25 + 9 * i, cfg.vocab_size)) for i in range(n)]
    samples = [(0.0, 0.9, 1.0), (0.7, 0.9, 1.2), (0.0, 0.9, 1.3)]
    unif = np.random.default_rng(1).random((steps, n))
    a = engine_from_tensors(cfg, tens, max_seqs=n)
    first = []
    for i, p in enumerate(prompts):
        a.prefill(p, 0, seq=i)
        first.append(a.sample_last(i))
    got = a.decode_batch(np.arange(n), first, [len(p) for p in prompts], steps, samples, unif)
    a.close()
    b = engine_from_tensors(cfg, tens, max_seqs=n)
    want = np.empty((steps, n), np.int32)
    for i, p in enumerate(prompts):
        b.prefill(p, 0, seq=i)
        tok, pos = b.sample_last(i), len(p)
        assert tok == first[i]
        for k in range(steps):
            T, P, R = samples[i]
            tok = b.step(tok, pos, seq=i, temperature=T, top_p=P, rep=R, uniform=float(unif[k, i]))
            want[k, i] = tok
            pos += 1
    b.close()
    assert (got == want).all()
