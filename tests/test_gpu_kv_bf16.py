"""The bf16 KV cache (GG_FLAG_KV_BF16, GemmaConfig.kv_dtype = "bf16") against the oracle with
the same option, on every path: serial prefill + decode kernel, batched prefill, batched decode.

The reference keeps f32 caches; with the option, k and v rows are rounded to bf16 (nearest
even) when stored and attention reads the rounded rows, the current position's included. The
oracle does the same (or_bf16_round), so the tolerances are test_gpu_parity.py's: logits within
2e-3 relative L2, identical greedy tokens.
"""
import dataclasses

import numpy as np
import pytest

from conftest import rel_l2, synthetic

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def _bf16(shape, seed, **kw):
    cfg, tens = synthetic(shape, seed)
    return dataclasses.replace(cfg, kv_dtype="bf16", **kw), tens


@pytest.mark.parametrize("serial", [True, False])
@pytest.mark.parametrize("shape,seed,plen,window", [("small", 3, 41, 0), ("mid", 5, 70, 0), ("small", 9, 45, 16)])
def test_bf16_kv_decode_matches_oracle(shape, seed, plen, window, serial, oracle_mod):
    from gemma_b200 import synth
    from gemma_b200.native import GG_FLAG_SERIAL_PREFILL, engine_from_tensors
    from oracle.oracle import OracleModel
    extra = dict(sliding_window=window, rope_theta_swa=10000.0, swa_period=2) if window else {}
    cfg, tens = _bf16(shape, seed, **extra)
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
    # stored rows are bf16 values
    for layer in (0, cfg.num_layers - 1):
        for which in (0, 1):
            row = eng.kv_row(layer, pos - 1, which)
            assert (row.view(np.uint32) & 0xFFFF == 0).all()
    eng.close()


def test_bf16_kv_rows_are_rounded_f32_rows(oracle_mod):
    """Position 0 of layer 0 sees identical inputs with either cache type: the bf16 row must be
    exactly the f32 row rounded to nearest even."""
    from gemma_b200 import synth
    from gemma_b200.native import GG_FLAG_SERIAL_PREFILL, engine_from_tensors
    cfg32, tens = synthetic("small", 3)
    cfg16 = dataclasses.replace(cfg32, kv_dtype="bf16")
    prompt = synth.make_prompt(3, 5, cfg32.vocab_size)
    rows = {}
    for name, cfg in (("f32", cfg32), ("bf16", cfg16)):
        eng = engine_from_tensors(cfg, tens, flags=GG_FLAG_SERIAL_PREFILL)
        eng.prefill(prompt, 0)
        rows[name] = [eng.kv_row(0, 0, w) for w in (0, 1)]
        eng.close()
    for w in (0, 1):
        want = oracle_mod.bf16_round(rows["f32"][w])
        assert (rows["bf16"][w].view(np.uint32) == want.view(np.uint32)).all()


def test_bf16_kv_batched_decode_matches_steps():
    """Batched decode (tensor-core GEMMs) against per-sequence steps (dp4a matvecs) with a bf16
    cache. The two paths round differently at the 1e-5 level, and a value that close to a bf16
    rounding boundary is stored one bf16 step apart on the two paths, so the comparison is on
    greedy rows and allows a row to diverge only at a near tie of the per-sequence logits
    (top two within 1e-3 of the largest magnitude); the rows are compared up to that point."""
    from gemma_b200 import synth
    from gemma_b200.native import engine_from_tensors
    cfg, tens = _bf16("small", 7)
    n, steps = 3, 8
    prompts = [list(synth.make_prompt(80 + i, 22 + 9 * i, cfg.vocab_size)) for i in range(n)]
    samples = [(0.0, 0.9, 1.0)] * n  # plain greedy: the pick is the argmax of the logits
    unif = np.zeros((steps, n))
    a = engine_from_tensors(cfg, tens, max_seqs=n)
    first = []
    for i, p in enumerate(prompts):
        a.prefill(p, 0, seq=i)
        first.append(a.sample_last(i))
    got = a.decode_batch(np.arange(n), first, [len(p) for p in prompts], steps, samples, unif)
    a.close()
    b = engine_from_tensors(cfg, tens, max_seqs=n)
    agreed = 0
    for i, p in enumerate(prompts):
        b.prefill(p, 0, seq=i)
        tok, pos = b.sample_last(i), len(p)
        assert tok == first[i]
        T, P, R = samples[i]
        for k in range(steps):
            tok = b.step(tok, pos, seq=i, temperature=T, top_p=P, rep=R, uniform=0.0)
            pos += 1
            if got[k, i] != tok:
                lg = b.logits()
                gap = abs(float(lg[tok]) - float(lg[got[k, i]]))
                assert gap < 1e-3 * float(np.abs(lg).max()), (i, k, tok, int(got[k, i]), gap)
                break
            agreed += 1
    b.close()
    assert agreed >= steps * n // 2
