"""gg_sample_logits_noalloc: sampling from device logits without allocating memory.

Some callers cannot call cudaMalloc: code that runs while another allocator owns the
device's memory (a framework's caching allocator, a fixed arena), and latency-bound loops
that cannot take the device-wide synchronisation cudaMalloc/cudaFree may cause. For them
the library offers one entry point that allocates nothing: it takes logits already on the
GPU and keeps its scratch in a static device array.

These tests call it through the C-ABI on consecutive calls (so the second call finds the
first one's scratch contents) and check each token against the existing entry points
gg_sample_last / gg_step on the same logits. Tokens are integers: they must match exactly.
This file is collected last so that a failure here stops a `-x` run after everything else.
"""
import ctypes

import numpy as np
import pytest

from conftest import synthetic

pytestmark = pytest.mark.gpu


def _bits(ids, vocab):
    words = np.zeros((vocab + 31) // 32, np.uint32)
    for t in ids:
        words[t >> 5] |= np.uint32(1 << (t & 31))
    return words


class NoAlloc:
    def __init__(self):
        import torch
        from gemma_b200 import native
        self.torch = torch
        self.lib = native.load()
        self.out = torch.full((1,), -7, dtype=torch.int32, device="cuda:0")

    def __call__(self, logits, seen_ids=None, temperature=0.0, top_p=0.9, rep=1.0, uniform=0.0):
        from gemma_b200.native import GGSample
        torch = self.torch
        vocab = int(logits.shape[0])
        lg = torch.from_numpy(np.ascontiguousarray(logits, np.float32)).to("cuda:0")
        seen = None
        if seen_ids is not None:
            seen = torch.from_numpy(_bits(seen_ids, vocab).view(np.int32)).to("cuda:0")
        torch.cuda.synchronize()
        s = GGSample(temperature, top_p, rep)
        rc = self.lib.gg_sample_logits_noalloc(ctypes.c_void_p(lg.data_ptr()), vocab,
                                               ctypes.c_void_p(seen.data_ptr()) if seen is not None else None,
                                               ctypes.byref(s), float(uniform),
                                               ctypes.c_void_p(self.out.data_ptr()), None)
        assert rc == 0, self.lib.gg_last_error(None)
        torch.cuda.synchronize()
        return int(self.out.item())


def test_noalloc_matches_sample_last_and_step():
    from gemma_b200 import synth
    from gemma_b200.native import engine_from_tensors
    cfg, tens = synthetic("mid", 3)  # vocab 16384: four CTAs meet at the end-of-launch ticket
    eng = engine_from_tensors(cfg, tens)
    noalloc = NoAlloc()
    prompt = [int(t) for t in synth.make_prompt(3, 6, cfg.vocab_size)]
    eng.prefill(prompt, 0)
    eng.seen_reset(0)

    # call 1: greedy
    ref1 = eng.sample_last(0)
    lg1 = eng.logits()
    assert noalloc(lg1) == ref1
    seen = {ref1}

    # call 2: temperature + top-p + repetition penalty on this turn's tokens
    top = [int(i) for i in np.argsort(-lg1, kind="stable")[:8]]
    eng.seen_add(top)
    seen |= set(top)
    ref2 = eng.sample_last(0, temperature=0.9, top_p=0.95, rep=1.5, uniform=0.61)
    lg2 = eng.logits()
    assert noalloc(lg2, sorted(seen), 0.9, 0.95, 1.5, 0.61) == ref2
    seen.add(ref2)

    # call 3: the next position's logits, through gg_step
    ref3 = eng.step(ref2, len(prompt), temperature=0.7, top_p=0.9, rep=1.3, uniform=0.25)
    lg3 = eng.logits()
    assert noalloc(lg3, sorted(seen), 0.7, 0.9, 1.3, 0.25) == ref3
    seen.add(ref3)

    # call 4: greedy with a penalty takes the sorted path
    ref4 = eng.step(ref3, len(prompt) + 1, temperature=0.0, top_p=0.9, rep=2.0, uniform=0.0)
    lg4 = eng.logits()
    assert noalloc(lg4, sorted(seen), 0.0, 0.9, 2.0, 0.0) == ref4
    eng.close()


def test_noalloc_large_vocab_then_small_matches():
    """A Gemma-3-sized call (64 CTAs) leaves its lane maxima in the scratch; the next,
    smaller call must not see them."""
    from oracle import oracle_np
    from gemma_b200.native import engine_from_tensors
    noalloc = NoAlloc()
    rng = np.random.default_rng(11)
    big = (rng.standard_normal(262144) * 2).astype(np.float32)
    big[123456] = big[1000] = np.float32(9.5)  # tie across lanes 64 and 232: lane 64 wins
    vals, ids = oracle_np.topk256(big)
    for T, top_p, rep, u in [(0.0, 0.9, 1.0, 0.0), (0.8, 0.9, 1.0, 0.3)]:
        want = oracle_np.sample(vals, ids, T, top_p, rep, set(), u)
        assert noalloc(big, None, T, top_p, rep, u) == want

    cfg, tens = synthetic("tiny", 7)  # vocab 4096: one CTA
    eng = engine_from_tensors(cfg, tens)
    eng.prefill([5, 6, 7], 0)
    ref = eng.sample_last(0)
    assert noalloc(eng.logits()) == ref
    eng.close()


@pytest.mark.parametrize("lanes", [(1, 2), (3, 5), (2, 1), (128, 64), (255, 127), (6, 10, 12), (0, 17, 34)])
def test_noalloc_greedy_ties_follow_the_reference_tree(lanes):
    """Equal maxima in several lanes of a 262,144-entry vocabulary: the greedy pick must be the
    reference's argmax tree result (smallest bit-reversed lane, shaders.ts:327-361), as the
    C oracle computes it, not the lowest lane. -0 and +0 tie inside a lane."""
    from oracle import oracle
    noalloc = NoAlloc()
    rng = np.random.default_rng(sum(lanes))
    lg = (rng.standard_normal(262144) * 0.5).astype(np.float32)
    for k, lane in enumerate(lanes):
        lg[lane + 256 * (100 + 37 * k)] = np.float32(7.25)
    want = oracle.argmax(lg)
    assert lg[want] == np.float32(7.25)
    assert noalloc(lg) == want
    z = np.full(4096, -1.0, np.float32)
    z[9], z[9 + 256 * 3] = np.float32(-0.0), np.float32(0.0)
    assert noalloc(z) == oracle.argmax(z) == 9


def test_noalloc_allocates_no_device_memory():
    """After one warm-up call, further calls leave the device's free memory unchanged."""
    import torch
    noalloc = NoAlloc()
    rng = np.random.default_rng(5)
    lg = (rng.standard_normal(262144)).astype(np.float32)
    dev = torch.from_numpy(lg).to("cuda:0")
    seen = torch.zeros(262144 // 32, dtype=torch.int32, device="cuda:0")
    from gemma_b200.native import GGSample
    s = GGSample(0.8, 0.9, 1.2)
    torch.cuda.synchronize()
    rc = noalloc.lib.gg_sample_logits_noalloc(ctypes.c_void_p(dev.data_ptr()), 262144, ctypes.c_void_p(seen.data_ptr()),
                                              ctypes.byref(s), 0.4, ctypes.c_void_p(noalloc.out.data_ptr()), None)
    assert rc == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    toks = []
    for i in range(8):
        rc = noalloc.lib.gg_sample_logits_noalloc(ctypes.c_void_p(dev.data_ptr()), 262144,
                                                  ctypes.c_void_p(seen.data_ptr()), ctypes.byref(s), 0.1 * i,
                                                  ctypes.c_void_p(noalloc.out.data_ptr()), None)
        assert rc == 0
        torch.cuda.synchronize()
        toks.append(int(noalloc.out.item()))
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0
    from oracle import oracle
    vals, ids = oracle.topk256(lg)
    for i, t in enumerate(toks):
        assert t == oracle.sample(vals, ids, 0.8, 0.9, 1.2, [], 0.1 * i, 262144)
