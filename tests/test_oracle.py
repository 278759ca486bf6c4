"""CPU oracle checks: pins, known answers, C oracle vs the numpy restatement, golden fixtures.

The reference ships no test vectors (parity unpinned); what can be pinned independently is
pinned here: f16ToF32 against IEEE binary16 for all 65536 patterns, the packQ8_0ForGPU byte
layout on hand-built blocks, and the argmax / topk256 / sampler rules on hand-built inputs.
"""
import json
import os

import numpy as np
import pytest

from conftest import rel_l2, synthetic

HERE = os.path.dirname(os.path.abspath(__file__))


def test_f16_to_f32_exhaustive(oracle_mod):
    from oracle import oracle_np
    bits = np.arange(65536, dtype=np.uint16)
    ieee = bits.view(np.float16).astype(np.float32)
    c = np.array([oracle_mod.f16_to_f32(int(b)) for b in bits], dtype=np.float32)
    npm = oracle_np.f16_to_f32(bits)
    for got in (c, npm):
        same = (got.view(np.uint32) == ieee.view(np.uint32)) | (np.isnan(got) & np.isnan(ieee))
        assert same.all()


def test_pack_q8_0_known_answer(oracle_mod):
    # one block: d = f16 0x3C00 (1.0), quants 0..31 as int8 with sign flips
    q = np.array([(i if i % 2 == 0 else -i) for i in range(32)], dtype=np.int8)
    raw = np.concatenate([np.array([0x00, 0x3C], np.uint8), q.view(np.uint8)])
    words = oracle_mod.pack_q8_0(raw)
    assert words.shape == (9,)
    assert words[0] == np.float32(1.0).view(np.uint32)
    for j in range(8):
        b = q.view(np.uint8)[4 * j:4 * j + 4].astype(np.uint32)
        assert words[1 + j] == (b[0] | (b[1] << 8) | (b[2] << 16) | (b[3] << 24))
    from gemma_b200 import gguf
    assert (gguf.pack_q8_0_for_gpu(raw, 32) == words).all()


def test_dequant_matches_pack(tiny_model):
    from gemma_b200 import gguf
    cfg, tens = tiny_model
    dims, t, raw = tens["blk.0.attn_q.weight"]
    n = int(np.prod(dims))
    deq = gguf.dequantize_q8_0(raw, n).reshape(-1, 32)
    packed = gguf.pack_q8_0_for_gpu(raw, n).reshape(-1, 9)
    q = packed[:, 1:].copy().view(np.int8).reshape(-1, 32).astype(np.float32)
    d = packed[:, 0].copy().view(np.float32)
    assert (deq == q * d[:, None]).all()  # q * f32(d) is exact


@pytest.mark.parametrize("m,n", [(7, 256), (33, 640), (19, 1152), (5, 6912)])
def test_linear_q8_c_vs_numpy_bit_exact(oracle_mod, m, n):
    from oracle import oracle_np
    rng = np.random.default_rng(m * 1000 + n)
    qs = rng.integers(-127, 128, size=m * n, dtype=np.int8)
    d = (np.abs(rng.standard_normal(m * n // 32)) * 1e-3).astype(np.float16)
    from gemma_b200 import gguf
    raw = gguf.q8_0_join(qs, d.view(np.uint16))
    packed = oracle_mod.pack_q8_0(raw)
    x = rng.standard_normal(n).astype(np.float32)
    yc = oracle_mod.linear_q8(x, packed, m, n)
    yn = oracle_np.linear_q8(x, packed, m, n)
    assert (yc.view(np.uint32) == yn.view(np.uint32)).all()


@pytest.mark.parametrize("n", [256, 640, 1152, 1000])
def test_norms_c_vs_numpy_bit_exact(oracle_mod, n):
    from oracle import oracle_np
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    w = (rng.standard_normal(n) * 0.1).astype(np.float32)
    r = rng.standard_normal(n).astype(np.float32)
    assert (oracle_mod.rmsnorm(x, w) == oracle_np.rmsnorm(x, w, 1e-6)).all()
    assert (oracle_mod.fused_norm_add(x, w, r) == oracle_np.fused_norm_add(x, w, r, 1e-6)).all()


def test_transcendental_ops_close(oracle_mod):
    from oracle import oracle_np
    rng = np.random.default_rng(5)
    g = (rng.standard_normal(4096) * 3).astype(np.float32)
    u = rng.standard_normal(4096).astype(np.float32)
    # 0.5*x*(1+tanh(t)) cancels for negative x: compare against the 0.5*x*up scale (tanh ulps)
    err = np.abs(oracle_mod.gelu_mul(g, u).astype(np.float64) - oracle_np.gelu_mul(g, u))
    assert (err <= 4e-7 * np.abs(0.5 * g.astype(np.float64) * u) + 1e-12).all()
    d = rng.standard_normal(5 * 256).astype(np.float32)
    w = (rng.standard_normal(256) * 0.1).astype(np.float32)
    for pos in (0, 1, 511, 2047):
        a = oracle_mod.fused_norm_rope(d, w, 5, 256, 1e-6, pos, 1e6)
        b = oracle_np.fused_norm_rope(d, w, 5, 256, 1e-6, pos, 1e6)
        assert rel_l2(a, b) < 1e-6
    q = rng.standard_normal(1024).astype(np.float32)
    kc = rng.standard_normal((300, 256)).astype(np.float32)
    vc = rng.standard_normal((300, 256)).astype(np.float32)
    for sl in (1, 7, 256, 300):
        a = oracle_mod.attention(q, kc, vc, 4, 1, 256, sl, 0.0625)
        b = oracle_np.attention(q, kc, vc, 4, 1, 256, sl, 0.0625)
        assert rel_l2(a, b) < 1e-6


def test_topk256_and_argmax_rules(oracle_mod):
    from oracle import oracle_np
    n = 4096
    lg = np.full(n, -5.0, np.float32)
    # lane 3 holds the max twice (indices 3 and 259): first index wins inside a lane
    lg[3] = 2.0
    lg[259] = 2.0
    # lane 1 holds an equal max at a larger index. Across lanes the shader's tree (strides 128,
    # 64, ..., 1, the lower slot kept on a tie) prefers the smallest bit-reversed lane index:
    # bitrev8(1) = 128 < bitrev8(3) = 192, so lane 1 wins here
    lg[257] = 2.0
    lg[10] = np.nan  # NaN is never selected
    v, i = oracle_mod.topk256(lg)
    assert i[3] == 3 and i[1] == 257 and v[3] == 2.0
    assert oracle_mod.argmax(lg) == 257
    assert oracle_np.argmax(lg) == 257
    # values at or below the -1e30 init never replace it (strict '>' from (-1e30, 0))
    lg2 = np.full(512, -1e30, np.float32)
    v2, i2 = oracle_mod.topk256(lg2)
    assert (i2 == 0).all() and (v2 == np.float32(-1e30)).all()
    assert oracle_mod.argmax(lg2) == 0


def bitrev8(x: int) -> int:
    return int(f"{x:08b}"[::-1], 2)


def tree_argmax(lg) -> int:
    """src/shaders.ts:327-361 written as plain loops: lane maxima with strict '>', then the
    stride-halving tree that keeps the lower slot on a tie."""
    m, ix = [np.float32(-1e30)] * 256, [0] * 256
    for i, v in enumerate(np.asarray(lg, np.float32)):
        if v > m[i % 256]:
            m[i % 256], ix[i % 256] = v, i
    stride = 128
    while stride:
        for t in range(stride):
            if m[t + stride] > m[t]:
                m[t], ix[t] = m[t + stride], ix[t + stride]
        stride >>= 1
    return ix[0]


@pytest.mark.parametrize("lanes,winner", [((1, 2), 2), ((3, 5), 5), ((2, 1), 2), ((0, 128), 0),
                                          ((128, 64), 128), ((255, 127), 127), ((6, 10, 12), 12)])
def test_argmax_tie_across_lanes_follows_the_tree(oracle_mod, lanes, winner):
    """Equal maxima in several lanes: the reference's tree reduce returns the lane with the
    smallest bit-reversed index (lanes 1 and 2 tied -> lane 2), not the lowest lane."""
    from oracle import oracle_np
    lg = np.full(1024, -3.0, np.float32)
    for k, lane in enumerate(lanes):
        lg[lane + 256 * (k % 4)] = 1.5
    want = [lane + 256 * (k % 4) for k, lane in enumerate(lanes) if lane == winner][0]
    assert min(lanes, key=bitrev8) == winner
    assert tree_argmax(lg) == want
    assert oracle_mod.argmax(lg) == want
    assert oracle_np.argmax(lg) == want


def test_argmax_signed_zeros_tie(oracle_mod):
    """-0 and +0 compare equal under '>': inside a lane the first index keeps the maximum."""
    lg = np.full(512, -1.0, np.float32)
    lg[7] = np.float32(-0.0)
    lg[263] = np.float32(0.0)
    v, i = oracle_mod.topk256(lg)
    assert i[7] == 7
    assert oracle_mod.argmax(lg) == tree_argmax(lg) == 7


def test_sampler_rules(oracle_mod):
    from oracle import oracle_np
    vocab = 4096
    rng = np.random.default_rng(9)
    vals = (rng.standard_normal(256) * 0.05).astype(np.float32)
    ids = rng.choice(vocab, size=256, replace=False).astype(np.uint32)
    vals[10] = vals[20]  # a tie: lane order decides (stable sort)
    seen = [int(ids[k]) for k in (0, 5, 10, 77)]
    for T, top_p, rep in [(0.0, 0.9, 1.0), (0.0, 0.9, 1.3), (0.7, 0.9, 1.2), (1.0, 0.5, 1.0), (0.3, 1.0, 2.0)]:
        for u in (0.0, 0.01, 0.5, 0.999999):
            a = oracle_mod.sample(vals, ids, T, top_p, rep, seen, u, vocab)
            b = oracle_np.sample(vals, ids, T, top_p, rep, set(seen), u)
            assert a == b, (T, top_p, rep, u)
    # greedy without penalty is the top candidate
    assert oracle_mod.sample(vals, ids, 0.0, 0.9, 1.0, [], 0.0, vocab) == int(ids[int(np.argmax(vals))])


def test_bf16_round_c_vs_numpy_vs_torch(oracle_mod):
    """The optional bf16 KV store's rounding: the C oracle's integer method, the numpy
    restatement by definition and torch's f32 -> bf16 cast agree on every value, ties included."""
    import torch
    from oracle import oracle_np
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(20000) * np.exp2(rng.integers(-30, 30, 20000))).astype(np.float32)
    u = x.view(np.uint32).copy()
    u[:4000] = (u[:4000] & np.uint32(0xFFFF0000)) | np.uint32(0x8000)  # exact ties, both parities
    u[4000:4100] = rng.integers(0, 1 << 23, 100).astype(np.uint32)   # subnormals
    u[4100:4200] = (u[4100:4200] & np.uint32(0xFFFF0000)) | np.uint32(0x7FFF)
    u[4200] = 0
    u[4201] = 0x80000000
    u[4202] = 0x7F7FFFFF  # largest finite f32 rounds up to infinity
    x = u.view(np.float32)
    c = oracle_mod.bf16_round(x)
    t = torch.from_numpy(x.copy()).to(torch.bfloat16).to(torch.float32).numpy()
    assert (c.view(np.uint32) == t.view(np.uint32)).all()
    fin = np.isfinite(x) & (np.abs(x) < 3e38)
    n = oracle_np.bf16_round(x[fin])
    assert (c[fin].view(np.uint32) == n.view(np.uint32)).all()


@pytest.mark.parametrize("kv_dtype", ["f32", "bf16"])
def test_tiny_forward_c_vs_numpy(kv_dtype):
    import dataclasses
    from oracle import oracle, oracle_np
    from gemma_b200 import synth
    cfg, tens = synthetic("tiny", 7)
    cfg = dataclasses.replace(cfg, kv_dtype=kv_dtype)
    store = oracle_np.bf16_round if kv_dtype == "bf16" else (lambda a: a)
    P = {}
    for name, (dims, t, raw) in tens.items():
        P[name] = oracle.pack_q8_0(raw) if t == 8 else raw.view(np.float32)
    H, Q, KV, I, HD, L = cfg.hidden_size, cfg.q_dim, cfg.kv_dim, cfg.intermediate_size, cfg.head_dim, cfg.num_layers
    prompt = synth.make_prompt(7, 4, cfg.vocab_size)
    kc = np.zeros((L, cfg.context_length, KV), np.float32)
    vc = np.zeros_like(kc)
    m = oracle.OracleModel.from_tensors(cfg, tens)
    for pos, tok in enumerate(prompt):
        hidden = oracle.embedding(P["token_embd.weight"], H, int(tok))
        for l in range(L):
            g = lambda k: P[f"blk.{l}.{k}.weight"]
            x = oracle_np.rmsnorm(hidden, g("attn_norm"), 1e-6)
            q = oracle_np.linear_q8(x, g("attn_q"), Q, H)
            k = oracle_np.linear_q8(x, g("attn_k"), KV, H)
            v = oracle_np.linear_q8(x, g("attn_v"), KV, H)
            q = oracle_np.fused_norm_rope(q, g("attn_q_norm"), 4, HD, 1e-6, pos, 1e6)
            k = oracle_np.fused_norm_rope(k, g("attn_k_norm"), 1, HD, 1e-6, pos, 1e6)
            kc[l, pos], vc[l, pos] = store(k), store(v)
            att = oracle_np.attention(q, kc[l], vc[l], 4, 1, HD, pos + 1, 0.0625)
            res = oracle_np.fused_norm_add(oracle_np.linear_q8(att, g("attn_output"), H, Q),
                                           g("post_attention_norm"), hidden, 1e-6)
            x = oracle_np.rmsnorm(res, g("ffn_norm"), 1e-6)
            mul = oracle_np.gelu_mul(oracle_np.linear_q8(x, g("ffn_gate"), I, H),
                                     oracle_np.linear_q8(x, g("ffn_up"), I, H))
            hidden = oracle_np.fused_norm_add(oracle_np.linear_q8(mul, g("ffn_down"), H, I),
                                              g("post_ffw_norm"), res, 1e-6)
        normed_np = oracle_np.rmsnorm(hidden, P["output_norm.weight"], 1e-6)
        normed_c = m.forward(int(tok), pos)
        assert rel_l2(normed_c, normed_np) < 1e-6
    lg_np = oracle_np.linear_q8(normed_np, P["token_embd.weight"], cfg.vocab_size, H)
    assert rel_l2(m.logits(), lg_np) < 1e-6


def test_golden_greedy_fixtures():
    from oracle import oracle
    from gemma_b200 import synth
    import hashlib
    with open(os.path.join(HERE, "golden", "greedy.json")) as f:
        gold = json.load(f)
    for case in gold["cases"]:
        cfg, tens = synthetic(case["shape"], case["seed"])
        prompt = synth.make_prompt(case["seed"], len(case["prompt"]), cfg.vocab_size)
        assert [int(t) for t in prompt] == case["prompt"]
        m = oracle.OracleModel.from_tensors(cfg, tens)
        toks, lgs = m.greedy(prompt, len(case["greedy"]), return_logits=True)
        assert toks == case["greedy"]
        assert hashlib.sha256(np.asarray(lgs[0], np.float32).tobytes()).hexdigest() == case["logits_first"]["sha256"]


def test_oracle_rejects_bad_input(oracle_mod):
    cfg, tens = synthetic("tiny", 7)
    m = oracle_mod.OracleModel.from_tensors(cfg, tens)
    with pytest.raises(ValueError):
        m.forward(cfg.vocab_size, 0)
    with pytest.raises(ValueError):
        m.forward(1, cfg.context_length)
    with pytest.raises(ValueError):
        m.set_tensor("blk.99.attn_q.weight", 8, np.zeros(34, np.uint8), 32)


def test_oracle_sliding_window_semantics():
    """A window at least as long as the prefix changes nothing; swa_period 1 makes every layer
    global (no window at all)."""
    import dataclasses
    from oracle import oracle
    from gemma_b200 import synth
    cfg, tens = synthetic("tiny", 7)
    prompt = synth.make_prompt(7, 12, cfg.vocab_size)

    def run(c):
        m = oracle.OracleModel.from_tensors(c, tens)
        for i, t in enumerate(prompt):
            out = m.forward(int(t), i)
        lg = m.logits()
        m.close()
        return lg

    base = run(cfg)
    assert (run(dataclasses.replace(cfg, sliding_window=64)) == base).all()
    assert (run(dataclasses.replace(cfg, sliding_window=4, swa_period=1)) == base).all()
    assert not (run(dataclasses.replace(cfg, sliding_window=4)) == base).all()


def test_sampler_known_answers(oracle_mod):
    """Hand-computed cases of engine.ts:862-901, independent of both restatements."""
    from oracle import oracle_np
    vocab = 1024
    ids = np.arange(256, dtype=np.uint32) + 500
    low = np.float32(-1e30)  # candidates that contribute exp(-inf) = 0

    def both(vals, T, top_p, rep, seen, u):
        a = oracle_mod.sample(vals, ids, T, top_p, rep, list(seen), u, vocab)
        b = oracle_np.sample(vals, ids, T, top_p, rep, set(seen), u)
        assert a == b
        return a

    # repetition penalty: a seen positive logit is divided (2.0 / 1.25 = 1.6 < 1.9) ...
    v = np.full(256, low, np.float32)
    v[0], v[1] = 2.0, 1.9
    assert both(v, 0.0, 0.9, 1.0, [], 0.0) == 500           # no penalty: greedy fast path
    assert both(v, 0.0, 0.9, 1.25, [500], 0.0) == 501       # penalised: the other candidate wins
    # ... and a seen negative logit is multiplied (-1.0 * 1.25 = -1.25 < -1.1)
    v[0], v[1] = -1.0, -1.1
    assert both(v, 0.0, 0.9, 1.25, [500], 0.0) == 501
    # ties keep lane order (the sort is stable)
    v[0], v[1] = 0.5, 0.5
    assert both(v, 0.0, 0.9, 1.5, [700], 0.0) == 500
    # top-p: probs 1, 1/2, 1/4 (T = 1), shares 4/7, 2/7, 1/7; top_p 0.8 keeps two (4/7 < 0.8 <= 6/7)
    v = np.full(256, low, np.float32)
    v[0], v[1], v[2] = 0.0, np.float32(np.log(0.5)), np.float32(np.log(0.25))
    assert both(v, 1.0, 0.8, 1.0, [], 0.6) == 500            # r = 0.6 * 1.5 = 0.9; 0.9 - 1 <= 0
    assert both(v, 1.0, 0.8, 1.0, [], 0.7) == 501            # r = 1.05; 1.05 - 1 > 0; 0.05 - 0.5 <= 0
    assert both(v, 1.0, 0.8, 1.0, [], 0.999999) == 501       # the third candidate is cut off
    assert both(v, 1.0, 1.0, 1.0, [], 0.999999) == 502       # top_p 1 keeps all three


def test_ops_known_answers(oracle_mod):
    """Each op against its formula evaluated in float64 (shaders.ts; see the op's reference lines)."""
    rng = np.random.default_rng(21)
    n = 640
    x = rng.standard_normal(n).astype(np.float32)
    w = (rng.standard_normal(n) * 0.1).astype(np.float32)
    res = rng.standard_normal(n).astype(np.float32)
    x64, w64 = x.astype(np.float64), w.astype(np.float64)
    rms = np.sqrt(np.mean(x64 * x64) + 1e-6)
    # rmsNorm is x * w / rms (shaders.ts:25-56): zero weights give zeros (not Gemma's (1 + w))
    assert rel_l2(oracle_mod.rmsnorm(x, w), x64 * w64 / rms) < 1e-6
    assert (oracle_mod.rmsnorm(x, np.zeros(n, np.float32)) == 0).all()
    # fusedNormAdd: res + x * w / rms(x) (shaders.ts:386-418)
    assert rel_l2(oracle_mod.fused_norm_add(x, w, res), res + x64 * w64 / rms) < 1e-6
    # GeGLU with the argument clamp at +-15 (shaders.ts:153-170)
    g = np.array([0.0, 1.0, -1.0, 20.0, -20.0], np.float32)
    u = np.array([3.0, 2.0, 2.0, 0.5, 0.5], np.float32)
    t = np.clip(0.7978845608028654 * g * (1 + 0.044715 * g.astype(np.float64) ** 2), -15, 15)
    want = 0.5 * g * (1 + np.tanh(t)) * u
    got = oracle_mod.gelu_mul(g, u).astype(np.float64)
    assert np.allclose(got, want, rtol=1e-6, atol=1e-12)
    assert got[3] == pytest.approx(10.0, rel=1e-6) and abs(got[4]) < 1e-9
    # per-head norm + RoPE (shaders.ts:420-467): position 0 is the norm alone; at pos p the pair
    # (i, i + 128) turns by p * theta^(-2i/256)
    hd = 256
    d = rng.standard_normal(hd).astype(np.float32)
    wn = (rng.standard_normal(hd) * 0.1 + 1.0).astype(np.float32)
    d64 = d.astype(np.float64)
    normed = d64 * wn.astype(np.float64) / np.sqrt(np.mean(d64 * d64) + 1e-6)
    assert rel_l2(oracle_mod.fused_norm_rope(d, wn, 1, hd, 1e-6, 0, 1e6), normed) < 1e-6
    pos, theta = 37, 1e4
    ang = pos * theta ** (-2.0 * np.arange(hd // 2) / hd)
    a0, a1 = normed[:hd // 2], normed[hd // 2:]
    rot = np.concatenate([a0 * np.cos(ang) - a1 * np.sin(ang), a0 * np.sin(ang) + a1 * np.cos(ang)])
    assert rel_l2(oracle_mod.fused_norm_rope(d, wn, 1, hd, 1e-6, pos, theta), rot) < 1e-5
    # attention over one key returns that key's value row for every head (softmax of one score)
    q = rng.standard_normal(4 * hd).astype(np.float32)
    kc = rng.standard_normal((1, hd)).astype(np.float32)
    vc = rng.standard_normal((1, hd)).astype(np.float32)
    out = oracle_mod.attention(q, kc, vc, 4, 1, hd, 1, 0.0625).reshape(4, hd)
    assert (out == vc[0]).all()


def test_linear_q8_and_embedding_known_answers(oracle_mod):
    """linearQ8 (shaders.ts:92-151): y[m] = sum over blocks of (sum_j q * x) * d; embedding
    (shaders.ts:2-23): h = q * d * sqrt(H). Small integers and power-of-two scales keep every
    step exact, so the expected values are exact."""
    def block(d_f16_bits, q):
        return np.concatenate([np.array([d_f16_bits & 255, d_f16_bits >> 8], np.uint8),
                               np.asarray(q, np.int8).view(np.uint8)])
    n, m = 64, 2                        # two rows of two blocks each
    q = np.arange(-16, 16, dtype=np.int8)
    raw = np.concatenate([block(0x3C00, q), block(0x4000, -q),        # row 0: d = 1, then d = 2
                          block(0x3800, np.ones(32)), block(0x3400, 2 * np.ones(32))])  # row 1: 0.5, 0.25
    packed = oracle_mod.pack_q8_0(raw)
    x = np.concatenate([np.ones(32), np.arange(32)]).astype(np.float32)
    y = oracle_mod.linear_q8(x, packed, m, n)
    want0 = q.astype(np.int64).sum() * 1.0 + (-q.astype(np.int64) * np.arange(32)).sum() * 2.0
    want1 = 32 * 0.5 + 2 * np.arange(32).sum() * 0.25
    assert y.tolist() == [float(want0), float(want1)]
    # embedding row 1 of a [2][64] table: h = q * d * sqrt(64) = q * d * 8
    h = oracle_mod.embedding(packed, n, 1)
    assert h.tolist() == [0.5 * 8.0] * 32 + [2 * 0.25 * 8.0] * 32
