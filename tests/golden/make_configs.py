"""Full-size golden fixtures for the benchmark configurations, made by the CPU oracle.

The reference (svenflow/webgpu-gemma) ships no vectors and cannot run here (it needs WebGPU and
a JS runtime), so its CPU restatement (oracle/gemma_oracle.c) produces them on the same seeded
synthetic models, prompts and draws that bench.py runs:

* cfg0 -- 270M shape, seed 0, 32-token prompt, 64 greedy tokens (src/engine.ts:923-1025);
* cfg1 -- 1B shape, seed 1, 512-token prompt, 256 greedy tokens;
* cfg3 -- 1B shape, two turns: 1536-token prompt + 128 tokens, then 256 ids (the last sampled
  token first) + 128 tokens, the last forward at position 2045 (engine.ts:968-990 KV reuse);
* cfg4 -- 1B shape, 4 of the 64 sampled streams (T 0.7, top-p 0.9, rep 1.2, per-stream Philox
  draws), 256-token prompts, 32 tokens each (engine.ts:862-901 with injected draws).

Each greedy fixture holds every step's token, its top-1 / top-2 logits (the margin shows a near
tie instead of hiding it) and the full logits of a few steps (float32). The GPU tests
(tests/test_gpu_configs.py) compare against these files without running the oracle.

    python tests/golden/make_configs.py [cfg0 cfg1 cfg3 cfg4]
"""
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "webgpu-gemma_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from gemma_b200 import synth  # noqa: E402
from gemma_b200.engine import philox_uniforms  # noqa: E402
from oracle import oracle  # noqa: E402

# Workloads, shared with bench.py and tests/test_gpu_configs.py.
CFG0 = dict(shape="270m", seed=0, prompt=32, new=64, logit_steps=(0, 63))
CFG1 = dict(shape="1b", seed=1, prompt=512, new=256, logit_steps=(0, 128, 255))
CFG3 = dict(shape="1b", seed=1, turns=((1536, 128), (256, 128)), logit_steps=((0, 0), (1, 127)))
CFG4 = dict(shape="1b", seed=1, seqs=64, prompt=256, new=32, streams=(0, 21, 42, 63), sample=(0.7, 0.9, 1.2))


def top2(lg: np.ndarray):
    i = int(oracle.argmax(lg))
    rest = np.delete(lg, i)
    return i, float(lg[i]), float(np.max(rest))


def cfg1_prompt(c):
    return synth.make_prompt(c["seed"], c["prompt"], 262144)


def cfg3_turn_ids(c, turn: int, last):
    ids = [int(t) for t in synth.make_prompt(c["seed"] * 1000 + turn, c["turns"][turn][0], 262144)]
    return ids if last is None else [int(last)] + ids[:-1]


def cfg4_prompt(c, sid: int):
    return synth.make_prompt(c["seed"] * 100003 + sid, c["prompt"], 262144)


def greedy_run(m, ids, start_pos, n_new, keep_steps):
    """Prefill `ids` at start_pos, then n_new greedy tokens. Returns tokens, top1, top2 and the
    kept steps' logits."""
    for i, t in enumerate(ids):
        m.forward(int(t), start_pos + i)
    pos = start_pos + len(ids)
    toks, t1, t2, kept = [], [], [], {}
    lg = m.logits()
    for s in range(n_new):
        if s > 0:
            m.forward(toks[-1], pos)
            pos += 1
            lg = m.logits()
        i, a, b = top2(lg)
        toks.append(i); t1.append(a); t2.append(b)
        if s in keep_steps:
            kept[s] = lg.copy()
    return toks, np.array(t1, np.float32), np.array(t2, np.float32), kept


def make_cfg0():
    c = CFG0
    shape = synth.SHAPES[c["shape"]]
    cfg = shape.config()
    m = oracle.OracleModel.from_tensors(cfg, synth.make_tensors(shape, c["seed"]))
    prompt = synth.make_prompt(c["seed"], c["prompt"], cfg.vocab_size)
    toks, t1, t2, kept = greedy_run(m, prompt, 0, c["new"], c["logit_steps"])
    np.savez_compressed(os.path.join(HERE, "cfg0_270m.npz"), prompt=prompt, tokens=np.array(toks, np.int32),
                        top1=t1, top2=t2, logit_steps=np.array(c["logit_steps"], np.int32),
                        logits=np.stack([kept[s] for s in c["logit_steps"]]))
    return toks, t1 - t2


def make_cfg1():
    c = CFG1
    shape = synth.SHAPES[c["shape"]]
    cfg = shape.config()
    m = oracle.OracleModel.from_tensors(cfg, synth.make_tensors(shape, c["seed"]))
    prompt = cfg1_prompt(c)
    toks, t1, t2, kept = greedy_run(m, prompt, 0, c["new"], c["logit_steps"])
    np.savez_compressed(os.path.join(HERE, "cfg1_1b.npz"), prompt=prompt, tokens=np.array(toks, np.int32),
                        top1=t1, top2=t2, logit_steps=np.array(c["logit_steps"], np.int32),
                        logits=np.stack([kept[s] for s in c["logit_steps"]]))
    return toks, t1 - t2


def make_cfg3():
    c = CFG3
    shape = synth.SHAPES[c["shape"]]
    cfg = shape.config()
    m = oracle.OracleModel.from_tensors(cfg, synth.make_tensors(shape, c["seed"]))
    out, pos, last, lgs = {}, 0, None, []
    for ti, (plen, ngen) in enumerate(c["turns"]):
        ids = cfg3_turn_ids(c, ti, last)
        keep = tuple(s for (t, s) in c["logit_steps"] if t == ti)
        toks, t1, t2, kept = greedy_run(m, ids, pos, ngen, keep)
        out[f"ids{ti}"] = np.array(ids, np.int32)
        out[f"tokens{ti}"] = np.array(toks, np.int32)
        out[f"top1_{ti}"], out[f"top2_{ti}"] = t1, t2
        out[f"start{ti}"] = np.int32(pos)
        lgs += [kept[s] for s in keep]
        pos += len(ids) + ngen - 1
        last = toks[-1]
    np.savez_compressed(os.path.join(HERE, "cfg3_1b.npz"), logit_steps=np.array(c["logit_steps"], np.int32),
                        logits=np.stack(lgs), **out)
    return [out["tokens0"], out["tokens1"]], None


def sample_gap(vals, temperature, top_p, u):
    """Distance of the draw from the nearest pick boundary, as a fraction of the kept mass
    (diagnostic only: a tiny gap means a low-bit difference could change the pick)."""
    v = np.sort(np.asarray(vals, np.float64))[::-1]
    p = np.exp((v - v[0]) / temperature).astype(np.float32).astype(np.float64)
    cum = np.cumsum(p / p.sum())
    cutoff = int(np.searchsorted(cum, top_p) + 1)
    sub = p[:cutoff].sum()
    edges = np.cumsum(p[:cutoff]) / sub
    return float(np.min(np.abs(edges - u)))


def make_cfg4():
    c = CFG4
    shape = synth.SHAPES[c["shape"]]
    cfg = shape.config()
    T, TP, R = c["sample"]
    streams = c["streams"]
    m = oracle.OracleModel.from_tensors(cfg, synth.make_tensors(shape, c["seed"]), max_seqs=len(streams))
    toks = np.zeros((c["new"], len(streams)), np.int32)
    gaps = np.zeros((c["new"], len(streams)), np.float64)
    for k, sid in enumerate(streams):
        prompt = cfg4_prompt(c, sid)
        draws = philox_uniforms(c["seed"], sid, c["new"] + 1)
        for i, t in enumerate(prompt):
            m.forward(int(t), i, k)
        seen = [int(t) for t in prompt]
        pos = len(prompt)
        for s in range(c["new"]):
            if s > 0:
                m.forward(int(toks[s - 1, k]), pos, k)
                pos += 1
            vals, ids = oracle.topk256(m.logits(k))
            tok = oracle.sample(vals, ids, T, TP, R, seen, float(draws[s]), cfg.vocab_size)
            gaps[s, k] = sample_gap(vals, T, TP, float(draws[s]))
            toks[s, k] = tok
            seen.append(tok)
        print("cfg4 stream", sid, toks[:, k].tolist(), flush=True)
    np.savez_compressed(os.path.join(HERE, "cfg4_1b.npz"), streams=np.array(streams, np.int32), tokens=toks,
                        draw_gap=gaps)
    return toks, gaps.min()


def main(names):
    oracle.build()
    print("oracle threads", oracle.use_all_host_cores(), flush=True)
    for name in names:
        t0 = time.time()
        toks, margin = {"cfg0": make_cfg0, "cfg1": make_cfg1, "cfg3": make_cfg3, "cfg4": make_cfg4}[name]()
        mm = None if margin is None else float(np.min(margin))
        print(f"{name}: done in {time.time() - t0:.0f} s, smallest margin {mm}", flush=True)


if __name__ == "__main__":
    main(sys.argv[1:] or ["cfg0", "cfg1", "cfg3", "cfg4"])
