"""Generate the golden fixtures in this directory from the CPU oracle (oracle/gemma_oracle.c).

The reference (svenflow/webgpu-gemma) ships no tests or vectors and cannot run here (it needs
WebGPU and a JS runtime), so these fixtures are the oracle's outputs on seeded synthetic models;
they pin the oracle against itself over time and let GPU tests check tokens without rerunning it.

    python tests/golden/make_golden.py
"""
import hashlib
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "webgpu-gemma_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

from gemma_b200 import synth  # noqa: E402
from oracle import oracle  # noqa: E402

CASES = [  # (shape, seed, prompt length, new tokens)
    ("tiny", 7, 5, 16),
    ("small", 3, 9, 12),
    ("mid", 5, 17, 8),
]


def logits_digest(lg: np.ndarray) -> dict:
    lg = np.asarray(lg, np.float32)
    return {"sha256": hashlib.sha256(lg.tobytes()).hexdigest(), "sum": float(lg.astype(np.float64).sum()),
            "l2": float(np.linalg.norm(lg.astype(np.float64))), "first8": [float(v) for v in lg[:8]]}


def main():
    oracle.build()
    out = {"generator": "tests/golden/make_golden.py", "cases": []}
    for shape_name, seed, plen, ngen in CASES:
        shape = synth.SHAPES[shape_name]
        cfg = shape.config()
        tens = synth.make_tensors(shape, seed)
        m = oracle.OracleModel.from_tensors(cfg, tens)
        prompt = synth.make_prompt(seed, plen, cfg.vocab_size)
        toks, lgs = m.greedy(prompt, ngen, return_logits=True)
        out["cases"].append({
            "shape": shape_name, "seed": seed, "prompt": [int(t) for t in prompt], "greedy": [int(t) for t in toks],
            "logits_first": logits_digest(lgs[0]), "logits_last": logits_digest(lgs[-1]),
        })
        print(shape_name, toks)
    with open(os.path.join(HERE, "greedy.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
