"""The numbers bench.py's roofline and sampled configs rest on, checked on the CPU.

* Algorithmic bytes per decode token: Q8_0 weights at 34 B per 32 weights (tied LM head
  included), f32 norm weights, one embedding row and the f32 KV rows of positions 0..pos,
  53,248 B per position at 1B (2 x 26 layers x 256 x 4 B).
* The injected sampling draws: one Philox4x32-10 stream per sequence, reproducible and in [0, 1).
"""
import numpy as np
import pytest

import bench
from gemma_b200 import synth
from gemma_b200.engine import philox_uniforms


@pytest.mark.parametrize("shape,seed,weights,kv_per_pos", [
    ("1b", 1, 741_371_904 + 320_864_256 + 537_088, 2 * 26 * 256 * 4),
    ("270m", 0, 106_536_960 + 178_257_920 + 223_744, 2 * 18 * 256 * 4),
])
def test_weight_bytes_and_kv_bytes_per_position(shape, seed, weights, kv_per_pos):
    sh = synth.SHAPES[shape]
    tensors = synth.make_tensors(sh, seed)
    assert bench.weight_bytes(tensors) == weights
    cfg = sh.config()
    assert 2 * cfg.num_layers * cfg.kv_dim * 4 == kv_per_pos
    if shape == "1b":
        assert bench.KV_BYTES_PER_POS == kv_per_pos
        emb_row = cfg.hidden_size + cfg.hidden_size // 16  # 1,152 quants + 36 f16 scales
        assert bench.algo_bytes_per_token(weights, cfg.hidden_size, 640) == weights + emb_row + kv_per_pos * 641


def test_roofline_traffic_is_close_to_the_algorithmic_bytes():
    """The committed ncu traffic per launch (position 641) is within 2 % of the algorithmic bytes:
    the weights cross HBM once."""
    algo = bench.algo_bytes_per_token(1_062_773_248, 1152, 641)
    assert abs(bench.NCU_TRAFFIC_PER_LAUNCH / algo - 1.0) < 0.02


def test_philox_draws_are_reproducible_per_stream():
    a = philox_uniforms(1, 5, 300)
    b = philox_uniforms(1, 5, 300)
    c = philox_uniforms(1, 6, 300)
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)
    assert a.dtype == np.float64 and a.min() >= 0.0 and a.max() < 1.0
    assert np.array_equal(philox_uniforms(1, 5, 100), a[:100])  # a prefix of the same stream
