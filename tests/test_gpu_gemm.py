"""Tensor-core Q8_0 GEMM (gg_linear, tcgen05) against the exactly dequantised weights.

y[b][m] = sum_k x[b][k] W[m][k] is compared with a float64 product of the dequantised
weights (q * f32(d) is exact, gguf.ts:107-124). The bound is relative to sum_k |x||W|:
the kernel splits weights and activations into bf16 hi + lo pairs (about 2^-17 each) and
accumulates in f32, so 1e-4 of that scale is a loose bound; the reference's own sequential
f32 loop has errors of the same order.
"""
import numpy as np
import pytest

from conftest import synthetic

pytestmark = pytest.mark.gpu

TOL = 1e-4


def dense(tens, name, rows, cols):
    from gemma_b200 import gguf
    dims, t, raw = tens[name]
    return gguf.dequantize_q8_0(raw, rows * cols).reshape(rows, cols).astype(np.float64)


def matrices(cfg, tens, layer):
    H, Q, KV, I, V = cfg.hidden_size, cfg.q_dim, cfg.kv_dim, cfg.intermediate_size, cfg.vocab_size
    b = f"blk.{layer}."
    qkv = np.concatenate([dense(tens, b + "attn_q.weight", Q, H), dense(tens, b + "attn_k.weight", KV, H),
                          dense(tens, b + "attn_v.weight", KV, H)])
    gate, up = dense(tens, b + "ffn_gate.weight", I, H), dense(tens, b + "ffn_up.weight", I, H)
    gu = np.empty((2 * I, H))
    gu[0::2], gu[1::2] = gate, up
    return {0: qkv, 1: dense(tens, b + "attn_output.weight", H, Q), 2: gu,
            3: dense(tens, b + "ffn_down.weight", H, I), 4: dense(tens, "token_embd.weight", V, H)}


def check(y, x, W):
    ref = x.astype(np.float64) @ W.T
    scale = np.abs(x.astype(np.float64)) @ np.abs(W).T
    err = np.abs(y - ref) / np.maximum(scale, 1e-30)
    assert err.max() < TOL, (err.max(), np.unravel_index(err.argmax(), err.shape))


@pytest.fixture(scope="module")
def mid():
    from gemma_b200.native import engine_from_tensors
    cfg, tens = synthetic("mid", 3)
    eng = engine_from_tensors(cfg, tens)
    yield cfg, tens, eng
    eng.close()


@pytest.fixture(params=[0, 1], ids=["dequant", "scaled"])
def kernel(request):
    """Runs the test with each kernel family of the tensor-core products, then restores it."""
    from gemma_b200.native import set_gemm_kernel
    prev = set_gemm_kernel(request.param)
    yield request.param
    set_gemm_kernel(prev)


@pytest.mark.parametrize("batch", [1, 2, 8, 9, 64, 65, 128, 200])
def test_gemm_all_matrices(mid, batch, kernel):
    cfg, tens, eng = mid
    W = matrices(cfg, tens, 1)
    rng = np.random.default_rng(batch)
    for which in range(5):
        K = W[which].shape[1]
        x = rng.standard_normal((batch, K)).astype(np.float32)
        y = eng.linear(which, 1, x)
        check(y, x, W[which])


def test_gemm_prefill_sized_batch_small_model(kernel):
    from gemma_b200.native import engine_from_tensors
    cfg, tens = synthetic("small", 5)
    eng = engine_from_tensors(cfg, tens)
    W = matrices(cfg, tens, 2)
    rng = np.random.default_rng(0)
    for which in (0, 3):
        x = (rng.standard_normal((512, W[which].shape[1])) * 3).astype(np.float32)
        check(eng.linear(which, 2, x), x, W[which])
    eng.close()
