"""Bit-exact dequantisation on the device ("bit-exact dequant").

The reference unpacks each 34-byte GGUF Q8_0 block into {f32 d, 8 x u32} on the host
(packQ8_0ForGPU + f16ToF32, src/gguf.ts:95-149) and its shader multiplies f32(q) * d. This
library uploads the raw blocks and repacks them on the device (row format for the decode kernel,
tiled copy for the tensor-core GEMM). gg_dequant_row reads a row back from either copy as
f32(q) * f32(d); every value must equal the oracle's unpacking bit for bit, including blocks
whose f16 scale is subnormal, negative zero or the largest finite value and quants of -128.
"""
import numpy as np
import pytest

from conftest import synthetic

pytestmark = pytest.mark.gpu

# f16 scale patterns planted in chosen blocks: smallest subnormal, -0, largest negative
# subnormal, largest finite, 1.0, a negative normal
SCALES = [0x0001, 0x8000, 0x83FF, 0x7BFF, 0x3C00, 0xB555]


def _plant(raw: np.ndarray, K: int, row: int, first_block: int) -> None:
    """Writes the SCALES patterns (and a -128 quant) into blocks of `row` of a raw Q8_0 tensor."""
    bpr = K // 32
    for j, bits in enumerate(SCALES):
        b = row * bpr + (first_block + j) % bpr
        raw[b * 34:b * 34 + 2] = np.frombuffer(np.uint16(bits).tobytes(), np.uint8)
        raw[b * 34 + 2 + j] = np.uint8(0x80)  # int8 -128


def _oracle_row(oracle_mod, raw: np.ndarray, K: int, row: int) -> np.ndarray:
    bpr = K // 32
    words = oracle_mod.pack_q8_0(raw[row * bpr * 34:(row + 1) * bpr * 34]).reshape(bpr, 9)
    d = words[:, 0].view(np.float32)
    q = words[:, 1:].copy().view(np.int8).reshape(bpr, 32).astype(np.float32)
    return (q * d[:, None]).reshape(-1).astype(np.float32)


def _source(cfg, tens, which, layer, r):
    """(raw tensor, K, row in that tensor) of row r of the engine's matrix `which`."""
    H, Q, KV = cfg.hidden_size, cfg.q_dim, cfg.kv_dim
    p = f"blk.{layer}."
    if which == 0:
        name, rr = (("attn_q", r) if r < Q else ("attn_k", r - Q) if r < Q + KV else ("attn_v", r - Q - KV))
        return tens[p + name + ".weight"][2], H, rr
    if which == 1:
        return tens[p + "attn_output.weight"][2], Q, r
    if which == 2:
        return tens[p + ("ffn_gate" if r % 2 == 0 else "ffn_up") + ".weight"][2], H, r // 2
    if which == 3:
        return tens[p + "ffn_down.weight"][2], cfg.intermediate_size, r
    return tens["token_embd.weight"][2], H, r


def test_device_rows_dequantise_bit_exact(oracle_mod):
    from gemma_b200.native import engine_from_tensors
    cfg, base = synthetic("mid", 5)
    tens = {k: (d, t, np.array(raw, copy=True)) for k, (d, t, raw) in base.items()}
    L = cfg.num_layers
    M = {0: cfg.q_dim + 2 * cfg.kv_dim, 1: cfg.hidden_size, 2: 2 * cfg.intermediate_size, 3: cfg.hidden_size,
         4: cfg.vocab_size}
    planted = []
    for which in range(5):
        for layer in ([0] if which == 4 else [0, L - 1]):
            for r in (0, M[which] // 3, M[which] - 1):
                raw, K, rr = _source(cfg, tens, which, layer, r)
                _plant(raw, K, rr, first_block=r % 7)
                planted.append((which, layer, r))
    eng = engine_from_tensors(cfg, tens)
    checked = 0
    rng = np.random.default_rng(0)
    rows = planted + [(w, int(rng.integers(0, L)) if w < 4 else 0, int(rng.integers(0, M[w]))) for w in range(5)
                      for _ in range(4)]
    for which, layer, r in rows:
        raw, K, rr = _source(cfg, tens, which, layer, r)
        want = _oracle_row(oracle_mod, raw, K, rr)
        for copy in (0, 1):
            got = eng.dequant_row(which, layer, r, copy)
            same = got.view(np.uint32) == want.view(np.uint32)
            assert same.all(), (which, layer, r, copy, int(np.argmin(same)), got[~same][:4], want[~same][:4])
            checked += 1
    eng.close()
    assert checked == 2 * len(rows)
    # the planted patterns really occur: a -0 scale gives signed zeros, a subnormal scale 2^-24 steps
    raw, K, rr = _source(cfg, tens, 4, 0, 0)
    w = _oracle_row(oracle_mod, raw, K, rr)
    assert (w[32:64] == 0).all() and np.signbit(w[32:64]).any()
    assert np.float32(w[0:32][w[0:32] != 0][0]) % np.float32(2.0 ** -24) == 0
