"""GGUF reader/writer (restating src/gguf.ts) and the synthetic model generator."""
import struct

import numpy as np
import pytest

from conftest import synthetic


def test_roundtrip_and_config(tmp_path):
    from gemma_b200 import gguf, synth
    from gemma_b200.config import default_config
    shape = synth.SHAPES["tiny"]
    path = synth.write_model(str(tmp_path / "m.gguf"), shape, 7)
    data = open(path, "rb").read()
    p = gguf.parse(data)
    assert p.version == 3 and p.data_offset % 32 == 0
    assert p.tensor_count == len(synth.tensor_shapes(shape))
    cfg = default_config()
    size = gguf.update_config_from_gguf(p, cfg)
    assert size == "270M"  # <= 18 layers (gguf.ts:218)
    assert (cfg.hidden_size, cfg.num_layers, cfg.intermediate_size, cfg.context_length) == (256, 2, 512, 256)
    assert cfg.q_dim == 4 * 256 and cfg.kv_dim == 256
    assert cfg.vocab_size == 262144  # never read from the file (types.ts:28)
    tens = synth.make_tensors(shape, 7)
    for t in p.tensors:
        dims, ty, raw = tens[t.name]
        assert list(t.dims) == list(dims) and t.type == ty
        assert bytes(p.tensor_bytes(t)) == raw.tobytes()
        assert t.offset % 32 == 0


def test_context_cap(tmp_path):
    from gemma_b200 import gguf, synth
    from gemma_b200.config import default_config
    path = synth.write_model(str(tmp_path / "m.gguf"), synth.SHAPES["mid"], 5)
    p = gguf.parse(open(path, "rb").read())
    cfg = default_config()
    gguf.update_config_from_gguf(p, cfg, 512)
    assert cfg.context_length == 512  # min(file ctx, requested cap) (gguf.ts:211-212)


def test_bad_magic_and_truncation():
    from gemma_b200 import gguf
    with pytest.raises(gguf.GGUFError, match="Invalid GGUF magic"):
        gguf.parse(struct.pack("<IIQQ", 0x12345678, 3, 0, 0) + b"\0" * 16)
    good = struct.pack("<IIQQ", gguf.GGUF_MAGIC, 3, 1, 1) + struct.pack("<Q", 4) + b"abcd"
    with pytest.raises(gguf.GGUFError):
        gguf.parse(good)


def test_tensor_byte_size_and_q8_helpers():
    from gemma_b200 import gguf
    t = gguf.GGUFTensor("x", [64, 3], gguf.GGML_TYPE_Q8_0, 0)
    assert gguf.tensor_byte_size(t) == 6 * 34
    assert gguf.tensor_byte_size(gguf.GGUFTensor("y", [10], gguf.GGML_TYPE_F32, 0)) == 40
    assert gguf.tensor_byte_size(gguf.GGUFTensor("z", [10], gguf.GGML_TYPE_F16, 0)) == 20
    with pytest.raises(gguf.GGUFError):
        gguf.tensor_byte_size(gguf.GGUFTensor("w", [32], 2, 0))
    rng = np.random.default_rng(0)
    qs = rng.integers(-127, 128, 96, dtype=np.int8)
    d = rng.standard_normal(3).astype(np.float16).view(np.uint16)
    q2, d2 = gguf.q8_0_split(gguf.q8_0_join(qs, d), 96)
    assert (q2 == qs).all() and (d2 == d).all()


def test_synthetic_distributions():
    cfg, tens = synthetic("tiny", 7)
    from gemma_b200 import gguf
    dims, t, raw = tens["blk.0.ffn_gate.weight"]
    qs, sb = gguf.q8_0_split(raw, int(np.prod(dims)))
    assert qs.min() >= -127 and qs.max() <= 127
    d = gguf.f16_to_f32(sb)
    assert (d >= 0).all() and 0.5e-4 < float(np.mean(d)) < 2e-4  # |N(0,1)| * 0.02/127 ~ 1.26e-4
    nw = tens["blk.0.attn_norm.weight"][2].view(np.float32)
    assert 0.05 < float(np.std(nw)) < 0.2
    from gemma_b200 import synth
    a, b = synth.make_prompt(1, 512), synth.make_prompt(1, 512)
    assert (a == b).all() and a.min() >= 2 and a.max() < 262144
