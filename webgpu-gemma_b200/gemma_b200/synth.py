"""Seeded synthetic Gemma 3 Q8_0 models (the benchmark's stand-in for real checkpoints).

There is no network here, so the benchmark configurations use random-init weights of the
real architectures. The distributions are fixed so that every machine builds the same bytes
from the same seed (numpy's PCG64 stream is platform independent):

* Q8_0 quants uniform in [-127, 127]; scale ``d = f16(|N(0,1)| * 0.02 / 127)``;
* norm weights (F32) ``N(0, 0.1)``;
* prompts: token ids uniform in [2, vocab) from a second stream ``default_rng([seed, 1])``.

Tensors are drawn in the order of :data:`TENSOR_ORDER` per layer, after ``token_embd`` and
``output_norm``. Tensor names and shapes follow what the reference loads
(src/engine.ts:229-259, 335-336).
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import numpy as np

from . import gguf
from .config import GemmaConfig

SPECIAL = {0: "<pad>", 1: "<eos>", 2: "<bos>", 3: "<unk>", 105: "<start_of_turn>", 106: "<end_of_turn>"}

Q8_NAMES = ("attn_q", "attn_k", "attn_v", "attn_output", "ffn_gate", "ffn_up", "ffn_down")
F32_NAMES = ("attn_norm", "ffn_norm", "attn_q_norm", "attn_k_norm", "post_attention_norm", "post_ffw_norm")
TENSOR_ORDER = ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_q_norm", "attn_k_norm", "attn_output",
                "post_attention_norm", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down", "post_ffw_norm")


@dataclass(frozen=True)
class ModelShape:
    name: str
    hidden: int
    layers: int
    inter: int
    q_heads: int = 4
    kv_heads: int = 1
    head_dim: int = 256
    vocab: int = 262144
    ctx: int = 2048

    def config(self) -> GemmaConfig:
        c = GemmaConfig(hidden_size=self.hidden, num_layers=self.layers, intermediate_size=self.inter,
                        num_q_heads=self.q_heads, num_kv_heads=self.kv_heads, head_dim=self.head_dim,
                        vocab_size=self.vocab, context_length=self.ctx)
        c.q_dim = self.q_heads * self.head_dim
        c.kv_dim = self.kv_heads * self.head_dim
        return c


# BASELINE configs 0 and 1, plus small shapes for tests.
SHAPES = {
    "270m": ModelShape("270m", hidden=640, layers=18, inter=2048),
    "1b": ModelShape("1b", hidden=1152, layers=26, inter=6912),
    # test shapes: same head geometry, small vocab / widths, ragged K (640, 2048) and 1152-wide rows
    "tiny": ModelShape("tiny", hidden=256, layers=2, inter=512, vocab=4096, ctx=256),
    "tiny1": ModelShape("tiny1", hidden=256, layers=1, inter=512, vocab=4096, ctx=256),
    "small": ModelShape("small", hidden=640, layers=3, inter=2048, vocab=8192, ctx=512),
    "mid": ModelShape("mid", hidden=1152, layers=2, inter=6912, vocab=16384, ctx=1024),
}
SEEDS = {"270m": 0, "1b": 1}


def tensor_shapes(shape: ModelShape) -> dict[str, tuple[list[int], int]]:
    """name -> (ggml dims (ne0 = input width first), ggml type)."""
    H, Q, KV, I = shape.hidden, shape.q_heads * shape.head_dim, shape.kv_heads * shape.head_dim, shape.inter
    out = {"token_embd.weight": ([H, shape.vocab], gguf.GGML_TYPE_Q8_0),
           "output_norm.weight": ([H], gguf.GGML_TYPE_F32)}
    per = {"attn_norm": [H], "attn_q": [H, Q], "attn_k": [H, KV], "attn_v": [H, KV],
           "attn_q_norm": [shape.head_dim], "attn_k_norm": [shape.head_dim], "attn_output": [Q, H],
           "post_attention_norm": [H], "ffn_norm": [H], "ffn_gate": [H, I], "ffn_up": [H, I],
           "ffn_down": [I, H], "post_ffw_norm": [H]}
    for il in range(shape.layers):
        for key in TENSOR_ORDER:
            t = gguf.GGML_TYPE_Q8_0 if key in Q8_NAMES else gguf.GGML_TYPE_F32
            out[f"blk.{il}.{key}.weight"] = (per[key], t)
    return out


def _q8_tensor(rng: np.random.Generator, n: int) -> np.ndarray:
    nb = n // 32
    qs = rng.integers(-127, 128, size=n, dtype=np.int8)
    d = (np.abs(rng.standard_normal(nb)) * (0.02 / 127)).astype(np.float16)
    return gguf.q8_0_join(qs, d.view(np.uint16))


def _f32_tensor(rng: np.random.Generator, n: int) -> np.ndarray:
    return rng.normal(0.0, 0.1, size=n).astype(np.float32)


def make_tensors(shape: ModelShape, seed: int) -> dict[str, tuple[list[int], int, np.ndarray]]:
    """Draw every tensor of the model: name -> (dims, ggml type, raw little-endian bytes as uint8)."""
    rng = np.random.default_rng(seed)
    out = {}
    for name, (dims, t) in tensor_shapes(shape).items():
        n = int(np.prod(dims))
        if t == gguf.GGML_TYPE_Q8_0:
            out[name] = (dims, t, _q8_tensor(rng, n))
        else:
            out[name] = (dims, t, _f32_tensor(rng, n).view(np.uint8))
    return out


def make_vocab(n: int) -> list[str]:
    """A synthetic vocabulary: the reference's special ids, printable characters, and filler words."""
    vocab = [""] * n
    for i, s in SPECIAL.items():
        if i < n:
            vocab[i] = s
    chars = ["▁"] + [chr(c) for c in range(0x21, 0x7F)] + ["\n"]
    nxt = 4
    for ch in chars:
        while nxt in SPECIAL:
            nxt += 1
        vocab[nxt] = ch
        nxt += 1
    for i in range(n):
        if not vocab[i]:
            vocab[i] = f"▁w{i}"
    return vocab


def make_prompt(seed: int, n: int, vocab: int = 262144) -> np.ndarray:
    return np.random.default_rng([seed, 1]).integers(2, vocab, size=n, dtype=np.int64).astype(np.int32)


def write_model(path: str, shape: ModelShape, seed: int, tensors=None) -> str:
    """Write the synthetic model as a GGUF v3 file that the reference's parser accepts."""
    if tensors is None:
        tensors = make_tensors(shape, seed)
    u32 = gguf.T_UINT32
    kv = [
        ("general.architecture", gguf.T_STRING, "gemma3"),
        ("general.name", gguf.T_STRING, f"synthetic-{shape.name}-seed{seed}"),
        ("gemma3.embedding_length", u32, shape.hidden),
        ("gemma3.block_count", u32, shape.layers),
        ("gemma3.feed_forward_length", u32, shape.inter),
        ("gemma3.attention.head_count", u32, shape.q_heads),
        ("gemma3.attention.head_count_kv", u32, shape.kv_heads),
        ("gemma3.attention.key_length", u32, shape.head_dim),
        ("gemma3.context_length", u32, shape.ctx),
        ("tokenizer.ggml.tokens", gguf.T_ARRAY, (gguf.T_STRING, make_vocab(shape.vocab))),
    ]
    tl = [(name, dims, t, data) for name, (dims, t, data) in tensors.items()]
    gguf.write_gguf(path, kv, tl)
    return path


def cached_model(shape_name: str, seed: int | None = None, cache_dir: str | None = None) -> str:
    """Path of the synthetic GGUF for a named shape, generating it once per cache directory."""
    shape = SHAPES[shape_name]
    if seed is None:
        seed = SEEDS.get(shape_name, 7)
    cache_dir = cache_dir or os.environ.get("GEMMA_B200_CACHE", "/tmp/gemma_b200_models")
    os.makedirs(cache_dir, exist_ok=True)
    path = os.path.join(cache_dir, f"{shape_name}_seed{seed}.gguf")
    if not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        write_model(tmp, shape, seed)
        os.replace(tmp, path)
    return path
