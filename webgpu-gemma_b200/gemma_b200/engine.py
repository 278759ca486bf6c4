"""Host-side mirror of the reference's public engine API.

The reference (svenflow/webgpu-gemma) exposes ``createGemmaEngine(options)`` returning a
``GemmaEngine`` with ``addUserMessage``, ``generate`` (async iterator of token strings),
``resetConversation``, ``dispose`` and ``config`` (src/index.ts:34-38, src/types.ts:86-97).
This module keeps the same names (snake_case), argument meaning, defaults and control flow
(src/engine.ts:957-1037); every GPU call goes to libgemma_b200.so through its C-ABI.
``generate`` is a plain generator here; ``Math.random`` is replaced by an injectable draw.
"""
from __future__ import annotations

import mmap
import os
import random as _random
from typing import Callable, Iterator

import numpy as np

from . import gguf, synth
from .config import GemmaConfig, default_config, gemma3_spec
from .conversation import build_chat_prompt
from .native import NativeEngine
from .tokenizer import Tokenizer

STOP_IDS = (0, 1, 106)  # engine.ts:1004, 1014


def _resolve_model(model: str) -> str:
    if model.startswith("synthetic:"):
        return synth.cached_model(model.split(":", 1)[1])
    if os.path.exists(model):
        return model
    raise ValueError(f"model '{model}': pass a local .gguf path or 'synthetic:<270m|1b|tiny|small|mid>' "
                     "(the reference's Hugging Face URLs need a network)")


class GemmaEngine:
    """``GemmaEngineImpl`` (src/engine.ts:30-1078) with the GPU parts in libgemma_b200.so."""

    def __init__(self, model: str = "synthetic:1b", on_progress: Callable[[dict], None] | None = None,
                 context_length: int | None = None, device: int = 0,
                 random: Callable[[], float] | None = None, kv_dtype: str = "f32", spec: bool = False):
        self.config: GemmaConfig = default_config()
        if context_length:
            self.config.context_length = context_length
        self._on_progress = on_progress
        self._random = random or _random.random
        self.conversation_history: list[dict] = []
        self.kv_position = 0
        path = _resolve_model(model)
        self._progress(0, 1, "Reading header...")
        with open(path, "rb") as f:
            self._mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        parsed = gguf.parse(memoryview(self._mm))
        gguf.update_config_from_gguf(parsed, self.config, context_length)
        # The reference keeps vocab_size at 262,144, the size of every Gemma 3 GGUF; taking it from
        # the embedding's row count gives the same value for those and also loads other sizes.
        embd = next((t for t in parsed.tensors if t.name == "token_embd.weight"), None)
        if embd is not None and len(embd.dims) == 2:
            self.config.vocab_size = int(embd.dims[1])
        # options beyond the reference's: KV element type, Gemma 3's sliding window + local theta
        self.config.kv_dtype = kv_dtype
        if spec:
            gemma3_spec(self.config)
        self.tokenizer = Tokenizer.from_gguf(parsed)
        self._native = NativeEngine(self.config, device=device)
        total = sum(gguf.tensor_byte_size(t) for t in parsed.tensors)
        loaded = 0
        for t in parsed.tensors:  # uploadWeightsStreaming (engine.ts:290-400)
            raw = np.frombuffer(parsed.tensor_bytes(t), dtype=np.uint8)
            self._native.upload_tensor(t.name, t.type, raw, t.dims)
            loaded += gguf.tensor_byte_size(t)
            self._progress(loaded, total, "Streaming weights to GPU...")
        del raw, parsed
        self._native.finalize()

    def _progress(self, loaded, total, status):
        if self._on_progress:
            self._on_progress({"loaded": loaded, "total": total, "status": status})

    # ----------------------------------------------------------------- public API

    def add_user_message(self, text: str) -> None:
        self.conversation_history.append({"role": "user", "text": text})

    def generate(self, temperature: float = 0.7, top_p: float = 0.9, rep_penalty: float = 1.2,
                 max_tokens: int = 32768, tools_json: str = "[]", signal=None) -> Iterator[str]:
        """``generate`` (engine.ts:957-1031): prefill the new turn, then sample token by token."""
        if self._native is None:
            raise RuntimeError("engine disposed")
        tok = self.tokenizer
        if self.kv_position == 0:
            new_tokens = tok.encode(build_chat_prompt(self.conversation_history, tools_json))
        else:
            last = self.conversation_history[-1]
            suffix = f"<end_of_turn>\n<start_of_turn>user\n{last['text']}<end_of_turn>\n<start_of_turn>model\n"
            new_tokens = tok.encode(suffix)[1:]
        if self.kv_position + len(new_tokens) >= self.config.context_length - 10:  # engine.ts:977-985
            last = self.conversation_history[-1]
            self.conversation_history = [{"role": "user", "text": last["text"]}]
            new_tokens = tok.encode(build_chat_prompt(self.conversation_history, tools_json))
            self._native.reset_kv(0)
            self.kv_position = 0
        sample = dict(temperature=temperature, top_p=top_p, rep=rep_penalty)
        self._native.seen_reset(0)  # allTokens = [...newTokens] (engine.ts:989)
        self._native.prefill(new_tokens, self.kv_position)
        self.kv_position += len(new_tokens)
        nxt = self._native.sample_last(0, uniform=self._random(), **sample)
        end_func = tok.func_tokens.get("<end_function_call>")
        generated = [nxt]
        gen_kv_writes = 0
        yield tok.decode_token(nxt)
        for _ in range(1, max_tokens):
            if nxt in STOP_IDS or (end_func is not None and nxt == end_func):
                break
            if signal is not None and (getattr(signal, "aborted", False) or
                                       (hasattr(signal, "is_set") and signal.is_set())):
                break
            pos = self.kv_position + gen_kv_writes
            if pos >= self.config.context_length - 1:
                break
            nxt = self._native.step(nxt, pos, 0, uniform=self._random(), **sample)
            gen_kv_writes += 1
            if nxt in STOP_IDS:
                break
            if end_func is not None and nxt == end_func:
                generated.append(nxt)
                break
            generated.append(nxt)
            yield tok.decode_token(nxt)
        self.conversation_history.append({"role": "model", "text": tok.decode_tokens(generated)})
        self.kv_position += gen_kv_writes

    def reset_conversation(self) -> None:
        self.conversation_history = []
        self.kv_position = 0
        self._native.reset_kv(0)

    def dispose(self) -> None:
        if self._native is not None:
            self._native.close()
            self._native = None
        if getattr(self, "_mm", None) is not None:
            self._mm.close()
            self._mm = None

    @property
    def native(self) -> NativeEngine:
        return self._native


def create_gemma_engine(model: str = "synthetic:1b", on_progress=None, context_length: int | None = None,
                        device: int = 0, random=None, kv_dtype: str = "f32", spec: bool = False) -> GemmaEngine:
    """``createGemmaEngine`` (src/index.ts:34-38). ``kv_dtype`` ("f32" as the reference, or
    "bf16") and ``spec`` (Gemma 3's 512-position window and local theta 1e4, off as in the
    reference) are options the reference does not have."""
    return GemmaEngine(model=model, on_progress=on_progress, context_length=context_length, device=device,
                       random=random, kv_dtype=kv_dtype, spec=spec)


def philox_uniforms(seed: int, stream: int, n: int) -> np.ndarray:
    """Per-sequence injected draws in [0, 1): Philox4x32-10 keyed by (seed, stream)."""
    g = np.random.Generator(np.random.Philox(key=[seed & 0xFFFFFFFFFFFFFFFF, stream]))
    return g.random(n)
