"""ctypes front end of the C oracle (gemma_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` as the
checker, and by bench.py for its CPU-baseline leg. The product (libgemma_b200.so and
the gemma_b200 package) never imports it.

PARITY UNPINNED: see the header of gemma_oracle.c.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

OR_FLAG_KV_BF16 = 2  # or_config.flags bit: bf16 KV cache (GG_FLAG_KV_BF16)
HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "gemma_oracle.c")
LIB = os.path.join(HERE, "liboracle.so")
# Portable x86-64-v3 (AVX2) code so the library built here also runs on the GPU box's host.
CFLAGS = ["-O3", "-march=x86-64-v3", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
          "-fPIC", "-shared", "-fvisibility=hidden", "-std=c11"]


def build(force: bool = False) -> str:
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        tmp = LIB + f".tmp{os.getpid()}"
        subprocess.check_call(["gcc", *CFLAGS, SRC, "-o", tmp, "-lm"])
        os.replace(tmp, LIB)
    return LIB


class OrConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "hidden_size", "q_dim", "kv_dim", "num_q_heads", "num_kv_heads", "head_dim",
        "intermediate_size", "vocab_size", "num_layers", "context_length")] + [
        ("rms_norm_eps", ctypes.c_float), ("rope_theta_global", ctypes.c_float),
        ("rope_theta_swa", ctypes.c_float), ("swa_period", ctypes.c_int32),
        ("max_seqs", ctypes.c_int32), ("flags", ctypes.c_int32), ("sliding_window", ctypes.c_int32)]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        L = ctypes.CDLL(build())
        P, I, F, D = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double
        i64 = ctypes.c_int64
        sig = {
            "or_f16_to_f32": (F, [ctypes.c_uint16]),
            "or_pack_q8_0": (None, [P, i64, P]),
            "or_embedding": (None, [P, I, I, P]),
            "or_rmsnorm": (None, [P, P, P, I, F]),
            "or_fused_norm_add": (None, [P, P, P, P, I, F]),
            "or_linear_q8": (None, [P, P, P, I, I]),
            "or_gelu_mul": (None, [P, P, P, I]),
            "or_fused_norm_rope": (None, [P, P, I, I, F, I, F]),
            "or_attention": (None, [P, P, P, I, I, I, I, F, P, P]),
            "or_topk256": (None, [P, I, P, P]),
            "or_argmax": (ctypes.c_uint32, [P, I]),
            "or_sample": (ctypes.c_int32, [P, P, D, D, D, P, I, D]),
            "or_create": (P, [ctypes.POINTER(OrConfig)]),
            "or_free": (None, [P]),
            "or_set_tensor": (I, [P, ctypes.c_char_p, I, P, i64]),
            "or_reset_kv": (None, [P, I]),
            "or_forward": (I, [P, I, I, I, P]),
            "or_lm_head": (I, [P, I, P]),
            "or_kv_row": (P, [P, I, I, I, I]),
            "or_set_threads": (None, [I]),
            "or_get_threads": (I, []),
            "or_bf16_round": (None, [P, P, i64]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# ----------------------------------------------------------------- op-level wrappers

def f16_to_f32(bits: int) -> float:
    return lib().or_f16_to_f32(bits)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """f32 values rounded to bf16 (nearest even) and widened back: the optional bf16 KV store."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty_like(x)
    lib().or_bf16_round(_p(x), _p(y), x.size)
    return y


def pack_q8_0(raw: np.ndarray) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    nb = raw.size // 34
    out = np.empty(nb * 9, dtype=np.uint32)
    lib().or_pack_q8_0(_p(raw), nb, _p(out))
    return out


def linear_q8(x: np.ndarray, packed: np.ndarray, m: int, n: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(m, dtype=np.float32)
    lib().or_linear_q8(_p(x), _p(np.ascontiguousarray(packed)), _p(y), m, n)
    return y


def rmsnorm(x, w, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    lib().or_rmsnorm(_p(x), _p(w), _p(out), x.size, eps)
    return out


def fused_norm_add(x, w, res, eps=1e-6):
    x = np.ascontiguousarray(x, np.float32); w = np.ascontiguousarray(w, np.float32)
    res = np.ascontiguousarray(res, np.float32)
    out = np.empty_like(x)
    lib().or_fused_norm_add(_p(x), _p(w), _p(res), _p(out), x.size, eps)
    return out


def gelu_mul(g, u):
    g = np.ascontiguousarray(g, np.float32); u = np.ascontiguousarray(u, np.float32)
    out = np.empty_like(g)
    lib().or_gelu_mul(_p(g), _p(u), _p(out), g.size)
    return out


def fused_norm_rope(data, w, nheads, hd, eps, pos, theta):
    d = np.array(data, dtype=np.float32, copy=True)
    w = np.ascontiguousarray(w, np.float32)
    lib().or_fused_norm_rope(_p(d), _p(w), nheads, hd, eps, pos, theta)
    return d


def attention(q, kc, vc, nqh, nkvh, hd, seq_len, scale):
    q = np.ascontiguousarray(q, np.float32)
    kc = np.ascontiguousarray(kc, np.float32); vc = np.ascontiguousarray(vc, np.float32)
    scores = np.empty(nqh * seq_len, np.float32)
    out = np.empty(nqh * hd, np.float32)
    lib().or_attention(_p(q), _p(kc), _p(vc), nqh, nkvh, hd, seq_len, scale, _p(scores), _p(out))
    return out


def embedding(packed, hidden, token):
    out = np.empty(hidden, np.float32)
    lib().or_embedding(_p(np.ascontiguousarray(packed)), hidden, token, _p(out))
    return out


def topk256(logits):
    logits = np.ascontiguousarray(logits, np.float32)
    v = np.empty(256, np.float32); i = np.empty(256, np.uint32)
    lib().or_topk256(_p(logits), logits.size, _p(v), _p(i))
    return v, i


def argmax(logits) -> int:
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().or_argmax(_p(logits), logits.size))


def sample(vals, ids, temperature, top_p, rep, seen_ids, u, vocab) -> int:
    seen = np.zeros((vocab + 7) // 8, np.uint8)
    n = 0
    for t in seen_ids:
        seen[t >> 3] |= np.uint8(1 << (t & 7)); n += 1
    vals = np.ascontiguousarray(vals, np.float32); ids = np.ascontiguousarray(ids, np.uint32)
    return int(lib().or_sample(_p(vals), _p(ids), temperature, top_p, rep, _p(seen), n, u))


# ----------------------------------------------------------------- model

class OracleModel:
    """The reference's whole token loop on the CPU (src/engine.ts:735-1031)."""

    def __init__(self, cfg, max_seqs: int = 1):
        c = OrConfig()
        for name, _ in OrConfig._fields_:
            if name == "max_seqs":
                c.max_seqs = max_seqs
            elif name == "flags":
                c.flags = OR_FLAG_KV_BF16 if getattr(cfg, "kv_dtype", "f32") == "bf16" else 0
            else:
                setattr(c, name, getattr(cfg, name, 0))
        self.cfg = cfg
        self.max_seqs = max_seqs
        self._h = lib().or_create(ctypes.byref(c))

    def close(self):
        if self._h:
            lib().or_free(self._h)
            self._h = None

    __del__ = close

    def set_tensor(self, name: str, ggml_type: int, raw: np.ndarray, n_elems: int):
        raw = np.ascontiguousarray(raw).view(np.uint8)
        if lib().or_set_tensor(self._h, name.encode(), ggml_type, _p(raw), n_elems) != 0:
            raise ValueError(f"oracle rejected tensor {name}")

    @classmethod
    def from_tensors(cls, cfg, tensors: dict, max_seqs: int = 1):
        m = cls(cfg, max_seqs)
        for name, (dims, t, raw) in tensors.items():
            m.set_tensor(name, t, raw, int(np.prod(dims)))
        return m

    def reset_kv(self, seq: int = 0):
        lib().or_reset_kv(self._h, seq)

    def forward(self, token: int, pos: int, seq: int = 0) -> np.ndarray:
        out = np.empty(self.cfg.hidden_size, np.float32)
        if lib().or_forward(self._h, seq, int(token), int(pos), _p(out)) != 0:
            raise ValueError("oracle forward: bad seq/pos/token")
        return out

    def logits(self, seq: int = 0) -> np.ndarray:
        out = np.empty(self.cfg.vocab_size, np.float32)
        lib().or_lm_head(self._h, seq, _p(out))
        return out

    def kv_row(self, layer: int, pos: int, which: int, seq: int = 0) -> np.ndarray:
        p = lib().or_kv_row(self._h, seq, layer, pos, which)
        return np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), (self.cfg.kv_dim,)).copy()

    def greedy(self, prompt, n_new: int, seq: int = 0, start_pos: int = 0, return_logits: bool = False):
        """Serial prefill then greedy decode with the argmax fast path (engine.ts:823, 923-1025)."""
        for i, t in enumerate(prompt):
            self.forward(int(t), start_pos + i, seq)
        pos = start_pos + len(prompt)
        lg = self.logits(seq)
        toks, all_logits = [argmax(lg)], [lg] if return_logits else None
        for _ in range(n_new - 1):
            self.forward(toks[-1], pos, seq)
            pos += 1
            lg = self.logits(seq)
            if return_logits:
                all_logits.append(lg)
            toks.append(argmax(lg))
        return (toks, all_logits) if return_logits else toks


def use_all_host_cores() -> int:
    """Run the parallel loops on every core this process may use; returns the thread count."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    lib().or_set_threads(n)
    return int(lib().or_get_threads())
