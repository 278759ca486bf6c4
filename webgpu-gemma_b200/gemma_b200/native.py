"""ctypes binding of libgemma_b200.so (declarations in include/gemma_b200.h).

There is no fallback: if the library is missing or fails to load, importing the engine
raises. The product path is the CUDA library only.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from .config import CConfig, GemmaConfig, to_cconfig

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libgemma_b200.so")

GG_OK, GG_E_ARG, GG_E_CUDA, GG_E_STATE, GG_E_DEVICE, GG_E_NOMEM = 0, -1, -2, -3, -4, -5

# Bytes a gg_step call moves: host->device, the launch's parameters (a whole GGState of 128 B
# carrying the token, position and sampling options, a flag and two pointers); device->host, the
# kernel's writes of GGState's device-owned tail into the mapped pinned state (epoch, ticket,
# error bits, sampled token, seen count, parity: 24 B).
STATE_H2D_BYTES = 128 + 4 + 8 + 8
STATE_D2H_BYTES = 24

# Every symbol the header declares, with (restype, argtypes).
_P, _I, _D = ctypes.c_void_p, ctypes.c_int, ctypes.c_double
_I32P = ctypes.POINTER(ctypes.c_int32)
SIGNATURES = {
    "gg_create": (_I, [ctypes.POINTER(CConfig), _I, ctypes.POINTER(_P)]),
    "gg_upload_tensor": (_I, [_P, ctypes.c_char_p, _I, _P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_uint64), _I]),
    "gg_finalize": (_I, [_P]),
    "gg_prefill": (_I, [_P, _I, _I32P, _I, _I]),
    "gg_sample_last": (_I, [_P, _I, _P, _D, _I32P]),
    "gg_step": (_I, [_P, _I, ctypes.c_int32, _I, _P, _D, _I32P]),
    "gg_decode": (_I, [_P, _I, ctypes.c_int32, _I, _I, _P, _P, _I32P]),
    "gg_get_logits": (_I, [_P, _P]),
    "gg_get_hidden": (_I, [_P, _P]),
    "gg_get_kv": (_I, [_P, _I, _I, _I, _I, _P]),
    "gg_debug_read": (_I, [_P, _I, _P, _I]),
    "gg_dequant_row": (_I, [_P, _I, _I, _I, _I, _P, _I]),
    "gg_seen_reset": (_I, [_P, _I]),
    "gg_seen_add": (_I, [_P, _I, _I32P, _I]),
    "gg_reset_kv": (_I, [_P, _I]),
    "gg_grid": (_I, [_P, ctypes.POINTER(ctypes.c_int)]),
    "gg_set_trace": (_I, [_P, _I]),
    "gg_read_trace": (_I, [_P, _P, _I]),
    "gg_linear": (_I, [_P, _I, _I, _P, _I, _P]),
    "gg_decode_batch": (_I, [_P, _I, _P, _P, _P, _I, _P, _P, _P]),
    "gg_selftest_wait": (_I, [_P, ctypes.c_uint64]),
    "gg_set_gemm_kernel": (_I, [_I]),
    "gg_sample_logits_noalloc": (_I, [_P, _I, _P, _P, _D, _P, _P]),
    "gg_set_timeout": (_I, [_P, ctypes.c_uint64]),
    "gg_last_device_ms": (_I, [_P, ctypes.POINTER(ctypes.c_float)]),
    "gg_destroy": (_I, [_P]),
    "gg_last_error": (ctypes.c_char_p, [_P]),
    "gg_version": (ctypes.c_char_p, []),
    "gg_tokenizer_create": (_I, [_P, _P, _I, ctypes.POINTER(_P)]),
    "gg_tokenizer_encode": (_I, [_P, ctypes.c_char_p, ctypes.c_size_t, _P, _I, ctypes.POINTER(ctypes.c_int)]),
    "gg_tokenizer_decode": (_I, [_P, _P, _I, _P, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "gg_tokenizer_token_id": (_I, [_P, ctypes.c_char_p, _I32P]),
    "gg_tokenizer_destroy": (None, [_P]),
}


GG_FLAG_SERIAL_PREFILL = 1  # prefill one token per launch (the reference's order)


class GGSample(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_double), ("top_p", ctypes.c_double), ("rep_penalty", ctypes.c_double)]


class GemmaB200Error(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None


def load(path: str | None = None) -> ctypes.CDLL:
    """Load the library (building it first when the source is newer and nvcc is present)."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise OSError(f"libgemma_b200.so not found at {path}; run webgpu-gemma_b200/build.py")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


GEMM_DEQUANT, GEMM_SCALED = 0, 1


def set_gemm_kernel(kind: int) -> int:
    """Process-wide kernel family of the tensor-core products (gg_set_gemm_kernel); returns the
    previous one. GEMM_DEQUANT (default) multiplies each Q8_0 block's scale into bf16 hi + lo
    operands, GEMM_SCALED applies it after the block's MMAs."""
    rc = load().gg_set_gemm_kernel(int(kind))
    if rc < 0:
        raise ValueError(f"unknown GEMM kernel family {kind}")
    return rc


def _i32p(a: np.ndarray):
    return a.ctypes.data_as(_I32P)


class NativeEngine:
    """Thin object wrapper over one gg_engine handle (one GPU, one stream)."""

    def __init__(self, cfg: GemmaConfig, device: int = 0, max_seqs: int = 1, flags: int = 0):
        self.lib = load()
        self.cfg = cfg
        self.max_seqs = max_seqs
        h = ctypes.c_void_p()
        cc = to_cconfig(cfg, max_seqs=max_seqs, flags=flags)
        rc = self.lib.gg_create(ctypes.byref(cc), device, ctypes.byref(h))
        if rc != GG_OK:
            raise GemmaB200Error(rc, self.lib.gg_last_error(None).decode())
        self.h = h

    def _check(self, rc: int):
        if rc != GG_OK:
            raise GemmaB200Error(rc, self.lib.gg_last_error(self.h).decode())

    def upload_tensor(self, name: str, ggml_type: int, raw, dims):
        buf = np.ascontiguousarray(np.frombuffer(raw, dtype=np.uint8) if not isinstance(raw, np.ndarray) else raw)
        d = (ctypes.c_uint64 * len(dims))(*[int(x) for x in dims])
        self._check(self.lib.gg_upload_tensor(self.h, name.encode(), ggml_type, buf.ctypes.data_as(_P),
                                              buf.nbytes, d, len(dims)))

    def finalize(self):
        self._check(self.lib.gg_finalize(self.h))

    def prefill(self, ids, start_pos: int, seq: int = 0):
        a = np.ascontiguousarray(ids, dtype=np.int32)
        self._check(self.lib.gg_prefill(self.h, seq, _i32p(a), a.size, start_pos))

    @staticmethod
    def _sample(temperature: float, top_p: float, rep: float) -> GGSample:
        return GGSample(float(temperature), float(top_p), float(rep))

    def sample_last(self, seq: int = 0, temperature=0.0, top_p=0.9, rep=1.0, uniform=0.0) -> int:
        out = ctypes.c_int32()
        s = self._sample(temperature, top_p, rep)
        self._check(self.lib.gg_sample_last(self.h, seq, ctypes.byref(s), float(uniform), ctypes.byref(out)))
        return out.value

    def step(self, token: int, pos: int, seq: int = 0, temperature=0.0, top_p=0.9, rep=1.0, uniform=0.0) -> int:
        out = ctypes.c_int32()
        s = self._sample(temperature, top_p, rep)
        self._check(self.lib.gg_step(self.h, seq, int(token), int(pos), ctypes.byref(s), float(uniform),
                                     ctypes.byref(out)))
        return out.value

    def decode(self, token: int, pos: int, n: int, seq: int = 0, temperature=0.0, top_p=0.9, rep=1.0,
               uniforms=None) -> np.ndarray:
        out = np.empty(n, np.int32)
        s = self._sample(temperature, top_p, rep)
        up = None
        if uniforms is not None:
            u = np.ascontiguousarray(uniforms, dtype=np.float64)
            up = u.ctypes.data_as(_P)
        self._check(self.lib.gg_decode(self.h, seq, int(token), int(pos), int(n), ctypes.byref(s), up, _i32p(out)))
        return out

    def logits(self) -> np.ndarray:
        out = np.empty(self.cfg.vocab_size, np.float32)
        self._check(self.lib.gg_get_logits(self.h, out.ctypes.data_as(_P)))
        return out

    def hidden(self) -> np.ndarray:
        out = np.empty(self.cfg.hidden_size, np.float32)
        self._check(self.lib.gg_get_hidden(self.h, out.ctypes.data_as(_P)))
        return out

    def kv_row(self, layer: int, pos: int, which: int, seq: int = 0) -> np.ndarray:
        out = np.empty(self.cfg.kv_dim, np.float32)
        self._check(self.lib.gg_get_kv(self.h, seq, layer, pos, which, out.ctypes.data_as(_P)))
        return out

    DEBUG_BUFFERS = ("qkv", "att", "proj", "act", "down", "hidden", "residual", "normed", "logits")

    def debug_read(self, which: str) -> np.ndarray:
        c = self.cfg
        n = {"qkv": c.q_dim + 2 * c.kv_dim, "att": c.q_dim, "proj": c.hidden_size, "act": c.intermediate_size,
             "down": c.hidden_size, "hidden": c.hidden_size, "residual": c.hidden_size, "normed": c.hidden_size,
             "logits": c.vocab_size}[which]
        out = np.empty(n, np.float32)
        self._check(self.lib.gg_debug_read(self.h, self.DEBUG_BUFFERS.index(which), out.ctypes.data_as(_P), n))
        return out

    def dequant_row(self, which: int, layer: int, row: int, copy: int = 0) -> np.ndarray:
        """Row `row` of matrix `which` (0 qkv, 1 o, 2 gate/up interleaved, 3 down, 4 embedding)
        dequantised from the device's copy (0 row format, 1 the GEMM's tiled copy)."""
        c = self.cfg
        k = {0: c.hidden_size, 1: c.q_dim, 2: c.hidden_size, 3: c.intermediate_size, 4: c.hidden_size}[which]
        out = np.empty(k, np.float32)
        self._check(self.lib.gg_dequant_row(self.h, which, layer, row, copy, out.ctypes.data_as(_P), k))
        return out

    def seen_reset(self, seq: int = 0):
        self._check(self.lib.gg_seen_reset(self.h, seq))

    def seen_add(self, ids, seq: int = 0):
        a = np.ascontiguousarray(ids, dtype=np.int32)
        self._check(self.lib.gg_seen_add(self.h, seq, _i32p(a), a.size))

    def reset_kv(self, seq: int = 0):
        self._check(self.lib.gg_reset_kv(self.h, seq))

    def set_trace(self, on: bool):
        self._check(self.lib.gg_set_trace(self.h, 1 if on else 0))

    def grid(self) -> int:
        """CTAs of the persistent decode kernel (one per SM)."""
        v = ctypes.c_int()
        self._check(self.lib.gg_grid(self.h, ctypes.byref(v)))
        return v.value

    def read_trace(self, n: int) -> np.ndarray:
        out = np.zeros(n, np.uint64)
        self._check(self.lib.gg_read_trace(self.h, out.ctypes.data_as(_P), n))
        return out

    def decode_batch(self, seqs, tokens, pos, steps: int, samples, uniforms) -> np.ndarray:
        """Batched decode: row i = KV slot seqs[i] fed tokens[i] at pos[i]; `samples` is one
        (temperature, top_p, rep) per row; uniforms [steps][n]. Returns tokens [steps][n]."""
        seqs = np.ascontiguousarray(seqs, np.int32)
        tokens = np.ascontiguousarray(tokens, np.int32)
        pos = np.ascontiguousarray(pos, np.int32)
        n = seqs.size
        sp = (GGSample * n)(*[GGSample(float(t), float(p), float(r)) for (t, p, r) in samples])
        u = np.ascontiguousarray(np.asarray(uniforms, np.float64).reshape(steps, n))
        out = np.empty((steps, n), np.int32)
        self._check(self.lib.gg_decode_batch(self.h, n, seqs.ctypes.data_as(_P), tokens.ctypes.data_as(_P),
                                             pos.ctypes.data_as(_P), int(steps), ctypes.cast(sp, _P),
                                             u.ctypes.data_as(_P), out.ctypes.data_as(_P)))
        return out

    def linear(self, which: int, layer: int, x: np.ndarray) -> np.ndarray:
        """y = x @ W.T for matrix `which` (0 qkv, 1 o, 2 gate/up interleaved, 3 down, 4 LM head)."""
        x = np.ascontiguousarray(x, dtype=np.float32)
        if x.ndim == 1:
            x = x[None, :]
        rows = {0: self.cfg.q_dim + 2 * self.cfg.kv_dim, 1: self.cfg.hidden_size, 2: 2 * self.cfg.intermediate_size,
                3: self.cfg.hidden_size, 4: self.cfg.vocab_size}[which]
        y = np.empty((x.shape[0], rows), np.float32)
        self._check(self.lib.gg_linear(self.h, which, layer, x.ctypes.data_as(_P), x.shape[0], y.ctypes.data_as(_P)))
        return y

    def selftest_wait(self, timeout_ns: int) -> int:
        """Runs the bounded-wait self-test; returns the status code (GG_E_DEVICE expected)."""
        return self.lib.gg_selftest_wait(self.h, int(timeout_ns))

    def last_error(self) -> str:
        return self.lib.gg_last_error(self.h).decode()

    def set_timeout(self, ns: int):
        self._check(self.lib.gg_set_timeout(self.h, int(ns)))

    def last_device_ms(self) -> float:
        v = ctypes.c_float()
        self._check(self.lib.gg_last_device_ms(self.h, ctypes.byref(v)))
        return v.value

    def close(self):
        if getattr(self, "h", None):
            self.lib.gg_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def engine_from_tensors(cfg: GemmaConfig, tensors: dict, device: int = 0, max_seqs: int = 1,
                        flags: int = 0) -> NativeEngine:
    """Create + upload every (name -> (dims, type, raw bytes)) tensor + finalize."""
    eng = NativeEngine(cfg, device=device, max_seqs=max_seqs, flags=flags)
    for name, (dims, t, raw) in tensors.items():
        eng.upload_tensor(name, t, raw, dims)
    eng.finalize()
    return eng
