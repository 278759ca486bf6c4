"""GGUF v3 reader and writer for Gemma 3 Q8_0 models.

The reader mirrors the reference's ``GGUFParser`` (src/gguf.ts:3-178): the same value
types, the same 32-byte data alignment, the same error on a bad magic, and the same
``updateConfigFromGGUF`` key set (src/gguf.ts:190-220). The writer is the inverse and
is used to produce seeded synthetic models (the build has no network, so no real
checkpoint can be fetched).

The device-side repacking of Q8_0 (the reference's ``packQ8_0ForGPU``) happens inside
the native library; this module hands it the raw 34-byte GGUF blocks.
"""
from __future__ import annotations

import math
import struct
from dataclasses import dataclass, field
from typing import Any

import numpy as np

from .config import GemmaConfig

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian (src/gguf.ts:69)
GGUF_ALIGNMENT = 32  # src/gguf.ts:90

# ggml tensor types the reference handles (src/gguf.ts:163-170, 181-186)
GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q8_0 = 8

Q8_0_BLOCK = 32
Q8_0_BLOCK_BYTES = 34  # f16 scale + 32 x int8

# GGUF metadata value types (src/gguf.ts:42-65)
T_UINT8, T_INT8, T_UINT16, T_INT16, T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_ARRAY, \
    T_UINT64, T_INT64, T_FLOAT64 = range(13)

_SCALAR_FMT = {
    T_UINT8: "<B", T_INT8: "<b", T_UINT16: "<H", T_INT16: "<h", T_UINT32: "<I",
    T_INT32: "<i", T_FLOAT32: "<f", T_BOOL: "<B", T_UINT64: "<Q", T_INT64: "<q",
    T_FLOAT64: "<d",
}
_TYPE_NAMES = {
    T_UINT8: "uint8", T_INT8: "int8", T_UINT16: "uint16", T_INT16: "int16", T_UINT32: "uint32",
    T_INT32: "int32", T_FLOAT32: "float32", T_BOOL: "bool", T_STRING: "string", T_ARRAY: "array",
    T_UINT64: "uint64", T_INT64: "int64", T_FLOAT64: "float64",
}


@dataclass
class GGUFValue:
    type: str
    value: Any


@dataclass
class GGUFTensor:
    name: str
    dims: list[int]
    type: int
    offset: int  # relative to data_offset

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= int(d)
        return n


@dataclass
class GGUFParsed:
    version: int
    tensor_count: int
    kv_count: int
    kv: dict[str, GGUFValue]
    tensors: list[GGUFTensor]
    data_offset: int
    buffer: memoryview = field(repr=False, default=None)

    def tensor(self, name: str) -> GGUFTensor | None:
        for t in self.tensors:
            if t.name == name:
                return t
        return None

    def tensor_bytes(self, t: GGUFTensor) -> memoryview:
        """Raw on-disk bytes of a tensor (``dataOffset + tensor.offset``, src/gguf.ts:161, 174)."""
        start = self.data_offset + int(t.offset)
        return self.buffer[start:start + tensor_byte_size(t)]


class GGUFError(ValueError):
    pass


class _Reader:
    def __init__(self, buf):
        self.buf = memoryview(buf).cast("B")
        self.off = 0

    def scalar(self, t: int):
        fmt = _SCALAR_FMT[t]
        (v,) = struct.unpack_from(fmt, self.buf, self.off)
        self.off += struct.calcsize(fmt)
        return v

    def u32(self) -> int:
        return self.scalar(T_UINT32)

    def u64(self) -> int:
        return self.scalar(T_UINT64)

    def string(self) -> str:
        n = self.u64()
        s = bytes(self.buf[self.off:self.off + n]).decode("utf-8", errors="replace")
        self.off += n
        return s

    def value(self, t: int) -> GGUFValue:
        """``readValue`` (src/gguf.ts:42-65)."""
        if t == T_STRING:
            return GGUFValue("string", self.string())
        if t == T_ARRAY:
            et = self.u32()
            count = self.u64()
            if et == T_STRING:
                out = []
                for _ in range(count):
                    out.append(GGUFValue("string", self.string()))
                return GGUFValue("array", out)
            if et in _SCALAR_FMT:
                fmt = _SCALAR_FMT[et]
                sz = struct.calcsize(fmt)
                vals = struct.unpack_from("<%d%s" % (count, fmt[1]), self.buf, self.off)
                self.off += sz * count
                name = _TYPE_NAMES[et]
                if et == T_BOOL:
                    return GGUFValue("array", [GGUFValue(name, v != 0) for v in vals])
                return GGUFValue("array", [GGUFValue(name, v) for v in vals])
            return GGUFValue("array", [self.value(et) for _ in range(count)])
        if t in _SCALAR_FMT:
            v = self.scalar(t)
            if t == T_BOOL:
                v = v != 0
            return GGUFValue(_TYPE_NAMES[t], v)
        return GGUFValue("unknown", None)


def parse(buf) -> GGUFParsed:
    """``GGUFParser.parse`` (src/gguf.ts:67-93)."""
    r = _Reader(buf)
    if len(r.buf) < 24:
        raise GGUFError("GGUF buffer too small")
    magic = r.u32()
    if magic != GGUF_MAGIC:
        raise GGUFError(f"Invalid GGUF magic: 0x{magic:x}")
    version = r.u32()
    tensor_count = r.u64()
    kv_count = r.u64()
    kv: dict[str, GGUFValue] = {}
    try:
        for _ in range(kv_count):
            key = r.string()
            vt = r.u32()
            kv[key] = r.value(vt)
        tensors = []
        for _ in range(tensor_count):
            name = r.string()
            n_dims = r.u32()
            dims = [r.u64() for _ in range(n_dims)]
            ttype = r.u32()
            offset = r.u64()
            tensors.append(GGUFTensor(name, dims, ttype, offset))
    except struct.error as e:  # truncated header
        raise GGUFError(f"truncated GGUF header: {e}") from None
    data_offset = int(math.ceil(r.off / GGUF_ALIGNMENT) * GGUF_ALIGNMENT)
    return GGUFParsed(version, tensor_count, kv_count, kv, tensors, data_offset, r.buf)


def tensor_byte_size(t: GGUFTensor) -> int:
    """``tensorByteSize`` (src/gguf.ts:181-187)."""
    n = t.n_elements
    if t.type == GGML_TYPE_Q8_0:
        return (n // Q8_0_BLOCK) * Q8_0_BLOCK_BYTES
    if t.type == GGML_TYPE_F32:
        return n * 4
    if t.type == GGML_TYPE_F16:
        return n * 2
    raise GGUFError(f"Unknown tensor type: {t.type}")


def update_config_from_gguf(gguf: GGUFParsed, config: GemmaConfig,
                            max_context_length: int | None = None) -> str:
    """``updateConfigFromGGUF`` (src/gguf.ts:190-220): the same 7 keys, ctx capped at 2048."""

    def get(key):
        e = gguf.kv.get(key)
        return None if e is None else int(e.value)

    hidden = get("gemma3.embedding_length")
    layers = get("gemma3.block_count")
    inter = get("gemma3.feed_forward_length")
    qh = get("gemma3.attention.head_count")
    kvh = get("gemma3.attention.head_count_kv")
    hd = get("gemma3.attention.key_length")
    ctx = get("gemma3.context_length")
    if hidden is not None:
        config.hidden_size = hidden
    if layers is not None:
        config.num_layers = layers
    if inter is not None:
        config.intermediate_size = inter
    if qh is not None:
        config.num_q_heads = qh
    if kvh is not None:
        config.num_kv_heads = kvh
    if hd is not None:
        config.head_dim = hd
    max_ctx = max_context_length if max_context_length is not None else 2048
    if ctx is not None:
        config.context_length = min(int(ctx), max_ctx)
    config.q_dim = config.num_q_heads * config.head_dim
    config.kv_dim = config.num_kv_heads * config.head_dim
    return "270M" if config.num_layers <= 18 else "1B"


# ---------------------------------------------------------------- Q8_0 helpers (numpy)

def f16_to_f32(h: np.ndarray) -> np.ndarray:
    """Bit-exact ``f16ToF32`` (src/gguf.ts:95-105) for an array of raw f16 bit patterns."""
    return np.asarray(h, dtype=np.uint16).view(np.float16).astype(np.float32)


def q8_0_split(raw: bytes | memoryview | np.ndarray, n_elements: int) -> tuple[np.ndarray, np.ndarray]:
    """Split raw Q8_0 bytes into (int8 quants [n], f16 scale bits [n/32])."""
    nb = n_elements // Q8_0_BLOCK
    a = np.frombuffer(raw, dtype=np.uint8, count=nb * Q8_0_BLOCK_BYTES).reshape(nb, Q8_0_BLOCK_BYTES)
    scales = a[:, :2].copy().view(np.uint16).reshape(nb)
    qs = a[:, 2:].copy().view(np.int8).reshape(nb * Q8_0_BLOCK)
    return qs, scales


def q8_0_join(qs: np.ndarray, scale_bits: np.ndarray) -> np.ndarray:
    """Inverse of :func:`q8_0_split`: build raw 34-byte GGUF Q8_0 blocks."""
    nb = scale_bits.size
    out = np.empty((nb, Q8_0_BLOCK_BYTES), dtype=np.uint8)
    out[:, :2] = np.ascontiguousarray(scale_bits, dtype=np.uint16).view(np.uint8).reshape(nb, 2)
    out[:, 2:] = np.ascontiguousarray(qs, dtype=np.int8).view(np.uint8).reshape(nb, Q8_0_BLOCK)
    return out.reshape(-1)


def dequantize_q8_0(raw, n_elements: int) -> np.ndarray:
    """``dequantizeQ8_0`` (src/gguf.ts:107-124): ``q * f32(d)``, exact in f32."""
    qs, sb = q8_0_split(raw, n_elements)
    d = f16_to_f32(sb)
    return (qs.reshape(-1, Q8_0_BLOCK).astype(np.float32) * d[:, None]).reshape(-1)


def pack_q8_0_for_gpu(raw, n_elements: int) -> np.ndarray:
    """``packQ8_0ForGPU`` (src/gguf.ts:126-149): 36-byte {f32 scale, 8 x u32} blocks as u32[9*nb]."""
    qs, sb = q8_0_split(raw, n_elements)
    nb = sb.size
    out = np.empty((nb, 9), dtype=np.uint32)
    out[:, 0] = f16_to_f32(sb).view(np.uint32)
    out[:, 1:] = qs.view(np.uint8).reshape(nb, 32).copy().view("<u4").reshape(nb, 8)
    return out.reshape(-1)


# ---------------------------------------------------------------- writer

def _enc_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _enc_value(vtype: int, v) -> bytes:
    if vtype == T_STRING:
        return _enc_str(v)
    if vtype == T_ARRAY:
        et, items = v
        head = struct.pack("<IQ", et, len(items))
        if et == T_STRING:
            return head + b"".join(_enc_str(s) for s in items)
        return head + struct.pack("<%d%s" % (len(items), _SCALAR_FMT[et][1]), *items)
    return struct.pack(_SCALAR_FMT[vtype], v)


def write_gguf(path: str, kv: list[tuple[str, int, Any]], tensors: list[tuple[str, list[int], int, Any]]):
    """Write a GGUF v3 file.

    ``kv``: (key, value_type, value); arrays are (T_ARRAY, (elem_type, list)).
    ``tensors``: (name, dims (ggml order: ne0 first), ggml_type, raw bytes or numpy array).
    Each tensor's data offset is aligned to 32 bytes, like llama.cpp's writer.
    """
    header = bytearray()
    header += struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(kv))
    for key, vt, v in kv:
        header += _enc_str(key) + struct.pack("<I", vt) + _enc_value(vt, v)
    offsets = []
    off = 0
    blobs = []
    for name, dims, ttype, data in tensors:
        blob = memoryview(np.ascontiguousarray(data).view(np.uint8).reshape(-1)) if isinstance(data, np.ndarray) \
            else memoryview(data)
        t = GGUFTensor(name, list(dims), ttype, 0)
        if blob.nbytes != tensor_byte_size(t):
            raise GGUFError(f"{name}: {blob.nbytes} bytes, expected {tensor_byte_size(t)}")
        off = (off + GGUF_ALIGNMENT - 1) // GGUF_ALIGNMENT * GGUF_ALIGNMENT
        offsets.append(off)
        off += blob.nbytes
        blobs.append(blob)
    for (name, dims, ttype, _), o in zip(tensors, offsets):
        header += _enc_str(name) + struct.pack("<I", len(dims)) + struct.pack("<%dQ" % len(dims), *dims)
        header += struct.pack("<IQ", ttype, o)
    pad = (-len(header)) % GGUF_ALIGNMENT
    header += b"\0" * pad
    with open(path, "wb") as f:
        f.write(header)
        pos = 0
        for blob, o in zip(blobs, offsets):
            if o > pos:
                f.write(b"\0" * (o - pos))
                pos = o
            f.write(blob)
            pos += blob.nbytes
