"""Model configuration for the Gemma 3 token loop.

Mirrors the reference's ``GemmaConfig`` (src/types.ts:1-44): the same fields, the
same defaults (Gemma 3 270M), the same SWA-period rule for picking the RoPE theta.
The defaults that the reference never reads from the GGUF (vocab 262144, eps 1e-6,
theta 1e6 on *every* layer) are kept exactly, because parity follows the reference,
not the Gemma 3 paper.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, asdict


@dataclass
class GemmaConfig:
    """Field-for-field restatement of ``GemmaConfig`` (src/types.ts:2-17)."""

    hidden_size: int = 640
    q_dim: int = 1024
    kv_dim: int = 256
    num_q_heads: int = 4
    num_kv_heads: int = 1
    head_dim: int = 256
    intermediate_size: int = 2048
    vocab_size: int = 262144
    num_layers: int = 18
    context_length: int = 2048
    rms_norm_eps: float = 1e-6
    rope_theta_global: float = 1000000.0
    # The reference sets the sliding-window layers' theta to 1e6 as well
    # (src/types.ts:32-33); a spec-faithful 10k is opt-in, not the default.
    rope_theta_swa: float = 1000000.0
    swa_period: int = 6
    # Not in the reference (which attends the whole prefix on every layer): > 0 limits the
    # sliding-window layers to the last `sliding_window` positions, as Gemma 3 is specified.
    sliding_window: int = 0
    # KV cache element type: "f32" as the reference (engine.ts:440-447), or "bf16" (rows
    # rounded to nearest even when stored; GG_FLAG_KV_BF16 in the C-ABI).
    kv_dtype: str = "f32"

    def as_dict(self) -> dict:
        return asdict(self)


def default_config() -> GemmaConfig:
    """``defaultConfig()`` (src/types.ts:19-36)."""
    return GemmaConfig()


def gemma3_spec(cfg: GemmaConfig, window: int = 512, theta_local: float = 10000.0) -> GemmaConfig:
    """The configuration as Gemma 3 is specified rather than as the reference runs it: sliding
    window of `window` positions and RoPE base `theta_local` on the local layers."""
    cfg.sliding_window = window
    cfg.rope_theta_swa = theta_local
    return cfg


def is_swa_layer(il: int, config: GemmaConfig) -> bool:
    """``isSwaLayer`` (src/types.ts:38-40): picks the RoPE theta, and the window when
    ``sliding_window`` > 0."""
    return (il % config.swa_period) < (config.swa_period - 1)


def get_rope_theta(il: int, config: GemmaConfig) -> float:
    """``getRopeTheta`` (src/types.ts:42-44)."""
    return config.rope_theta_swa if is_swa_layer(il, config) else config.rope_theta_global


class CConfig(ctypes.Structure):
    """Layout of ``gg_config`` in include/gemma_b200.h (the C-ABI view of GemmaConfig)."""

    _fields_ = [
        ("hidden_size", ctypes.c_int32),
        ("q_dim", ctypes.c_int32),
        ("kv_dim", ctypes.c_int32),
        ("num_q_heads", ctypes.c_int32),
        ("num_kv_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("intermediate_size", ctypes.c_int32),
        ("vocab_size", ctypes.c_int32),
        ("num_layers", ctypes.c_int32),
        ("context_length", ctypes.c_int32),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta_global", ctypes.c_float),
        ("rope_theta_swa", ctypes.c_float),
        ("swa_period", ctypes.c_int32),
        ("max_seqs", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("sliding_window", ctypes.c_int32),
    ]


GG_FLAG_KV_BF16 = 2  # include/gemma_b200.h


def kv_flags(cfg) -> int:
    """gg_config.flags bits that follow from the configuration itself (the KV element type)."""
    kv = getattr(cfg, "kv_dtype", "f32")
    if kv not in ("f32", "bf16"):
        raise ValueError(f"kv_dtype must be 'f32' or 'bf16', not {kv!r}")
    return GG_FLAG_KV_BF16 if kv == "bf16" else 0


def to_cconfig(cfg: GemmaConfig, max_seqs: int = 1, flags: int = 0) -> CConfig:
    c = CConfig()
    for name, _ in CConfig._fields_:
        if name == "max_seqs":
            c.max_seqs = max_seqs
        elif name == "flags":
            c.flags = flags | kv_flags(cfg)
        else:
            setattr(c, name, getattr(cfg, name))
    return c
