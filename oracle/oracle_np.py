"""Numpy restatement of the reference's shader math, for small shapes.

TEST INFRASTRUCTURE ONLY: a second, independent restatement used to cross-check the C
oracle (gemma_oracle.c). Nothing in the product imports it.

Each function follows the same reference lines as its C twin (svenflow/webgpu-gemma
src/shaders.ts, src/engine.ts); every float32 operation is one numpy float32 operation
in the shader's order, so results agree with the C oracle bit for bit except in the
transcendental functions, which are evaluated in f64 and rounded to f32 (a correctly rounded
libm; glibc's float functions can differ by an ulp). PARITY UNPINNED, as for the C oracle: the reference has no tests or fixtures.
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    """src/gguf.ts:95-105 restated with the formula (not numpy's float16 cast)."""
    h = np.asarray(bits, dtype=np.uint32)
    sign = np.where((h >> 15) & 1, -1.0, 1.0)
    ex = ((h >> 10) & 0x1F).astype(np.int64)
    mant = (h & 0x3FF).astype(np.float64)
    sub = sign * (2.0 ** -14) * (mant / 1024.0)
    nrm = sign * np.power(2.0, (ex - 15).astype(np.float64)) * (1.0 + mant / 1024.0)
    inf_nan = np.where(mant == 0, sign * np.inf, np.nan)
    v = np.where(ex == 0, sub, np.where(ex == 31, inf_nan, nrm))
    return v.astype(np.float32)


def bf16_round(x: np.ndarray) -> np.ndarray:
    """The optional bf16 KV store (not in the reference): each f32 value goes to the nearer of
    the two bf16 values around it, ties to the one with an even last mantissa bit, and is
    widened back to f32. Stated by that definition (distances in f64), independently of the C
    oracle's integer rounding; finite inputs only."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    lo_u = u & np.uint32(0xFFFF0000)                # truncation: toward zero
    hi_u = lo_u + np.uint32(0x10000)                # next bf16 value away from zero
    lo = lo_u.view(np.float32).astype(np.float64)
    hi = hi_u.view(np.float32).astype(np.float64)
    xd = x.astype(np.float64)
    dlo, dhi = np.abs(xd - lo), np.abs(hi - xd)
    lo_even = ((lo_u >> np.uint32(16)) & np.uint32(1)) == 0
    pick_lo = (dlo < dhi) | ((dlo == dhi) & lo_even)
    return np.where(pick_lo, lo_u, hi_u).astype(np.uint32).view(np.float32)


def unpack(packed: np.ndarray, m: int, n: int) -> tuple[np.ndarray, np.ndarray]:
    """packQ8_0ForGPU words -> (q int8 [m, n/32, 32], scale f32 [m, n/32])."""
    w = np.asarray(packed, dtype=np.uint32).reshape(m, n // 32, 9)
    scale = w[:, :, 0].copy().view(np.float32)
    q = w[:, :, 1:].copy().view(np.int8).reshape(m, n // 32, 32)
    return q, scale


def sumsq_tree(x: np.ndarray) -> f32:
    """256 strided partials then the 128->1 tree (src/shaders.ts:37-49)."""
    n = x.shape[0]
    s = np.zeros(256, dtype=f32)
    for base in range(0, n, 256):
        seg = x[base:base + 256]
        s[:seg.shape[0]] = s[:seg.shape[0]] + seg * seg
    stride = 128
    while stride > 0:
        s[:stride] = s[:stride] + s[stride:2 * stride]
        stride >>= 1
    return s[0]


def rmsnorm(x, w, eps):
    rms = np.sqrt(f32(sumsq_tree(x) / f32(x.shape[0]) + f32(eps)))
    return (x * w) / rms


def fused_norm_add(x, w, res, eps):
    rms = np.sqrt(f32(sumsq_tree(x) / f32(x.shape[0]) + f32(eps)))
    return res + (x * w) / rms


def linear_q8(x: np.ndarray, packed: np.ndarray, m: int, n: int) -> np.ndarray:
    """src/shaders.ts:92-151, sequential over j within a block and over blocks."""
    q, scale = unpack(packed, m, n)
    qf = q.astype(f32)
    xb = x.reshape(n // 32, 32)
    total = np.zeros(m, dtype=f32)
    for b in range(n // 32):
        bs = np.zeros(m, dtype=f32)
        for j in range(32):
            bs = bs + qf[:, b, j] * xb[b, j]
        total = total + bs * scale[:, b]
    return total


def gelu_mul(gate, up):
    S, A = f32(0.7978845608028654), f32(0.044715)
    t = np.clip(S * gate * (f32(1.0) + A * gate * gate), f32(-15.0), f32(15.0))
    g = f32(0.5) * gate * (f32(1.0) + np.tanh(t.astype(np.float64)).astype(f32))
    return g * up


def fused_norm_rope(data: np.ndarray, w, nheads, hd, eps, pos, theta):
    d = data.reshape(nheads, hd).copy()
    half = hd // 2
    i = np.arange(half)
    # transcendental functions in f64, rounded to f32: a correctly rounded libm, like glibc's
    freq = f32(1.0) / np.power(np.float64(f32(theta)), ((i * 2).astype(f32) / f32(hd)).astype(np.float64)).astype(f32)
    ang = f32(pos) * freq
    c, s = np.cos(ang.astype(np.float64)).astype(f32), np.sin(ang.astype(np.float64)).astype(f32)
    for h in range(nheads):
        d[h] = rmsnorm(d[h], w, eps)
        x0, x1 = d[h, :half].copy(), d[h, half:].copy()
        d[h, :half] = x0 * c - x1 * s
        d[h, half:] = x0 * s + x1 * c
    return d.reshape(-1)


def attention(q, kc, vc, nqh, nkvh, hd, seq_len, scale):
    kvs = nkvh * hd
    out = np.zeros(nqh * hd, dtype=f32)
    for h in range(nqh):
        kvh = h * nkvh // nqh
        K = kc[:seq_len].reshape(seq_len, kvs)[:, kvh * hd:(kvh + 1) * hd]
        V = vc[:seq_len].reshape(seq_len, kvs)[:, kvh * hd:(kvh + 1) * hd]
        dot = np.zeros(seq_len, dtype=f32)
        for dd in range(hd):
            dot = dot + q[h * hd + dd] * K[:, dd]
        s = dot * f32(scale)
        sm = np.full(256, f32(-1e30), dtype=f32)
        for base in range(0, seq_len, 256):
            seg = s[base:base + 256]
            sm[:seg.shape[0]] = np.maximum(sm[:seg.shape[0]], seg)
        mx = sm.max()
        e = np.exp((s - mx).astype(np.float64)).astype(f32)
        ss = np.zeros(256, dtype=f32)
        for base in range(0, seq_len, 256):
            seg = e[base:base + 256]
            ss[:seg.shape[0]] = ss[:seg.shape[0]] + seg
        stride = 128
        while stride > 0:
            ss[:stride] = ss[:stride] + ss[stride:2 * stride]
            stride >>= 1
        p = e / ss[0]
        acc = np.zeros(hd, dtype=f32)
        for t in range(seq_len):
            acc = acc + p[t] * V[t]
        out[h * hd:(h + 1) * hd] = acc
    return out


def topk256(logits: np.ndarray):
    n = logits.shape[0]
    vals = np.full(256, f32(-1e30), dtype=f32)
    idx = np.zeros(256, dtype=np.uint32)
    for base in range(0, n, 256):
        seg = logits[base:base + 256]
        k = seg.shape[0]
        better = seg > vals[:k]
        vals[:k] = np.where(better, seg, vals[:k])
        idx[:k] = np.where(better, np.arange(base, base + k, dtype=np.uint32), idx[:k])
    return vals, idx


def argmax(logits: np.ndarray) -> int:
    m, ix = topk256(logits)
    m, ix = m.copy(), ix.copy()
    stride = 128
    while stride > 0:
        upd = m[stride:2 * stride] > m[:stride]
        m[:stride] = np.where(upd, m[stride:2 * stride], m[:stride])
        ix[:stride] = np.where(upd, ix[stride:2 * stride], ix[:stride])
        stride >>= 1
    return int(ix[0])


def sample(vals, ids, temperature, top_p, rep, seen: set, u: float) -> int:
    """src/engine.ts:862-901 with Python floats (IEEE doubles, like JS numbers)."""
    cand = [[float(vals[i]), int(ids[i])] for i in range(256)]
    if rep > 1.0 and len(seen) > 0:
        for c in cand:
            if c[1] in seen:
                c[0] = c[0] / rep if c[0] > 0 else c[0] * rep
    cand.sort(key=lambda c: -c[0])  # Python's sort is stable, like Array.prototype.sort
    if temperature == 0:
        return cand[0][1]
    mx = cand[0][0]
    import math
    probs = [float(np.float32(math.exp((c[0] - mx) / temperature))) for c in cand]
    s = 0.0
    for p in probs:
        s += p
    cum, cutoff = 0.0, 256
    for i, p in enumerate(probs):
        cum += p / s
        if cum >= top_p:
            cutoff = i + 1
            break
    sub = 0.0
    for i in range(cutoff):
        sub += probs[i]
    r = u * sub
    for i in range(cutoff):
        r -= probs[i]
        if r <= 0:
            return cand[i][1]
    return cand[cutoff - 1][1]
