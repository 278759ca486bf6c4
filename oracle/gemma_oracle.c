/*
 * gemma_oracle.c -- CPU restatement of the reference's Gemma 3 token loop.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the parity checker for the CUDA path in
 * libgemma_b200.so and the timed CPU baseline of bench.py; no product code path
 * links, loads or calls it.
 *
 * What it restates (paths are inside the reference project svenflow/webgpu-gemma):
 *   - src/gguf.ts:95-105   f16ToF32                  -> or_f16_to_f32
 *   - src/gguf.ts:126-149  packQ8_0ForGPU            -> or_pack_q8_0
 *   - src/shaders.ts:2-23    embeddingLookup         -> or_embedding
 *   - src/shaders.ts:25-56   rmsNorm                 -> or_rmsnorm
 *   - src/shaders.ts:92-151  linearQ8                -> or_linear_q8
 *   - src/shaders.ts:153-170 geluMul                 -> or_gelu_mul
 *   - src/shaders.ts:209-227 kvCacheStore            -> (inline in or_forward)
 *   - src/shaders.ts:229-325 attnScore/softmax/attnOutput -> or_attention
 *   - src/shaders.ts:327-361 argmax                  -> or_argmax
 *   - src/shaders.ts:363-384 topk256                 -> or_topk256
 *   - src/shaders.ts:386-418 fusedNormAdd            -> or_fused_norm_add
 *   - src/shaders.ts:420-467 fusedPerHeadNormRope    -> or_fused_norm_rope
 *   - src/engine.ts:735-802  encodeTransformerPass   -> or_forward
 *   - src/engine.ts:817-821  LM head dispatch        -> or_lm_head
 *   - src/engine.ts:862-901  CPU sampler (JS doubles)-> or_sample
 *
 * Arithmetic: every WGSL f32 operation is one C float operation, evaluated in the
 * shader's order, built with -ffp-contract=off (no fused multiply-add: the WGSL spec
 * leaves contraction to the implementation; rounding each product is one valid reading).
 * The 256-thread strided partial sums and 128->1 tree reductions of the shaders are
 * reproduced exactly. exp/tanh/pow/sin/cos/sqrt use libm's float functions (the WGSL
 * builtins have implementation-defined accuracy, so ULP-level differences from any real
 * WebGPU driver are expected).
 *
 * PARITY UNPINNED: the reference ships no tests, golden vectors or fixtures, and it
 * cannot run in this build environment (it needs a WebGPU device and a JS runtime).
 * Only f16ToF32 is pinned independently (exhaustively, against IEEE binary16).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <stdio.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ dequant */

/* gguf.ts:95-105. Computed in double as JS does, then stored as f32 (Float32Array). */
OR_EXPORT float or_f16_to_f32(uint16_t h) {
    int sign = (h >> 15) & 1, ex = (h >> 10) & 0x1f, mant = h & 0x3ff;
    double v;
    if (ex == 0) {
        if (mant == 0) return sign ? -0.0f : 0.0f;
        v = (sign ? -1.0 : 1.0) * pow(2.0, -14) * (mant / 1024.0);
    } else if (ex == 31) {
        return mant == 0 ? (sign ? -INFINITY : INFINITY) : NAN;
    } else {
        v = (sign ? -1.0 : 1.0) * pow(2.0, ex - 15) * (1.0 + mant / 1024.0);
    }
    return (float)v;
}

/* gguf.ts:126-149: 34-byte GGUF blocks -> 9 x u32 {f32 scale, 8 words, byte k at bits 8k}. */
OR_EXPORT void or_pack_q8_0(const uint8_t *src, int64_t nblocks, uint32_t *dst) {
    for (int64_t b = 0; b < nblocks; b++) {
        const uint8_t *s = src + b * 34;
        float sc = or_f16_to_f32((uint16_t)(s[0] | (s[1] << 8)));
        memcpy(&dst[b * 9], &sc, 4);
        for (int j = 0; j < 8; j++) {
            uint32_t p = 0;
            for (int k = 0; k < 4; k++) p |= (uint32_t)s[2 + j * 4 + k] << (k * 8);
            dst[b * 9 + 1 + j] = p;
        }
    }
}

static inline float q8_at(uint32_t word, int byte) {
    /* extractBits(bitcast<i32>(packed), byte*8, 8): signed extract */
    return (float)(int8_t)((word >> (byte * 8)) & 0xff);
}

static inline float u32_as_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------ kernels */

/* shaders.ts:2-23 */
OR_EXPORT void or_embedding(const uint32_t *emb, int H, int token, float *out) {
    int bpr = H / 32;
    const float sq = sqrtf((float)H);
    for (int i = 0; i < H; i++) {
        int64_t row_off = (int64_t)token * bpr * 9;
        int64_t boff = row_off + (i / 32) * 9;
        float scale = u32_as_f32(emb[boff]);
        int e = i % 32;
        float q = q8_at(emb[boff + 1 + e / 4], e % 4);
        out[i] = q * scale * sq;
    }
}

/* 256-thread strided partial sums of x*x followed by the 128->1 tree (shaders.ts:37-49). */
static float sumsq_tree(const float *x, int n) {
    float s[256];
    for (int t = 0; t < 256; t++) {
        float p = 0.0f;
        for (int i = t; i < n; i += 256) { float v = x[i]; p += v * v; }
        s[t] = p;
    }
    for (int stride = 128; stride > 0; stride >>= 1)
        for (int t = 0; t < stride; t++) s[t] += s[t + stride];
    return s[0];
}

/* shaders.ts:25-56 */
OR_EXPORT void or_rmsnorm(const float *x, const float *w, float *out, int n, float eps) {
    float rms = sqrtf(sumsq_tree(x, n) / (float)n + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * w[i] / rms;
}

/* shaders.ts:386-418: out = residual + x*w/rms(x) */
OR_EXPORT void or_fused_norm_add(const float *x, const float *w, const float *res, float *out, int n, float eps) {
    float rms = sqrtf(sumsq_tree(x, n) / (float)n + eps);
    for (int i = 0; i < n; i++) out[i] = res[i] + x[i] * w[i] / rms;
}

/* shaders.ts:92-151: y[m] = sum_b (sum_{j<32} q*x) * d, sequential in j then b.
 * Eight rows are processed together so the compiler can vectorise across rows; each
 * row's arithmetic is still the shader's exact sequence. */
OR_EXPORT void or_linear_q8(const float *x, const uint32_t *w, float *y, int M, int N) {
    const int bpr = N / 32;
    #pragma omp parallel for schedule(static) if (M >= 1024)
    for (int m0 = 0; m0 < M; m0 += 8) {
        int nr = M - m0 < 8 ? M - m0 : 8;
        float tot[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int b = 0; b < bpr; b++) {
            float bs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            for (int r = 0; r < nr; r++) {
                const uint32_t *blk = w + ((int64_t)(m0 + r) * bpr + b) * 9;
                float acc = 0.0f;
                for (int j = 0; j < 32; j++) acc += q8_at(blk[1 + j / 4], j % 4) * x[b * 32 + j];
                bs[r] = acc;
            }
            for (int r = 0; r < nr; r++) {
                const uint32_t *blk = w + ((int64_t)(m0 + r) * bpr + b) * 9;
                tot[r] += bs[r] * u32_as_f32(blk[0]);
            }
        }
        for (int r = 0; r < nr; r++) y[m0 + r] = tot[r];
    }
}

/* shaders.ts:153-170 */
OR_EXPORT void or_gelu_mul(const float *gate, const float *up, float *out, int n) {
    const float S = (float)0.7978845608028654, A = 0.044715f;
    for (int i = 0; i < n; i++) {
        float x = gate[i];
        float t = S * x * (1.0f + A * x * x);
        t = t < -15.0f ? -15.0f : (t > 15.0f ? 15.0f : t);
        float g = 0.5f * x * (1.0f + tanhf(t));
        out[i] = g * up[i];
    }
}

/* shaders.ts:420-467: per-head RMSNorm (in place) then NeoX RoPE of pairs (i, i+hd/2). */
OR_EXPORT void or_fused_norm_rope(float *data, const float *w, int nheads, int hd, float eps, int pos, float theta) {
    for (int h = 0; h < nheads; h++) {
        float *d = data + (int64_t)h * hd;
        float rms = sqrtf(sumsq_tree(d, hd) / (float)hd + eps);
        for (int i = 0; i < hd; i++) d[i] = d[i] * w[i] / rms;
        int half = hd / 2;
        for (int i = 0; i < half; i++) {
            float freq = 1.0f / powf(theta, (float)(i * 2) / (float)hd);
            float ang = (float)pos * freq;
            float c = cosf(ang), s = sinf(ang);
            float x0 = d[i], x1 = d[i + half];
            d[i] = x0 * c - x1 * s;
            d[i + half] = x0 * s + x1 * c;
        }
    }
}

/* shaders.ts:229-325: scores (sequential d), softmax (strided/tree), output (sequential p).
 * kcache/vcache are [ctx][nkvh][hd]; attends to positions 0..seq_len-1, no window. */
OR_EXPORT void or_attention(const float *q, const float *kc, const float *vc, int nqh, int nkvh, int hd,
                            int seq_len, float scale, float *scores /* [nqh*seq_len] */, float *out) {
    int kvs = nkvh * hd;
    for (int h = 0; h < nqh; h++) {
        int kvh = h * nkvh / nqh;
        for (int p = 0; p < seq_len; p++) {
            float dot = 0.0f;
            const float *kr = kc + (int64_t)p * kvs + kvh * hd;
            for (int dd = 0; dd < hd; dd++) dot += q[h * hd + dd] * kr[dd];
            scores[h * seq_len + p] = dot * scale;
        }
    }
    for (int h = 0; h < nqh; h++) {
        float *s = scores + (int64_t)h * seq_len;
        float sm[256], ss[256];
        for (int t = 0; t < 256; t++) {
            float lm = -1e30f;
            for (int i = t; i < seq_len; i += 256) lm = fmaxf(lm, s[i]);
            sm[t] = lm;
        }
        for (int stride = 128; stride > 0; stride >>= 1)
            for (int t = 0; t < stride; t++) sm[t] = fmaxf(sm[t], sm[t + stride]);
        float mx = sm[0];
        for (int t = 0; t < 256; t++) {
            float ls = 0.0f;
            for (int i = t; i < seq_len; i += 256) { float e = expf(s[i] - mx); s[i] = e; ls += e; }
            ss[t] = ls;
        }
        for (int stride = 128; stride > 0; stride >>= 1)
            for (int t = 0; t < stride; t++) ss[t] += ss[t + stride];
        float sum = ss[0];
        for (int i = 0; i < seq_len; i++) s[i] = s[i] / sum;
    }
    for (int h = 0; h < nqh; h++) {
        int kvh = h * nkvh / nqh;
        for (int dd = 0; dd < hd; dd++) {
            float acc = 0.0f;
            for (int p = 0; p < seq_len; p++) acc += scores[h * seq_len + p] * vc[(int64_t)p * kvs + kvh * hd + dd];
            out[h * hd + dd] = acc;
        }
    }
}

/* shaders.ts:363-384: for lane t, max over i = t (mod 256) with strict '>' from (-1e30, 0). */
OR_EXPORT void or_topk256(const float *logits, int n, float *vals, uint32_t *idx) {
    for (int t = 0; t < 256; t++) {
        float lm = -1e30f; uint32_t li = 0;
        for (int i = t; i < n; i += 256) if (logits[i] > lm) { lm = logits[i]; li = (uint32_t)i; }
        vals[t] = lm; idx[t] = li;
    }
}

/* shaders.ts:327-361: the same lanes, then a tree reduce with strict '>' (lower lane wins ties). */
OR_EXPORT uint32_t or_argmax(const float *logits, int n) {
    float m[256]; uint32_t ix[256];
    or_topk256(logits, n, m, ix);
    for (int stride = 128; stride > 0; stride >>= 1)
        for (int t = 0; t < stride; t++)
            if (m[t + stride] > m[t]) { m[t] = m[t + stride]; ix[t] = ix[t + stride]; }
    return ix[0];
}

/* engine.ts:862-901, in JS double arithmetic. `seen` is a bitmap over the vocabulary of
 * this turn's tokens (allTokens); `u` replaces Math.random(). Stable sort descending by
 * value (Array.prototype.sort is stable): ties keep lane order. */
OR_EXPORT int32_t or_sample(const float *vals, const uint32_t *ids, double temperature, double top_p,
                            double rep, const uint8_t *seen, int n_seen_tokens, double u) {
    double v[256]; uint32_t id[256]; int ord[256];
    for (int i = 0; i < 256; i++) { v[i] = (double)vals[i]; id[i] = ids[i]; ord[i] = i; }
    if (rep > 1.0 && n_seen_tokens > 0 && seen) {
        for (int i = 0; i < 256; i++) {
            uint32_t t = id[i];
            if (seen[t >> 3] & (1u << (t & 7))) {
                if (v[i] > 0) v[i] /= rep; else v[i] *= rep;
            }
        }
    }
    /* stable insertion sort on (value desc) */
    for (int i = 1; i < 256; i++) {
        int k = ord[i], j = i - 1;
        while (j >= 0 && v[ord[j]] < v[k]) { ord[j + 1] = ord[j]; j--; }
        ord[j + 1] = k;
    }
    if (temperature == 0.0) return (int32_t)id[ord[0]];
    double mx = v[ord[0]];
    float probs[256];
    double sum = 0.0;
    for (int i = 0; i < 256; i++) { probs[i] = (float)exp((v[ord[i]] - mx) / temperature); sum += probs[i]; }
    double cum = 0.0; int cutoff = 256;
    for (int i = 0; i < 256; i++) { cum += probs[i] / sum; if (cum >= top_p) { cutoff = i + 1; break; } }
    double sub = 0.0;
    for (int i = 0; i < cutoff; i++) sub += probs[i];
    double r = u * sub;
    for (int i = 0; i < cutoff; i++) { r -= probs[i]; if (r <= 0) return (int32_t)id[ord[i]]; }
    return (int32_t)id[ord[cutoff - 1]];
}

/* ------------------------------------------------------------------ bf16 KV option */

/* Not in the reference (its caches are f32, engine.ts:440-447): the optional bf16 KV cache.
 * f32 -> bf16 with round-to-nearest-even on the upper 16 bits (add 0x7fff plus the lowest kept
 * bit, truncate); NaN stays NaN (quiet bit set), infinities stay infinite. Returns the
 * rounded value widened back to f32, which is what attention reads. */
static float or_bf16_round1(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) {
        if (u & 0x007fffffu) u |= 0x00400000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u);
    }
    u &= 0xffff0000u;
    memcpy(&x, &u, 4);
    return x;
}

OR_EXPORT void or_bf16_round(const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = or_bf16_round1(x[i]);
}

#define OR_FLAG_KV_BF16 2 /* the engine's GG_FLAG_KV_BF16 */

/* ------------------------------------------------------------------ model */

typedef struct {
    int32_t hidden_size, q_dim, kv_dim, num_q_heads, num_kv_heads, head_dim, intermediate_size,
        vocab_size, num_layers, context_length;
    float rms_norm_eps, rope_theta_global, rope_theta_swa;
    int32_t swa_period, max_seqs, flags;
    int32_t sliding_window; /* 0: whole prefix (the reference); W: last W positions on SWA layers */
} or_config;

typedef struct {
    uint32_t *q, *k, *v, *o, *gate, *up, *down; /* packed 36-byte blocks */
    float *attn_norm, *ffn_norm, *q_norm, *k_norm, *post_attn_norm, *post_ffw_norm;
} or_layer;

typedef struct {
    or_config c;
    uint32_t *embd;
    float *out_norm;
    or_layer *L;
    float *kc, *vc; /* [seq][layer][ctx][kv_dim] */
    /* per-seq work buffers (engine.ts:402-438) */
    float *hidden, *residual, *normed, *qb, *kb, *vb, *att, *proj, *scores, *gate, *upb, *mul, *down;
} or_model;

static size_t kv_layer_elems(const or_config *c) { return (size_t)c->context_length * c->kv_dim; }

OR_EXPORT or_model *or_create(const or_config *cfg) {
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->c = *cfg;
    if (m->c.max_seqs < 1) m->c.max_seqs = 1;
    const or_config *c = &m->c;
    m->L = (or_layer *)calloc(c->num_layers, sizeof(or_layer));
    size_t kv = kv_layer_elems(c) * c->num_layers * c->max_seqs;
    m->kc = (float *)calloc(kv, sizeof(float));
    m->vc = (float *)calloc(kv, sizeof(float));
    int S = c->max_seqs, H = c->hidden_size, Q = c->q_dim, KV = c->kv_dim, I = c->intermediate_size;
    m->hidden = calloc((size_t)S * H, 4); m->residual = calloc((size_t)S * H, 4); m->normed = calloc((size_t)S * H, 4);
    m->qb = calloc((size_t)S * Q, 4); m->kb = calloc((size_t)S * KV, 4); m->vb = calloc((size_t)S * KV, 4);
    m->att = calloc((size_t)S * Q, 4); m->proj = calloc((size_t)S * H, 4);
    m->scores = calloc((size_t)S * c->num_q_heads * c->context_length, 4);
    m->gate = calloc((size_t)S * I, 4); m->upb = calloc((size_t)S * I, 4); m->mul = calloc((size_t)S * I, 4);
    m->down = calloc((size_t)S * H, 4);
    return m;
}

OR_EXPORT void or_free(or_model *m) {
    if (!m) return;
    for (int l = 0; l < m->c.num_layers; l++) {
        or_layer *L = &m->L[l];
        free(L->q); free(L->k); free(L->v); free(L->o); free(L->gate); free(L->up); free(L->down);
        free(L->attn_norm); free(L->ffn_norm); free(L->q_norm); free(L->k_norm); free(L->post_attn_norm); free(L->post_ffw_norm);
    }
    free(m->L); free(m->embd); free(m->out_norm); free(m->kc); free(m->vc);
    free(m->hidden); free(m->residual); free(m->normed); free(m->qb); free(m->kb); free(m->vb);
    free(m->att); free(m->proj); free(m->scores); free(m->gate); free(m->upb); free(m->mul); free(m->down);
    free(m);
}

/* Accepts a GGUF tensor's raw bytes: Q8_0 is packed like packQ8_0ForGPU, F32 copied,
 * F16 converted with f16ToF32 (engine.ts:302-330). Returns 0, or -1 on an unknown name/type. */
OR_EXPORT int or_set_tensor(or_model *m, const char *name, int type, const void *data, int64_t n_elems) {
    void *buf = NULL;
    if (type == 8) {
        buf = malloc((size_t)(n_elems / 32) * 36);
        or_pack_q8_0((const uint8_t *)data, n_elems / 32, (uint32_t *)buf);
    } else if (type == 0) {
        buf = malloc((size_t)n_elems * 4);
        memcpy(buf, data, (size_t)n_elems * 4);
    } else if (type == 1) {
        float *f = (float *)malloc((size_t)n_elems * 4);
        const uint16_t *h = (const uint16_t *)data;
        for (int64_t i = 0; i < n_elems; i++) f[i] = or_f16_to_f32(h[i]);
        buf = f;
    } else {
        return -1;
    }
    if (!strcmp(name, "token_embd.weight")) { if (type != 8) { free(buf); return -1; } m->embd = (uint32_t *)buf; return 0; }
    if (!strcmp(name, "output_norm.weight")) { m->out_norm = (float *)buf; return 0; }
    int il; char key[64];
    if (sscanf(name, "blk.%d.%63[^.].weight", &il, key) == 2 && il >= 0 && il < m->c.num_layers) {
        or_layer *L = &m->L[il];
        struct { const char *k; void **p; int q8; } tab[] = {
            {"attn_q", (void **)&L->q, 1}, {"attn_k", (void **)&L->k, 1}, {"attn_v", (void **)&L->v, 1},
            {"attn_output", (void **)&L->o, 1}, {"ffn_gate", (void **)&L->gate, 1}, {"ffn_up", (void **)&L->up, 1},
            {"ffn_down", (void **)&L->down, 1}, {"attn_norm", (void **)&L->attn_norm, 0},
            {"ffn_norm", (void **)&L->ffn_norm, 0}, {"attn_q_norm", (void **)&L->q_norm, 0},
            {"attn_k_norm", (void **)&L->k_norm, 0}, {"post_attention_norm", (void **)&L->post_attn_norm, 0},
            {"post_ffw_norm", (void **)&L->post_ffw_norm, 0},
        };
        for (size_t i = 0; i < sizeof(tab) / sizeof(tab[0]); i++) {
            if (!strcmp(key, tab[i].k)) {
                if (tab[i].q8 != (type == 8)) { free(buf); return -1; }
                free(*tab[i].p); *tab[i].p = buf; return 0;
            }
        }
    }
    free(buf);
    return -1;
}

OR_EXPORT void or_reset_kv(or_model *m, int seq) {
    size_t n = kv_layer_elems(&m->c) * m->c.num_layers;
    memset(m->kc + (size_t)seq * n, 0, n * 4);
    memset(m->vc + (size_t)seq * n, 0, n * 4);
}

static float rope_theta(const or_config *c, int il) {
    /* types.ts:38-44 */
    int swa = (il % c->swa_period) < (c->swa_period - 1);
    return swa ? c->rope_theta_swa : c->rope_theta_global;
}

/* engine.ts:735-802: one token through every layer; leaves the final-normed hidden state
 * in the seq's `normed` buffer (and copies it to normed_out when given). */
OR_EXPORT int or_forward(or_model *m, int seq, int token, int pos, float *normed_out) {
    const or_config *c = &m->c;
    int H = c->hidden_size, Q = c->q_dim, KV = c->kv_dim, I = c->intermediate_size, HD = c->head_dim;
    int NQH = c->num_q_heads, NKH = c->num_kv_heads, ctx = c->context_length;
    if (seq < 0 || seq >= c->max_seqs || pos < 0 || pos >= ctx || token < 0 || token >= c->vocab_size) return -1;
    float eps = c->rms_norm_eps;
    float *hidden = m->hidden + (size_t)seq * H, *residual = m->residual + (size_t)seq * H;
    float *normed = m->normed + (size_t)seq * H, *q = m->qb + (size_t)seq * Q, *k = m->kb + (size_t)seq * KV;
    float *v = m->vb + (size_t)seq * KV, *att = m->att + (size_t)seq * Q, *proj = m->proj + (size_t)seq * H;
    float *scores = m->scores + (size_t)seq * NQH * ctx, *gate = m->gate + (size_t)seq * I;
    float *up = m->upb + (size_t)seq * I, *mul = m->mul + (size_t)seq * I, *down = m->down + (size_t)seq * H;
    const float scale = (float)(1.0 / sqrt((double)HD)); /* engine.ts:200 */
    int seq_len = pos + 1;

    or_embedding(m->embd, H, token, hidden);
    for (int il = 0; il < c->num_layers; il++) {
        or_layer *L = &m->L[il];
        float *kc = m->kc + ((size_t)seq * c->num_layers + il) * kv_layer_elems(c);
        float *vc = m->vc + ((size_t)seq * c->num_layers + il) * kv_layer_elems(c);
        float theta = rope_theta(c, il);
        or_rmsnorm(hidden, L->attn_norm, normed, H, eps);
        or_linear_q8(normed, L->q, q, Q, H);
        or_linear_q8(normed, L->k, k, KV, H);
        or_linear_q8(normed, L->v, v, KV, H);
        or_fused_norm_rope(q, L->q_norm, NQH, HD, eps, pos, theta);
        or_fused_norm_rope(k, L->k_norm, NKH, HD, eps, pos, theta);
        if (c->flags & OR_FLAG_KV_BF16) {
            or_bf16_round(k, kc + (size_t)pos * KV, KV);
            or_bf16_round(v, vc + (size_t)pos * KV, KV);
        } else {
            memcpy(kc + (size_t)pos * KV, k, (size_t)KV * 4);
            memcpy(vc + (size_t)pos * KV, v, (size_t)KV * 4);
        }
        /* Gemma 3's sliding window on the local layers (off unless sliding_window > 0) */
        int lo = 0;
        if (c->sliding_window > 0 && (il % c->swa_period) < (c->swa_period - 1) && pos + 1 > c->sliding_window)
            lo = pos + 1 - c->sliding_window;
        or_attention(q, kc + (size_t)lo * KV, vc + (size_t)lo * KV, NQH, NKH, HD, seq_len - lo, scale, scores, att);
        or_linear_q8(att, L->o, proj, H, Q);
        or_fused_norm_add(proj, L->post_attn_norm, hidden, residual, H, eps);
        or_rmsnorm(residual, L->ffn_norm, normed, H, eps);
        or_linear_q8(normed, L->gate, gate, I, H);
        or_linear_q8(normed, L->up, up, I, H);
        or_gelu_mul(gate, up, mul, I);
        or_linear_q8(mul, L->down, down, H, I);
        or_fused_norm_add(down, L->post_ffw_norm, residual, hidden, H, eps);
    }
    or_rmsnorm(hidden, m->out_norm, normed, H, eps);
    if (normed_out) memcpy(normed_out, normed, (size_t)H * 4);
    return 0;
}

/* engine.ts:817-821: tied LM head over the seq's final-normed hidden state. */
OR_EXPORT int or_lm_head(or_model *m, int seq, float *logits) {
    if (seq < 0 || seq >= m->c.max_seqs) return -1;
    or_linear_q8(m->normed + (size_t)seq * m->c.hidden_size, m->embd, logits, m->c.vocab_size, m->c.hidden_size);
    return 0;
}

/* Read-only views for tests (KV rows and the last hidden state). */
OR_EXPORT const float *or_kv_row(or_model *m, int seq, int layer, int pos, int which) {
    size_t off = ((size_t)seq * m->c.num_layers + layer) * kv_layer_elems(&m->c) + (size_t)pos * m->c.kv_dim;
    return (which ? m->vc : m->kc) + off;
}

/* Thread count of the parallel loops (the benchmark's CPU legs pin it to the host's cores, since
 * process launchers may set OMP_NUM_THREADS=1). */
OR_EXPORT void or_set_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

OR_EXPORT int or_get_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
