// gg_decode.cu -- the batch-1 Gemma 3 token step as one persistent sm_100a kernel.
//
// One CTA per SM (cooperative launch). Warp GG_NCW is a producer: it streams this CTA's
// share of every weight matrix of the step (and its attention KV rows) through a ring of
// shared-memory stages with cp.async.bulk, completing on mbarriers; it never waits on
// activations, only on free slots, so HBM streaming runs ahead across layer boundaries.
// Warps 0..GG_NCW-1 consume the stages. Between phases the CTAs exchange activations as
// tagged 64-bit words (f32 value | epoch << 32), so each word is its own ready flag.
//
// Phases per layer (reference: src/engine.ts:766-795):
//   A  rmsNorm(hidden) -> fused QKV matvec                       (shaders.ts:25-56, 92-151)
//   B  q/k per-head norm + RoPE, KV store, split attention       (shaders.ts:209-325, 420-467)
//   B2 combine of the attention splits (online-softmax merge)
//   C  O projection                                              (shaders.ts:92-151)
//   D  post-attn norm + residual, ffn rmsNorm, gate/up + GeGLU   (shaders.ts:153-170, 386-418)
//   E  down projection                                           (shaders.ts:92-151)
// then F: post-ffw norm + residual, final rmsNorm, tied LM head with per-lane maxima
// (engine.ts:797-821, shaders.ts:327-384), and the sampler in the last CTA (engine.ts:823-901).
#include "gg_device.cuh"
#include "gg_model.h"

namespace gg {

constexpr int NCW = GG_NCW;
constexpr int NCT = GG_NCT;
constexpr int PH_PER_LAYER = 6;

GG_DEV void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

GG_DEV uint32_t make_tag(uint32_t base, int phase) { return 0x80000000u | ((base + (uint32_t)phase) & 0x7fffffffu); }

GG_DEV void part(int M, int G, int c, int& b, int& e) {
  b = (int)((long long)c * M / G);
  e = (int)((long long)(c + 1) * M / G);
}

// Logical x element -> float index in the swizzled shared x vector.
GG_DEV int xs_index(int e) {
  int c = e >> 4, k = e & 15;
  return 4 * xswz(c, k >> 2) + (k & 3);
}

struct Smem {
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  float4* xs4;
  float* xs;
  float* hid;
  float* res;
  float* tmp;
  float* cs;    // RoPE cos (first HD/2) and sin (next HD/2)
  float* red;   // cross-warp partial sums
  float* sc;    // attention scores / combine scratch
  float* cmb;   // combine: max, sum, weight per split
  unsigned long long* keys;
  float* scal;
  int* flag;
};

GG_DEV unsigned long long init_lane_key() {
  return ((unsigned long long)f32_order_key(-1e30f) << 32) | 0xffffffffull;
}

// sum over a row's 16-byte chunks [c0, c1) of (dot of 16 int8 with x) * block scale
GG_DEV float row_dot(const uint8_t* rowp, int K, const float4* xs4, int c0, int c1, int lane) {
  float acc = 0.f;
#pragma unroll 2
  for (int c = c0 + lane; c < c1; c += 32) {
    uint4 w = *reinterpret_cast<const uint4*>(rowp + 16 * c);
    float s = __half2float(*reinterpret_cast<const __half*>(rowp + K + 2 * (c >> 1)));
    float4 a = xs4[xswz(c, 0)], b = xs4[xswz(c, 1)], cc = xs4[xswz(c, 2)], d = xs4[xswz(c, 3)];
    acc = fmaf(dot16(w, a, b, cc, d), s, acc);
  }
  return warp_sum(acc);
}

GG_DEV void row_dot2(const uint8_t* r0, const uint8_t* r1, int K, const float4* xs4, int lane, float& o0,
                     float& o1) {
  float a0 = 0.f, a1 = 0.f;
  const int nch = K >> 4;
#pragma unroll 2
  for (int c = lane; c < nch; c += 32) {
    uint4 w0 = *reinterpret_cast<const uint4*>(r0 + 16 * c);
    uint4 w1 = *reinterpret_cast<const uint4*>(r1 + 16 * c);
    float s0 = __half2float(*reinterpret_cast<const __half*>(r0 + K + 2 * (c >> 1)));
    float s1 = __half2float(*reinterpret_cast<const __half*>(r1 + K + 2 * (c >> 1)));
    float4 a = xs4[xswz(c, 0)], b = xs4[xswz(c, 1)], cc = xs4[xswz(c, 2)], d = xs4[xswz(c, 3)];
    a0 = fmaf(dot16(w0, a, b, cc, d), s0, a0);
    a1 = fmaf(dot16(w1, a, b, cc, d), s1, a1);
  }
  o0 = warp_sum(a0);
  o1 = warp_sum(a1);
}

// Sum over the consumer threads; every consumer thread gets the same total.
GG_DEV float csum(float v, float* scal) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) scal[warp] = v;
  cbar();
  float t = lane < NCW ? scal[lane] : 0.f;
  t = warp_sum(t);
  cbar();
  return t;
}

GG_DEV float gelu_tanh(float x) {
  // shaders.ts:153-170
  const float S = 0.7978845608028654f, A = 0.044715f;
  float t = S * x * (1.0f + A * x * x);
  t = fminf(fmaxf(t, -15.0f), 15.0f);
  return 0.5f * x * (1.0f + tanhf(t));
}

struct Ctx {
  const GGModelDev* m;
  GGState* st;
  Smem S;
  SpinCtl sc;
  int mode, token, pos, seq, nsplit;
  uint32_t tagbase;
  uint32_t idx;  // ring position (per warp for consumers, lane 0 for the producer)
};

// ---------------------------------------------------------------------------------- producer

struct Producer {
  Ctx& x;
  uint64_t pol;
  bool ok = true;

  GG_DEV void issue(const void* s0, uint32_t b0, const void* s1, uint32_t b1, uint32_t off1) {
    const GGModelDev& m = *x.m;
    int slot = x.idx % m.nstages;
    uint32_t use = x.idx / m.nstages;
    if (use > 0 && ok) ok = mbar_wait(&x.S.empty[slot], (use - 1) & 1, x.sc);
    if (!ok) return;
    uint8_t* dst = x.S.ring + (size_t)slot * m.stage_bytes;
    mbar_arrive_expect_tx(&x.S.full[slot], b0 + b1);
    if (b0) bulk_g2s(dst, s0, b0, &x.S.full[slot], pol);
    if (b1) bulk_g2s(dst + off1, s1, b1, &x.S.full[slot], pol);
    x.idx++;
  }
  GG_DEV void rows(const uint8_t* W, int rs, int rb, int re, int rps) {
    for (int r = rb; r < re && ok; r += rps) {
      int n = min(rps, re - r);
      issue(W + (size_t)r * rs, (uint32_t)(n * rs), nullptr, 0, 0);
    }
  }
  GG_DEV void run() {
    const GGModelDev& m = *x.m;
    const int c = blockIdx.x, G = m.grid;
    int b, e;
    if (x.mode & GG_RUN_LAYERS) {
      for (int l = 0; l < m.L && ok; l++) {
        const GGLayerW& Lw = m.layers[l];
        part(m.Q + 2 * m.KV, G, c, b, e);
        rows(Lw.wqkv, m.rs_h, b, e, m.rps_h);
        const int rot = (l * x.nsplit) % G;
        for (int s = (c - rot + G) % G; s < x.nsplit && ok; s += G) {
          int p0 = s * m.pos_per_split, pc = min(p0 + m.pos_per_split, x.pos);
          uint32_t nb = pc > p0 ? (uint32_t)((pc - p0) * m.KV * 4) : 0u;
          size_t off = (size_t)x.seq * m.kv_seq_stride + ((size_t)l * m.CTX + p0) * m.KV;
          issue(m.kcache + off, nb, m.vcache + off, nb, (uint32_t)(m.pos_per_split * m.KV * 4));
        }
        part(m.H, G, c, b, e);
        rows(Lw.wo, m.rs_q, b, e, m.rps_q);
        part(m.I, G, c, b, e);
        rows(Lw.wgu, m.rs_h, 2 * b, 2 * e, 2 * m.pps_gu);
        part(m.H, G, c, b, e);
        rows(Lw.wdown, m.rs_i, b, e, m.rps_i);
      }
    }
    if ((x.mode & GG_RUN_LM) && ok) {
      part(m.V, G, c, b, e);
      rows(m.embd, m.rs_h, b, e, m.rps_h);
    }
    // Drain: wait until every copy issued into the ring has landed before the CTA may exit.
    SpinCtl drain = x.sc;
    uint32_t n = x.idx < (uint32_t)m.nstages ? x.idx : (uint32_t)m.nstages;
    for (uint32_t k = x.idx - n; k < x.idx; k++) {
      int slot = k % m.nstages;
      uint32_t par = (k / m.nstages) & 1;
      uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&x.S.full[slot], par)) {
        if (global_timer_ns() - t0 > drain.timeout_ns) { atomicOr(drain.err, GG_ERR_WAIT_MBAR); break; }
      }
    }
  }
};

// ---------------------------------------------------------------------------------- consumers

struct Consumer {
  Ctx& x;
  int tid, lane, warp;
  // Once a ring wait gives up, this warp stops waiting on and releasing slots, so the
  // producer can never refill a slot whose copy might still be landing; it drains and exits.
  bool dead = false;

  GG_DEV uint8_t* stage_acquire() {
    const GGModelDev& m = *x.m;
    int slot = x.idx % m.nstages;
    if (!dead) {
      bool ok = mbar_wait(&x.S.full[slot], (x.idx / m.nstages) & 1, x.sc);
      dead = !__all_sync(0xffffffffu, ok);
    }
    return x.S.ring + (size_t)slot * m.stage_bytes;
  }
  GG_DEV void stage_release() {
    __syncwarp();
    if (lane == 0 && !dead) mbar_arrive(&x.S.empty[x.idx % x.m->nstages]);
    x.idx++;
  }

  // Wait for n tagged words and store them (optionally swizzled) into shared memory.
  GG_DEV void gather(const uint64_t* src, int n, uint32_t tag, float* dst, bool swz) {
    for (int i = tid; i < n; i += NCT) {
      float v = tag_wait(src + i, tag, x.sc);
      dst[swz ? xs_index(i) : i] = v;
    }
  }

  // Rows [rb, re) of a matrix, one warp per row (round robin), whole rows per stage.
  template <class Epi>
  GG_DEV void rows_ks1(int rb, int re, int rps, int K, int rs, Epi epi) {
    const int nrows = re - rb, nch = K >> 4;
    for (int r0 = 0; r0 < nrows; r0 += rps) {
      const uint8_t* stg = stage_acquire();
      const int r1 = min(r0 + rps, nrows);
      for (int u = r0 + ((warp - r0) % NCW + NCW) % NCW; u < r1; u += NCW) {
        float v = row_dot(stg + (size_t)(u - r0) * rs, K, x.S.xs4, 0, nch, lane);
        epi(rb + u, v);
      }
      stage_release();
    }
  }

  // Rows [rb, re) split in `ks` K-slices (units spread over warps); the slice partials are
  // summed in a fixed order after the phase, then passed to epi(row, value) by one thread.
  template <class Epi>
  GG_DEV void rows_ksn(int rb, int re, int rps, int K, int rs, int ks, Epi epi) {
    const int nrows = re - rb, nch = K >> 4, cpk = nch / ks;
    for (int r0 = 0; r0 < nrows; r0 += rps) {
      const uint8_t* stg = stage_acquire();
      const int r1 = min(r0 + rps, nrows);
      const int u0 = r0 * ks, u1 = r1 * ks;
      for (int u = u0 + ((warp - u0) % NCW + NCW) % NCW; u < u1; u += NCW) {
        int r = u / ks, s = u % ks;
        float v = row_dot(stg + (size_t)(r - r0) * rs, K, x.S.xs4, s * cpk, (s + 1) * cpk, lane);
        if (lane == 0) x.S.red[u] = v;
      }
      stage_release();
    }
    cbar();
    for (int r = tid; r < nrows; r += NCT) {
      float v = 0.f;
      for (int s = 0; s < ks; s++) v += x.S.red[r * ks + s];
      epi(rb + r, v);
    }
  }

  // x = rmsNorm(v) * w into the swizzled x vector (shaders.ts:25-56)
  GG_DEV void norm_to_xs(const float* v, const float* w, int n) {
    const GGModelDev& m = *x.m;
    float ss = 0.f;
    for (int i = tid; i < n; i += NCT) ss += v[i] * v[i];
    ss = csum(ss, x.S.scal);
    float rms = sqrtf(ss / (float)n + m.eps);
    for (int i = tid; i < n; i += NCT) x.S.xs[xs_index(i)] = v[i] * w[i] / rms;
  }

  // out = base + v * w / rms(v)   (shaders.ts:386-418)
  GG_DEV void norm_add(const float* v, const float* w, const float* base, float* out, int n) {
    const GGModelDev& m = *x.m;
    float ss = 0.f;
    for (int i = tid; i < n; i += NCT) ss += v[i] * v[i];
    ss = csum(ss, x.S.scal);
    float rms = sqrtf(ss / (float)n + m.eps);
    for (int i = tid; i < n; i += NCT) out[i] = base[i] + v[i] * w[i] / rms;
  }

  // hidden = residual + post_ffw_norm(down)  (the end of layer l, engine.ts:794)
  GG_DEV void finish_layer(int l) {
    const GGModelDev& m = *x.m;
    gather(m.t_down, m.H, make_tag(x.tagbase, l * PH_PER_LAYER + 5), x.S.tmp, false);
    cbar();
    norm_add(x.S.tmp, m.layers[l].post_ffw_norm, x.S.res, x.S.hid, m.H);
    cbar();
    if (blockIdx.x == 0)
      for (int i = tid; i < m.H; i += NCT) m.dbg_hidden[i] = x.S.hid[i];
  }

  GG_DEV void embed() {
    // shaders.ts:2-23: h[i] = q * d * sqrt(H), evaluated left to right in f32
    const GGModelDev& m = *x.m;
    const uint8_t* row = m.embd + (size_t)x.token * m.rs_h;
    const float sq = sqrtf((float)m.H);
    for (int i = tid; i < m.H; i += NCT) {
      float q = (float)(int8_t)row[i];
      float d = __half2float(*reinterpret_cast<const __half*>(row + m.H + 2 * (i >> 5)));
      float v = q * d;
      x.S.hid[i] = v * sq;
    }
    cbar();
  }

  GG_DEV void phase_qkv(int l) {
    const GGModelDev& m = *x.m;
    if (l == 0) embed();
    else finish_layer(l - 1);
    norm_to_xs(x.S.hid, m.layers[l].attn_norm, m.H);
    cbar();
    int b, e;
    part(m.Q + 2 * m.KV, m.grid, blockIdx.x, b, e);
    const uint32_t tag = make_tag(x.tagbase, l * PH_PER_LAYER + 0);
    uint64_t* out = m.t_qkv;
    rows_ks1(b, e, m.rps_h, m.H, m.rs_h, [&](int row, float v) {
      if (lane == 0) tag_store(out + row, v, tag);
    });
  }

  GG_DEV void phase_attn(int l) {
    const GGModelDev& m = *x.m;
    const int G = m.grid, c = blockIdx.x, rot = (l * x.nsplit) % G;
    int s = (c - rot + G) % G;
    if (s >= x.nsplit) return;
    const int Q = m.Q, KV = m.KV, HD = m.HD, NQH = m.NQH, NKH = m.NKH, PPS = m.pos_per_split;
    const GGLayerW& Lw = m.layers[l];
    float* t = x.S.tmp;  // q [Q] | k [KV] | v [KV]
    cbar();              // tmp may still be read by a slow warp of the previous phase prologue
    gather(m.t_qkv, Q + 2 * KV, make_tag(x.tagbase, l * PH_PER_LAYER + 0), t, false);
    // RoPE table for this position (shaders.ts:457-460)
    for (int i = tid; i < HD / 2; i += NCT) {
      float freq = 1.0f / powf(Lw.theta, (float)(i * 2) / (float)HD);
      float ang = (float)x.pos * freq;
      x.S.cs[i] = cosf(ang);
      x.S.cs[HD / 2 + i] = sinf(ang);
    }
    cbar();
    // per-head RMSNorm of q heads and k heads (shaders.ts:433-452)
    const int nh = NQH + NKH;
    for (int h = warp; h < nh; h += NCW) {
      const float* d = t + h * HD;
      float ss = 0.f;
      for (int i = lane; i < HD; i += 32) ss += d[i] * d[i];
      ss = warp_sum(ss);
      if (lane == 0) x.S.scal[64 + h] = sqrtf(ss / (float)HD + m.eps);
    }
    cbar();
    for (int i = tid; i < nh * HD; i += NCT) {
      int h = i / HD, dd = i % HD;
      const float* w = h < NQH ? Lw.q_norm : Lw.k_norm;
      t[i] = t[i] * w[dd] / x.S.scal[64 + h];
    }
    cbar();
    // RoPE of pairs (i, i + HD/2) (shaders.ts:454-466)
    for (int i = tid; i < nh * (HD / 2); i += NCT) {
      int h = i / (HD / 2), k = i % (HD / 2);
      float* d = t + h * HD;
      float cs = x.S.cs[k], sn = x.S.cs[HD / 2 + k];
      float x0 = d[k], x1 = d[k + HD / 2];
      d[k] = x0 * cs - x1 * sn;
      d[k + HD / 2] = x0 * sn + x1 * cs;
    }
    cbar();
    const uint32_t tag = make_tag(x.tagbase, l * PH_PER_LAYER + 1);
    for (; s < x.nsplit; s += G) {
      const int p0 = s * PPS, p1 = min(p0 + PPS, x.pos + 1), np = p1 - p0;
      const uint8_t* stg = stage_acquire();
      const float* Kst = reinterpret_cast<const float*>(stg);
      const float* Vst = reinterpret_cast<const float*>(stg + (size_t)PPS * KV * 4);
      if (p1 == x.pos + 1) {  // this split owns the new position: store it (shaders.ts:209-227)
        size_t off = (size_t)x.seq * m.kv_seq_stride + ((size_t)l * m.CTX + x.pos) * KV;
        for (int i = tid; i < KV; i += NCT) {
          m.kcache[off + i] = t[Q + i];
          m.vcache[off + i] = t[Q + KV + i];
        }
      }
      // scores (shaders.ts:229-252)
      for (int pr = warp; pr < NQH * np; pr += NCW) {
        int h = pr / np, j = pr % np, kvh = h * NKH / NQH;
        const float* kr = (p0 + j < x.pos) ? Kst + (size_t)j * KV + kvh * HD : t + Q + kvh * HD;
        const float* qh = t + h * HD;
        float d = 0.f;
        for (int i = lane; i < HD; i += 32) d = fmaf(qh[i], kr[i], d);
        d = warp_sum(d);
        if (lane == 0) x.S.sc[h * PPS + j] = d * m.attn_scale;
      }
      cbar();
      if (tid < NQH) {  // local softmax statistics of this split
        int h = tid;
        float mx = -1e30f;
        for (int j = 0; j < np; j++) mx = fmaxf(mx, x.S.sc[h * PPS + j]);
        float sum = 0.f;
        for (int j = 0; j < np; j++) {
          float ev = expf(x.S.sc[h * PPS + j] - mx);
          x.S.sc[h * PPS + j] = ev;
          sum += ev;
        }
        tag_store(m.t_ml + ((size_t)s * NQH + h) * 2 + 0, mx, tag);
        tag_store(m.t_ml + ((size_t)s * NQH + h) * 2 + 1, sum, tag);
      }
      cbar();
      for (int o = tid; o < NQH * HD; o += NCT) {  // (shaders.ts:302-325)
        int h = o / HD, dd = o % HD, kvh = h * NKH / NQH;
        float acc = 0.f;
        for (int j = 0; j < np; j++) {
          const float* vr = (p0 + j < x.pos) ? Vst + (size_t)j * KV : t + Q + KV;
          acc = fmaf(x.S.sc[h * PPS + j], vr[kvh * HD + dd], acc);
        }
        tag_store(m.t_o + (size_t)s * Q + o, acc, tag);
      }
      stage_release();
      cbar();
    }
  }

  GG_DEV void phase_combine(int l) {
    const GGModelDev& m = *x.m;
    const int Q = m.Q, HD = m.HD, NQH = m.NQH, DPC = m.dims_per_comb;
    const uint32_t tagB = make_tag(x.tagbase, l * PH_PER_LAYER + 1);
    const uint32_t tagC = make_tag(x.tagbase, l * PH_PER_LAYER + 2);
    float* cm = x.S.cmb;
    float* cl = cm + m.max_splits;
    float* cw = cl + m.max_splits;
    for (int cc = blockIdx.x; cc < m.ncomb; cc += m.grid) {
      const int d0 = cc * DPC, h = d0 / HD;
      for (int s = tid; s < x.nsplit; s += NCT) {
        cm[s] = tag_wait(m.t_ml + ((size_t)s * NQH + h) * 2 + 0, tagB, x.sc);
        cl[s] = tag_wait(m.t_ml + ((size_t)s * NQH + h) * 2 + 1, tagB, x.sc);
      }
      cbar();
      if (warp == 0) {
        float mx = -INFINITY;
        for (int s = lane; s < x.nsplit; s += 32) mx = fmaxf(mx, cm[s]);
        mx = warp_max(mx);
        float lsum = 0.f;
        for (int s = lane; s < x.nsplit; s += 32) {
          float w = expf(cm[s] - mx);
          cw[s] = w;
          lsum = fmaf(w, cl[s], lsum);
        }
        lsum = warp_sum(lsum);
        if (lane == 0) x.S.scal[127] = lsum;
      }
      cbar();
      const float inv = 1.0f / x.S.scal[127];
      for (int k = warp; k < DPC; k += NCW) {
        const int d = d0 + k;
        float acc = 0.f;
        for (int s = lane; s < x.nsplit; s += 32)
          acc = fmaf(cw[s], tag_wait(m.t_o + (size_t)s * Q + d, tagB, x.sc), acc);
        acc = warp_sum(acc);
        if (lane == 0) tag_store(m.t_att + d, acc * inv, tagC);
      }
      cbar();
    }
  }

  GG_DEV void phase_o(int l) {
    const GGModelDev& m = *x.m;
    cbar();  // x vector is about to be overwritten
    gather(m.t_att, m.Q, make_tag(x.tagbase, l * PH_PER_LAYER + 2), x.S.xs, true);
    cbar();
    int b, e;
    part(m.H, m.grid, blockIdx.x, b, e);
    const uint32_t tag = make_tag(x.tagbase, l * PH_PER_LAYER + 3);
    uint64_t* out = m.t_proj;
    if (m.ks_o > 1)
      rows_ksn(b, e, m.rps_q, m.Q, m.rs_q, m.ks_o, [&](int row, float v) { tag_store(out + row, v, tag); });
    else
      rows_ks1(b, e, m.rps_q, m.Q, m.rs_q, [&](int row, float v) {
        if (lane == 0) tag_store(out + row, v, tag);
      });
  }

  GG_DEV void phase_ffn_up(int l) {
    const GGModelDev& m = *x.m;
    const GGLayerW& Lw = m.layers[l];
    gather(m.t_proj, m.H, make_tag(x.tagbase, l * PH_PER_LAYER + 3), x.S.tmp, false);
    cbar();
    // residual = hidden + post_attention_norm(proj)  (engine.ts:785)
    norm_add(x.S.tmp, Lw.post_attn_norm, x.S.hid, x.S.res, m.H);
    cbar();
    if (blockIdx.x == 0)
      for (int i = tid; i < m.H; i += NCT) m.dbg_residual[i] = x.S.res[i];
    norm_to_xs(x.S.res, Lw.ffn_norm, m.H);  // engine.ts:786
    cbar();
    int b, e;
    part(m.I, m.grid, blockIdx.x, b, e);
    const uint32_t tag = make_tag(x.tagbase, l * PH_PER_LAYER + 4);
    const int npair = e - b, pps = m.pps_gu, rs = m.rs_h;
    for (int q0 = 0; q0 < npair; q0 += pps) {
      const uint8_t* stg = stage_acquire();
      const int q1 = min(q0 + pps, npair);
      for (int u = q0 + ((warp - q0) % NCW + NCW) % NCW; u < q1; u += NCW) {
        const uint8_t* rg = stg + (size_t)(2 * (u - q0)) * rs;
        float g, up;
        row_dot2(rg, rg + rs, m.H, x.S.xs4, lane, g, up);
        if (lane == 0) tag_store(m.t_act + b + u, gelu_tanh(g) * up, tag);  // shaders.ts:153-170
      }
      stage_release();
    }
  }

  GG_DEV void phase_down(int l) {
    const GGModelDev& m = *x.m;
    cbar();
    gather(m.t_act, m.I, make_tag(x.tagbase, l * PH_PER_LAYER + 4), x.S.xs, true);
    cbar();
    int b, e;
    part(m.H, m.grid, blockIdx.x, b, e);
    const uint32_t tag = make_tag(x.tagbase, l * PH_PER_LAYER + 5);
    uint64_t* out = m.t_down;
    if (m.ks_down > 1)
      rows_ksn(b, e, m.rps_i, m.I, m.rs_i, m.ks_down, [&](int row, float v) { tag_store(out + row, v, tag); });
    else
      rows_ks1(b, e, m.rps_i, m.I, m.rs_i, [&](int row, float v) {
        if (lane == 0) tag_store(out + row, v, tag);
      });
  }

  GG_DEV void phase_lm() {
    const GGModelDev& m = *x.m;
    if (x.mode & GG_RUN_LAYERS) {
      finish_layer(m.L - 1);
    } else {  // LM head on the state a previous launch left behind
      for (int i = tid; i < m.H; i += NCT) x.S.hid[i] = m.dbg_hidden[i];
      cbar();
    }
    norm_to_xs(x.S.hid, m.out_norm, m.H);  // engine.ts:797-801
    for (int i = tid; i < 256; i += NCT) x.S.keys[i] = init_lane_key();
    cbar();
    if (blockIdx.x == 0)
      for (int i = tid; i < m.H; i += NCT) {
        m.dbg_normed[i] = x.S.xs[xs_index(i)];
        m.dbg_hidden[i] = x.S.hid[i];
      }
    int b, e;
    part(m.V, m.grid, blockIdx.x, b, e);
    float* logits = m.logits;
    unsigned long long* keys = x.S.keys;
    rows_ks1(b, e, m.rps_h, m.H, m.rs_h, [&](int row, float v) {
      if (lane == 0) {
        logits[row] = v;
        if (!isnan(v)) {  // topk256 lane rule: strict '>' from (-1e30, 0), first index wins
          unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - (uint32_t)row);
          atomicMax(&keys[row & 255], k);
        }
      }
    });
    cbar();
    const unsigned long long ik = init_lane_key();
    for (int i = tid; i < 256; i += NCT)
      if (x.S.keys[i] != ik) atomicMax(&m.lane_keys[i], x.S.keys[i]);
  }

  GG_DEV void run() {
    const GGModelDev& m = *x.m;
    if (x.mode & GG_RUN_LAYERS) {
      for (int l = 0; l < m.L; l++) {
        phase_qkv(l);
        phase_attn(l);
        phase_combine(l);
        phase_o(l);
        phase_ffn_up(l);
        phase_down(l);
      }
      if (!(x.mode & GG_RUN_LM)) {  // leave hidden/residual for a later LM-head launch
        finish_layer(m.L - 1);
      }
    }
    if (x.mode & GG_RUN_LM) phase_lm();
  }
};

// ---------------------------------------------------------------------------------- sampler

// Runs in the last CTA to finish, all GG_NTHREADS threads. engine.ts:823-901.
GG_DEV int sample_token(const GGModelDev& m, GGState* st, Smem& S) {
  __shared__ double sv[256];
  __shared__ int sl[256];
  __shared__ int result;
  const int tid = threadIdx.x;
  const int seq = st->seq;
  float val = 0.f;
  uint32_t idx = 0;
  if (tid < 256) {
    unsigned long long k = __ldcg(&m.lane_keys[tid]);
    val = f32_from_order_key((uint32_t)(k >> 32));
    idx = 0xffffffffu - (uint32_t)k;
  }
  const float T = st->temperature, rep = st->rep_penalty;
  if (T == 0.0f && rep <= 1.0f) {
    // argmax (shaders.ts:327-361): max value, ties -> lowest lane
    __shared__ unsigned long long wk[8];
    unsigned long long key = 0;
    if (tid < 256) key = ((unsigned long long)f32_order_key(val) << 32) | (uint32_t)(255 - tid);
    if (tid < 256) {
      for (int o = 16; o > 0; o >>= 1) {
        unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
      }
      if ((tid & 31) == 0) wk[tid >> 5] = key;
    }
    __syncthreads();
    if (tid == 0) {
      unsigned long long best = wk[0];
      for (int w = 1; w < 8; w++) best = wk[w] > best ? wk[w] : best;
      int lane = 255 - (int)(uint32_t)(best & 0xffffffffu);
      result = lane;
    }
    __syncthreads();
    int lane = result;
    __syncthreads();
    if (tid == lane) result = (int)idx;
    __syncthreads();
    return result;
  }
  // Candidate values in double, repetition penalty on this turn's tokens (engine.ts:868-876)
  if (tid < 256) {
    double v = (double)val;
    const uint8_t* seen = m.seen + (size_t)seq * m.seen_stride;
    if (rep > 1.0f && st->seen_count > 0 && idx < (uint32_t)m.V && (seen[idx >> 3] >> (idx & 7)) & 1)
      v = v > 0 ? v / (double)rep : v * (double)rep;
    sv[tid] = v;
    sl[tid] = tid;
  }
  __syncthreads();
  // Stable descending sort == sort by (value desc, lane asc): bitonic network on that total order.
  for (int k = 2; k <= 256; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (tid < 256) {
        int p = tid ^ j;
        if (p > tid) {
          double a = sv[tid], bb = sv[p];
          int la = sl[tid], lb = sl[p];
          bool a_first = (a > bb) || (a == bb && la < lb);
          bool up = (tid & k) == 0;
          if (up != a_first) {
            sv[tid] = bb; sv[p] = a; sl[tid] = lb; sl[p] = la;
          }
        }
      }
      __syncthreads();
    }
  }
  __shared__ uint32_t cid[256];
  if (tid < 256) cid[tid] = idx;
  __syncthreads();
  if (tid == 0) {
    int pick;
    if (T == 0.0f) {
      pick = 0;
    } else {
      // engine.ts:881-901, JS numbers are doubles; probs is a Float32Array
      const double temp = (double)T, top_p = (double)st->top_p;
      __shared__ float probs[256];
      double mx = sv[0], sum = 0.0;
      for (int i = 0; i < 256; i++) {
        probs[i] = (float)exp((sv[i] - mx) / temp);
        sum += (double)probs[i];
      }
      double cum = 0.0;
      int cutoff = 256;
      for (int i = 0; i < 256; i++) {
        cum += (double)probs[i] / sum;
        if (cum >= top_p) { cutoff = i + 1; break; }
      }
      double sub = 0.0;
      for (int i = 0; i < cutoff; i++) sub += (double)probs[i];
      double u = st->uniforms ? st->uniforms[0] : st->uniform;
      double r = u * sub;
      pick = cutoff - 1;
      for (int i = 0; i < cutoff; i++) {
        r -= (double)probs[i];
        if (r <= 0) { pick = i; break; }
      }
    }
    result = (int)cid[sl[pick]];
  }
  __syncthreads();
  return result;
}

// ---------------------------------------------------------------------------------- kernel

extern "C" __global__ void __launch_bounds__(GG_NTHREADS, 1)
    gg_decode_kernel(const GGModelDev* __restrict__ mp, GGState* __restrict__ st) {
  extern __shared__ __align__(128) uint8_t smem[];
  const GGModelDev& m = *mp;
  Ctx x;
  x.m = mp;
  x.st = st;
  x.mode = st->mode;
  x.token = st->token;
  x.pos = st->pos;
  x.seq = st->seq;
  x.tagbase = st->epoch;
  x.sc.err = &st->error;
  x.sc.timeout_ns = st->timeout_ns;
  x.idx = 0;
  // carve shared memory
  uint8_t* p = smem;
  x.S.ring = p; p += (size_t)m.nstages * m.stage_bytes;
  x.S.full = reinterpret_cast<uint64_t*>(p); p += 8 * m.nstages;
  x.S.empty = reinterpret_cast<uint64_t*>(p); p += 8 * m.nstages;
  x.S.keys = reinterpret_cast<unsigned long long*>(p); p += 8 * 256;
  x.S.xs4 = reinterpret_cast<float4*>(p); x.S.xs = reinterpret_cast<float*>(p); p += 4 * (size_t)m.xs_floats;
  x.S.hid = reinterpret_cast<float*>(p); p += 4 * (size_t)m.H;
  x.S.res = reinterpret_cast<float*>(p); p += 4 * (size_t)m.H;
  x.S.tmp = reinterpret_cast<float*>(p); p += 4 * (size_t)m.tmp_floats;
  x.S.cs = reinterpret_cast<float*>(p); p += 4 * (size_t)m.HD;
  x.S.red = reinterpret_cast<float*>(p); p += 4 * 1024;
  x.S.sc = reinterpret_cast<float*>(p); p += 4 * (size_t)(m.NQH * m.pos_per_split + 32);
  x.S.cmb = reinterpret_cast<float*>(p); p += 4 * (size_t)(3 * m.max_splits);
  x.S.scal = reinterpret_cast<float*>(p); p += 4 * 128;
  x.S.flag = reinterpret_cast<int*>(p); p += 16;

  const bool bad = x.token < 0 || x.token >= m.V || x.pos < 0 || x.pos >= m.CTX || x.seq < 0 || x.seq >= m.max_seqs;
  if (bad) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&st->error, GG_ERR_BAD_INPUT);
    x.mode = 0;
  }
  x.nsplit = (x.pos + m.pos_per_split) / m.pos_per_split;  // ceil((pos + 1) / PPS)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < m.nstages; i++) {
      mbar_init(&x.S.full[i], 1);
      mbar_init(&x.S.empty[i], NCW);
    }
    mbar_fence_init();
  }
  __syncthreads();

  if (warp == NCW) {
    if (lane == 0) {
      Producer pr{x, l2_policy_evict_first()};
      pr.run();
    }
  } else {
    Consumer cs{x, (int)threadIdx.x, lane, warp};
    cs.run();
  }
  __syncthreads();

  // End of launch: the last CTA to arrive runs the sampler and hands the state on.
  if (threadIdx.x == 0) {
    __threadfence();
    uint32_t t = atomicAdd(&st->done, 1u);
    *x.S.flag = (t == (uint32_t)m.grid - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!*x.S.flag) return;
  __threadfence();
  int tok = -1;
  if (x.mode & GG_RUN_SAMPLE) tok = sample_token(m, st, x.S);
  __syncthreads();
  if (threadIdx.x < 256) m.lane_keys[threadIdx.x] = init_lane_key();
  if (threadIdx.x == 0) {
    st->epoch = st->epoch + (uint32_t)(m.L * PH_PER_LAYER + 1);
    st->done = 0;
    if (x.mode & GG_RUN_SAMPLE) {
      st->out_token = tok;
      if (tok >= 0 && tok < m.V) {
        uint8_t* seen = m.seen + (size_t)x.seq * m.seen_stride;
        seen[tok >> 3] |= (uint8_t)(1u << (tok & 7));
        st->seen_count = st->seen_count + 1;
      }
      if (st->token_ring && st->ring_len > 0) st->token_ring[st->step_index % st->ring_len] = tok;
      st->step_index = st->step_index + 1;
      if (st->uniforms) st->uniforms = st->uniforms + 1;
      st->token = tok;
      st->pos = x.pos + 1;
    } else if (x.mode & GG_PREFILL_ADVANCE) {
      if (st->prefill_left > 0) {
        st->token = *st->prefill_ids;
        st->prefill_ids = st->prefill_ids + 1;
        st->prefill_left = st->prefill_left - 1;
      }
      st->pos = x.pos + 1;
    }
  }
}

}  // namespace gg
