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
//   A  post-ffw norm + residual of the previous layer, rmsNorm, fused QKV matvec
//                                                     (shaders.ts:25-56, 92-151, 386-418)
//   B  q/k per-head norm + RoPE, KV store, split attention       (shaders.ts:209-325, 420-467)
//   B2 merge of the attention splits (online softmax)
//   C  O projection                                              (shaders.ts:92-151)
//   D  post-attn norm + residual, ffn rmsNorm, gate/up + GeGLU   (shaders.ts:153-170, 386-418)
//   E  down projection                                           (shaders.ts:92-151)
// then F: post-ffw norm + residual, final rmsNorm, tied LM head with per-lane maxima
// (engine.ts:797-821, shaders.ts:327-384), and the sampler in the last CTA (engine.ts:823-901).
//
// Matvec arithmetic: x is held as 24-bit fixed point per 16-element chunk in three byte
// planes; q . x is three exact int32 dp4a sums per chunk, recombined in f32 and scaled by the
// chunk exponent and the Q8_0 block scale (accumulation order differs from the shader's
// sequential f32 loop; results agree within f32 rounding).
#include "gg_device.cuh"
#include "gg_launch.h"
#include "gg_model.h"

namespace gg {

constexpr int NCW = GG_NCW;
constexpr int NCT = GG_NCT;
constexpr int PH_PER_LAYER = 6;
constexpr uint32_t NS = GG_RING_STAGES;  // ring slots (GGModelDev::nstages holds the same value)

GG_DEV void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

GG_DEV uint32_t make_tag(uint32_t base, int phase) { return 0x80000000u | ((base + (uint32_t)phase) & 0x7fffffffu); }

// Rows [b, e) of M that CTA c of G takes. 32-bit: the host checks grid * rows < 2^31.
GG_DEV void part(int M, int G, int c, int& b, int& e) {
  b = (int)(((uint32_t)c * (uint32_t)M) / (uint32_t)G);
  e = (int)(((uint32_t)(c + 1) * (uint32_t)M) / (uint32_t)G);
}

// This CTA's share of each matvec, computed once per launch (Smem::rows): the range is the same
// in every layer, and recomputing it after each phase's barrier would put two integer divisions
// on every hand-over's critical path.
enum { RG_QKV = 0, RG_H = 2, RG_I = 4, RG_V = 6, RG_N = 8 };

// x operand of the dot products: each 16-element chunk as 24-bit fixed point (shared exponent)
// split into three byte planes; p0 holds the signed top byte, p1/p2 the unsigned lower bytes.
struct XPlanes {
  uint8_t* p0;
  uint8_t* p1;
  uint8_t* p2;
  float* inv;  // 2^(e-23) per chunk: multiply the integer dot by this to get back to x's scale
};

struct Smem {
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  XPlanes xp[2];  // double buffer: a phase builds one while the previous phase may still read the other
  float* hid;     // residual stream (hidden state), identical in every CTA
  float* res;     // residual after the attention block
  float* tmp;     // attention: q | k | v of the current token
  float* red;     // K-slice partial sums
  int* rcnt;      // per-row count of finished K-slices
  unsigned long long* keys;
  float* scal;
  int* flag;
  int* rows;  // [RG_N]: [b, e) of the q/k/v rows, the H rows (O, down), the I gate/up pairs, the V rows
};

GG_DEV unsigned long long init_lane_key() {
  return ((unsigned long long)f32_order_key(-1e30f) << 32) | 0xffffffffull;
}

GG_DEV void ld2_volatile(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// Dot products of R Q8_0 rows (rowp, rowp + rs, ...) with x over the rows' 16-byte chunks
// [c0, c1), by a group of GS lanes (gl = lane within the group): sum over chunks of
// d_block * (q . x). The int8 x int8 products of q with the three byte planes of x accumulate
// exactly in int32 (dp4a); the three partial sums are recombined in f32 and scaled by the
// chunk's exponent and the block scale. The R rows share the loads of the x planes. Every
// lane of the group receives the row totals.
template <int GS, int R>
GG_DEV void group_dot(const uint8_t* rowp, int rs, int K, const XPlanes& P, int c0, int c1, int gl, float* out) {
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; r++) acc[r] = 0.f;
#pragma unroll 3
  for (int c = c0 + gl; c < c1; c += GS) {
    const uint4 a0 = *reinterpret_cast<const uint4*>(P.p0 + 16 * c);
    const uint4 a1 = *reinterpret_cast<const uint4*>(P.p1 + 16 * c);
    const uint4 a2 = *reinterpret_cast<const uint4*>(P.p2 + 16 * c);
    const float is = P.inv[c];
#pragma unroll
    for (int r = 0; r < R; r++) {
      const uint8_t* rp = rowp + (size_t)r * rs;
      const uint4 w = *reinterpret_cast<const uint4*>(rp + 16 * c);
      const float sc = __half2float(*reinterpret_cast<const __half*>(rp + K + 2 * (c >> 1))) * is;
      int s0 = dp4a_ss((int)w.x, (int)a0.x, 0);
      s0 = dp4a_ss((int)w.y, (int)a0.y, s0);
      s0 = dp4a_ss((int)w.z, (int)a0.z, s0);
      s0 = dp4a_ss((int)w.w, (int)a0.w, s0);
      int s1 = dp4a_su((int)w.x, (int)a1.x, 0);
      s1 = dp4a_su((int)w.y, (int)a1.y, s1);
      s1 = dp4a_su((int)w.z, (int)a1.z, s1);
      s1 = dp4a_su((int)w.w, (int)a1.w, s1);
      int s2 = dp4a_su((int)w.x, (int)a2.x, 0);
      s2 = dp4a_su((int)w.y, (int)a2.y, s2);
      s2 = dp4a_su((int)w.z, (int)a2.z, s2);
      s2 = dp4a_su((int)w.w, (int)a2.w, s2);
      acc[r] = fmaf(fmaf((float)s0, 65536.f, (float)(s1 * 256 + s2)), sc, acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < R; r++) {
#pragma unroll
    for (int o = GS / 2; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
    out[r] = acc[r];
  }
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

// First attention split holding a position inside this layer's window, and the first such
// position (0, 0 when the layer attends the whole prefix).
GG_DEV int window_lo(const GGLayerW& Lw, int pos) {
  return (Lw.window > 0 && pos + 1 > Lw.window) ? pos + 1 - Lw.window : 0;
}

template <bool KV16>
struct Producer {
  Ctx& x;
  uint64_t pol;
  bool ok = true;

  GG_DEV void issue(const void* s0, uint32_t b0, const void* s1, uint32_t b1, uint32_t off1) {
    const GGModelDev& m = *x.m;
    int slot = x.idx % NS;
    uint32_t use = x.idx / NS;
    if (use > 0 && ok) ok = mbar_wait(&x.S.empty[slot], (use - 1) & 1, x.sc);
    if (!ok) return;
    uint8_t* dst = x.S.ring + (size_t)slot * m.stage_bytes;
    if ((x.mode & GG_TRACE) && blockIdx.x == 0 && x.idx < 480)  // stage issue times (CTA 0)
      m.trace[(size_t)160 * 4 + x.idx] = global_timer_ns();
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
    if (x.mode & GG_RUN_LAYERS) {
      for (int l = 0; l < m.L && ok; l++) {
        const GGLayerW& Lw = m.layers[l];
        rows(Lw.wqkv, m.rs_h, x.S.rows[RG_QKV], x.S.rows[RG_QKV + 1], m.ph_qkv.rps);
        const int rot = (l * x.nsplit) % G, slo = window_lo(Lw, x.pos) / m.pos_per_split;
        for (int s = slo + (c - rot + G) % G; s < x.nsplit && ok; s += G) {
          int p0 = s * m.pos_per_split, pc = min(p0 + m.pos_per_split, x.pos);
          constexpr int es = KV16 ? 2 : 4;  // bytes per cache element
          uint32_t nb = pc > p0 ? (uint32_t)((pc - p0) * m.KV * es) : 0u;
          size_t off = ((size_t)x.seq * m.kv_seq_stride + ((size_t)l * m.CTX + p0) * m.KV) * es;
          issue(m.kcache + off, nb, m.vcache + off, nb, (uint32_t)(m.pos_per_split * m.KV * es));
        }
        const int hb = x.S.rows[RG_H], he = x.S.rows[RG_H + 1];
        rows(Lw.wo, m.rs_q, hb, he, m.ph_o.rps);
        rows(Lw.wgu, m.rs_h, 2 * x.S.rows[RG_I], 2 * x.S.rows[RG_I + 1], 2 * m.pps_gu);
        rows(Lw.wdown, m.rs_i, hb, he, m.ph_down.rps);
      }
    }
    if ((x.mode & GG_RUN_LM) && ok) {
      rows(m.embd, m.rs_h, x.S.rows[RG_V], x.S.rows[RG_V + 1], m.ph_lm.rps);
    }
    // Drain: wait until every copy issued into the ring has landed before the CTA may exit.
    SpinCtl drain = x.sc;
    uint32_t n = x.idx < NS ? x.idx : NS;
    for (uint32_t k = x.idx - n; k < x.idx; k++) {
      int slot = k % NS;
      uint32_t par = (k / NS) & 1;
      uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&x.S.full[slot], par)) {
        if (global_timer_ns() - t0 > drain.timeout_ns) { atomicOr(drain.err, GG_ERR_WAIT_MBAR); break; }
      }
    }
  }
};

// ---------------------------------------------------------------------------------- consumers

// KV16: the KV cache holds bf16 elements (GG_FLAG_KV_BF16); one kernel is built per element
// type so neither carries the other's attention code.
template <bool KV16>
struct Consumer {
  Ctx& x;
  int tid, lane, warp;
  // Once a ring wait gives up, this warp stops waiting on and releasing slots, so the
  // producer can never refill a slot whose copy might still be landing; it drains and exits.
  bool dead = false;
  uint64_t ring_wait_ns = 0;  // trace: time warp 0 spent waiting for ring slots in this phase
  int cslot = 0;              // rotating scratch slot of csum

  GG_DEV uint8_t* stage_acquire() {
    const GGModelDev& m = *x.m;
    int slot = x.idx % NS;
    if (!dead) {
      const bool tr = (x.mode & GG_TRACE) && tid == 0;
      const uint64_t t0 = tr ? global_timer_ns() : 0;
      bool ok = mbar_wait(&x.S.full[slot], (x.idx / NS) & 1, x.sc);
      dead = !__all_sync(0xffffffffu, ok);
      if (tr) ring_wait_ns += global_timer_ns() - t0;
      if (tr && blockIdx.x == 0 && x.idx < 480) {  // stage acquire times of warp 0 (CTA 0)
        x.m->trace[(size_t)300 * 4 + x.idx] = global_timer_ns();
        x.m->trace[(size_t)420 * 4 + x.idx] = t0;
      }
    }
    return x.S.ring + (size_t)slot * m.stage_bytes;
  }
  GG_DEV void stage_release() {
    __syncwarp();
    if (lane == 0 && !dead) mbar_arrive(&x.S.empty[x.idx % NS]);
    x.idx++;
  }

  // Trace stamps (GG_TRACE launches only): globaltimer of event ev (0 enter, 1 inputs ready,
  // 2 done) of phase ph, per CTA: trace[(cta * GG_TRACE_PHASES + ph) * 4 + ev]; event 3 holds
  // the ring-wait time of warp 0 during the phase.
  GG_DEV void trace(int ph, int ev) {
    if ((x.mode & GG_TRACE) && ev == 2) cbar();  // "done" = every warp of the CTA finished the phase
    if ((x.mode & GG_TRACE) && tid == 0 && ph < GG_TRACE_PHASES) {
      unsigned long long* t = x.m->trace + ((size_t)blockIdx.x * GG_TRACE_PHASES + ph) * 4;
      t[ev] = global_timer_ns();
      if (ev == 2) {
        t[3] = ring_wait_ns;
        ring_wait_ns = 0;
      }
    }
  }

  // Four consecutive tagged words (16-byte aligned): two vector loads, re-polled as vectors
  // until every tag matches. Bounded: on timeout (or an error raised elsewhere) the missing
  // words read as 0 and the error word is set.
  GG_DEV void load4(const uint64_t* p, uint32_t tag, float* v) {
    uint64_t w0, w1, w2, w3;
    ld2_volatile(p, w0, w1);
    ld2_volatile(p + 2, w2, w3);
    bool a = (uint32_t)(w0 >> 32) == tag && (uint32_t)(w1 >> 32) == tag;
    bool b = (uint32_t)(w2 >> 32) == tag && (uint32_t)(w3 >> 32) == tag;
    for (int it = 0; it < 512 && !(a && b); ++it) {  // fast path: polls only, no clock reads
      if (!a) {
        ld2_volatile(p, w0, w1);
        a = (uint32_t)(w0 >> 32) == tag && (uint32_t)(w1 >> 32) == tag;
      }
      if (!b) {
        ld2_volatile(p + 2, w2, w3);
        b = (uint32_t)(w2 >> 32) == tag && (uint32_t)(w3 >> 32) == tag;
      }
    }
    if (!(a && b)) {
      const uint64_t t0 = global_timer_ns();
      for (uint32_t it = 1; !(a && b); ++it) {
        if (!a) {
          ld2_volatile(p, w0, w1);
          a = (uint32_t)(w0 >> 32) == tag && (uint32_t)(w1 >> 32) == tag;
        }
        if (!b) {
          ld2_volatile(p + 2, w2, w3);
          b = (uint32_t)(w2 >> 32) == tag && (uint32_t)(w3 >> 32) == tag;
        }
        if ((it & 31u) == 0) {
          const uint64_t dt = global_timer_ns() - t0;
          if (dt > GG_QUIET_SPIN_NS && (*(volatile uint32_t*)x.sc.err || dt > x.sc.timeout_ns)) {
            if (dt > x.sc.timeout_ns) atomicOr(x.sc.err, GG_ERR_WAIT_FLAG);
            w0 = w1 = w2 = w3 = 0;
            break;
          }
        }
      }
    }
    v[0] = __uint_as_float((uint32_t)w0);
    v[1] = __uint_as_float((uint32_t)w1);
    v[2] = __uint_as_float((uint32_t)w2);
    v[3] = __uint_as_float((uint32_t)w3);
  }

  // NV sums over the consumer threads with one barrier; every thread of warps 0..nw-1 gets the
  // same totals (same summation order everywhere). Scratch slots rotate, so no second barrier.
  // Only warps 0..nw-1 hold data: the others (whose values are all zero) only take part in
  // the barrier and leave v as it is; skipping their zero terms leaves every total unchanged.
  template <int NV>
  GG_DEV void csum(float* v, int nw) {
    // slot layout [warp][4]: a warp's NV (<= 4) partials are one 16-byte store and load
    static_assert(NV <= 4, "at most four sums per call");
    float4* s = reinterpret_cast<float4*>(x.S.scal) + (cslot & 3) * 16;
    cslot++;
    if (warp < nw) {
      float t[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int k = 0; k < NV; k++) t[k] = warp_sum(v[k]);
      if (lane == 0) s[warp] = make_float4(t[0], t[1], t[2], t[3]);
    }
    cbar();
    if (warp < nw) {
      float t[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < NCW; w++)
        if (w < nw) {
          const float4 f = s[w];
          t[0] += f.x; t[1] += f.y; t[2] += f.z; t[3] += f.w;
        }
#pragma unroll
      for (int k = 0; k < NV; k++) v[k] = t[k];
    }
  }

  // One element quad (4 consecutive x values) of the planes, by the thread owning quad k.
  // The four quads of a 16-element chunk sit on four consecutive lanes and share the chunk
  // maximum by shuffles, so every lane of the warp must call this (ok = false: no quad).
  // Chunk c: e = exponent of max|x| (max|x| < 2^e), X = round(x * 2^(23-e)) in (-2^23, 2^23),
  // X = 65536*p0 + 256*p1 + p2.
  GG_DEV void plane_quad(const XPlanes& P, int k, bool ok, const float* v) {
    float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    if (!ok) return;
    const int e = max((int)((__float_as_uint(mx) >> 23) & 255) - 126, -100);
    const float s = __int_as_float((127 + 23 - e) << 23);
    uint32_t X[4];
#pragma unroll
    for (int j = 0; j < 4; j++) X[j] = (uint32_t)min(max(__float2int_rn(v[j] * s), -8388607), 8388607);
    // byte b of X[j] goes to byte j of plane 2 - b (b = 0, 1, 2: the 24-bit two's complement)
    const uint32_t lo01 = __byte_perm(X[0], X[1], 0x5140), lo23 = __byte_perm(X[2], X[3], 0x5140);
    const uint32_t hi01 = __byte_perm(X[0], X[1], 0x0062), hi23 = __byte_perm(X[2], X[3], 0x0062);
    const uint32_t b2 = __byte_perm(lo01, lo23, 0x5410), b1 = __byte_perm(lo01, lo23, 0x7632);
    const uint32_t b0 = __byte_perm(hi01, hi23, 0x5410);
    reinterpret_cast<uint32_t*>(P.p0)[k] = b0;
    reinterpret_cast<uint32_t*>(P.p1)[k] = b1;
    reinterpret_cast<uint32_t*>(P.p2)[k] = b2;
    if ((k & 3) == 0) P.inv[k >> 2] = __int_as_float((127 - 23 + e) << 23);
  }

  // Planes straight from n tagged words (no normalisation): phases C and E.
  GG_DEV void planes_tagged(const XPlanes& P, const uint64_t* src, uint32_t tag, int n) {
    const int nq = n >> 2;
    for (int base = 0; base < nq; base += NCT) {
      const int k = base + tid;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (k < nq) load4(src + 4 * k, tag, v);
      plane_quad(P, k, k < nq, v);
    }
  }

  // out = base + v * wa / r1, r1 = rms(v) (shaders.ts:386-418, v = tagged words), then the
  // planes of out * wb / r2, r2 = rms(out) (shaders.ts:25-56). One barrier: the sums of v^2,
  // base^2, base*v*wa and (v*wa)^2 give both norms. The weights are fetched before the wait
  // on v. Thread t owns element quad t (hidden_size <= 4 * GG_NCT).
  GG_DEV void add_norm_planes(const XPlanes& P, const uint64_t* src, uint32_t tag, const float* wa,
                              const float* base, float* out, const float* wb, float* dbg_out, float* dbg_x) {
    const GGModelDev& m = *x.m;
    const int nq = m.H >> 2, k = tid, nw = (nq + 31) >> 5;
    const bool ok = k < nq;
    float4 fa = make_float4(0.f, 0.f, 0.f, 0.f), fb = fa, fbase = fa;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      fa = __ldg(reinterpret_cast<const float4*>(wa) + k);
      fb = __ldg(reinterpret_cast<const float4*>(wb) + k);
      fbase = reinterpret_cast<const float4*>(base)[k];
      load4(src + 4 * k, tag, v);
    }
    const float wav[4] = {fa.x, fa.y, fa.z, fa.w}, wbv[4] = {fb.x, fb.y, fb.z, fb.w};
    const float bv[4] = {fbase.x, fbase.y, fbase.z, fbase.w};
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      const float vw = v[j] * wav[j];
      s[0] += v[j] * v[j];
      s[1] += bv[j] * bv[j];
      s[2] += bv[j] * vw;
      s[3] += vw * vw;
    }
    csum<4>(s, nw);
    if (warp >= nw) return;  // no element quads in this warp: nothing to normalise or store
    const float r1 = sqrtf(s[0] / (float)m.H + m.eps);
    const float ss_out = s[1] + 2.f * s[2] / r1 + s[3] / (r1 * r1);
    const float r2 = sqrtf(ss_out / (float)m.H + m.eps);
    float o[4], xv[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      o[j] = bv[j] + v[j] * wav[j] / r1;
      xv[j] = o[j] * wbv[j] / r2;
    }
    if (ok) {
      reinterpret_cast<float4*>(out)[k] = make_float4(o[0], o[1], o[2], o[3]);
      if (dbg_out) reinterpret_cast<float4*>(dbg_out)[k] = make_float4(o[0], o[1], o[2], o[3]);
      if (dbg_x) reinterpret_cast<float4*>(dbg_x)[k] = make_float4(xv[0], xv[1], xv[2], xv[3]);
    }
    plane_quad(P, k, ok, xv);
  }

  // shaders.ts:2-23: h[i] = q * d * sqrt(H), evaluated left to right in f32; then the planes
  // of rmsNorm(h) * wb.
  GG_DEV void embed_planes(const XPlanes& P, const float* wb) {
    const GGModelDev& m = *x.m;
    const uint8_t* row = m.embd + (size_t)x.token * m.rs_h;
    const float sq = sqrtf((float)m.H);
    const int nq = m.H >> 2, k = tid, nw = (nq + 31) >> 5;
    const bool ok = k < nq;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    float4 fb = make_float4(0.f, 0.f, 0.f, 0.f);
    float s[1] = {0.f};
    if (ok) {
      fb = __ldg(reinterpret_cast<const float4*>(wb) + k);
      const float d = __half2float(*reinterpret_cast<const __half*>(row + m.H + 2 * ((4 * k) >> 5)));
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float qv = (float)(int8_t)row[4 * k + j];
        float vv = qv * d;
        vv = vv * sq;
        o[j] = vv;
        s[0] += vv * vv;
      }
      reinterpret_cast<float4*>(x.S.hid)[k] = make_float4(o[0], o[1], o[2], o[3]);
    }
    csum<1>(s, nw);
    if (warp >= nw) return;
    const float r = sqrtf(s[0] / (float)m.H + m.eps);
    const float wbv[4] = {fb.x, fb.y, fb.z, fb.w};
    float xv[4];
#pragma unroll
    for (int j = 0; j < 4; j++) xv[j] = o[j] * wbv[j] / r;
    plane_quad(P, k, ok, xv);
  }

  // Epilogue of a matvec row: a tagged activation word, or an LM-head logit (+ its lane key).
  enum { EPI_TAG = 0, EPI_LOGIT = 1 };
  GG_DEV void epilogue(int kind, uint64_t* out, uint32_t tag, int row, float v) {
    if (kind == EPI_TAG) {
      tag_store(out + row, v, tag);
    } else {
      x.m->logits[row] = v;
      if (!isnan(v)) {  // topk256 lane rule: strict '>' from (-1e30, 0), first index wins
        if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal under '>': key them alike
        unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - (uint32_t)row);
        atomicMax(&x.S.keys[row & 255], k);
      }
    }
  }

  // Rows [rb, re) of one phase, rps whole rows per ring stage. A unit is 32/GS lane groups x
  // R rows per lane, times one of ks K-slices. Units go round robin over the consumer warps.
  // ks == 1: the epilogue runs on the lane holding a row's total. ks > 1: each slice partial
  // goes to shared memory and the warp that completes a row's last slice sums the partials
  // in slice order and runs the epilogue (no CTA barrier).
  template <int GS, int R>
  GG_DEV void rows_phase(const XPlanes& P, int rb, int re, int rps, int K, int rs, int ks, int kind, uint64_t* out,
                         uint32_t tag) {
    constexpr int UR = (32 / GS) * R;
    const int nrows = re - rb, nch = K >> 4, cpk = nch / ks;
    const int g = lane / GS, gl = lane % GS;
    int ubase = 0;
    for (int r0 = 0; r0 < nrows; r0 += rps) {
      const uint8_t* stg = stage_acquire();
      const int r1 = min(r0 + rps, nrows);
      const int nunits = ((r1 - r0 + UR - 1) / UR) * ks;
      for (int u = ubase + ((warp - ubase) % NCW + NCW) % NCW; u < ubase + nunits; u += NCW) {
        const int lu = u - ubase, grp = lu / ks, sl = lu % ks;
        const int rl = grp * UR + g * R;  // first row (within the stage) of this lane's rows
        float v[R];
        group_dot<GS, R>(stg + (size_t)rl * rs, rs, K, P, sl * cpk, (sl + 1) * cpk, gl, v);
        if (ks == 1) {
          if (gl == 0)
#pragma unroll
            for (int r = 0; r < R; r++)
              if (r0 + rl + r < r1) epilogue(kind, out, tag, rb + r0 + rl + r, v[r]);
        } else {
          if (gl == 0)
#pragma unroll
            for (int r = 0; r < R; r++)
              if (r0 + rl + r < r1) {
                const int row = r0 + rl + r;
                x.S.red[row * ks + sl] = v[r];
                __threadfence_block();
                if (atomicAdd(&x.S.rcnt[row], 1) == ks - 1) {
                  __threadfence_block();
                  float t = 0.f;
                  for (int k = 0; k < ks; k++) t += *(volatile float*)&x.S.red[row * ks + k];
                  x.S.rcnt[row] = 0;
                  epilogue(kind, out, tag, rb + row, t);
                }
              }
        }
      }
      ubase += nunits;
      stage_release();
    }
  }

  GG_DEV void rows_dispatch(const XPlanes& P, const GGPhaseCfg& pc, int rb, int re, int K, int rs, int kind,
                            uint64_t* out, uint32_t tag) {
    if (pc.gs == 8) rows_phase<8, 1>(P, rb, re, pc.rps, K, rs, pc.ks, kind, out, tag);
    else rows_phase<16, 1>(P, rb, re, pc.rps, K, rs, pc.ks, kind, out, tag);
  }

  GG_DEV void phase_qkv(int l) {
    const GGModelDev& m = *x.m;
    const XPlanes& P = x.S.xp[0];
    if (l == 0) {
      embed_planes(P, m.layers[0].attn_norm);
    } else {  // hidden = residual + post_ffw_norm(down) (engine.ts:794), attn rmsNorm (768)
      add_norm_planes(P, m.t_down, make_tag(x.tagbase, (l - 1) * PH_PER_LAYER + 5), m.layers[l - 1].post_ffw_norm,
                      x.S.res, x.S.hid, m.layers[l].attn_norm, blockIdx.x == 0 ? m.dbg_hidden : nullptr, nullptr);
    }
    cbar();
    trace(l * 6 + 0, 1);
    const int b = x.S.rows[RG_QKV], e = x.S.rows[RG_QKV + 1];
    rows_dispatch(P, m.ph_qkv, b, e, m.H, m.rs_h, EPI_TAG, m.t_qkv, make_tag(x.tagbase, l * PH_PER_LAYER + 0));
  }

  // q/k per-head RMSNorm + RoPE (shaders.ts:420-467), the KV store (shaders.ts:209-227) and a
  // split of the attention (shaders.ts:229-325) with local softmax statistics. One warp per
  // head: lane l holds elements l + 32j of its head, so the RoPE pair (i, i + HD/2) is in one
  // lane and nothing needs a barrier except handing the heads to the split loop.
  GG_DEV void phase_attn(int l) {
    const GGModelDev& m = *x.m;
    const int G = m.grid, c = blockIdx.x, rot = (l * x.nsplit) % G;
    const int plo = window_lo(m.layers[l], x.pos), slo = plo / m.pos_per_split;
    int s = slo + (c - rot + G) % G;
    if (s >= x.nsplit) return;
    const int HD = m.HD, NQH = m.NQH, NKH = m.NKH;
    constexpr int NJ = GG_HEAD_DIM / 32;  // elements per lane of a head
    const GGLayerW& Lw = m.layers[l];
    float* t = x.S.tmp;  // q [Q] | k [KV] | v [KV]
    const uint32_t tagA = make_tag(x.tagbase, l * PH_PER_LAYER + 0);
    const int nh = NQH + NKH;
    for (int h = warp; h < nh + NKH; h += NCW) {
      const uint64_t* src = m.t_qkv + h * HD;
      // inputs that do not depend on this step's activations are fetched before the wait
      float nwv[NJ];
      float2 cr[NJ / 2];
      if (h < nh) {
        const float* nw = h < NQH ? Lw.q_norm : Lw.k_norm;
#pragma unroll
        for (int j = 0; j < NJ; j++) nwv[j] = __ldg(nw + lane + 32 * j);
#pragma unroll
        for (int j = 0; j < NJ / 2; j++) cr[j] = __ldg(Lw.rope + (size_t)x.pos * (HD / 2) + lane + 32 * j);
      }
      uint64_t w[NJ];
#pragma unroll
      for (int j = 0; j < NJ; j++) w[j] = tag_load(src + lane + 32 * j);
      float v[NJ];
#pragma unroll
      for (int j = 0; j < NJ; j++)
        v[j] = ((uint32_t)(w[j] >> 32) == tagA) ? __uint_as_float((uint32_t)w[j]) : tag_wait(src + lane + 32 * j, tagA, x.sc);
      if (h < nh) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < NJ; j++) ss += v[j] * v[j];
        const float rms = sqrtf(warp_sum(ss) / (float)HD + m.eps);
#pragma unroll
        for (int j = 0; j < NJ; j++) v[j] = v[j] * nwv[j] / rms;
#pragma unroll
        for (int j = 0; j < NJ / 2; j++) {
          const float cs = cr[j].x, sn = cr[j].y;  // (cos, sin) of pos * freq_i, i = lane + 32 j
          const float x0 = v[j], x1 = v[j + NJ / 2];
          v[j] = x0 * cs - x1 * sn;
          v[j + NJ / 2] = x0 * sn + x1 * cs;
        }
      }
      if (KV16 && h >= NQH) {  // bf16 cache: attention reads the stored (rounded) k, v
#pragma unroll
        for (int j = 0; j < NJ; j++) v[j] = bf16_rne(v[j]);
      }
#pragma unroll
      for (int j = 0; j < NJ; j++) t[h * HD + lane + 32 * j] = v[j];
    }
    cbar();
    trace(l * 6 + 1, 1);
    const uint32_t tag = make_tag(x.tagbase, l * PH_PER_LAYER + 1);
    for (; s < x.nsplit; s += G) {
      const uint8_t* stg = stage_acquire();
      attn_split(l, s, plo, stg, tag);
      stage_release();
    }
  }

  // One split of PPS positions: K rows at the start of the stage, V rows after PPS K rows; the
  // current position's k and v come from the scratch vector instead (stored here as well).
  GG_DEV void attn_split(int l, int s, int plo, const uint8_t* stg, uint32_t tag) {
    using KT = kv_t<KV16>;
    const GGModelDev& m = *x.m;
    const int Q = m.Q, KV = m.KV, HD = m.HD, NQH = m.NQH, NKH = m.NKH, PPS = m.pos_per_split;
    static_assert(GG_HEAD_DIM == 8 * 32, "a lane holds 8 dims of a head");
    const float* t = x.S.tmp;
    const int p0 = s * PPS, p1 = min(p0 + PPS, x.pos + 1), np = p1 - p0;
    const int pv = max(plo - p0, 0);  // positions before pv are outside the window
    const KT* Kst = reinterpret_cast<const KT*>(stg);
    const KT* Vst = reinterpret_cast<const KT*>(stg + (size_t)PPS * KV * sizeof(KT));
    if (p1 == x.pos + 1) {  // this split owns the new position: store it
      const size_t off = (size_t)x.seq * m.kv_seq_stride + ((size_t)l * m.CTX + x.pos) * KV;
      KT* kc = reinterpret_cast<KT*>(m.kcache);
      KT* vc = reinterpret_cast<KT*>(m.vcache);
      for (int i = tid; i < KV; i += NCT) {
        kc[off + i] = kv_narrow<KV16>(t[Q + i]);
        vc[off + i] = kv_narrow<KV16>(t[Q + KV + i]);
      }
    }
    // lane l takes dims 8l..8l+7 of a head: one 16-byte shared load per K or V row
    const auto row8 = [&](const KT* st_row, const float* cur_row, bool cached, float* f) {
      if (cached && KV16) {
        bf16x8_widen(*reinterpret_cast<const uint4*>(st_row + 8 * lane), f);
      } else {
        if (cached) cur_row = reinterpret_cast<const float*>(st_row);  // f32 cache: same as scratch
        const float4 a = reinterpret_cast<const float4*>(cur_row + 8 * lane)[0];
        const float4 b = reinterpret_cast<const float4*>(cur_row + 8 * lane)[1];
        f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
        f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
      }
    };
    // Every position of the split reads a valid row (positions outside [pv, np) read row pv
    // instead and get weight 0), so the eight dot products, their warp sums and the P.V loads
    // carry no per-position branch and overlap. Each warp sum keeps the butterfly order, and a
    // masked position adds an exact zero, so the results equal a loop over the valid rows only.
    const float scale = m.attn_scale;
    for (int h = warp; h < NQH; h += NCW) {
      const int kvh = h * NKH / NQH;
      float qv[8];
      row8(nullptr, t + h * HD, false, qv);
      float sc[GG_POS_PER_SPLIT];
#pragma unroll
      for (int p = 0; p < GG_POS_PER_SPLIT; p++) {
        const int pp = (p >= pv && p < np) ? p : pv;
        float kf[8];
        row8(Kst + (size_t)pp * KV + kvh * HD, t + Q + kvh * HD, p0 + pp < x.pos, kf);
        float d = 0.f;
#pragma unroll
        for (int j = 0; j < 8; j++) d = fmaf(qv[j], kf[j], d);
        sc[p] = d;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int p = 0; p < GG_POS_PER_SPLIT; p++) sc[p] += __shfl_xor_sync(0xffffffffu, sc[p], o);
      float mx = -1e30f;
#pragma unroll
      for (int p = 0; p < GG_POS_PER_SPLIT; p++) {
        sc[p] *= scale;
        if (p >= pv && p < np) mx = fmaxf(mx, sc[p]);
      }
      float sum = 0.f;
#pragma unroll
      for (int p = 0; p < GG_POS_PER_SPLIT; p++) {
        sc[p] = (p >= pv && p < np) ? expf(sc[p] - mx) : 0.f;
        sum += sc[p];
      }
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < GG_POS_PER_SPLIT; p++) {
        const int pp = (p >= pv && p < np) ? p : pv;
        float vf[8];
        row8(Vst + (size_t)pp * KV + kvh * HD, t + Q + KV + kvh * HD, p0 + pp < x.pos, vf);
#pragma unroll
        for (int j = 0; j < 8; j++) acc[j] = fmaf(sc[p], vf[j], acc[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; j++) tag_store(m.t_o + (size_t)s * Q + h * HD + 8 * lane + j, acc[j], tag);
      if (lane == 0) {
        tag_store(m.t_ml + ((size_t)s * NQH + h) * 2 + 0, mx, tag);
        tag_store(m.t_ml + ((size_t)s * NQH + h) * 2 + 1, sum, tag);
      }
    }
  }

  // Merge of the attention splits (online softmax): one warp per output dimension. Every
  // lane loads the (max, sum, value) triples of its splits in one batch; every warp recomputes
  // the head's global max and denominator itself, so no barrier is needed.
  GG_DEV void phase_combine(int l) {
    const GGModelDev& m = *x.m;
    const int Q = m.Q, HD = m.HD, NQH = m.NQH, DPC = m.dims_per_comb;
    const uint32_t tagB = make_tag(x.tagbase, l * PH_PER_LAYER + 1);
    const uint32_t tagC = make_tag(x.tagbase, l * PH_PER_LAYER + 2);
    constexpr int SPL = 4;  // splits per lane per batch
    for (int cc = blockIdx.x; cc < m.ncomb; cc += m.grid) {
      const int d0 = cc * DPC, h = d0 / HD;
      for (int k = warp; k < DPC; k += NCW) {
        const int d = d0 + k;
        float mx = -INFINITY, lsum = 0.f, acc = 0.f;
        for (int s0 = window_lo(m.layers[l], x.pos) / m.pos_per_split; s0 < x.nsplit; s0 += 32 * SPL) {
          uint64_t wm[SPL], wl[SPL], wo[SPL];
#pragma unroll
          for (int q = 0; q < SPL; q++) {
            const int s = s0 + q * 32 + lane;
            if (s < x.nsplit) {
              wm[q] = tag_load(m.t_ml + ((size_t)s * NQH + h) * 2);
              wl[q] = tag_load(m.t_ml + ((size_t)s * NQH + h) * 2 + 1);
              wo[q] = tag_load(m.t_o + (size_t)s * Q + d);
            }
          }
          float fm[SPL], fl[SPL], fo[SPL];
#pragma unroll
          for (int q = 0; q < SPL; q++) {
            const int s = s0 + q * 32 + lane;
            fm[q] = -INFINITY; fl[q] = 0.f; fo[q] = 0.f;
            if (s < x.nsplit) {
              const uint64_t* pm = m.t_ml + ((size_t)s * NQH + h) * 2;
              fm[q] = ((uint32_t)(wm[q] >> 32) == tagB) ? __uint_as_float((uint32_t)wm[q]) : tag_wait(pm, tagB, x.sc);
              fl[q] = ((uint32_t)(wl[q] >> 32) == tagB) ? __uint_as_float((uint32_t)wl[q]) : tag_wait(pm + 1, tagB, x.sc);
              fo[q] = ((uint32_t)(wo[q] >> 32) == tagB) ? __uint_as_float((uint32_t)wo[q])
                                                         : tag_wait(m.t_o + (size_t)s * Q + d, tagB, x.sc);
            }
          }
          // rescale the running (max, sums) to include this batch (online softmax merge)
          float bm = -INFINITY;
#pragma unroll
          for (int q = 0; q < SPL; q++) bm = fmaxf(bm, fm[q]);
          const float nm = fmaxf(mx, bm);
          const float sc0 = (mx == -INFINITY) ? 0.f : expf(mx - nm);
          lsum *= sc0;
          acc *= sc0;
#pragma unroll
          for (int q = 0; q < SPL; q++) {
            if (fm[q] != -INFINITY) {
              const float w = expf(fm[q] - nm);
              lsum = fmaf(w, fl[q], lsum);
              acc = fmaf(w, fo[q], acc);
            }
          }
          mx = nm;
        }
        // merge lanes: global max, then rescale each lane's sums
        const float gm = warp_max(mx);
        const float f = (mx == -INFINITY) ? 0.f : expf(mx - gm);
        lsum = warp_sum(lsum * f);
        acc = warp_sum(acc * f);
        if (lane == 0) tag_store(m.t_att + d, acc / lsum, tagC);
      }
    }
  }

  GG_DEV void phase_o(int l) {
    const GGModelDev& m = *x.m;
    const XPlanes& P = x.S.xp[1];
    planes_tagged(P, m.t_att, make_tag(x.tagbase, l * PH_PER_LAYER + 2), m.Q);
    cbar();
    trace(l * 6 + 3, 1);
    const int b = x.S.rows[RG_H], e = x.S.rows[RG_H + 1];
    rows_dispatch(P, m.ph_o, b, e, m.Q, m.rs_q, EPI_TAG, m.t_proj, make_tag(x.tagbase, l * PH_PER_LAYER + 3));
  }

  GG_DEV void phase_ffn_up(int l) {
    const GGModelDev& m = *x.m;
    const GGLayerW& Lw = m.layers[l];
    const XPlanes& P = x.S.xp[0];
    // residual = hidden + post_attention_norm(proj) (engine.ts:785), then ffn rmsNorm (786)
    add_norm_planes(P, m.t_proj, make_tag(x.tagbase, l * PH_PER_LAYER + 3), Lw.post_attn_norm, x.S.hid, x.S.res,
                    Lw.ffn_norm, blockIdx.x == 0 ? m.dbg_residual : nullptr, nullptr);
    cbar();
    trace(l * 6 + 4, 1);
    const int b = x.S.rows[RG_I], e = x.S.rows[RG_I + 1];
    const uint32_t tag = make_tag(x.tagbase, l * PH_PER_LAYER + 4);
    // gate_i and up_i are adjacent rows: with 8 lanes per row and 2 rows per lane, one lane
    // holds both sums of a pair and applies GeGLU itself (shaders.ts:153-170).
    const int npair = e - b, pps = m.pps_gu, rs = m.rs_h, nch = m.H >> 4;
    const int g = lane >> 3, gl = lane & 7;
    int ubase = 0;
    for (int q0 = 0; q0 < npair; q0 += pps) {
      const uint8_t* stg = stage_acquire();
      const int q1 = min(q0 + pps, npair);
      const int nunits = (q1 - q0 + 3) / 4;  // 4 pairs per warp unit
      const int u_first = ((warp - ubase) % NCW + NCW) % NCW;
      ubase += nunits;
      for (int u = u_first; u < nunits; u += NCW) {
        const int pr = 4 * u + g;  // pair within the stage
        float v[2];
        group_dot<8, 2>(stg + (size_t)(2 * pr) * rs, rs, m.H, P, 0, nch, gl, v);
        if (gl == 0 && q0 + pr < q1) tag_store(m.t_act + b + q0 + pr, gelu_tanh(v[0]) * v[1], tag);
      }
      stage_release();
    }
  }

  GG_DEV void phase_down(int l) {
    const GGModelDev& m = *x.m;
    const XPlanes& P = x.S.xp[1];
    planes_tagged(P, m.t_act, make_tag(x.tagbase, l * PH_PER_LAYER + 4), m.I);
    cbar();
    trace(l * 6 + 5, 1);
    const int b = x.S.rows[RG_H], e = x.S.rows[RG_H + 1];
    rows_dispatch(P, m.ph_down, b, e, m.I, m.rs_i, EPI_TAG, m.t_down, make_tag(x.tagbase, l * PH_PER_LAYER + 5));
  }

  GG_DEV void phase_lm() {
    const GGModelDev& m = *x.m;
    const XPlanes& P = x.S.xp[0];
    for (int i = tid; i < 256; i += NCT) x.S.keys[i] = init_lane_key();
    if (x.mode & GG_RUN_LAYERS) {  // hidden = residual + post_ffw_norm(down), final rmsNorm (engine.ts:797-801)
      add_norm_planes(P, m.t_down, make_tag(x.tagbase, (m.L - 1) * PH_PER_LAYER + 5), m.layers[m.L - 1].post_ffw_norm,
                      x.S.res, x.S.hid, m.out_norm, blockIdx.x == 0 ? m.dbg_hidden : nullptr,
                      blockIdx.x == 0 ? m.dbg_normed : nullptr);
    } else {  // LM head on the hidden state a previous launch left behind
      const int nq = m.H >> 2, k = tid, nw = (nq + 31) >> 5;
      const bool ok = k < nq;
      float h[4] = {0.f, 0.f, 0.f, 0.f};
      float4 fw = make_float4(0.f, 0.f, 0.f, 0.f);
      float s[1] = {0.f};
      if (ok) {
        const float4 f = reinterpret_cast<const float4*>(m.dbg_hidden)[k];
        fw = __ldg(reinterpret_cast<const float4*>(m.out_norm) + k);
        h[0] = f.x; h[1] = f.y; h[2] = f.z; h[3] = f.w;
#pragma unroll
        for (int j = 0; j < 4; j++) s[0] += h[j] * h[j];
        reinterpret_cast<float4*>(x.S.hid)[k] = f;
      }
      csum<1>(s, nw);
      if (warp < nw) {
        const float r = sqrtf(s[0] / (float)m.H + m.eps);
        const float wv[4] = {fw.x, fw.y, fw.z, fw.w};
        float xv[4];
#pragma unroll
        for (int j = 0; j < 4; j++) xv[j] = h[j] * wv[j] / r;
        if (ok && blockIdx.x == 0) reinterpret_cast<float4*>(m.dbg_normed)[k] = make_float4(xv[0], xv[1], xv[2], xv[3]);
        plane_quad(P, k, ok, xv);
      }
    }
    cbar();
    const int b = x.S.rows[RG_V], e = x.S.rows[RG_V + 1];
    // Two rows per 8-lane group: each load of the x planes serves both rows' dot products,
    // halving the LM head's shared-memory reads of the planes (each row's sum is unchanged).
    if (m.ph_lm.gs == 8 && m.ph_lm.r == 2) rows_phase<8, 2>(P, b, e, m.ph_lm.rps, m.H, m.rs_h, 1, EPI_LOGIT, nullptr, 0);
    else rows_dispatch(P, m.ph_lm, b, e, m.H, m.rs_h, EPI_LOGIT, nullptr, 0);
    cbar();
    const unsigned long long ik = init_lane_key();
    for (int i = tid; i < 256; i += NCT)
      if (x.S.keys[i] != ik) atomicMax(&m.lane_keys[i], x.S.keys[i]);
  }

  GG_DEV void run() {
    const GGModelDev& m = *x.m;
    for (int i = tid; i < 256; i += NCT) x.S.rcnt[i] = 0;
    cbar();
    if (x.mode & GG_RUN_LAYERS) {
      for (int l = 0; l < m.L; l++) {
        trace(l * 6 + 0, 0);
        phase_qkv(l);
        trace(l * 6 + 0, 2);
        trace(l * 6 + 1, 0);
        phase_attn(l);
        trace(l * 6 + 1, 2);
        trace(l * 6 + 2, 0);
        phase_combine(l);
        trace(l * 6 + 2, 2);
        trace(l * 6 + 3, 0);
        phase_o(l);
        trace(l * 6 + 3, 2);
        trace(l * 6 + 4, 0);
        phase_ffn_up(l);
        trace(l * 6 + 4, 2);
        trace(l * 6 + 5, 0);
        phase_down(l);
        trace(l * 6 + 5, 2);
      }
      if (!(x.mode & GG_RUN_LM)) {  // leave the hidden state for a later LM-head launch
        add_norm_planes(x.S.xp[0], m.t_down, make_tag(x.tagbase, (m.L - 1) * PH_PER_LAYER + 5),
                        m.layers[m.L - 1].post_ffw_norm, x.S.res, x.S.hid, m.out_norm,
                        blockIdx.x == 0 ? m.dbg_hidden : nullptr, nullptr);
      }
    }
    if (x.mode & GG_RUN_LM) {
      trace(m.L * 6, 0);
      phase_lm();
      trace(m.L * 6, 2);
    }
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
  const double T = st->temperature, rep = st->rep_penalty;
  if (T == 0.0 && rep <= 1.0) {
    // argmax (shaders.ts:327-361): the largest lane maximum. The shader's tree keeps the lower
    // slot on a tie at every stride (128, 64, ..., 1), so bit 0 of the lane is decided last and
    // weighs most: among equal maxima the lane with the smallest bit-reversed 8-bit index wins
    // (lanes 1 and 2 tied: lane 2). The low word keys that order for the max below.
    __shared__ unsigned long long wk[8];
    unsigned long long key = 0;
    if (tid < 256) key = ((unsigned long long)f32_order_key(val) << 32) | (uint32_t)(255u - (__brev((uint32_t)tid) >> 24));
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
      result = (int)(__brev(255u - (uint32_t)(best & 0xffffffffu)) >> 24);  // back from bit-reversed order
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
    if (rep > 1.0 && st->seen_count > 0 && idx < (uint32_t)m.V && (seen[idx >> 3] >> (idx & 7)) & 1)
      v = v > 0 ? v / rep : v * rep;
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
  if (T == 0.0) {
    if (tid == 0) result = (int)cid[sl[0]];
    __syncthreads();
    return result;
  }
  // engine.ts:881-901, JS numbers are doubles; probs is a Float32Array. The element-wise terms
  // (exp, the division by the sum) are computed by one thread each; every running sum is taken
  // by one thread in index order, as the reference does, so the result is the same bit for bit.
  __shared__ float probs[256];
  __shared__ double share[256];
  __shared__ double sum_all;
  const double temp = T, top_p = st->top_p;
  if (tid < 256) probs[tid] = (float)exp((sv[tid] - sv[0]) / temp);
  __syncthreads();
  if (tid == 0) {
    double sum = 0.0;
    for (int i = 0; i < 256; i++) sum += (double)probs[i];
    sum_all = sum;
  }
  __syncthreads();
  if (tid < 256) share[tid] = (double)probs[tid] / sum_all;
  __syncthreads();
  if (tid == 0) {
    double cum = 0.0;
    int cutoff = 256;
    for (int i = 0; i < 256; i++) {
      cum += share[i];
      if (cum >= top_p) { cutoff = i + 1; break; }
    }
    double sub = 0.0;
    for (int i = 0; i < cutoff; i++) sub += (double)probs[i];
    double u = st->uniforms ? st->uniforms[0] : st->uniform;
    double r = u * sub;
    int pick = cutoff - 1;
    for (int i = 0; i < cutoff; i++) {
      r -= (double)probs[i];
      if (r <= 0) { pick = i; break; }
    }
    result = (int)cid[sl[pick]];
  }
  __syncthreads();
  return result;
}

// ---------------------------------------------------------------------------------- kernel

template <bool KV16>
GG_DEV void decode_body(const GGModelDev* __restrict__ mp, GGState* __restrict__ st) {
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
  // carve shared memory (sizes: GGModelDev::smem_bytes, computed by the host the same way)
  uint8_t* p = smem;
  x.S.ring = p; p += (size_t)NS * m.stage_bytes;
  x.S.full = reinterpret_cast<uint64_t*>(p); p += 8 * NS;
  x.S.empty = reinterpret_cast<uint64_t*>(p); p += 8 * NS;
  x.S.keys = reinterpret_cast<unsigned long long*>(p); p += 8 * 256;
  const int xsz[2] = {m.xs0, m.xs1};
  for (int b = 0; b < 2; b++) {
    x.S.xp[b].p0 = p; p += xsz[b];
    x.S.xp[b].p1 = p; p += xsz[b];
    x.S.xp[b].p2 = p; p += xsz[b];
    x.S.xp[b].inv = reinterpret_cast<float*>(p); p += xsz[b] / 4;
  }
  x.S.hid = reinterpret_cast<float*>(p); p += 4 * (size_t)m.H;
  x.S.res = reinterpret_cast<float*>(p); p += 4 * (size_t)m.H;
  x.S.tmp = reinterpret_cast<float*>(p); p += 4 * (size_t)m.tmp_floats;
  x.S.red = reinterpret_cast<float*>(p); p += 4 * 1024;
  x.S.rcnt = reinterpret_cast<int*>(p); p += 4 * 256;
  x.S.scal = reinterpret_cast<float*>(p); p += 4 * 256;  // 4 rotating csum slots of 16 warps x float4
  x.S.flag = reinterpret_cast<int*>(p); p += 16;
  x.S.rows = reinterpret_cast<int*>(p); p += 4 * RG_N;

  const bool bad = x.token < 0 || x.token >= m.V || x.pos < 0 || x.pos >= m.CTX || x.seq < 0 || x.seq >= m.max_seqs;
  if (bad) {
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicOr(&st->error, GG_ERR_BAD_INPUT);
    x.mode = 0;
  }
  x.nsplit = (x.pos + m.pos_per_split) / m.pos_per_split;  // ceil((pos + 1) / PPS)

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < (int)NS; i++) {
      mbar_init(&x.S.full[i], 1);
      mbar_init(&x.S.empty[i], NCW);
    }
    mbar_fence_init();
    part(m.Q + 2 * m.KV, m.grid, blockIdx.x, x.S.rows[RG_QKV], x.S.rows[RG_QKV + 1]);
    part(m.H, m.grid, blockIdx.x, x.S.rows[RG_H], x.S.rows[RG_H + 1]);
    part(m.I, m.grid, blockIdx.x, x.S.rows[RG_I], x.S.rows[RG_I + 1]);
    part(m.V, m.grid, blockIdx.x, x.S.rows[RG_V], x.S.rows[RG_V + 1]);
  }
  __syncthreads();

  if (warp == NCW) {
    if (lane == 0) {
      Producer<KV16> pr{x, l2_policy_evict_first()};
      pr.run();
    }
  } else {
    Consumer<KV16> cs{x, (int)threadIdx.x, lane, warp};
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
        if (m.seen_cnt) m.seen_cnt[x.seq] += 1;
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

extern "C" __global__ void __launch_bounds__(GG_NTHREADS, 1)
    gg_decode_kernel(const GGModelDev* __restrict__ mp, GGState* __restrict__ st) {
  decode_body<false>(mp, st);
}

// The same kernel for a bf16 KV cache (GG_FLAG_KV_BF16).
extern "C" __global__ void __launch_bounds__(GG_NTHREADS, 1)
    gg_decode_kernel_kv16(const GGModelDev* __restrict__ mp, GGState* __restrict__ st) {
  decode_body<true>(mp, st);
}

}  // namespace gg

namespace gg {

// ---------------------------------------------------------------------- batched sampling

// One CTA per row of a [B][V] logits matrix: the 256 lane maxima of the row, then the sampler
// (sample_token, engine.ts:823-901) with that row's parameters, draw and KV slot's seen set.
// The sampled token is added to the slot's seen set, becomes the row's next input token, and
// the row's position advances.
__global__ void __launch_bounds__(512)
    gg_batch_sample_kernel(const float* __restrict__ logits, int V, const int32_t* __restrict__ seqs,
                           const GGSampleDev* __restrict__ sp, const double* __restrict__ unif, uint8_t* seen,
                           int seen_stride, int32_t* seen_cnt, unsigned long long* keys, int32_t* tokens,
                           int32_t* pos, int32_t* out) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  __shared__ GGModelDev sm;
  __shared__ GGState ss;
  __shared__ unsigned long long sk[8][256];
  const int b = blockIdx.x, t = threadIdx.x;
  const float* row = logits + (size_t)b * V;
  const unsigned long long ik = init_lane_key();
  // Element i belongs to lane i % 256. Thread t reads 16-byte groups c = t, t + 512, ... (eight
  // loads in flight): elements 4c..4c+3 are lanes 4 (c % 64) + j, shared by the eight threads
  // t % 64 + 64 k.
  unsigned long long best[4] = {ik, ik, ik, ik};
  const int n4 = V >> 2;
  auto take = [&](const float4 f, int c) {
    const float fv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float v = fv[j];
      if (!isnan(v)) {
        if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal under '>': key them alike
        const uint32_t i = 4u * (uint32_t)c + j;
        const unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - i);
        best[j] = k > best[j] ? k : best[j];
      }
    }
  };
  const float4* row4 = reinterpret_cast<const float4*>(row);
  int c = t;
  for (; c + 7 * 512 < n4; c += 8 * 512) {
    float4 f[8];
#pragma unroll
    for (int u = 0; u < 8; u++) f[u] = __ldcs(row4 + c + u * 512);
#pragma unroll
    for (int u = 0; u < 8; u++) take(f[u], c + u * 512);
  }
  for (; c < n4; c += 512) take(__ldcs(row4 + c), c);
#pragma unroll
  for (int j = 0; j < 4; j++) sk[t >> 6][4 * (t & 63) + j] = best[j];
  __syncthreads();
  unsigned long long kb = ik;
  if (t < 256) {
#pragma unroll
    for (int q = 0; q < 8; q++) kb = sk[q][t] > kb ? sk[q][t] : kb;
    for (int i = 4 * n4; i < V; i++) {  // tail when V % 4 != 0 (< 4 elements): lane i % 256
      if ((i & 255) != t) continue;
      float v = row[i];
      if (!isnan(v)) {
        if (v == 0.0f) v = 0.0f;
        const unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - (uint32_t)i);
        kb = k > kb ? k : kb;
      }
    }
  }
  unsigned long long* rk = keys + (size_t)b * 256;
  if (t < 256) rk[t] = kb;
  const int seq = seqs[b];
  if (t == 0) {
    sm.lane_keys = rk;
    sm.seen = seen;
    sm.seen_stride = seen_stride;
    sm.V = V;
    ss.seq = seq;
    ss.temperature = sp[b].temperature;
    ss.top_p = sp[b].top_p;
    ss.rep_penalty = sp[b].rep_penalty;
    ss.uniform = unif[b];
    ss.uniforms = nullptr;
    ss.seen_count = seen_cnt[seq];
  }
  __threadfence_block();
  __syncthreads();
  Smem unused{};
  const int tok = sample_token(sm, &ss, unused);
  if (t == 0) {
    out[b] = tok;
    if (tok >= 0 && tok < V) {
      atomicOr(reinterpret_cast<unsigned int*>(seen + (size_t)seq * seen_stride) + (tok >> 5), 1u << (tok & 31));
      seen_cnt[seq] += 1;
    }
    tokens[b] = tok;
    pos[b] += 1;
  }
}

}  // namespace gg

cudaError_t gg_batch_sample(const float* logits, int B, int V, const int32_t* seqs, const GGSampleDev* sp,
                            const double* unif, uint8_t* seen, int seen_stride, int32_t* seen_cnt,
                            unsigned long long* keys, int32_t* tokens, int32_t* pos, int32_t* out, cudaStream_t s) {
  if (B <= 0) return cudaErrorInvalidValue;
  return gg::launch_pdl(gg::gg_batch_sample_kernel, dim3(B), dim3(512), 0, s, logits, V, seqs, sp, unif, seen,
                        seen_stride, seen_cnt, keys, tokens, pos, out);
}

// ------------------------------------------------------------------ sampling without allocation
//
// gg_sample_logits_noalloc: the step kernel's last stage -- the 256 per-lane maxima of the
// logits (shaders.ts:363-384) and the sampler (engine.ts:823-901) -- as a kernel of its own over
// logits the caller already holds on the device. Its scratch (per-CTA lane maxima and an
// end-of-launch ticket) lives in a static device array, so a call allocates no memory.

#include <cuda.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "gemma_b200.h"

namespace gg {

constexpr int SL_THREADS = 256;                                   // thread t owns top-256 lane t
constexpr int SL_ROWS_PER_THREAD = 16;
constexpr int SL_ROWS_PER_CTA = SL_THREADS * SL_ROWS_PER_THREAD;  // 4096 logits per CTA
constexpr int SL_MAX_CTAS = 128;
constexpr int SL_MAX_VOCAB = SL_MAX_CTAS * SL_ROWS_PER_CTA;       // 524,288 (Gemma 3: 262,144)
constexpr int SL_KEYS_OFF = 32;  // word 0: ticket; from word 32: SL_MAX_CTAS x 256 lane keys
constexpr size_t SL_SCRATCH_WORDS = SL_KEYS_OFF + (size_t)SL_MAX_CTAS * SL_THREADS;

// 262,400 bytes on every GPU that loads the library, held until the process exits. Shared by
// all calls: the ticket (word 0) must be zero when a launch starts and is cleared by the host
// before each launch; every CTA overwrites its own lane-key slot before anything reads it.
static __device__ __align__(256) unsigned long long g_sample_scratch[SL_SCRATCH_WORDS];

__global__ void __launch_bounds__(SL_THREADS)
    gg_sample_logits_kernel(const float* __restrict__ logits, int V, const uint32_t* __restrict__ seen_bits,
                            double temperature, double top_p, double rep_penalty, double uniform,
                            int32_t* __restrict__ out_token, unsigned long long* __restrict__ scratch) {
  __shared__ int is_last;
  __shared__ GGModelDev sm;
  __shared__ GGState ss;
  const int t = threadIdx.x;
  unsigned long long* keys = scratch + SL_KEYS_OFF;
  // Rows base + t + 256 j all fall in lane t: (value, lowest row) maximum, strict '>' from
  // (-1e30, 0), NaN never taken; -0 is keyed as +0 since the two compare equal.
  const unsigned long long ik = init_lane_key();
  unsigned long long best = ik;
  const int base = blockIdx.x * SL_ROWS_PER_CTA;
#pragma unroll 4
  for (int j = 0; j < SL_ROWS_PER_THREAD; j++) {
    const int row = base + t + j * SL_THREADS;
    if (row < V) {
      float v = __ldg(logits + row);
      if (!isnan(v)) {
        if (v == 0.0f) v = 0.0f;
        const unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - (uint32_t)row);
        best = k > best ? k : best;
      }
    }
  }
  keys[(size_t)blockIdx.x * SL_THREADS + t] = best;
  __threadfence();
  __syncthreads();
  if (t == 0) is_last = atomicAdd(scratch, 1ull) == (unsigned long long)(gridDim.x - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  unsigned long long k = ik;
  for (int c = 0; c < (int)gridDim.x; c++) {
    const unsigned long long o = __ldcg(keys + (size_t)c * SL_THREADS + t);
    k = o > k ? o : k;
  }
  keys[t] = k;  // slot 0 now holds the merged maxima; thread t reads back only its own lane
  if (t == 0) {
    sm.lane_keys = keys;
    sm.seen = reinterpret_cast<uint8_t*>(const_cast<uint32_t*>(seen_bits));
    sm.seen_stride = 0;
    sm.V = V;
    ss.seq = 0;
    ss.temperature = temperature;
    ss.top_p = top_p;
    ss.rep_penalty = rep_penalty;
    ss.uniform = uniform;
    ss.uniforms = nullptr;
    ss.seen_count = seen_bits ? 1 : 0;
  }
  __threadfence_block();
  __syncthreads();
  Smem unused{};
  const int tok = sample_token(sm, &ss, unused);
  if (t == 0) *out_token = tok;
}

}  // namespace gg

void gg_set_engineless_error(const char* msg);  // gg_engine.cu: the message gg_last_error(NULL) returns

namespace {

constexpr int SL_MAX_DEVICES = 64;
std::mutex g_sl_mu;
// Device address of the array per device, with the id of the context it was looked up in: a
// context that replaced that one (after cudaDeviceReset, or another context made current) has
// its own copy of the array at a possibly different address, so the lookup is redone there.
struct SlSlot {
  unsigned long long ctx_id = 0;
  unsigned long long* addr = nullptr;
};
SlSlot g_sl_scratch[SL_MAX_DEVICES];

typedef CUresult (*PfnCtxGetCurrent)(CUcontext*);
typedef CUresult (*PfnCtxGetId)(CUcontext, unsigned long long*);

// Unique id (for the life of the process) of the calling thread's current context, or 0.
unsigned long long current_ctx_id() {
  static PfnCtxGetCurrent get_cur = nullptr;
  static PfnCtxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<PfnCtxGetCurrent>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PfnCtxGetId>(f);
  });
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (!get_cur || !get_id || get_cur(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int sl_fail(int code, const char* fmt, ...) {
  char buf[320];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  gg_set_engineless_error(buf);
  return code;
}

}  // namespace

extern "C" int gg_sample_logits_noalloc(const float* logits, int vocab, const uint32_t* seen_bits,
                                        const gg_sample* sp, double uniform, int32_t* out_token, void* stream) {
  using namespace gg;
  if (!logits || !sp || !out_token) return sl_fail(GG_E_ARG, "gg_sample_logits_noalloc: null logits, sample or out_token");
  if (vocab < 1 || vocab > SL_MAX_VOCAB)
    return sl_fail(GG_E_ARG,
                   "gg_sample_logits_noalloc: vocab %d outside 1..%d (its static scratch holds the lane maxima "
                   "of %d blocks of %d logits)", vocab, SL_MAX_VOCAB, SL_MAX_CTAS, SL_ROWS_PER_CTA);
  int dev = -1;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return sl_fail(GG_E_CUDA, "gg_sample_logits_noalloc: cudaGetDevice: %s", cudaGetErrorString(r));
  if (dev < 0 || dev >= SL_MAX_DEVICES) return sl_fail(GG_E_ARG, "gg_sample_logits_noalloc: device %d >= %d", dev, SL_MAX_DEVICES);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (s) {  // the kernel and the memset run on the current device: the stream must belong to it
    int sdev = -1;
    r = cudaStreamGetDevice(s, &sdev);
    if (r != cudaSuccess) return sl_fail(GG_E_ARG, "gg_sample_logits_noalloc: cudaStreamGetDevice: %s", cudaGetErrorString(r));
    if (sdev != dev)
      return sl_fail(GG_E_ARG, "gg_sample_logits_noalloc: stream belongs to device %d, the current device is %d", sdev, dev);
  }
  unsigned long long* scratch = nullptr;
  {
    // First call on a device (or in a new context on it): look up the array's device address
    // with that device current. The host-side name g_sample_scratch is not a device address and
    // is never passed to a kernel.
    std::lock_guard<std::mutex> g(g_sl_mu);
    SlSlot& slot = g_sl_scratch[dev];
    const unsigned long long ctx = current_ctx_id();  // 0 before the runtime made a context current
    if (!slot.addr || ctx == 0 || slot.ctx_id != ctx) {
      void* p = nullptr;
      r = cudaGetSymbolAddress(&p, g_sample_scratch);  // also makes the primary context current
      if (r != cudaSuccess || !p)
        return sl_fail(GG_E_CUDA, "gg_sample_logits_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                       cudaGetErrorString(r));
      slot.addr = static_cast<unsigned long long*>(p);
      slot.ctx_id = current_ctx_id();
    }
    scratch = slot.addr;
  }
  r = cudaMemsetAsync(scratch, 0, sizeof(unsigned long long), s);  // the ticket starts at zero
  if (r != cudaSuccess) return sl_fail(GG_E_CUDA, "gg_sample_logits_noalloc: clearing the ticket: %s", cudaGetErrorString(r));
  const int grid = (vocab + SL_ROWS_PER_CTA - 1) / SL_ROWS_PER_CTA;
  gg_sample_logits_kernel<<<grid, SL_THREADS, 0, s>>>(logits, vocab, seen_bits, sp->temperature, sp->top_p,
                                                      sp->rep_penalty, uniform, out_token, scratch);
  r = cudaGetLastError();
  if (r != cudaSuccess) return sl_fail(GG_E_CUDA, "gg_sample_logits_noalloc: launch: %s", cudaGetErrorString(r));
  return GG_OK;
}
