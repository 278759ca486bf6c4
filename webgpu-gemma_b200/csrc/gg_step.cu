// gg_step.cu -- the batch-1 Gemma 3 token step as one persistent sm_100a kernel.
//
// One CTA per SM (cooperative launch), 16 consumer warps and one producer warp. The producer's
// lane 0 walks the whole token's weight schedule -- per layer this CTA's rows of Wqkv, the KV rows
// of its attention splits, its rows of Wo, Wgu and Wdown, then its LM-head rows -- and streams
// them with cp.async.bulk into a ring of 16 KB shared-memory stages completing on mbarriers. It
// only ever waits for free stages, so weight streaming runs ahead across phase and layer
// boundaries while the consumers wait for activations.
//
// Between phases the CTAs exchange activations as tagged 64-bit words (f32 value | tag << 32,
// the tag naming the launch and phase), so each word is its own ready flag. A CTA's outputs of a
// phase occupy its own slot of whole 32-byte sectors: producers never share a sector, and a
// consumer loads every word it needs with 16-byte loads that are all in flight before it checks
// any tag.
//
// Phases per layer (reference: src/engine.ts:766-795):
//   0  post-ffw norm + residual of the previous layer, attention rmsNorm, fused QKV matvec
//                                                      (shaders.ts:25-56, 92-151, 386-418)
//   1  q/k per-head norm + RoPE, KV store, attention splits of 8 positions (shaders.ts:209-325, 420-467)
//   2  merge of the splits (online softmax): one warp per 8 output dimensions
//   3  O projection                                               (shaders.ts:92-151)
//   4  post-attn norm + residual, ffn rmsNorm, gate/up + GeGLU    (shaders.ts:153-170, 386-418)
//   5  down projection                                            (shaders.ts:92-151)
// then the final norm, the tied LM head with per-lane maxima (engine.ts:797-821, shaders.ts:327-384)
// and the sampler in the last CTA to finish (engine.ts:823-901).
//
// Matvec arithmetic: x is held as 24-bit fixed point per 16-element chunk in three byte planes
// (one exponent per chunk); q . x is three exact int32 dp4a sums per chunk, recombined in f32 and
// scaled by the chunk exponent and the Q8_0 block scale. A warp computes one row (two for the
// gate/up pairs and the LM head) with its lanes over the row's chunks.
//
// Code size is kept small on purpose: one dot-product routine per row count serves every matvec
// phase, so the per-layer loop stays resident in the SM's instruction cache.
#include "gg_device.cuh"
#include "gg_model.h"
#include "gg_sample.cuh"

namespace gg {
namespace step {

constexpr int NCW = GG_STEP_NCW;
constexpr int NCT = NCW * 32;
constexpr int NTH = NCT + 32;
constexpr uint32_t NS = GG_STEP_STAGES;
constexpr int PH = 6;  // phases (tags) per layer
static_assert(sizeof(SampleScratch) <= (size_t)GG_STEP_STAGES * GG_STEP_STAGE_BYTES, "the sampler works in the idle ring");

#define GG_NOINLINE __device__ __noinline__

GG_DEV void cbar() { asm volatile("bar.sync 1, %0;" ::"n"(NCT) : "memory"); }

GG_DEV uint32_t make_tag(uint32_t base, int phase) { return 0x80000000u | ((base + (uint32_t)phase) & 0x7fffffffu); }

// Quad partition: quads [qpart(c), qpart(c + 1)) of nq go to CTA c of G (32-bit: the host checks
// G * nq < 2^31), and the CTA that owns quad q.
GG_DEV int qpart(int nq, int c) { return (int)(((uint32_t)c * (uint32_t)nq) / (uint32_t)GG_STEP_GRID); }
// (division by nq as a multiply by mq = ceil(2^40 / nq): n * nq < 2^40 here, so it is exact)
GG_DEV int qowner(unsigned long long mq, int q) {
  return (int)(((unsigned long long)(((uint32_t)q + 1u) * (uint32_t)GG_STEP_GRID - 1u) * mq) >> 40);
}
// Word offset of element quad q in a slot layout (CTA c's words start at c * sl).
GG_DEV int slot_word(int nq, unsigned long long mq, int sl, int q) {
  const int c = qowner(mq, q);
  return c * sl + 4 * (q - qpart(nq, c));
}

// The planes of one x vector, as shared-window addresses.
struct XPlanes {
  uint32_t p0;   // signed top byte of each element's 24-bit fixed point value
  uint32_t p1;   // middle byte (unsigned)
  uint32_t p2;   // low byte (unsigned)
  uint32_t inv;  // f32 2^(e - 23) per 16-element chunk
};

enum { RG_QKV = 0, RG_H = 2, RG_I = 4, RG_V = 6, RG_N = 8 };  // this CTA's [begin, end) rows / pairs

struct Smem {
  uint8_t* ring;
  uint64_t* full;
  uint64_t* empty;
  float* lmv;   // this CTA's LM-head logits (rows [RG_V, RG_V + 1))
  XPlanes xa;   // H-wide inputs: QKV, gate/up, LM head
  XPlanes xb;   // Q- and I-wide inputs: O, down
  float* hid;   // residual stream (identical in every CTA)
  float* res;   // residual after the attention block
  float* tmp;   // q | k | v of the current token
  float4* scal;
  float* red;   // [16 rows][NCW slices] partial sums of the small matvecs
  int* flag;
  int* rows;
};

// Rows per ring stage of a phase whose n rows (n <= NCW) are computed one per warp, and the
// number of such stages.
GG_DEV int shared_rps(int rps_max, int n) { return max(min(rps_max, n), 1); }
GG_DEV int shared_nst(int rps_max, int n) { const int d = shared_rps(rps_max, n); return (n + d - 1) / d; }

// Work map of a small matvec phase (q/k/v, down) for one consumer warp, fixed for a launch: the
// ring offsets of its four rows ((stage << 16) | byte offset; rows past n repeat the last row),
// its 16-element chunk slice [c0, c1), its row group g (0xff: no rows) and slice index sl.
struct MvWarp {
  uint32_t roff[4];
  uint16_t c0, c1;
  uint8_t g, sl;
  uint16_t pad;
};
struct MvPhase {
  int n, nst, S;  // rows, ring stages, K slices per row group
  MvWarp w[GG_STEP_NCW];
};

// Per-launch constants, held in shared memory (filled by thread 0 at the start): keeping them out
// of registers leaves the hot loops free of register spills.
struct Ctx {
  const GGModelDev* m;
  GGState* st;
  Smem S;
  SpinCtl sc;
  int mode, token, pos, seq, nsplit;
  uint32_t tagbase;
  uint32_t par;  // accumulator set of this launch (0 or 1)
  MvPhase mv[2];  // matvec maps: 0 q/k/v, 1 down
};

// The matvec map of phase p for warp w (integer divisions, once per launch): the CTA's n rows in
// stages of d = shared_rps(rps_max, n) rows of rs bytes, K inputs; groups of four rows, each split
// into S = NCW / groups K slices.
GG_DEV void mv_map(MvPhase& ph, int w, int n, int rps_max, int K, int rs) {
  MvWarp& e = ph.w[w];
  if (n <= 0) {  // a CTA without rows in this phase (narrow models): no stages, every warp idle
    if (w == 0) {
      ph.n = 0;
      ph.nst = 0;
      ph.S = 1;
    }
    e.g = 0xff;
    e.sl = 0;
    e.c0 = e.c1 = 0;
    for (int k = 0; k < 4; k++) e.roff[k] = 0;
    return;
  }
  const int d = shared_rps(rps_max, n), ng = (n + 3) >> 2, S = GG_STEP_NCW / ng, nch = K >> 4;
  if (w == 0) {
    ph.n = n;
    ph.nst = (n + d - 1) / d;
    ph.S = S;
  }
  const int g = w / S, sl = w % S;
  e.g = g < ng ? (uint8_t)g : (uint8_t)0xff;
  e.sl = (uint8_t)sl;
  e.c0 = (uint16_t)(sl * nch / S);
  e.c1 = (uint16_t)((sl + 1) * nch / S);
  for (int k = 0; k < 4; k++) {
    const int r = min(4 * g + k, n - 1);
    e.roff[k] = ((uint32_t)(r / d) << 16) | (uint32_t)((r % d) * rs);
  }
}


GG_DEV int window_lo(const GGLayerW& Lw, int pos) { return (Lw.window > 0 && pos + 1 > Lw.window) ? pos + 1 - Lw.window : 0; }

// First split of this CTA in layer l (splits s >= slo with s - slo = (c - rot) mod G).
GG_DEV int first_split(const GGModelDev& m, int l, int pos, int nsplit, int c) {
  constexpr int G = GG_STEP_GRID;
  const int rot = (l * nsplit) % G;
  return window_lo(m.layers[l], pos) / GG_POS_PER_SPLIT + (c - rot + G) % G;
}

// ---------------------------------------------------------------------------------- producer

template <bool KV16>
struct Producer {
  Ctx& x;
  uint64_t pol;
  bool ok = true;
  uint32_t idx = 0;  // ring position

  GG_DEV void issue(const void* s0, uint32_t b0, const void* s1, uint32_t b1, uint32_t off1) {
    const int slot = idx % NS;
    const uint32_t use = idx / NS;
    if (use > 0 && ok) ok = mbar_wait_suspend(&x.S.empty[slot], (use - 1) & 1, x.sc);
    if (!ok) return;
    uint8_t* dst = x.S.ring + (size_t)slot * GG_STEP_STAGE_BYTES;
    mbar_arrive_expect_tx(&x.S.full[slot], b0 + b1);
    if (b0) bulk_g2s(dst, s0, b0, &x.S.full[slot], pol);
    if (b1) bulk_g2s(dst + off1, s1, b1, &x.S.full[slot], pol);
    idx++;
    *(volatile uint32_t*)(x.S.flag + 1) = idx;  // stages issued so far (read by the LM head's owners)
  }
  GG_DEV void rows(const uint8_t* W, int rs, int rb, int re, int rps) {
    for (int r = rb; r < re && ok; r += rps) issue(W + (size_t)r * rs, (uint32_t)(min(rps, re - r) * rs), nullptr, 0, 0);
  }
  GG_DEV void run() {
    const GGModelDev& m = *x.m;
    const int c = blockIdx.x, G = m.grid;
    const int* R = x.S.rows;
    if (x.mode & GG_RUN_LAYERS) {
      for (int l = 0; l < m.L && ok; l++) {
        const GGLayerW& Lw = m.layers[l];
        rows(Lw.wqkv, m.rs_h, R[RG_QKV], R[RG_QKV + 1], shared_rps(m.rps_h, R[RG_QKV + 1] - R[RG_QKV]));
        for (int s = first_split(m, l, x.pos, x.nsplit, c); s < x.nsplit && ok; s += G) {
          const int p0 = s * m.pos_per_split, pc = min(p0 + m.pos_per_split, x.pos);
          constexpr int es = KV16 ? 2 : 4;
          const uint32_t nb = pc > p0 ? (uint32_t)((pc - p0) * m.KV * es) : 0u;
          const size_t off = ((size_t)x.seq * m.kv_seq_stride + ((size_t)l * m.CTX + p0) * m.KV) * es;
          issue(m.kcache + off, nb, m.vcache + off, nb, (uint32_t)(m.pos_per_split * m.KV * es));
        }
        if (c < m.ncomb) issue(Lw.wo_cols + (size_t)c * m.H * 10, (uint32_t)(m.H * 10), nullptr, 0, 0);
        rows(Lw.wgu, m.rs_h, 2 * R[RG_I], 2 * R[RG_I + 1], m.rps_gu);
        rows(Lw.wdown, m.rs_i, R[RG_H], R[RG_H + 1], shared_rps(m.rps_i, R[RG_H + 1] - R[RG_H]));
      }
    }
    if ((x.mode & GG_RUN_LM) && ok) rows(m.embd, m.rs_h, R[RG_V], R[RG_V + 1], m.rps_gu);
    // Drain: every copy issued into the ring must land before the CTA may exit.
    const uint32_t n = idx < NS ? idx : NS;
    for (uint32_t k = idx - n; k < idx; k++) {
      const uint64_t t0 = global_timer_ns();
      while (!mbar_try_wait(&x.S.full[k % NS], (k / NS) & 1)) {
        if (global_timer_ns() - t0 > x.sc.timeout_ns) { atomicOr(x.sc.err, GG_ERR_WAIT_MBAR); break; }
      }
    }
  }
};

// Deadline of a tagged-word wait, checked every 32 passes after the first 512 (which read no
// clock): after GG_QUIET_SPIN_NS the wait gives up once an error is raised elsewhere, and after
// the timeout it raises GG_ERR_WAIT_FLAG itself.
GG_NOINLINE bool spin_gave_up(const SpinCtl sc, uint64_t t0) {
  const uint64_t dt = global_timer_ns() - t0;
  if (dt <= GG_QUIET_SPIN_NS) return false;
  if (dt > sc.timeout_ns) {
    atomicOr(sc.err, GG_ERR_WAIT_FLAG);
    return true;
  }
  return *(volatile uint32_t*)sc.err != 0;
}

struct SpinClock {
  uint32_t it = 0;
  uint64_t t0 = 0;
  GG_DEV bool expired(const SpinCtl& sc) {
    ++it;
    if (it == 512) t0 = global_timer_ns();
    if (it <= 512 || (it & 31u)) return false;
    return spin_gave_up(sc, t0);
  }
};

GG_DEV bool quad_ready(const uint64_t (&w)[4], uint32_t tag) {
  return (uint32_t)(w[0] >> 32) == tag && (uint32_t)(w[1] >> 32) == tag && (uint32_t)(w[2] >> 32) == tag &&
         (uint32_t)(w[3] >> 32) == tag;
}
// A quad that takes part in a warp wait without a load: four tagged zeros.
GG_DEV void quad_idle(uint64_t (&w)[4], uint32_t tag) {
#pragma unroll
  for (int j = 0; j < 4; j++) w[j] = (uint64_t)tag << 32;
}
GG_DEV void quad_vals(const uint64_t (&w)[4], float* v) {
#pragma unroll
  for (int j = 0; j < 4; j++) v[j] = __uint_as_float((uint32_t)w[j]);
}

// K-split reductions: an f32 partial added into a u64 accumulator as (round(v * 2^32) << 8) + 1:
// the high 56 bits sum the 2^-32 fixed-point partials (sums up to 2^23 in magnitude) and the low
// byte counts the contributions (at most 255 adders). Integer addition is exact and associative, so the sum is the same whatever
// order the CTAs arrive in, and a reader knows a word is complete when its count is full: no
// fence or separate arrival counter is needed.
GG_DEV void acc_add(unsigned long long* p, float v) {
  const long long q = __float2ll_rn(v * 4294967296.0f);
  const unsigned long long w = ((unsigned long long)q << 8) + 1ull;
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
GG_DEV float acc_value(unsigned long long w) { return (float)((long long)w >> 8) * 0x1p-32f; }
GG_DEV uint32_t acc_count(unsigned long long w) { return (uint32_t)(w & 0xffull); }

// ---------------------------------------------------------------------------------- dot products

// q . x over one Q8_0 row of K inputs held in shared memory (K int8 quants, then K/32 f16 scales):
// lane l takes the 16-element chunks l, l + 32, ...; each chunk is three exact dp4a sums against
// the byte planes of x, recombined in f32 and scaled by the chunk's 2^(e-23) and the block scale.
// Every lane receives the row total.
GG_DEV float dot_row(uint32_t row, int K, const XPlanes P) {
  const int lane = threadIdx.x & 31, nch = K >> 4;
  float acc = 0.f;
#pragma unroll 2
  for (int c = lane; c < nch; c += 32) {
    const uint4 a0 = lds128(P.p0 + 16 * c);
    const uint4 a1 = lds128(P.p1 + 16 * c);
    const uint4 a2 = lds128(P.p2 + 16 * c);
    const uint4 w = lds128(row + 16 * c);
    const float sc = lds_half(row + K + 2 * (c >> 1)) * ldsf(P.inv + 4 * c);
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
    acc = fmaf(fmaf((float)s0, 65536.f, (float)(s1 * 256 + s2)), sc, acc);
  }
  return warp_sum(acc);
}

// Four rows (addresses r[0..3], equal width K) over the chunks [c0, c1): lane l takes chunks
// c0 + l, c0 + l + 32, ...; each load of the x planes serves all four rows. Every lane receives
// the four slice totals.
GG_DEV float4 dot_rows4(const uint32_t (&r)[4], int K, int c0, int c1, const XPlanes& P) {
  const int lane = threadIdx.x & 31;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int c = c0 + lane; c < c1; c += 32) {
    const uint4 a0 = lds128(P.p0 + 16 * c);
    const uint4 a1 = lds128(P.p1 + 16 * c);
    const uint4 a2 = lds128(P.p2 + 16 * c);
    const float is = ldsf(P.inv + 4 * c);
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint4 w = lds128(r[k] + 16 * c);
      const float sc = lds_half(r[k] + K + 2 * (c >> 1)) * is;
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
      acc[k] = fmaf(fmaf((float)s0, 65536.f, (float)(s1 * 256 + s2)), sc, acc[k]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1)
#pragma unroll
    for (int k = 0; k < 4; k++) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
  return make_float4(acc[0], acc[1], acc[2], acc[3]);
}

// Row pairs by lane groups: the 8 lanes of group g (lane / 8) compute rows (ra, ra + rs) over the
// chunks c = lane % 8, lane % 8 + 8, ...; the pair totals end up in every lane of the group.
GG_DEV float2 dot_pair8(uint32_t ra, int rs, int K, const XPlanes& P) {
  const int gl = threadIdx.x & 7, nch = K >> 4;
  const uint32_t rb = ra + rs;
  float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 1  // (unrolling measured no faster: the loop is bound by shared-memory bandwidth)
  for (int c = gl; c < nch; c += 8) {
    const uint4 a0 = lds128(P.p0 + 16 * c);
    const uint4 a1 = lds128(P.p1 + 16 * c);
    const uint4 a2 = lds128(P.p2 + 16 * c);
    const float is = ldsf(P.inv + 4 * c);
    const uint4 wa = lds128(ra + 16 * c);
    const uint4 wb = lds128(rb + 16 * c);
    const float sa = lds_half(ra + K + 2 * (c >> 1)) * is;
    const float sb = lds_half(rb + K + 2 * (c >> 1)) * is;
    int x0 = dp4a_ss((int)wa.x, (int)a0.x, 0), y0 = dp4a_ss((int)wb.x, (int)a0.x, 0);
    x0 = dp4a_ss((int)wa.y, (int)a0.y, x0); y0 = dp4a_ss((int)wb.y, (int)a0.y, y0);
    x0 = dp4a_ss((int)wa.z, (int)a0.z, x0); y0 = dp4a_ss((int)wb.z, (int)a0.z, y0);
    x0 = dp4a_ss((int)wa.w, (int)a0.w, x0); y0 = dp4a_ss((int)wb.w, (int)a0.w, y0);
    int x1 = dp4a_su((int)wa.x, (int)a1.x, 0), y1 = dp4a_su((int)wb.x, (int)a1.x, 0);
    x1 = dp4a_su((int)wa.y, (int)a1.y, x1); y1 = dp4a_su((int)wb.y, (int)a1.y, y1);
    x1 = dp4a_su((int)wa.z, (int)a1.z, x1); y1 = dp4a_su((int)wb.z, (int)a1.z, y1);
    x1 = dp4a_su((int)wa.w, (int)a1.w, x1); y1 = dp4a_su((int)wb.w, (int)a1.w, y1);
    int x2 = dp4a_su((int)wa.x, (int)a2.x, 0), y2 = dp4a_su((int)wb.x, (int)a2.x, 0);
    x2 = dp4a_su((int)wa.y, (int)a2.y, x2); y2 = dp4a_su((int)wb.y, (int)a2.y, y2);
    x2 = dp4a_su((int)wa.z, (int)a2.z, x2); y2 = dp4a_su((int)wb.z, (int)a2.z, y2);
    x2 = dp4a_su((int)wa.w, (int)a2.w, x2); y2 = dp4a_su((int)wb.w, (int)a2.w, y2);
    acc0 = fmaf(fmaf((float)x0, 65536.f, (float)(x1 * 256 + x2)), sa, acc0);
    acc1 = fmaf(fmaf((float)y0, 65536.f, (float)(y1 * 256 + y2)), sb, acc1);
  }
#pragma unroll
  for (int o = 4; o > 0; o >>= 1) {
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, o);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, o);
  }
  return make_float2(acc0, acc1);
}

// ---------------------------------------------------------------------------------- consumers

template <bool KV16>
struct Consumer {
  Ctx& x;
  int tid, lane, warp;
  // Once a ring wait gives up, this warp stops waiting on and releasing slots, so the producer
  // can never refill a slot whose copy might still be landing; it drains and exits.
  bool dead = false;
  int cslot = 0;
  uint32_t idx = 0;  // ring position

  // Ring protocol. Every warp walks the ring in the producer's order (idx). A slot is waited on
  // for use u only after its use u - 1 has been consumed and released, so a parity wait can never
  // mistake use u - 1 for use u.
  // * Gated phases (all stages resident at once: q/k/v, O, gate/up, down): warp k waits for stage
  //   k of the phase before a CTA barrier, every warp reads the stages after it, and once every
  //   warp is past a later barrier thread 0 releases them all (release_all).
  // * Attention KV: the warps of split k wait for stage k and release it themselves.
  // * Streaming phase (LM head): every warp waits for and releases every stage (stage_wait,
  //   stage_done), computing on the stages it owns.
  GG_DEV uint8_t* stage_wait() { return stage_wait_ahead(0); }
  // Wait for the stage k places after the next one to release (k < NS).
  GG_DEV uint8_t* stage_wait_ahead(int k) {
    const uint32_t i = idx + (uint32_t)k;
    const int slot = i % NS;
    if (!dead) dead = !__all_sync(0xffffffffu, mbar_wait(&x.S.full[slot], (i / NS) & 1, x.sc));
    return x.S.ring + (size_t)slot * GG_STEP_STAGE_BYTES;
  }
  GG_DEV void stage_done() {
    __syncwarp();
    if (lane == 0 && !dead) mbar_arrive(&x.S.empty[idx % NS]);
    idx++;
  }
  // Gated phase, before its CTA barrier: warp k (< nst) waits for stage k of the phase.
  GG_DEV void gate(int nst) {
    if (warp < nst) stage_wait_ahead(warp);
  }
  // Gated phase, after a CTA barrier that every use of its nst stages precedes: release them
  // (NCW arrivals each, by one thread). After an error nothing is released: the producer's waits
  // then run out instead of refilling a slot whose copy may still be landing.
  GG_DEV void release_all(int nst) {
    if (tid == 0 && !dead && !*(volatile uint32_t*)x.sc.err)
      for (int k = 0; k < nst; k++) mbar_arrive_cnt(&x.S.empty[(idx + (uint32_t)k) % NS], NCW);
    idx += (uint32_t)nst;
  }

  // Phase boundaries and trace stamps (GG_TRACE launches): globaltimer of event ev (0 enter,
  // 1 inputs ready, 2 done) of phase ph: trace[(cta * GG_TRACE_PHASES + ph) * 4 + ev].
  // Every phase ends with a CTA barrier, traced or not: a warp that ran ahead into the next
  // phase would poll L2 for its inputs while the CTA's other warps still work on this one, and
  // its polls cost them issue slots (measured: 0.705 -> 0.679 ms per token at 1B).
  GG_DEV void trace(int ph, int ev) {
    if (ev == 2) cbar();  // "done" = every warp of the CTA finished the phase
    if (!(x.mode & GG_TRACE)) return;
    if (tid == 0 && ph < GG_TRACE_PHASES)
      x.m->trace[((size_t)blockIdx.x * GG_TRACE_PHASES + ph) * 4 + ev] = global_timer_ns();
  }

  // Warp-uniform wait for NQ quads per lane, first loaded by issue4 (or quad_idle): each pass
  // re-reads every quad of the warp that does not carry `tag` yet, all in flight together, and the
  // warp leaves together once every quad does. No lane spins alone while the rest of its warp
  // waits at a reconvergence point. Bounded (SpinClock); after giving up the values read 0.
  template <int NQ>
  GG_DEV void settle_warp(const uint64_t* const (&p)[NQ], uint32_t tag, uint64_t (&w)[NQ][4]) {
    SpinClock clk;
#pragma unroll 1
    for (;;) {
      bool ok = true;
#pragma unroll
      for (int k = 0; k < NQ; k++) ok = ok && quad_ready(w[k], tag);
      if (__all_sync(0xffffffffu, ok)) return;
#pragma unroll
      for (int k = 0; k < NQ; k++)
        if (!quad_ready(w[k], tag)) issue4(p[k], w[k]);
      if (__any_sync(0xffffffffu, clk.expired(x.sc))) {
#pragma unroll
        for (int k = 0; k < NQ; k++) quad_idle(w[k], tag);
        return;
      }
    }
  }
  // One tagged quad in one 32-byte load (p is 32-byte aligned at every call site: quads start at
  // multiples of 4 words of cudaMalloc'd buffers; two 16-byte loads made the step 5 % slower).
  GG_DEV void issue4(const uint64_t* p, uint64_t (&w)[4]) { ld4_relaxed(p, w); }

  // NV sums over the consumer threads with one barrier; warps 0..nw-1 hold data and receive the
  // totals (same summation order everywhere); the other warps only take part in the barrier.
  template <int NV>
  GG_DEV void csum(float* v, int nw) {
    static_assert(NV <= 4, "at most four sums per call");
    float4* s = x.S.scal + (cslot & 3) * NCW;
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
      for (int w = 0; w < nw; w++) {
        const float4 f = s[w];
        t[0] += f.x; t[1] += f.y; t[2] += f.z; t[3] += f.w;
      }
#pragma unroll
      for (int k = 0; k < NV; k++) v[k] = t[k];
    }
  }

  // One element quad (4 consecutive values) of the planes, by the thread owning quad k. The four
  // quads of a 16-element chunk sit on four consecutive lanes and share the chunk maximum by
  // shuffles, so every lane of the warp must call this (ok = false: no quad).
  // Chunk exponent e: max|x| < 2^e; X = round(x * 2^(23-e)) in (-2^23, 2^23), X = 65536*p0 + 256*p1 + p2.
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
    sts32(P.p0 + 4 * k, __byte_perm(hi01, hi23, 0x5410));
    sts32(P.p1 + 4 * k, __byte_perm(lo01, lo23, 0x7632));
    sts32(P.p2 + 4 * k, __byte_perm(lo01, lo23, 0x5410));
    if ((k & 3) == 0) sts32(P.inv + 4 * (k >> 2), (uint32_t)((127 - 23 + e) << 23));
  }

  // Planes of nq element quads held in a slot layout (sl words per CTA slot) or contiguously
  // (sl = 0), without normalisation: the inputs of the O and down projections. QPT quads per
  // thread are in flight before any tag is checked (one round trip when nq <= QPT * NCT).
  template <int QPT>
  GG_DEV void planes_gather(const XPlanes& P, const uint64_t* src, int nq, unsigned long long mq, int sl, uint32_t tag) {
    for (int base = 0; base < nq; base += QPT * NCT) {
      uint64_t w[QPT][4];
      const uint64_t* pk[QPT];
#pragma unroll
      for (int k = 0; k < QPT; k++) {
        const int q = base + tid + k * NCT;
        pk[k] = q < nq ? src + (sl ? slot_word(nq, mq, sl, q) : 4 * q) : src;
        if (q < nq)
          issue4(pk[k], w[k]);
        else
          quad_idle(w[k], tag);
      }
      settle_warp<QPT>(pk, tag, w);
#pragma unroll
      for (int k = 0; k < QPT; k++) {
        const int q = base + tid + k * NCT;
        if (base + k * NCT >= nq) break;  // uniform over the CTA
        float v[4];
        quad_vals(w[k], v);
        plane_quad(P, q, q < nq, v);
      }
    }
  }

  // out = base + v * wa / r1 with r1 = rms(v) (shaders.ts:386-418; v = the tagged words of a
  // slot layout), then the planes of out * wb / r2 with r2 = rms(out) (shaders.ts:25-56). One
  // barrier: the sums of v^2, base^2, base*v*wa and (v*wa)^2 give both norms. Thread t owns
  // element quad t; the weights are fetched before the wait.
  GG_DEV void add_norm_planes(const XPlanes& P, const uint64_t* src, uint32_t tag, const float* wa, const float* base,
                              float* out, const float* wb, float* dbg_out, float* dbg_x) {
    const GGModelDev& m = *x.m;
    const int nq = m.H >> 2, k = tid;
    const bool ok = k < nq;
    float4 fa = make_float4(0.f, 0.f, 0.f, 0.f), fb = fa, fbase = fa;
    float v[4];
    const uint64_t* p[1] = {src + slot_word(nq, m.mq_h, m.sl_h, ok ? k : 0)};
    uint64_t w[1][4];
    if (ok) {
      issue4(p[0], w[0]);
      fa = __ldg(reinterpret_cast<const float4*>(wa) + k);
      fb = __ldg(reinterpret_cast<const float4*>(wb) + k);
      fbase = reinterpret_cast<const float4*>(base)[k];
    } else {
      quad_idle(w[0], tag);
    }
    settle_warp<1>(p, tag, w);
    quad_vals(w[0], v);
    add_norm_tail(P, v, fa, fb, fbase, out, dbg_out, dbg_x);
  }

  // The same on the fixed-point sums of a K-split reduction: each warp polls its quads of
  // accumulators (every pass re-reads the lanes' incomplete words, the warp leaves together) until
  // every word counts `target` contributions. Bounded: after giving up the sums read 0.
  GG_DEV void add_norm_sums(const XPlanes& P, const unsigned long long* acc, uint32_t target, const float* wa,
                            const float* base, float* out, const float* wb, float* dbg_out, float* dbg_x) {
    const GGModelDev& m = *x.m;
    const int nq = m.H >> 2, k = tid;
    const bool ok = k < nq;
    float4 fa = make_float4(0.f, 0.f, 0.f, 0.f), fb = fa, fbase = fa;
    if (ok) {
      fa = __ldg(reinterpret_cast<const float4*>(wa) + k);
      fb = __ldg(reinterpret_cast<const float4*>(wb) + k);
      fbase = reinterpret_cast<const float4*>(base)[k];
    }
    const uint64_t* p = reinterpret_cast<const uint64_t*>(acc) + GG_ACC_QUAD_WORDS * (ok ? k : 0);
    uint64_t w[4] = {target, target, target, target};  // lanes without a quad: complete
    if (ok) issue4(p, w);
    {
      SpinClock clk;
#pragma unroll 1
      for (;;) {
        const bool done = acc_count(w[0]) == target && acc_count(w[1]) == target && acc_count(w[2]) == target &&
                          acc_count(w[3]) == target;
        if (__all_sync(0xffffffffu, done)) break;
        if (!done) issue4(p, w);
        if (__any_sync(0xffffffffu, clk.expired(x.sc))) {
          w[0] = w[1] = w[2] = w[3] = 0ull;
          break;
        }
      }
    }
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
#pragma unroll
      for (int j = 0; j < 4; j++) v[j] = acc_value(w[j]);
    }
    add_norm_tail(P, v, fa, fb, fbase, out, dbg_out, dbg_x);
  }

  GG_DEV void add_norm_tail(const XPlanes& P, const float* v, float4 fa, float4 fb, float4 fbase, float* out,
                            float* dbg_out, float* dbg_x) {
    const GGModelDev& m = *x.m;
    const int nq = m.H >> 2, k = tid, nw = (nq + 31) >> 5;
    const bool ok = k < nq;
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
    if (warp >= nw) return;
    // one square root and one division per norm (x * w / rms as x * w * (1 / rms))
    const float invh = 1.0f / (float)m.H;
    const float i1 = 1.0f / sqrtf(s[0] * invh + m.eps);
    const float i2 = 1.0f / sqrtf((s[1] + 2.f * s[2] * i1 + s[3] * (i1 * i1)) * invh + m.eps);
    float o[4], xv[4];
#pragma unroll
    for (int j = 0; j < 4; j++) {
      o[j] = bv[j] + v[j] * wav[j] * i1;
      xv[j] = o[j] * wbv[j] * i2;
    }
    if (ok) {
      reinterpret_cast<float4*>(out)[k] = make_float4(o[0], o[1], o[2], o[3]);
      if (dbg_out) reinterpret_cast<float4*>(dbg_out)[k] = make_float4(o[0], o[1], o[2], o[3]);
      if (dbg_x) reinterpret_cast<float4*>(dbg_x)[k] = make_float4(xv[0], xv[1], xv[2], xv[3]);
    }
    plane_quad(P, k, ok, xv);
  }

  // x = rmsNorm(h) * wb for a hidden state h already in hand (thread t: quad t), as planes.
  GG_DEV void norm_planes(const XPlanes& P, const float* h, bool ok, const float* wb, float* dbg_x) {
    const GGModelDev& m = *x.m;
    const int k = tid, nw = ((m.H >> 2) + 31) >> 5;
    float4 fb = make_float4(0.f, 0.f, 0.f, 0.f);
    float s[1] = {0.f};
    if (ok) {
      fb = __ldg(reinterpret_cast<const float4*>(wb) + k);
#pragma unroll
      for (int j = 0; j < 4; j++) s[0] += h[j] * h[j];
    }
    csum<1>(s, nw);
    if (warp >= nw) return;
    const float ir = 1.0f / sqrtf(s[0] * (1.0f / (float)m.H) + m.eps);
    const float wbv[4] = {fb.x, fb.y, fb.z, fb.w};
    float xv[4];
#pragma unroll
    for (int j = 0; j < 4; j++) xv[j] = h[j] * wbv[j] * ir;
    if (ok && dbg_x) reinterpret_cast<float4*>(dbg_x)[k] = make_float4(xv[0], xv[1], xv[2], xv[3]);
    plane_quad(P, k, ok, xv);
  }

  // shaders.ts:2-23: h[i] = q * d * sqrt(H), evaluated left to right in f32; then the planes of
  // rmsNorm(h) * wb.
  GG_DEV void embed_planes(const XPlanes& P, const float* wb) {
    const GGModelDev& m = *x.m;
    const uint8_t* row = m.embd + (size_t)x.token * m.rs_h;
    const float sq = sqrtf((float)m.H);
    const int k = tid;
    const bool ok = k < (m.H >> 2);
    float o[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      const float d = __half2float(*reinterpret_cast<const __half*>(row + m.H + 2 * ((4 * k) >> 5)));
#pragma unroll
      for (int j = 0; j < 4; j++) {
        float vv = (float)(int8_t)row[4 * k + j] * d;
        o[j] = vv * sq;
      }
      reinterpret_cast<float4*>(x.S.hid)[k] = make_float4(o[0], o[1], o[2], o[3]);
    }
    norm_planes(P, o, ok, wb, nullptr);
  }

  // The CTA's n rows (n <= 16) of a phase, in the ph.nst ring stages of its map (all resident at
  // once: the host checks nst < NS; the caller gated them before its barrier). Work units are
  // (group of four rows, K slice), as mv_map assigns them, so the four rows share every load of
  // the x planes. The slice totals meet in shared memory; thread r < n sums them in
  // slice order and stores the row total as tagged word out[r]. Every consumer warp must call
  // this (it holds a CTA barrier).
  GG_DEV void matvec(const XPlanes& P, const MvPhase& ph, int K, uint64_t* out, uint32_t tag) {
    const MvWarp& e = ph.w[warp];
    const int n = ph.n, S = ph.S, g = e.g;
    float* red = x.S.red;  // [row][slice]
    if (g != 0xff) {
      uint32_t ra[4];
      const uint32_t ring = smem_u32(x.S.ring);
#pragma unroll
      for (int k = 0; k < 4; k++) {  // rows past n repeat the last row; their sums are dropped
        const uint32_t o = e.roff[k];
        ra[k] = ring + ((idx + (o >> 16)) % NS) * GG_STEP_STAGE_BYTES + (o & 0xffffu);
      }
      const float4 v = dot_rows4(ra, K, e.c0, e.c1, P);
      if (lane == 0) {
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; k++)
          if (4 * g + k < n) red[(4 * g + k) * S + e.sl] = vv[k];
      }
    }
    cbar();
    release_all(ph.nst);
    if (tid < n) {
      float t = 0.f;
      for (int k = 0; k < S; k++) t += red[tid * S + k];
      tag_store(out + tid, t, tag);
    }
  }

  // Row pairs (2j, 2j + 1), rps / 2 pairs per ring stage, in units of four pairs: unit n goes to
  // warp n % NCW, whose four 8-lane groups take one pair each; the group's first lane passes the
  // pair to epi(j, row 2j, row 2j + 1).
  // gated: the stages are resident and were gated by the caller (who releases them after a
  // barrier); otherwise they stream in and every warp waits for and releases each.
  template <class Epi>
  GG_DEV void matvec_pairs(const XPlanes& P, int npairs, int rps, int K, int rs, bool gated, Epi epi) {
    const int pps = rps >> 1, g = lane >> 3;
    int unit = 0, k = 0;
    for (int j0 = 0; j0 < npairs; j0 += pps, k++) {
      const int j1 = min(j0 + pps, npairs);
      const int nu = (j1 - j0 + 3) >> 2;  // units in this stage (one per warp: NCW > 1)
      const int mine = (warp - unit % NCW + NCW) % NCW;  // which of this stage's units is this warp's
      if (mine < nu) {
        const uint8_t* stg = gated ? x.S.ring + (size_t)((idx + (uint32_t)k) % NS) * GG_STEP_STAGE_BYTES : owner_wait(k);
        const int j = j0 + 4 * mine + g;
        const float2 v = dot_pair8(smem_u32(stg) + (uint32_t)(2 * (min(j, j1 - 1) - j0) * rs), rs, K, P);
        if ((lane & 7) == 0 && j < j1) epi(j, v.x, v.y);
        if (!gated) {  // the stage's owners release it: NCW arrivals in all, the first owner giving the rest
          __syncwarp();
          if (lane == 0 && !dead && !*(volatile uint32_t*)x.sc.err)
            mbar_arrive_cnt(&x.S.empty[(idx + (uint32_t)k) % NS], mine == 0 ? (uint32_t)(NCW - nu + 1) : 1u);
        }
      }
      unit += nu;
    }
    if (!gated) idx += (uint32_t)k;
  }

  // Streamed stage k places after the ring position, waited for only by the warps that compute
  // on it: first until the producer has issued it (so the slot's previous use was released and
  // the parity wait below cannot match it), then for its copy. Bounded.
  GG_DEV const uint8_t* owner_wait(int k) {
    const uint32_t want = idx + (uint32_t)k + 1u;
    SpinClock clk;
#pragma unroll 1
    while ((int)(*(volatile uint32_t*)(x.S.flag + 1) - want) < 0) {
      if (__any_sync(0xffffffffu, clk.expired(x.sc))) {
        dead = true;
        break;
      }
    }
    return stage_wait_ahead(k);
  }

  GG_DEV void phase_qkv(int l) {
    const GGModelDev& m = *x.m;
    if (l == 0) {
      embed_planes(x.S.xa, m.layers[0].attn_norm);
    } else {  // hidden = residual + post_ffw_norm(down) (engine.ts:794), attention rmsNorm (768)
      add_norm_planes(x.S.xa, m.t_down, make_tag(x.tagbase, (l - 1) * PH + 5), m.layers[l - 1].post_ffw_norm, x.S.res,
                      x.S.hid, m.layers[l].attn_norm, blockIdx.x == 0 ? m.dbg_hidden : nullptr, nullptr);
    }
    gate(x.mv[0].nst);
    cbar();
    trace(l * PH + 0, 1);
    uint64_t* out = m.t_qkv + (size_t)blockIdx.x * m.sl_qkv;
    const uint32_t tag = make_tag(x.tagbase, l * PH + 0);
    matvec(x.S.xa, x.mv[0], m.H, out, tag);
  }

  // q/k per-head RMSNorm + RoPE (shaders.ts:420-467), the KV store (shaders.ts:209-227) and this
  // CTA's attention splits (shaders.ts:229-325) with local softmax statistics.
  GG_DEV void phase_attn(int l) {
    const GGModelDev& m = *x.m;
    const GGLayerW& Lw = m.layers[l];
    constexpr int G = GG_STEP_GRID;
    const int s0 = first_split(m, l, x.pos, x.nsplit, blockIdx.x);
    const int att_nst = s0 < x.nsplit ? (x.nsplit - 1 - s0) / G + 1 : 0;  // this CTA's splits (KV stages)
    if (s0 >= x.nsplit) return;
    constexpr int HD = GG_HEAD_DIM;
    const int NQH = m.NQH, NKH = m.NKH, Q = m.Q, KV = m.KV;
    float* t = x.S.tmp;  // q [Q] | k [KV] | v [KV]
    const uint32_t tagA = make_tag(x.tagbase, l * PH + 0);
    // One warp per q, k or v head. Lane l takes quads l and l + 32 of its head (elements 4l..4l+3
    // and HD/2 + 4l..): the RoPE pairs (i, i + HD/2) sit in one lane, and the norm weights and the
    // RoPE row are fetched in the same round trip as the head's values.
    static_assert(GG_HEAD_DIM == 256, "two quads per lane cover a head");
    const int nq = (Q + 2 * KV) >> 2;
    for (int h = warp; h < NQH + 2 * NKH; h += NCW) {
      const bool normed = h < NQH + NKH;  // q and k heads; v is stored as is
      const int q0 = h * (HD / 4) + lane, q1 = q0 + HD / 8;
      const uint64_t* pq[2] = {m.t_qkv + slot_word(nq, m.mq_qkv, m.sl_qkv, q0), m.t_qkv + slot_word(nq, m.mq_qkv, m.sl_qkv, q1)};
      uint64_t w[2][4];
      issue4(pq[0], w[0]);
      issue4(pq[1], w[1]);
      float4 n0 = make_float4(1.f, 1.f, 1.f, 1.f), n1 = n0, c0 = make_float4(1.f, 0.f, 1.f, 0.f), c1 = c0;
      if (normed) {
        const float4* nw = reinterpret_cast<const float4*>(h < NQH ? Lw.q_norm : Lw.k_norm);
        n0 = __ldg(nw + lane);
        n1 = __ldg(nw + lane + HD / 8);
        const float4* cr = reinterpret_cast<const float4*>(Lw.rope + (size_t)x.pos * (HD / 2) + 4 * lane);  // (cos, sin) x 4
        c0 = __ldg(cr);
        c1 = __ldg(cr + 1);
      }
      settle_warp<2>(pq, tagA, w);
      float a[4], b[4];
      quad_vals(w[0], a);
      quad_vals(w[1], b);
      if (normed) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 4; j++) ss += a[j] * a[j] + b[j] * b[j];
        const float ir = 1.0f / sqrtf(warp_sum(ss) * (1.0f / (float)HD) + m.eps);
        const float na[4] = {n0.x, n0.y, n0.z, n0.w}, nb[4] = {n1.x, n1.y, n1.z, n1.w};
        const float cs[4] = {c0.x, c0.z, c1.x, c1.z}, sn[4] = {c0.y, c0.w, c1.y, c1.w};
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float x0 = a[j] * na[j] * ir, x1 = b[j] * nb[j] * ir;
          a[j] = x0 * cs[j] - x1 * sn[j];
          b[j] = x0 * sn[j] + x1 * cs[j];
        }
      }
      if (KV16 && h >= NQH) {  // bf16 cache: attention reads the stored (rounded) k and v
#pragma unroll
        for (int j = 0; j < 4; j++) {
          a[j] = bf16_rne(a[j]);
          b[j] = bf16_rne(b[j]);
        }
      }
      reinterpret_cast<float4*>(t)[q0] = make_float4(a[0], a[1], a[2], a[3]);
      reinterpret_cast<float4*>(t)[q1] = make_float4(b[0], b[1], b[2], b[3]);
    }
    cbar();
    trace(l * PH + 1, 1);
    // the CTA whose splits include the new position stores its k and v
    if (x.pos / GG_POS_PER_SPLIT >= s0 && (x.pos / GG_POS_PER_SPLIT - s0) % G == 0) {
      using KT = kv_t<KV16>;
      const size_t off = (size_t)x.seq * m.kv_seq_stride + ((size_t)l * m.CTX + x.pos) * KV;
      KT* kc = reinterpret_cast<KT*>(m.kcache);
      KT* vc = reinterpret_cast<KT*>(m.vcache);
      for (int i = tid; i < KV; i += NCT) {
        kc[off + i] = kv_narrow<KV16>(t[Q + i]);
        vc[off + i] = kv_narrow<KV16>(t[Q + KV + i]);
      }
    }
    const uint32_t tag = make_tag(x.tagbase, l * PH + 1);
    const int plo = window_lo(Lw, x.pos);
    // Split k of this CTA is handled by warps NQH*k .. NQH*k + NQH - 1 (one per query head), which
    // wait for its KV stage themselves and release it when done: NCW arrivals in all, the first
    // warp giving those of the warps that do not read it. Every later ring wait follows the
    // merge's CTA barrier, which these arrivals precede.
    const int k = warp / NQH;
    if (k < att_nst) {
      attn_split(s0 + k * G, plo, stage_wait_ahead(k), warp % NQH, tag);
      __syncwarp();
      if (lane == 0 && !dead && !*(volatile uint32_t*)x.sc.err)
        mbar_arrive_cnt(&x.S.empty[(idx + (uint32_t)k) % NS], warp % NQH == 0 ? (uint32_t)(NCW - NQH + 1) : 1u);
    }
    idx += (uint32_t)att_nst;
  }

  // One split of PPS = 8 positions for query head h (one warp): K rows at the start of the stage,
  // V rows after PPS K rows; the current position's k and v come from the scratch vector.
  // Scores: lane (p, j) = (lane / 4, lane % 4) takes position p over head dims [64j, 64j + 64)
  // (its 16-byte chunks rotated by 2j + p % 2, so the eight lanes of a quarter warp read eight
  // different bank groups), and
  // two shuffles finish the dot product: all eight positions are scored at once. Softmax over the
  // positions inside the window by three shuffle levels; then lane l accumulates dims 8l..8l+7 of
  // the weighted V rows. Output: the split's unnormalised o (256 values), its max and its sum of
  // exp, into the split's slot of the exchange buffer.
  __device__ __noinline__ void attn_split(int s, int plo, const uint8_t* stg, int h, uint32_t tag) {
    using KT = kv_t<KV16>;
    const GGModelDev& m = *x.m;
    const int Q = m.Q, KV = m.KV, NQH = m.NQH, NKH = m.NKH;
    constexpr int HD = GG_HEAD_DIM;
    static_assert(GG_HEAD_DIM == 256 && GG_POS_PER_SPLIT == 8, "lanes are 8 positions x 4 quarters of a head");
    constexpr int PPS = GG_POS_PER_SPLIT;
    const float* t = x.S.tmp;
    const int p0 = s * PPS, np = min(p0 + PPS, x.pos + 1) - p0;
    const int pv = max(plo - p0, 0);  // positions before pv are outside the window (pv < np)
    const int kvh = h * NKH / NQH;
    const KT* Kst = reinterpret_cast<const KT*>(stg) + kvh * HD;
    const KT* Vst = reinterpret_cast<const KT*>(stg + (size_t)PPS * KV * sizeof(KT)) + kvh * HD;
    const float* qh = t + h * HD;
    const float* kcur = t + Q + kvh * HD;
    const float* vcur = t + Q + KV + kvh * HD;
    // ---- scores (every lane reads a row of the split: positions outside [pv, np) read row pv)
    const int p = lane >> 2, j = lane & 3, rot = 2 * j + (p & 1);
    const bool valid = p >= pv && p < np;
    const int pk = valid ? p : pv;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    const auto dot_f32 = [&](const float* kr) {  // kr: the row's quarter j
#pragma unroll 4
      for (int i = 0; i < 16; i++) {
        const int r = (i + rot) & 15;
        const float4 k4 = reinterpret_cast<const float4*>(kr)[r];
        const float4 q4 = reinterpret_cast<const float4*>(qh + 64 * j)[r];
        d[0] = fmaf(q4.x, k4.x, d[0]);
        d[1] = fmaf(q4.y, k4.y, d[1]);
        d[2] = fmaf(q4.z, k4.z, d[2]);
        d[3] = fmaf(q4.w, k4.w, d[3]);
      }
    };
    if (p0 + pk < x.pos) {
      if constexpr (KV16) {
        const KT* kr = Kst + (size_t)pk * KV + 64 * j;
#pragma unroll 4
        for (int i = 0; i < 8; i++) {
          const int r = (i + rot) & 7;
          float kf[8];
          bf16x8_widen(reinterpret_cast<const uint4*>(kr)[r], kf);
          const float4 qa = reinterpret_cast<const float4*>(qh + 64 * j)[2 * r];
          const float4 qb = reinterpret_cast<const float4*>(qh + 64 * j)[2 * r + 1];
          d[0] = fmaf(qa.x, kf[0], d[0]);
          d[1] = fmaf(qa.y, kf[1], d[1]);
          d[2] = fmaf(qa.z, kf[2], d[2]);
          d[3] = fmaf(qa.w, kf[3], d[3]);
          d[0] = fmaf(qb.x, kf[4], d[0]);
          d[1] = fmaf(qb.y, kf[5], d[1]);
          d[2] = fmaf(qb.z, kf[6], d[2]);
          d[3] = fmaf(qb.w, kf[7], d[3]);
        }
      } else {
        dot_f32(reinterpret_cast<const float*>(Kst + (size_t)pk * KV) + 64 * j);
      }
    } else {
      dot_f32(kcur + 64 * j);
    }
    float sc = (d[0] + d[1]) + (d[2] + d[3]);
    sc += __shfl_xor_sync(0xffffffffu, sc, 1);
    sc += __shfl_xor_sync(0xffffffffu, sc, 2);
    sc *= m.attn_scale;
    float mx = valid ? sc : -INFINITY;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float e = valid ? __expf(sc - mx) : 0.f;
    float sum = e;
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    // ---- o = sum_p e_p v_p (invalid positions weigh 0 and read row pv)
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int q = 0; q < PPS; q++) {
      const float w = __shfl_sync(0xffffffffu, e, 4 * q);
      const int pq = (q >= pv && q < np) ? q : pv;
      float vf[8];
      if (p0 + pq < x.pos && KV16) {
        bf16x8_widen(*reinterpret_cast<const uint4*>(Vst + (size_t)pq * KV + 8 * lane), vf);
      } else {
        // lanes 4..7 of each quarter warp load their two 16-byte halves in the other order, so the
        // quarter's first loads cover all eight bank groups
        const float* vr = p0 + pq < x.pos ? reinterpret_cast<const float*>(Vst + (size_t)pq * KV) : vcur;
        const int sw = (lane >> 2) & 1;
        const float4 u = reinterpret_cast<const float4*>(vr + 8 * lane)[sw];
        const float4 v = reinterpret_cast<const float4*>(vr + 8 * lane)[sw ^ 1];
        const float4 a = sw ? v : u, b = sw ? u : v;
        vf[0] = a.x; vf[1] = a.y; vf[2] = a.z; vf[3] = a.w;
        vf[4] = b.x; vf[5] = b.y; vf[6] = b.z; vf[7] = b.w;
      }
#pragma unroll
      for (int jj = 0; jj < 8; jj++) acc[jj] = fmaf(w, vf[jj], acc[jj]);
    }
    uint64_t* o = m.t_o + (size_t)s * m.att_slot + (size_t)h * (HD + 4);
    // One 32-byte sector per store (att_slot and HD + 4 are multiples of 4 words, so every quad
    // is sector-aligned). Written as 8-byte stores 64 bytes apart, the split's 2 KB made the step
    // 0.644 instead of 0.583 ms per token.
    static_assert((HD + 4) % 4 == 0, "split slots of whole sectors");
#pragma unroll
    for (int jj = 0; jj < 8; jj += 4) tag_store4(o + 8 * lane + jj, acc[jj], acc[jj + 1], acc[jj + 2], acc[jj + 3], tag);
    if (lane == 0) tag_store4(o + HD, mx, sum, 0.f, 0.f, tag);  // header quad: max, sum of exp, two zeros
  }

  // Merge of the attention splits (online softmax) for 8 output dimensions per unit. The unit's
  // splits are spread over W = ceil(splits / 32) warps, one split per lane, every load in flight
  // before any check; each warp merges its lanes, and warp 0 merges the W warp results from
  // shared memory in warp order and stores the unit's outputs.
  GG_DEV void phase_combine(int l) {
    const GGModelDev& m = *x.m;
    constexpr int HD = GG_HEAD_DIM;
    const int ncomb = m.Q >> 3;
    const uint32_t tagB = make_tag(x.tagbase, l * PH + 1);
    const uint32_t tagC = make_tag(x.tagbase, l * PH + 2);
    const int slo = window_lo(m.layers[l], x.pos) / GG_POS_PER_SPLIT;
    const int ns = x.nsplit - slo, W = min((ns + 31) >> 5, NCW);
    float* part = x.S.red;  // [warp][10]: max, sum, 8 outputs
    const int u = blockIdx.x;
    const bool have = u < ncomb;  // one unit per CTA (the host checks Q / 8 <= grid)
    const int d0 = 8 * u, h = d0 / HD, dh = d0 % HD;
    if (have && warp < W) {
      float mx = -INFINITY, lsum = 0.f, acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int sb = slo + warp * 32; sb < x.nsplit; sb += 32 * W) {  // uniform over the warp
        const int s = sb + lane;
        const bool act = s < x.nsplit;
        const uint64_t* pb = m.t_o + (size_t)(act ? s : sb) * m.att_slot + (size_t)h * (HD + 4);
        const uint64_t* pq[3] = {pb + HD, pb + dh, pb + dh + 4};
        uint64_t w[3][4];
#pragma unroll
        for (int k = 0; k < 3; k++) {
          if (act)
            issue4(pq[k], w[k]);
          else
            quad_idle(w[k], tagB);
        }
        settle_warp<3>(pq, tagB, w);
        if (!act) continue;
        float fml[4], f0[4], f1[4];
        quad_vals(w[0], fml);
        quad_vals(w[1], f0);
        quad_vals(w[2], f1);
        const float nm = fmaxf(mx, fml[0]);
        const float a = (mx == -INFINITY) ? 0.f : expf(mx - nm);
        const float b = expf(fml[0] - nm);
        lsum = fmaf(b, fml[1], lsum * a);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          acc[j] = fmaf(b, f0[j], acc[j] * a);
          acc[4 + j] = fmaf(b, f1[j], acc[4 + j] * a);
        }
        mx = nm;
      }
      const float gm = warp_max(mx);
      const float f = (mx == -INFINITY) ? 0.f : expf(mx - gm);
      lsum = warp_sum(lsum * f);
      float res = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        const float a = warp_sum(acc[j] * f);
        if (lane == j) res = a;
      }
      if (lane == 0) {
        part[warp * 10] = gm;
        part[warp * 10 + 1] = lsum;
      }
      if (lane < 8) part[warp * 10 + 2 + lane] = res;
    }
    cbar();  // the other warps wait here instead of polling the merged words
    if (!have) return;  // uniform over the CTA
    float* av = x.S.red + 16 * ((10 * NCW + 15) / 16);  // the unit's 8 merged values, after part[]
    if (warp == 0) {
      float gm = -INFINITY;
      for (int w = 0; w < W; w++) gm = fmaxf(gm, part[w * 10]);
      float lsum = 0.f, o = 0.f;
      for (int w = 0; w < W; w++) {
        const float wm = part[w * 10];
        const float f = (wm == -INFINITY) ? 0.f : expf(wm - gm);
        lsum = fmaf(f, part[w * 10 + 1], lsum);
        if (lane < 8) o = fmaf(f, part[w * 10 + 2 + lane], o);
      }
      if (lane < 8) {
        av[lane] = o / lsum;
        tag_store(m.t_att + d0 + lane, o / lsum, tagC);  // kept for gg_debug_read
      }
    }
    // O projection by columns (shaders.ts matmul of attn_output, engine.ts:783): this unit adds
    // Wo[r][d0..d0+7] . o for every row r into the layer's accumulators, then counts itself in.
    constexpr int nst = 1;  // the host checks H <= wo_rows_per_stage
    gate(nst);
    cbar();
    float a[8];
#pragma unroll
    for (int j = 0; j < 8; j++) a[j] = av[j];
    unsigned long long* acc = m.acc + ((size_t)x.par * m.L + l) * m.acc_stride;
    const uint32_t slice = smem_u32(x.S.ring) + (idx % NS) * GG_STEP_STAGE_BYTES;
    for (int r = tid; r < m.H; r += NCT) {
      const uint2 w = lds64(slice + 8u * (uint32_t)r);
      const uint32_t q[2] = {w.x, w.y};
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 8; j++) sum = fmaf((float)((int)(q[j >> 2] << (24 - 8 * (j & 3))) >> 24), a[j], sum);
      acc_add(acc + ((r >> 2) * GG_ACC_QUAD_WORDS + (r & 3)), sum * lds_half(slice + 8u * (uint32_t)m.H + 2u * (uint32_t)r));
    }
    cbar();
    release_all(nst);
  }

  GG_DEV void phase_ffn_up(int l) {
    const GGModelDev& m = *x.m;
    const GGLayerW& Lw = m.layers[l];
    // residual = hidden + post_attention_norm(proj) (engine.ts:785), then ffn rmsNorm (786)
    const size_t ai = (size_t)x.par * m.L + l;
    add_norm_sums(x.S.xa, m.acc + ai * m.acc_stride, (uint32_t)m.ncomb, Lw.post_attn_norm, x.S.hid,
                  x.S.res, Lw.ffn_norm, blockIdx.x == 0 ? m.dbg_residual : nullptr, nullptr);
    const int n = x.S.rows[RG_I + 1] - x.S.rows[RG_I];
    const int nst = (n + (m.rps_gu >> 1) - 1) / (m.rps_gu >> 1);
    gate(nst);
    cbar();
    trace(l * PH + 4, 1);
    uint64_t* out = m.t_act + (size_t)blockIdx.x * m.sl_i;
    const uint32_t tag = make_tag(x.tagbase, l * PH + 4);
    // gate_i and up_i are adjacent rows (2i, 2i + 1): GeGLU on the pair (shaders.ts:153-170)
    matvec_pairs(x.S.xa, n, m.rps_gu, m.H, m.rs_h, true,
                 [&](int j, float g, float u) { tag_store(out + j, gelu_tanh(g) * u, tag); });
    cbar();
    release_all(nst);
  }

  GG_DEV void phase_down(int l) {
    const GGModelDev& m = *x.m;
    planes_gather<4>(x.S.xb, m.t_act, m.I >> 2, m.mq_i, m.sl_i, make_tag(x.tagbase, l * PH + 4));
    gate(x.mv[1].nst);
    cbar();
    trace(l * PH + 5, 1);
    uint64_t* out = m.t_down + (size_t)blockIdx.x * m.sl_h;
    const uint32_t tag = make_tag(x.tagbase, l * PH + 5);
    matvec(x.S.xb, x.mv[1], m.I, out, tag);
  }

  GG_DEV void phase_lm() {
    const GGModelDev& m = *x.m;
    if (x.mode & GG_RUN_LAYERS) {  // hidden = residual + post_ffw_norm(down), final rmsNorm (engine.ts:797-801)
      add_norm_planes(x.S.xa, m.t_down, make_tag(x.tagbase, (m.L - 1) * PH + 5), m.layers[m.L - 1].post_ffw_norm,
                      x.S.res, x.S.hid, m.out_norm, blockIdx.x == 0 ? m.dbg_hidden : nullptr,
                      blockIdx.x == 0 ? m.dbg_normed : nullptr);
    } else {  // LM head on the hidden state a previous launch left behind
      const bool ok = tid < (m.H >> 2);
      float h[4] = {0.f, 0.f, 0.f, 0.f};
      if (ok) {
        const float4 f = reinterpret_cast<const float4*>(m.dbg_hidden)[tid];
        h[0] = f.x; h[1] = f.y; h[2] = f.z; h[3] = f.w;
        reinterpret_cast<float4*>(x.S.hid)[tid] = f;
      }
      norm_planes(x.S.xa, h, ok, m.out_norm, blockIdx.x == 0 ? m.dbg_normed : nullptr);
    }
    cbar();
    const int rb = x.S.rows[RG_V], re = x.S.rows[RG_V + 1];
    float* lg = x.S.lmv;  // this CTA's logits, row rb + i at i
    float2* gl = reinterpret_cast<float2*>(m.logits + rb);
    matvec_pairs(x.S.xa, (re - rb) >> 1, m.rps_gu, m.H, m.rs_h, false, [&](int j, float a, float b) {
      reinterpret_cast<float2*>(lg)[j] = make_float2(a, b);
      gl[j] = make_float2(a, b);
    });
    cbar();
    // topk256 lanes (shaders.ts:363-384): lane t keeps the largest logit among rows = t (mod 256)
    // with strict '>' from (-1e30, 0), so the first index wins a tie; NaN is never taken and -0
    // is keyed as +0. One thread per lane scans this CTA's rows of that lane in index order.
    if (tid < 256) {
      const unsigned long long ik = init_lane_key();
      unsigned long long best = ik;
      for (int r = rb + ((tid - rb) & 255); r < re; r += 256) {
        float v = lg[r - rb];
        if (!isnan(v)) {
          if (v == 0.0f) v = 0.0f;
          const unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - (uint32_t)r);
          best = k > best ? k : best;
        }
      }
      if (best != ik) atomicMax(&m.lane_keys[tid], best);
    }
  }

  GG_DEV void run() {
    const GGModelDev& m = *x.m;
    if (x.mode & GG_RUN_LAYERS) {
      for (int l = 0; l < m.L; l++) {
        trace(l * PH + 0, 0);
        phase_qkv(l);
        trace(l * PH + 0, 2);
        trace(l * PH + 1, 0);
        phase_attn(l);
        trace(l * PH + 1, 2);
        trace(l * PH + 2, 0);
        phase_combine(l);
        trace(l * PH + 2, 2);
        trace(l * PH + 4, 0);
        phase_ffn_up(l);
        trace(l * PH + 4, 2);
        trace(l * PH + 5, 0);
        phase_down(l);
        trace(l * PH + 5, 2);
      }
      if (!(x.mode & GG_RUN_LM)) {  // leave the hidden state for a later LM-head launch
        add_norm_planes(x.S.xa, m.t_down, make_tag(x.tagbase, (m.L - 1) * PH + 5), m.layers[m.L - 1].post_ffw_norm,
                        x.S.res, x.S.hid, m.out_norm, blockIdx.x == 0 ? m.dbg_hidden : nullptr, nullptr);
      }
    }
    if (x.mode & GG_RUN_LM) {
      trace(m.L * PH, 0);
      phase_lm();
      trace(m.L * PH, 2);
    }
  }
};

// ---------------------------------------------------------------------------------- kernel

template <bool KV16>
GG_DEV void step_body(const GGModelDev* __restrict__ mp, GGState* __restrict__ st, const GGState& in, int use_in,
                      GGState* host_st) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ Ctx x;
  const GGModelDev& m = *mp;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the descriptor's copy in shared memory (its size is a multiple of 8 bytes)
  GGModelDev* msm = reinterpret_cast<GGModelDev*>(smem + m.sm_model);
  {
    const int nw = (int)(GG_MODEL_BYTES(m.L) / 8);
    const uint64_t* src = reinterpret_cast<const uint64_t*>(mp);
    uint64_t* dst = reinterpret_cast<uint64_t*>(msm);
    for (int i = threadIdx.x; i < nw; i += blockDim.x) dst[i] = src[i];
  }
  if (threadIdx.x == 0) {
  x.m = msm;
  x.st = st;
  // host inputs from the launch's parameters (gg_step) or from the device state (chained launches)
  x.mode = use_in ? in.mode : st->mode;
  x.token = use_in ? in.token : st->token;
  x.pos = use_in ? in.pos : st->pos;
  x.seq = use_in ? in.seq : st->seq;
  x.tagbase = st->epoch;
  x.par = st->parity & 1u;
  x.sc.err = &st->error;
  x.sc.timeout_ns = use_in ? in.timeout_ns : st->timeout_ns;
  // carve shared memory (offsets and GGModelDev::smem_bytes computed by the host)
  x.S.ring = smem;
  x.S.full = reinterpret_cast<uint64_t*>(smem + (size_t)NS * GG_STEP_STAGE_BYTES);
  x.S.empty = x.S.full + NS;
  XPlanes* xp[2] = {&x.S.xa, &x.S.xb};
  const int xsz[2] = {m.xs0, m.xs1}, xoff[2] = {m.sm_xa, m.sm_xb};
  for (int b = 0; b < 2; b++) {
    const uint32_t a = smem_u32(smem + xoff[b]);
    xp[b]->p0 = a;
    xp[b]->p1 = a + xsz[b];
    xp[b]->p2 = a + 2 * xsz[b];
    xp[b]->inv = a + 3 * xsz[b];
  }
  x.S.hid = reinterpret_cast<float*>(smem + m.sm_hid);
  x.S.res = reinterpret_cast<float*>(smem + m.sm_res);
  x.S.tmp = reinterpret_cast<float*>(smem + m.sm_tmp);
  x.S.lmv = reinterpret_cast<float*>(smem + m.sm_lmv);
  x.S.scal = reinterpret_cast<float4*>(smem + m.sm_scal);
  x.S.red = reinterpret_cast<float*>(smem + m.sm_red);
  x.S.flag = reinterpret_cast<int*>(smem + m.sm_flag);
  x.S.rows = reinterpret_cast<int*>(smem + m.sm_rows);

  x.S.flag[1] = 0;  // stages issued by the producer
  const bool bad = x.token < 0 || x.token >= m.V || x.pos < 0 || x.pos >= m.CTX || x.seq < 0 || x.seq >= m.max_seqs;
  if (bad) {
    if (blockIdx.x == 0) atomicOr(&st->error, GG_ERR_BAD_INPUT);
    x.mode = 0;
  }
  x.nsplit = (x.pos + GG_POS_PER_SPLIT) / GG_POS_PER_SPLIT;  // ceil((pos + 1) / PPS)
    for (int i = 0; i < (int)NS; i++) {
      mbar_init(&x.S.full[i], 1);
      mbar_init(&x.S.empty[i], NCW);
    }
    mbar_fence_init();
    const int c = blockIdx.x;
    const int nq[4] = {(m.Q + 2 * m.KV) >> 2, m.H >> 2, m.I >> 2, m.V >> 2};
    for (int k = 0; k < 4; k++) {
      x.S.rows[2 * k] = 4 * qpart(nq[k], c);
      x.S.rows[2 * k + 1] = 4 * qpart(nq[k], c + 1);
    }
  }
  __syncthreads();
  if (threadIdx.x < 2 * NCW) {  // the matvec maps of the q/k/v (0) and down (1) phases
    const int p = threadIdx.x / NCW, w = threadIdx.x % NCW;
    if (p == 0)
      mv_map(x.mv[0], w, x.S.rows[RG_QKV + 1] - x.S.rows[RG_QKV], m.rps_h, m.H, m.rs_h);
    else
      mv_map(x.mv[1], w, x.S.rows[RG_H + 1] - x.S.rows[RG_H], m.rps_i, m.I, m.rs_i);
  }
  {  // zero this CTA's share of the other accumulator set (the next launch's)
    unsigned long long* a = m.acc + (size_t)(x.par ^ 1u) * m.L * m.acc_stride;
    const int n = m.L * m.acc_stride, stride = m.grid * (int)blockDim.x;
    for (int i = blockIdx.x * (int)blockDim.x + (int)threadIdx.x; i < n; i += stride) a[i] = 0ull;
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
    const uint32_t t = atomicAdd(&st->done, 1u);
    *x.S.flag = (t == (uint32_t)m.grid - 1) ? 1 : 0;
  }
  __syncthreads();
  if (!*x.S.flag) return;
  __threadfence();
  if (use_in && threadIdx.x == 0) {  // the launch's inputs become the device state (sampler, chains)
    st->token = in.token;
    st->pos = in.pos;
    st->seq = in.seq;
    st->mode = in.mode;
    st->temperature = in.temperature;
    st->top_p = in.top_p;
    st->rep_penalty = in.rep_penalty;
    st->step_index = in.step_index;
    st->uniform = in.uniform;
    st->uniforms = in.uniforms;
    st->timeout_ns = in.timeout_ns;
    st->prefill_ids = in.prefill_ids;
    st->prefill_left = in.prefill_left;
    st->ring_len = in.ring_len;
    st->token_ring = in.token_ring;
  }
  __syncthreads();
  int tok = -1;
  if (x.mode & GG_RUN_SAMPLE) tok = sample_token(m, st, *reinterpret_cast<SampleScratch*>(smem));  // ring is idle
  __syncthreads();
  if (threadIdx.x < 256) m.lane_keys[threadIdx.x] = init_lane_key();
  if (threadIdx.x == 0) {
    st->epoch = st->epoch + (uint32_t)(m.L * PH + 1);
    st->done = 0;
    st->parity = x.par ^ 1u;
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
    if (host_st) {  // the device-owned tail straight into the caller's mapped pinned state
      volatile GGState* h = host_st;
      h->epoch = st->epoch;
      h->done = 0;
      h->error = *(volatile uint32_t*)&st->error;
      h->out_token = st->out_token;
      h->seen_count = st->seen_count;
      h->parity = st->parity;
      __threadfence_system();
    }
  }
}

}  // namespace step

extern "C" __global__ void __launch_bounds__(step::NTH, 1)
    gg_step_kernel(const GGModelDev* __restrict__ mp, GGState* __restrict__ st, const GGState in, int use_in,
                   GGState* host_st) {
  step::step_body<false>(mp, st, in, use_in, host_st);
}

// The same kernel for a bf16 KV cache (GG_FLAG_KV_BF16).
extern "C" __global__ void __launch_bounds__(step::NTH, 1)
    gg_step_kernel_kv16(const GGModelDev* __restrict__ mp, GGState* __restrict__ st, const GGState in, int use_in,
                        GGState* host_st) {
  step::step_body<true>(mp, st, in, use_in, host_st);
}

}  // namespace gg
