// gg_prefill.cu -- the kernels between the tensor-core GEMMs of a batched prefill.
//
// The reference prefills serially, one full forward per prompt token (engine.ts:923-928).
// Here a chunk of T prompt tokens moves through each layer together: the matrices become
// GEMMs over T rows (gg_gemm.cu), and the per-token work between them -- norms, residual adds,
// q/k norm + RoPE, the KV store, causal attention over the cache, GeGLU -- runs in the
// kernels below, one CTA per token row (attention: per block of query rows and key range). The math per token
// is the reference's (formulas of shaders.ts, f32 throughout); only the order of some sums
// differs, within f32 rounding.
#include "gg_gemm_dev.cuh"
#include "gg_launch.h"
#include "gg_prefill.h"

namespace gg {

constexpr int PF_THREADS = 256;
constexpr int PF_MAX_H = 4096;
constexpr int PF_HD = 256;

// 16-byte global -> shared copies that stay in flight together (cp.async), then one wait.
GG_DEV void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
GG_DEV void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// Sum of `splits` planes at offset o (loads issued four at a time, added in plane order).
GG_DEV float sum_planes(const float* __restrict__ part, int splits, long long plane, long long o) {
  float v = part[o];
  int z = 1;
  for (; z + 3 < splits; z += 4) {
    const float a = part[(long long)z * plane + o], b = part[(long long)(z + 1) * plane + o];
    const float c = part[(long long)(z + 2) * plane + o], d = part[(long long)(z + 3) * plane + o];
    v += a;
    v += b;
    v += c;
    v += d;
  }
  for (; z < splits; z++) v += part[(long long)z * plane + o];
  return v;
}

GG_DEV float block_sum256(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < PF_THREADS / 32; i++) s += red[i];
  return s;
}

__global__ void __launch_bounds__(PF_THREADS) pf_embed_kernel(const int32_t* __restrict__ ids,
                                                              const uint8_t* __restrict__ embd, int rs, int H,
                                                              float* __restrict__ hidden) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  const int t = blockIdx.x;
  const uint8_t* row = embd + (size_t)ids[t] * rs;
  const float sq = sqrtf((float)H);
  for (int i = threadIdx.x; i < H; i += PF_THREADS) {
    const float d = __half2float(*reinterpret_cast<const __half*>(row + H + 2 * (i >> 5)));
    float v = (float)(int8_t)row[i] * d;
    hidden[(size_t)t * H + i] = v * sq;
  }
}

// One CTA per row; thread k owns the element quad 4k..4k+3 (H / 4 threads, up to 1024), so
// every load of the row (all split planes, residual, weights) is in flight at once.
__global__ void __launch_bounds__(1024)
    pf_addnorm_kernel(const float* __restrict__ part, int splits, long long plane, const float* __restrict__ w_post,
                      const float* rin, float* rout, const float* __restrict__ w_norm, uint8_t* thi, uint8_t* tlo,
                      int H, float eps) {
  pdl_trigger();
  __shared__ float red[2][32];
  const int t = blockIdx.x, k = threadIdx.x, nq = H >> 2;
  const bool ok = k < nq;
  const long long base = (long long)t * H + 4 * k;
  // the norm weights are constant: fetched before waiting for the previous kernel
  const float4 wp = (ok && part) ? __ldg(reinterpret_cast<const float4*>(w_post) + k) : make_float4(0.f, 0.f, 0.f, 0.f);
  const float4 wn = (ok && w_norm) ? __ldg(reinterpret_cast<const float4*>(w_norm) + k) : make_float4(0.f, 0.f, 0.f, 0.f);
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  float r[4] = {0.f, 0.f, 0.f, 0.f};
  if (ok) {
    const float4 ri = *reinterpret_cast<const float4*>(rin + base);
    r[0] = ri.x; r[1] = ri.y; r[2] = ri.z; r[3] = ri.w;
  }
  // block sum with one barrier: every warp adds the per-warp partials itself (in lane order, so
  // all warps get the same bits); the two sums use their own slots, so no second barrier guards
  // the slots' reuse
  auto bsum = [&](float v, int slot) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[slot][threadIdx.x >> 5] = v;
    __syncthreads();
    const int ln = threadIdx.x & 31;
    return warp_sum(ln < (int)(blockDim.x >> 5) ? red[slot][ln] : 0.f);
  };
  if (part) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (ok) {
      // split planes summed in plane order; up to eight loads in flight at a time
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int z0 = 0; z0 < splits; z0 += 8) {
        float4 a[8];
#pragma unroll
        for (int u = 0; u < 8; u++)
          if (z0 + u < splits) a[u] = *reinterpret_cast<const float4*>(part + (long long)(z0 + u) * plane + base);
#pragma unroll
        for (int u = 0; u < 8; u++) {
          if (z0 + u >= splits) break;
          if (z0 + u == 0) {
            acc = a[0];
          } else {
            acc.x += a[u].x; acc.y += a[u].y; acc.z += a[u].z; acc.w += a[u].w;
          }
        }
      }
      v[0] = acc.x; v[1] = acc.y; v[2] = acc.z; v[3] = acc.w;
    }
    const float rms = sqrtf(bsum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3], 0) / (float)H + eps);
    if (ok) {
      const float wv[4] = {wp.x, wp.y, wp.z, wp.w};
#pragma unroll
      for (int j = 0; j < 4; j++) r[j] = r[j] + v[j] * wv[j] / rms;
    }
  }
  if (ok && rout && (part || rout != rin))
    *reinterpret_cast<float4*>(rout + base) = make_float4(r[0], r[1], r[2], r[3]);
  if (!w_norm) return;
  const float rms2 = sqrtf(bsum(r[0] * r[0] + r[1] * r[1] + r[2] * r[2] + r[3] * r[3], 1) / (float)H + eps);
  // two quads per tile chunk of 8: the even thread gathers its neighbour's quad
  float x[4] = {r[0] * wn.x / rms2, r[1] * wn.y / rms2, r[2] * wn.z / rms2, r[3] * wn.w / rms2};
  float y[4];
#pragma unroll
  for (int j = 0; j < 4; j++) y[j] = __shfl_down_sync(0xffffffffu, x[j], 1);
  if (ok && (k & 1) == 0) {
    float v8[8] = {x[0], x[1], x[2], x[3], y[0], y[1], y[2], y[3]};
    xtile_put8(thi, tlo, H / 64, t, 4 * k, v8);
  }
}

// BATCH: row t is a different sequence, in KV slot seq_arr[t] (slot stride seq_stride floats)
// at position pos_arr[t]; otherwise row t is prompt position p0 + t of one slot.
// Element i of a bf16 hi / lo pair of planes (lo n elements after hi) from the value the cache
// holds: hi = f rounded to bf16, lo = (f - hi) rounded, as pf_kv_split_kernel makes them.
GG_DEV void split_put(uint16_t* hi, long long n, long long i, float f) {
  const __nv_bfloat16 h = __float2bfloat16_rn(f);
  hi[i] = __bfloat16_as_ushort(h);
  hi[n + i] = __bfloat16_as_ushort(__float2bfloat16_rn(f - __bfloat162float(h)));
}

template <bool BATCH, bool KV16>
__global__ void __launch_bounds__(PF_THREADS)
    pf_qk_kernel(const float* __restrict__ part, int splits, long long plane, const float* __restrict__ q_norm,
                 const float* __restrict__ k_norm, const float2* __restrict__ rope, int p0, int NQH, int NKH, float eps,
                 float* __restrict__ q_out, kv_t<KV16>* __restrict__ kc, kv_t<KV16>* __restrict__ vc,
                 const int32_t* __restrict__ pos_arr, const int32_t* __restrict__ seq_arr, size_t seq_stride,
                 uint16_t* __restrict__ ksplit, int ctx) {
  pdl_trigger();
  constexpr int NJ = PF_HD / 32;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int QD = NQH * PF_HD, KVD = NKH * PF_HD, W = QD + 2 * KVD;
  const long long base = (long long)t * W;
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  const int pos = BATCH ? pos_arr[t] : p0 + t;
  if (BATCH) {
    kc += (size_t)seq_arr[t] * seq_stride;
    vc += (size_t)seq_arr[t] * seq_stride;
  }
  for (int h = warp; h < NQH + NKH; h += PF_THREADS / 32) {
    // norm weights, RoPE table and the head's elements of every split plane issued together
    // (two planes in flight), the planes summed in plane order
    const float* nw = h < NQH ? q_norm : k_norm;
    float nwv[NJ];
    float2 cr[NJ / 2];  // (cos, sin) of pos * freq_i, i = lane + 32 j
#pragma unroll
    for (int j = 0; j < NJ; j++) nwv[j] = __ldg(nw + lane + 32 * j);
#pragma unroll
    for (int j = 0; j < NJ / 2; j++) cr[j] = rope[(size_t)pos * (PF_HD / 2) + lane + 32 * j];
    const long long ob = base + h * PF_HD + lane;
    float v[NJ];
#pragma unroll
    for (int j = 0; j < NJ; j++) v[j] = part[ob + 32 * j];
    for (int z = 1; z < splits; z += 2) {
      float a[NJ], b2[NJ];
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        a[j] = part[(long long)z * plane + ob + 32 * j];
        b2[j] = z + 1 < splits ? part[(long long)(z + 1) * plane + ob + 32 * j] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        v[j] += a[j];
        if (z + 1 < splits) v[j] += b2[j];
      }
    }
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; j++) ss += v[j] * v[j];
    const float rms = sqrtf(warp_sum(ss) / (float)PF_HD + eps);
#pragma unroll
    for (int j = 0; j < NJ; j++) v[j] = v[j] * nwv[j] / rms;
#pragma unroll
    for (int j = 0; j < NJ / 2; j++) {
      const float cs = cr[j].x, sn = cr[j].y;
      const float x0 = v[j], x1 = v[j + NJ / 2];
      v[j] = x0 * cs - x1 * sn;
      v[j + NJ / 2] = x0 * sn + x1 * cs;
    }
#pragma unroll
    for (int j = 0; j < NJ; j++) {
      const int i = lane + 32 * j;
      if (h < NQH) {
        const long long qi = (long long)t * QD + h * PF_HD + i;
        if constexpr (BATCH) {
          q_out[qi] = v[j];
        } else {  // prompt chunk: q as bf16 hi / lo halves (hi at q_out, lo T * QD elements later)
          uint16_t* qs = reinterpret_cast<uint16_t*>(q_out);
          const __nv_bfloat16 hi = __float2bfloat16_rn(v[j]);
          qs[qi] = __bfloat16_as_ushort(hi);
          qs[(long long)gridDim.x * QD + qi] = __bfloat16_as_ushort(__float2bfloat16_rn(v[j] - __bfloat162float(hi)));
        }
      }
      else {
        const long long ki = (long long)pos * KVD + (h - NQH) * PF_HD + i;
        const kv_t<KV16> kk = kv_narrow<KV16>(v[j]);
        kc[ki] = kk;
        if (!BATCH && ksplit) split_put(ksplit, (long long)ctx * KVD, ki, kv_widen(kk));
      }
    }
  }
  for (int i = threadIdx.x; i < KVD; i += PF_THREADS) {
    const long long vi = (long long)pos * KVD + i;
    const kv_t<KV16> vv = kv_narrow<KV16>(sum_planes(part, splits, plane, base + QD + KVD + i));
    vc[vi] = vv;
    if (!BATCH && ksplit) split_put(ksplit + 2 * (size_t)ctx * KVD, (long long)ctx * KVD, vi, kv_widen(vv));
  }
}

// Causal attention, split over key ranges. A work item is (a block of 32 query rows, a range
// of 64 keys): the rows are QT = 32/G consecutive tokens times the G query heads that share
// one KV head, so each K/V row serves all of them. An item leaves unnormalised partial results
// (running max m, sum l, output o) that pf_attn_merge combines with the usual online-softmax
// rescaling.
constexpr int PA_ROWS = 32;
constexpr int PA_KC = 64;                      // keys per work item (two CTAs per SM fill the GPU)
constexpr int PA_PART = PA_ROWS * PF_HD + 2 * PA_ROWS;  // floats per item: o, then m, then l

// The work item runs on the tensor cores: mma.sync m16n8k16 with bf16 operands and f32
// accumulation. Every f32 operand is split into bf16 hi + lo (hi + lo = x to ~2^-16) and each
// product is the sum of three MMAs (hi*hi + hi*lo + lo*hi), which keeps the scores and outputs
// within ~1e-5 of f32.
//   warp w: query rows 16*((w>>1)&1).. (one m16 tile), output dims 128*(w&1).., keys
//   16*(w>>2)..+15 of every 32-key block; both dim halves compute the scores of their rows and
//   keys, so the probabilities never leave registers (the score accumulators are re-packed as
//   the A operand of P.V). The two key halves keep their own softmax statistics and are merged
//   through shared memory at the end.
// K and V blocks of 32 keys are converted to swizzled bf16 hi/lo tiles in shared memory (16-byte
// chunk c of row r stored at chunk c ^ (r & 7), so ldmatrix reads 8 rows without bank conflicts).
constexpr int TA_KB = 32;                          // keys per shared-memory block
constexpr int TA_THREADS = 256;                   // 8 warps: row tile x dim half x key half
constexpr int TA_TILE = PF_HD * 2;                 // bytes of one bf16 row of 256 dims
constexpr int TA_SMEM = (PA_ROWS * 2 + TA_KB * 4) * TA_TILE;  // Q hi/lo, K hi/lo, V hi/lo

GG_DEV uint32_t ta_off(int r, int col) {  // byte offset of bf16 element (r, col) in a swizzled tile
  return (uint32_t)(r * TA_TILE + ((((col >> 3) ^ (r & 7)) & 31) << 4) + (col & 7) * 2);
}
GG_DEV void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
GG_DEV void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}
GG_DEV void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// Eight f32 -> one 16-byte chunk of bf16 hi and one of bf16 lo (lo = x - hi, rounded).
GG_DEV void split8(const float* f, uint4& hi, uint4& lo) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const __nv_bfloat16 h0 = __float2bfloat16_rn(f[2 * i]), h1 = __float2bfloat16_rn(f[2 * i + 1]);
    const __nv_bfloat16 l0 = __float2bfloat16_rn(f[2 * i] - __bfloat162float(h0));
    const __nv_bfloat16 l1 = __float2bfloat16_rn(f[2 * i + 1] - __bfloat162float(h1));
    h[i] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
    l[i] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
  }
  hi = make_uint4(h[0], h[1], h[2], h[3]);
  lo = make_uint4(l[0], l[1], l[2], l[3]);
}
GG_DEV uint32_t pack2(float a, float b) {  // a in the low half (lower column)
  return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
         ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
}

// K and V rows [r0, r1) of a layer's cache -> bf16 hi / lo copies (row-major [row][KVD]), once per
// layer and chunk, so the attention CTAs that read a row all copy ready operand halves.
template <bool KV16>
__global__ void __launch_bounds__(256)
    pf_kv_split_kernel(const kv_t<KV16>* __restrict__ kc, const kv_t<KV16>* __restrict__ vc, int r0, int r1, int KVD,
                       uint16_t* __restrict__ khi, uint16_t* __restrict__ klo, uint16_t* __restrict__ vhi,
                       uint16_t* __restrict__ vlo) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  const long long n8 = (long long)(r1 - r0) * (KVD / 8);
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < n8; i += (long long)gridDim.x * 256) {
    const long long e = (long long)r0 * KVD + 8 * i;
    float fk[8], fv[8];
    if constexpr (KV16) {
      bf16x8_widen(__ldg(reinterpret_cast<const uint4*>(kc + e)), fk);
      bf16x8_widen(__ldg(reinterpret_cast<const uint4*>(vc + e)), fv);
    } else {
      const float4 k0 = __ldg(reinterpret_cast<const float4*>(kc + e)), k1 = __ldg(reinterpret_cast<const float4*>(kc + e) + 1);
      const float4 v0 = __ldg(reinterpret_cast<const float4*>(vc + e)), v1 = __ldg(reinterpret_cast<const float4*>(vc + e) + 1);
      fk[0] = k0.x; fk[1] = k0.y; fk[2] = k0.z; fk[3] = k0.w; fk[4] = k1.x; fk[5] = k1.y; fk[6] = k1.z; fk[7] = k1.w;
      fv[0] = v0.x; fv[1] = v0.y; fv[2] = v0.z; fv[3] = v0.w; fv[4] = v1.x; fv[5] = v1.y; fv[6] = v1.z; fv[7] = v1.w;
    }
    uint4 hi, lo;
    split8(fk, hi, lo);
    *reinterpret_cast<uint4*>(khi + e) = hi;
    *reinterpret_cast<uint4*>(klo + e) = lo;
    split8(fv, hi, lo);
    *reinterpret_cast<uint4*>(vhi + e) = hi;
    *reinterpret_cast<uint4*>(vlo + e) = lo;
  }
}

__global__ void __launch_bounds__(TA_THREADS, 2)
    pf_attn_tc_kernel(const uint16_t* __restrict__ qhi, const uint16_t* __restrict__ qlo,
                      const uint16_t* __restrict__ khi, const uint16_t* __restrict__ klo,
                      const uint16_t* __restrict__ vhi, const uint16_t* __restrict__ vlo, int T, int p0, int NQH, int NKH,
                      float scale, int window, int maxc, float* __restrict__ part) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  extern __shared__ __align__(128) uint8_t ta_smem[];
  uint8_t* qh = ta_smem;
  uint8_t* ql = qh + PA_ROWS * TA_TILE;
  uint8_t* kh = ql + PA_ROWS * TA_TILE;
  uint8_t* kl = kh + TA_KB * TA_TILE;
  uint8_t* vh = kl + TA_KB * TA_TILE;
  uint8_t* vl = vh + TA_KB * TA_TILE;
  const int G = NQH / NKH, QT = PA_ROWS / G;
  const int c = blockIdx.x, b = blockIdx.y, kvh = blockIdx.z;
  const int t0 = b * QT, nq = min(QT, T - t0);
  const int kmax = p0 + t0 + nq - 1;
  const int k_begin = c * PA_KC;
  if (k_begin > kmax) return;
  const int k_end = min(k_begin + PA_KC, kmax + 1);
  const int klo0 = window > 0 ? max(0, p0 + t0 + 1 - window) : 0;
  if (k_end <= klo0) return;
  const int QD = NQH * PF_HD, KVD = NKH * PF_HD;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // query rows r = token * G + g -> head kvh * G + g of token t0 + token: the bf16 hi / lo halves
  // written by the q/k kernel, copied into the swizzled tiles (their cp.async group completes
  // with the first K/V block's)
  for (int i = tid; i < PA_ROWS * (PF_HD / 8); i += TA_THREADS) {
    const int r = i / (PF_HD / 8), c8 = i % (PF_HD / 8);
    const int tok = r / G, hq = kvh * G + r % G;
    const uint32_t off = ta_off(r, 8 * c8);
    if (tok < nq) {
      const long long e = (long long)(t0 + tok) * QD + hq * PF_HD + 8 * c8;
      cp_async16(qh + off, qhi + e);
      cp_async16(ql + off, qlo + e);
    } else {
      *reinterpret_cast<uint4*>(qh + off) = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(ql + off) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  const int rt = (warp >> 1) & 1, dh = warp & 1, kh2 = warp >> 2;  // row tile, dim half, key half
  const int g = lane >> 2, tq = lane & 3;   // mma fragment coordinates
  const int ra = 16 * rt + g, rb = ra + 8;  // this thread's two rows
  const int pos_a = p0 + t0 + ra / G, pos_b = p0 + t0 + rb / G;
  const bool va = ra / G < nq, vb = rb / G < nq;
  const int lo_a = window > 0 ? max(0, pos_a + 1 - window) : 0, lo_b = window > 0 ? max(0, pos_b + 1 - window) : 0;
  float m_a = -1e30f, m_b = -1e30f, l_a = 0.f, l_b = 0.f;
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;

  for (int j0 = k_begin; j0 < k_end; j0 += TA_KB) {
    const int nk = min(TA_KB, k_end - j0);
    __syncthreads();  // the previous block's tiles are no longer read (and Q is written)
    // K and V rows j0.. as bf16 hi/lo tiles: 16-byte async copies of the split rows into the
    // swizzled layout; rows past nk are zero
    for (int i = tid; i < TA_KB * (PF_HD / 8); i += TA_THREADS) {
      const int r = i / (PF_HD / 8), c8 = i % (PF_HD / 8);
      const uint32_t off = ta_off(r, 8 * c8);
      if (r < nk) {
        const long long e = (long long)(j0 + r) * KVD + kvh * PF_HD + 8 * c8;
        cp_async16(kh + off, khi + e);
        cp_async16(kl + off, klo + e);
        cp_async16(vh + off, vhi + e);
        cp_async16(vl + off, vlo + e);
      } else {
        const uint4 z = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(kh + off) = z;
        *reinterpret_cast<uint4*>(kl + off) = z;
        *reinterpret_cast<uint4*>(vh + off) = z;
        *reinterpret_cast<uint4*>(vl + off) = z;
      }
    }
    cp_async_wait_all();
    __syncthreads();
    // S = Q K^T for this warp's 16 rows x 16 keys (2 n-tiles of 8 keys: keys 16*kh2 ..)
    float sacc[2][4];
#pragma unroll
    for (int n = 0; n < 2; n++) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
    const int arow = 16 * rt + (lane & 15), acol = 8 * (lane >> 4);              // A (Q) ldmatrix lanes
    const int brow = (lane & 7) + 8 * (lane >> 4), bcol = 8 * ((lane >> 3) & 1);  // B (K) ldmatrix lanes
#pragma unroll 4
    for (int ks = 0; ks < PF_HD / 16; ks++) {
      uint32_t ah[4], al[4], bh[4], bl[4];
      ldsm_x4(smem_u32(qh + ta_off(arow, 16 * ks + acol)), ah);
      ldsm_x4(smem_u32(ql + ta_off(arow, 16 * ks + acol)), al);
      ldsm_x4(smem_u32(kh + ta_off(16 * kh2 + brow, 16 * ks + bcol)), bh);
      ldsm_x4(smem_u32(kl + ta_off(16 * kh2 + brow, 16 * ks + bcol)), bl);
      // the three products alternate over the two accumulators
#pragma unroll
      for (int n = 0; n < 2; n++) mma_bf16(sacc[n], ah, bh[2 * n], bh[2 * n + 1]);
#pragma unroll
      for (int n = 0; n < 2; n++) mma_bf16(sacc[n], ah, bl[2 * n], bl[2 * n + 1]);
#pragma unroll
      for (int n = 0; n < 2; n++) mma_bf16(sacc[n], al, bh[2 * n], bh[2 * n + 1]);
    }
    // causal / window / range mask, scale, and the online softmax of rows ra (d0, d1) and rb (d2, d3)
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; n++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        const int key = j0 + 16 * kh2 + 8 * n + 2 * tq + e;
        const bool in = key < j0 + nk;
        sacc[n][e] = (in && va && key <= pos_a && key >= lo_a) ? sacc[n][e] * scale : -INFINITY;
        sacc[n][2 + e] = (in && vb && key <= pos_b && key >= lo_b) ? sacc[n][2 + e] * scale : -INFINITY;
        mx_a = fmaxf(mx_a, sacc[n][e]);
        mx_b = fmaxf(mx_b, sacc[n][2 + e]);
      }
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
    mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
    mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
    const float nm_a = fmaxf(m_a, mx_a), nm_b = fmaxf(m_b, mx_b);
    const float al_a = expf(m_a - nm_a), al_b = expf(m_b - nm_b);
    m_a = nm_a;
    m_b = nm_b;
    float ps_a = 0.f, ps_b = 0.f;
#pragma unroll
    for (int n = 0; n < 2; n++)
#pragma unroll
      for (int e = 0; e < 2; e++) {
        sacc[n][e] = sacc[n][e] == -INFINITY ? 0.f : expf(sacc[n][e] - nm_a);
        sacc[n][2 + e] = sacc[n][2 + e] == -INFINITY ? 0.f : expf(sacc[n][2 + e] - nm_b);
        ps_a += sacc[n][e];
        ps_b += sacc[n][2 + e];
      }
    l_a = l_a * al_a + ps_a;  // this thread's columns; the quad is summed at the end
    l_b = l_b * al_b + ps_b;
#pragma unroll
    for (int n = 0; n < 16; n++) {
      o[n][0] *= al_a;
      o[n][1] *= al_a;
      o[n][2] *= al_b;
      o[n][3] *= al_b;
    }
    // O += P V: P (16 rows x this warp's 16 keys) from the score registers as bf16 hi/lo A fragments
    const int vrow = (lane & 7) + 8 * ((lane >> 3) & 1), vcol = 8 * (lane >> 4);  // V ldmatrix.trans lanes
    {
      const int kk = kh2;
      float pf[8] = {sacc[0][0], sacc[0][1], sacc[0][2], sacc[0][3], sacc[1][0], sacc[1][1], sacc[1][2], sacc[1][3]};
      uint32_t ph[4], pl[4];
#pragma unroll
      for (int i = 0; i < 4; i++) {
        // A fragment order: (row g, keys 2t..), (row g+8, keys 2t..), (row g, keys 2t+8..), (row g+8, keys 2t+8..)
        const float x0 = pf[(i & 1) * 2 + (i >> 1) * 4], x1 = pf[(i & 1) * 2 + (i >> 1) * 4 + 1];
        ph[i] = pack2(x0, x1);
        const float h0 = __uint_as_float((ph[i] & 0xffffu) << 16), h1 = __uint_as_float(ph[i] & 0xffff0000u);
        pl[i] = pack2(x0 - h0, x1 - h1);
      }
#pragma unroll
      for (int np = 0; np < 8; np += 2) {  // dims 128*dh + 16*np .. (two pairs of n-tiles at a time)
        uint32_t bh[2][4], bl[2][4];
#pragma unroll
        for (int u = 0; u < 2; u++) {
          const int dcol = 128 * dh + 16 * (np + u) + vcol;
          ldsm_x4_t(smem_u32(vh + ta_off(16 * kk + vrow, dcol)), bh[u]);
          ldsm_x4_t(smem_u32(vl + ta_off(16 * kk + vrow, dcol)), bl[u]);
        }
#pragma unroll
        for (int n = 0; n < 4; n++) mma_bf16(o[2 * np + n], ph, bh[n >> 1][2 * (n & 1)], bh[n >> 1][2 * (n & 1) + 1]);
#pragma unroll
        for (int n = 0; n < 4; n++) mma_bf16(o[2 * np + n], ph, bl[n >> 1][2 * (n & 1)], bl[n >> 1][2 * (n & 1) + 1]);
#pragma unroll
        for (int n = 0; n < 4; n++) mma_bf16(o[2 * np + n], pl, bh[n >> 1][2 * (n & 1)], bh[n >> 1][2 * (n & 1) + 1]);
      }
    }
  }
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  // merge the key halves: the upper-half warp leaves (m, l, o) in shared memory (the K/V tiles
  // are free now) and the lower-half warp of the same rows and dims folds them in
  __syncthreads();
  float* xo = reinterpret_cast<float*>(kh) + ((rt * 2 + dh) * 32 + lane) * 68;  // 64 o + 4 stats per lane
  if (kh2 == 1) {
#pragma unroll
    for (int n = 0; n < 16; n++)
      *reinterpret_cast<float4*>(xo + 4 * n) = make_float4(o[n][0], o[n][1], o[n][2], o[n][3]);
    *reinterpret_cast<float4*>(xo + 64) = make_float4(m_a, m_b, l_a, l_b);
  }
  __syncthreads();
  if (kh2 == 1) return;
  {
    const float4 st = *reinterpret_cast<const float4*>(xo + 64);
    const float nm_a = fmaxf(m_a, st.x), nm_b = fmaxf(m_b, st.y);
    const float s0a = expf(m_a - nm_a), s1a = expf(st.x - nm_a), s0b = expf(m_b - nm_b), s1b = expf(st.y - nm_b);
#pragma unroll
    for (int n = 0; n < 16; n++) {
      const float4 u = *reinterpret_cast<const float4*>(xo + 4 * n);
      o[n][0] = o[n][0] * s0a + u.x * s1a;
      o[n][1] = o[n][1] * s0a + u.y * s1a;
      o[n][2] = o[n][2] * s0b + u.z * s1b;
      o[n][3] = o[n][3] * s0b + u.w * s1b;
    }
    l_a = l_a * s0a + st.z * s1a;
    l_b = l_b * s0b + st.w * s1b;
    m_a = nm_a;
    m_b = nm_b;
  }
  float* dst = part + ((size_t)(kvh * gridDim.y + b) * maxc + c) * PA_PART;
#pragma unroll
  for (int n = 0; n < 16; n++) {
    const int d = 128 * dh + 8 * n + 2 * tq;
    *reinterpret_cast<float2*>(dst + ra * PF_HD + d) = make_float2(o[n][0], o[n][1]);
    *reinterpret_cast<float2*>(dst + rb * PF_HD + d) = make_float2(o[n][2], o[n][3]);
  }
  if (dh == 0 && tq == 0) {
    dst[PA_ROWS * PF_HD + ra] = m_a;
    dst[PA_ROWS * PF_HD + rb] = m_b;
    dst[PA_ROWS * PF_HD + PA_ROWS + ra] = l_a;
    dst[PA_ROWS * PF_HD + PA_ROWS + rb] = l_b;
  }
}

// Merge the key-range items of one row block and write the attention output as tiles.
__global__ void __launch_bounds__(PF_THREADS)
    pf_attn_merge_kernel(const float* __restrict__ part, int T, int p0, int NQH, int NKH, int window, int maxc,
                         uint8_t* thi, uint8_t* tlo) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  __shared__ float wm[32][PA_ROWS], wl[32][PA_ROWS];  // (max, sum) of every key range and row
  const int G = NQH / NKH, QT = PA_ROWS / G;
  const int b = blockIdx.x, kvh = blockIdx.y;
  const int t0 = b * QT, nq = min(QT, T - t0);
  const int nch = min(maxc, (p0 + t0 + nq - 1) / PA_KC + 1);
  const int c0 = window > 0 ? max(0, p0 + t0 + 1 - window) / PA_KC : 0;  // as in the part kernel
  const int nc = nch - c0;
  const float* base = part + ((size_t)(kvh * gridDim.x + b) * maxc + c0) * PA_PART;
  for (int i = threadIdx.x; i < nc * PA_ROWS; i += PF_THREADS) {  // every pair in one round of loads
    const float* pc = base + (size_t)(i / PA_ROWS) * PA_PART + PA_ROWS * PF_HD + i % PA_ROWS;
    wm[i / PA_ROWS][i % PA_ROWS] = pc[0];
    wl[i / PA_ROWS][i % PA_ROWS] = pc[PA_ROWS];
  }
  __syncthreads();
  // thread: row r, 8 dims of this CTA's quarter of the head (blockIdx.z)
  const int r = threadIdx.x / 8, c8 = 8 * blockIdx.z + threadIdx.x % 8;
  const int tok = r / G, hq = kvh * G + r % G;
  if (tok >= nq) return;
  float M = -1e30f;
  for (int i = 0; i < nc; i++) M = fmaxf(M, wm[i][r]);
  float L = 0.f, v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  constexpr int MB = 8;  // key ranges whose outputs are loaded together (one round for 512 keys)
  for (int i0 = 0; i0 < nc; i0 += MB) {
    float4 va[MB], vb[MB];
#pragma unroll
    for (int k = 0; k < MB; k++) {
      if (i0 + k < nc) {
        const float4* src = reinterpret_cast<const float4*>(base + (size_t)(i0 + k) * PA_PART + r * PF_HD + 8 * c8);
        va[k] = src[0];
        vb[k] = src[1];
      }
    }
#pragma unroll
    for (int k = 0; k < MB; k++) {
      if (i0 + k >= nc) break;
      const float w = expf(wm[i0 + k][r] - M);
      L = fmaf(wl[i0 + k][r], w, L);
      v[0] = fmaf(va[k].x, w, v[0]); v[1] = fmaf(va[k].y, w, v[1]); v[2] = fmaf(va[k].z, w, v[2]); v[3] = fmaf(va[k].w, w, v[3]);
      v[4] = fmaf(vb[k].x, w, v[4]); v[5] = fmaf(vb[k].y, w, v[5]); v[6] = fmaf(vb[k].z, w, v[6]); v[7] = fmaf(vb[k].w, w, v[7]);
    }
  }
  const float inv = 1.0f / L;
#pragma unroll
  for (int j = 0; j < 8; j++) v[j] *= inv;
  xtile_put8(thi, tlo, NQH * PF_HD / 64, t0 + tok, hq * PF_HD + 8 * c8, v);
}

// Decode attention for a batch of sequences: row b has one query token (NQH = 4 heads sharing
// the single KV head) at position pos[b] of KV slot seqs[b]. A work item (CTA) is (row, 64-key
// range); each of its warps takes 16 of the keys, lane l holding dims 8l..8l+7 of the four
// query heads, so a key row is one coalesced 1 KB (f32) or 512 B (bf16) warp load straight into
// registers, four keys' K and V rows in flight at a time. The warp keeps an online softmax
// (running max, sum, output) per head; the CTA merges its warps in shared memory and leaves one
// partial result per work item, merged over the ranges by bd_attn_merge_kernel.
constexpr int BD_NH = 4;
constexpr int BD_KC = 64;                  // keys per work item
constexpr int BD_WARPS = 4;                // warps per work item
constexpr int BD_KW = BD_KC / BD_WARPS;    // keys per warp
constexpr int BD_KB = 4;                   // keys per batch (rows in flight per warp)
constexpr int BD_PART = BD_NH * PF_HD + 2 * BD_NH;
static_assert(PF_HD == 8 * 32, "a lane holds 8 dims of a 256-wide head");

// Eight consecutive cache elements as f32: f32 one 32-byte load (p 32-byte aligned: the cache
// base, its slot and layer strides and pos * 256 are multiples of 8 floats), bf16 one 16-byte
// load.
template <bool KV16>
GG_DEV void kv_load8(const kv_t<KV16>* p, float* f) {
  if constexpr (KV16) {
    bf16x8_widen(__ldg(reinterpret_cast<const uint4*>(p)), f);
  } else {
    asm volatile("ld.global.nc.v8.f32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=f"(f[0]), "=f"(f[1]), "=f"(f[2]), "=f"(f[3]), "=f"(f[4]), "=f"(f[5]), "=f"(f[6]), "=f"(f[7])
                 : "l"(p));
  }
}

// The q/k work of pf_qk_kernel for one head of batch row b (warp-wide): the head's elements of
// every split plane of the q/k/v GEMM summed in plane order, RMSNorm with weights nw, RoPE at pos.
// Lane l holds elements l + 32 j.
GG_DEV void bd_head_norm_rope(const float* __restrict__ qkv, int splits, long long plane, long long ob,
                              const float* __restrict__ nw, const float2* __restrict__ rope, int pos, float eps, float* v) {
  constexpr int NJ = PF_HD / 32;
  const int lane = threadIdx.x & 31;
  float nwv[NJ];
  float2 cr[NJ / 2];
#pragma unroll
  for (int j = 0; j < NJ; j++) nwv[j] = __ldg(nw + lane + 32 * j);
#pragma unroll
  for (int j = 0; j < NJ / 2; j++) cr[j] = rope[(size_t)pos * (PF_HD / 2) + lane + 32 * j];
#pragma unroll
  for (int j = 0; j < NJ; j++) v[j] = qkv[ob + lane + 32 * j];
  for (int z = 1; z < splits; z++)
#pragma unroll
    for (int j = 0; j < NJ; j++) v[j] += qkv[(long long)z * plane + ob + lane + 32 * j];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NJ; j++) ss += v[j] * v[j];
  const float rms = sqrtf(warp_sum(ss) / (float)PF_HD + eps);
#pragma unroll
  for (int j = 0; j < NJ; j++) v[j] = v[j] * nwv[j] / rms;
#pragma unroll
  for (int j = 0; j < NJ / 2; j++) {
    const float cs = cr[j].x, sn = cr[j].y;
    const float x0 = v[j], x1 = v[j + NJ / 2];
    v[j] = x0 * cs - x1 * sn;
    v[j + NJ / 2] = x0 * sn + x1 * cs;
  }
}

// Fused with the q/k step (shaders.ts:420-467, 209-227): every CTA of row b builds the row's
// normed, rotated q in shared memory from the q/k/v GEMM's split planes, and the CTA whose range
// holds position pos also computes the new k and v, stores them in the cache and keeps them in
// shared memory for its own key pos (the cache loads below take the read-only path, which does
// not see this launch's stores).
template <bool KV16>
__global__ void __launch_bounds__(BD_WARPS * 32)
    bd_attn_part_kernel(const float* __restrict__ qkv, int splits, long long plane, const float* __restrict__ q_norm,
                        const float* __restrict__ k_norm, const float2* __restrict__ rope, float eps,
                        kv_t<KV16>* __restrict__ kc, kv_t<KV16>* __restrict__ vc, const int32_t* __restrict__ pos_arr,
                        const int32_t* __restrict__ seq_arr, size_t seq_stride, float scale, int window, int maxc,
                        float* __restrict__ part) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  static_assert(BD_WARPS == BD_NH, "one warp per query head builds q");
  __shared__ float sm_m[BD_WARPS][BD_NH], sm_l[BD_WARPS][BD_NH];
  __shared__ __align__(16) float sm_o[BD_WARPS][BD_NH][PF_HD];
  __shared__ __align__(16) float sm_q[BD_NH][PF_HD];
  __shared__ __align__(16) float sm_kv[2][PF_HD];  // the new position's k and v (as the cache holds them)
  const int c = blockIdx.x, b = blockIdx.y;
  const int pos = pos_arr[b];
  const int k_begin = c * BD_KC;
  if (k_begin > pos) return;
  const int k_end = min(k_begin + BD_KC, pos + 1);
  const int klo = window > 0 ? max(0, pos + 1 - window) : 0;  // sliding window
  if (k_end <= klo) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int W = BD_NH * PF_HD + 2 * PF_HD;  // one row of the q/k/v GEMM output (NKH = 1)
  const long long rb = (long long)b * W;
  const bool owner = k_end == pos + 1;  // this range holds the new position
  {
    float v[PF_HD / 32];
    bd_head_norm_rope(qkv, splits, plane, rb + warp * PF_HD, q_norm, rope, pos, eps, v);
#pragma unroll
    for (int j = 0; j < PF_HD / 32; j++) sm_q[warp][lane + 32 * j] = v[j];
    if (owner) {
      kv_t<KV16>* krow = kc + (size_t)seq_arr[b] * seq_stride + (size_t)pos * PF_HD;
      kv_t<KV16>* vrow = vc + (size_t)seq_arr[b] * seq_stride + (size_t)pos * PF_HD;
      if (warp == 0) {
        bd_head_norm_rope(qkv, splits, plane, rb + BD_NH * PF_HD, k_norm, rope, pos, eps, v);
#pragma unroll
        for (int j = 0; j < PF_HD / 32; j++) {
          const kv_t<KV16> kk = kv_narrow<KV16>(v[j]);
          krow[lane + 32 * j] = kk;
          sm_kv[0][lane + 32 * j] = kv_widen(kk);
        }
      } else {
        for (int i = threadIdx.x - 32; i < PF_HD; i += (BD_WARPS - 1) * 32) {
          const kv_t<KV16> vv = kv_narrow<KV16>(sum_planes(qkv, splits, plane, rb + BD_NH * PF_HD + PF_HD + i));
          vrow[i] = vv;
          sm_kv[1][i] = kv_widen(vv);
        }
      }
    }
  }
  __syncthreads();
  const kv_t<KV16>* kb = kc + (size_t)seq_arr[b] * seq_stride + 8 * lane;
  const kv_t<KV16>* vb = vc + (size_t)seq_arr[b] * seq_stride + 8 * lane;
  float qv[BD_NH][8];
#pragma unroll
  for (int h = 0; h < BD_NH; h++) {
    const float4* qp = reinterpret_cast<const float4*>(&sm_q[h][8 * lane]);
    const float4 a = qp[0], bq = qp[1];
    qv[h][0] = a.x; qv[h][1] = a.y; qv[h][2] = a.z; qv[h][3] = a.w;
    qv[h][4] = bq.x; qv[h][5] = bq.y; qv[h][6] = bq.z; qv[h][7] = bq.w;
  }
  float m[BD_NH], l[BD_NH], o[BD_NH][8];
#pragma unroll
  for (int h = 0; h < BD_NH; h++) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int d = 0; d < 8; d++) o[h][d] = 0.f;
  }
  const int w0 = max(k_begin + warp * BD_KW, klo), w1 = min(k_begin + (warp + 1) * BD_KW, k_end);
  for (int j0 = w0; j0 < w1; j0 += BD_KB) {
    float kf[BD_KB][8], vf[BD_KB][8];
#pragma unroll
    for (int k = 0; k < BD_KB; k++) {
      if (j0 + k == pos) {  // the new position: from shared memory
        const float4* kp = reinterpret_cast<const float4*>(&sm_kv[0][8 * lane]);
        const float4* vp = reinterpret_cast<const float4*>(&sm_kv[1][8 * lane]);
        const float4 k0 = kp[0], k1 = kp[1], v0 = vp[0], v1 = vp[1];
        kf[k][0] = k0.x; kf[k][1] = k0.y; kf[k][2] = k0.z; kf[k][3] = k0.w;
        kf[k][4] = k1.x; kf[k][5] = k1.y; kf[k][6] = k1.z; kf[k][7] = k1.w;
        vf[k][0] = v0.x; vf[k][1] = v0.y; vf[k][2] = v0.z; vf[k][3] = v0.w;
        vf[k][4] = v1.x; vf[k][5] = v1.y; vf[k][6] = v1.z; vf[k][7] = v1.w;
      } else if (j0 + k < w1) {
        kv_load8<KV16>(kb + (size_t)(j0 + k) * PF_HD, kf[k]);
        kv_load8<KV16>(vb + (size_t)(j0 + k) * PF_HD, vf[k]);
      } else {
#pragma unroll
        for (int d = 0; d < 8; d++) kf[k][d] = vf[k][d] = 0.f;
      }
    }
    static_assert(BD_KB * BD_NH == 16, "one 16-value warp reduction per batch");
    float dots[16];
#pragma unroll
    for (int k = 0; k < BD_KB; k++)
#pragma unroll
      for (int h = 0; h < BD_NH; h++) {
        float a = 0.f;
#pragma unroll
        for (int d = 0; d < 8; d++) a = fmaf(qv[h][d], kf[k][d], a);
        dots[k * BD_NH + h] = a;
      }
    warp_sum16(dots);
    float sc[BD_KB][BD_NH];
#pragma unroll
    for (int k = 0; k < BD_KB; k++)
#pragma unroll
      for (int h = 0; h < BD_NH; h++) sc[k][h] = j0 + k < w1 ? dots[k * BD_NH + h] * scale : -INFINITY;
#pragma unroll
    for (int h = 0; h < BD_NH; h++) {
      float bm = sc[0][h];
#pragma unroll
      for (int k = 1; k < BD_KB; k++) bm = fmaxf(bm, sc[k][h]);
      const float nm = fmaxf(m[h], bm);  // finite: key j0 is in range
      const float alpha = expf(m[h] - nm);
      float p[BD_KB], ps = 0.f;
#pragma unroll
      for (int k = 0; k < BD_KB; k++) {
        p[k] = expf(sc[k][h] - nm);
        ps += p[k];
      }
      l[h] = l[h] * alpha + ps;
      m[h] = nm;
#pragma unroll
      for (int d = 0; d < 8; d++) {
        float acc = o[h][d] * alpha;
#pragma unroll
        for (int k = 0; k < BD_KB; k++) acc = fmaf(p[k], vf[k][d], acc);
        o[h][d] = acc;
      }
    }
  }
  // merge the warps: each keeps (m, l, o) of its keys; a warp without keys has m = -inf
#pragma unroll
  for (int h = 0; h < BD_NH; h++) {
    float4* op = reinterpret_cast<float4*>(&sm_o[warp][h][8 * lane]);
    op[0] = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
    op[1] = make_float4(o[h][4], o[h][5], o[h][6], o[h][7]);
    if (lane == 0) {
      sm_m[warp][h] = m[h];
      sm_l[warp][h] = l[h];
    }
  }
  __syncthreads();
  float* dst = part + ((size_t)b * maxc + c) * BD_PART;
  for (int i = threadIdx.x; i < BD_NH * PF_HD; i += BD_WARPS * 32) {
    const int h = i / PF_HD, d = i % PF_HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < BD_WARPS; w++) M = fmaxf(M, sm_m[w][h]);
    float acc = 0.f;
#pragma unroll
    for (int w = 0; w < BD_WARPS; w++)
      if (sm_m[w][h] != -INFINITY) acc = fmaf(expf(sm_m[w][h] - M), sm_o[w][h][d], acc);
    dst[i] = acc;
    if (d == 0) {
      float L = 0.f;
#pragma unroll
      for (int w = 0; w < BD_WARPS; w++)
        if (sm_m[w][h] != -INFINITY) L = fmaf(expf(sm_m[w][h] - M), sm_l[w][h], L);
      dst[BD_NH * PF_HD + h] = M;
      dst[BD_NH * PF_HD + BD_NH + h] = L;
    }
  }
}

__global__ void __launch_bounds__(PF_THREADS)
    bd_attn_merge_kernel(const float* __restrict__ part, const int32_t* __restrict__ pos_arr, int window, int maxc,
                         uint8_t* thi, uint8_t* tlo) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  __shared__ float wm[32][BD_NH], wl[32][BD_NH];  // (max, sum) of every key range and head
  const int b = blockIdx.x;
  const int nch = min(maxc, pos_arr[b] / BD_KC + 1);
  const int c0 = window > 0 ? max(0, pos_arr[b] + 1 - window) / BD_KC : 0;
  const int nc = nch - c0;
  const float* base = part + ((size_t)b * maxc + c0) * BD_PART;
  for (int i = threadIdx.x; i < nc * BD_NH; i += PF_THREADS) {  // all pairs in one round of loads
    const float* pc = base + (size_t)(i / BD_NH) * BD_PART + BD_NH * PF_HD + i % BD_NH;
    wm[i / BD_NH][i % BD_NH] = pc[0];
    wl[i / BD_NH][i % BD_NH] = pc[BD_NH];
  }
  __syncthreads();
  if (threadIdx.x >= BD_NH * (PF_HD / 8)) return;
  const int h = threadIdx.x / (PF_HD / 8), c8 = threadIdx.x % (PF_HD / 8);
  float M = -1e30f;
  for (int i = 0; i < nc; i++) M = fmaxf(M, wm[i][h]);
  float L = 0.f, v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  constexpr int MB = 8;  // key ranges whose outputs are loaded together
  for (int i0 = 0; i0 < nc; i0 += MB) {
    float4 va[MB], vb[MB];
#pragma unroll
    for (int k = 0; k < MB; k++) {
      if (i0 + k < nc) {
        const float4* src = reinterpret_cast<const float4*>(base + (size_t)(i0 + k) * BD_PART + h * PF_HD + 8 * c8);
        va[k] = src[0];
        vb[k] = src[1];
      }
    }
#pragma unroll
    for (int k = 0; k < MB; k++) {
      if (i0 + k >= nc) break;
      const float w = expf(wm[i0 + k][h] - M);
      L = fmaf(wl[i0 + k][h], w, L);
      v[0] = fmaf(va[k].x, w, v[0]); v[1] = fmaf(va[k].y, w, v[1]);
      v[2] = fmaf(va[k].z, w, v[2]); v[3] = fmaf(va[k].w, w, v[3]);
      v[4] = fmaf(vb[k].x, w, v[4]); v[5] = fmaf(vb[k].y, w, v[5]);
      v[6] = fmaf(vb[k].z, w, v[6]); v[7] = fmaf(vb[k].w, w, v[7]);
    }
  }
  const float inv = 1.0f / L;
#pragma unroll
  for (int jj = 0; jj < 8; jj++) v[jj] *= inv;
  xtile_put8(thi, tlo, BD_NH * PF_HD / 64, b, h * PF_HD + 8 * c8, v);
}

__global__ void __launch_bounds__(PF_THREADS) pf_geglu_kernel(const float* __restrict__ gu, int splits, long long plane,
                                                              int T, int I, uint8_t* thi, uint8_t* tlo) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  const int c8 = I / 8;
  const long long n = (long long)T * c8;
  for (long long idx = blockIdx.x * (long long)PF_THREADS + threadIdx.x; idx < n;
       idx += (long long)gridDim.x * PF_THREADS) {
    const int t = (int)(idx / c8), c = (int)(idx % c8);
    float g[16];
    for (int z = 0; z < splits; z++) {
      const float4* src = reinterpret_cast<const float4*>(gu + (long long)z * plane + (long long)t * 2 * I + 16 * c);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const float4 f = src[j];
        if (z == 0) {
          g[4 * j] = f.x; g[4 * j + 1] = f.y; g[4 * j + 2] = f.z; g[4 * j + 3] = f.w;
        } else {
          g[4 * j] += f.x; g[4 * j + 1] += f.y; g[4 * j + 2] += f.z; g[4 * j + 3] += f.w;
        }
      }
    }
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = gelu_tanh(g[2 * j]) * g[2 * j + 1];
    xtile_put8(thi, tlo, I / 64, t, 8 * c, v);
  }
}

// RoPE table: (cos, sin) of pos * freq_i, freq_i = 1 / theta^(2i/HD), the same f32 expressions
// the shader evaluates per step (shaders.ts:420-467).
__global__ void pf_rope_table_kernel(float theta, int HD, int ctx, float2* out) {
  const int half = HD / 2;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < ctx * half; idx += gridDim.x * blockDim.x) {
    const int pos = idx / half, i = idx % half;
    const float freq = 1.0f / powf(theta, (float)(i * 2) / (float)HD);
    const float ang = (float)pos * freq;
    out[idx] = make_float2(cosf(ang), sinf(ang));
  }
}

}  // namespace gg

using namespace gg;

cudaError_t gg_rope_table(float theta, int HD, int ctx, float2* out, cudaStream_t s) {
  pf_rope_table_kernel<<<148 * 4, 256, 0, s>>>(theta, HD, ctx, out);
  return cudaGetLastError();
}

cudaError_t pf_embed(const int32_t* ids, int T, const uint8_t* embd, int rs, int H, float* hidden, cudaStream_t s) {
  if (T <= 0) return cudaErrorInvalidValue;
  return launch_pdl(pf_embed_kernel, dim3(T), dim3(PF_THREADS), 0, s, ids, embd, rs, H, hidden);
}

cudaError_t pf_addnorm(const float* part, int splits, long long plane, const float* w_post, const float* resid_in,
                       float* resid_out, const float* w_norm, uint8_t* thi, uint8_t* tlo, int T, int H, float eps,
                       cudaStream_t s) {
  if (T <= 0 || H > PF_MAX_H || H % 64) return cudaErrorInvalidValue;
  const int threads = ((H / 4) + 31) / 32 * 32;
  return launch_pdl(pf_addnorm_kernel, dim3(T), dim3(threads), 0, s, part, splits, plane, w_post, resid_in, resid_out,
                    w_norm, thi, tlo, H, eps);
}

cudaError_t pf_qk_rope_store(const float* part, int splits, long long plane, const float* q_norm,
                             const float* k_norm, const float2* rope, int T, int p0, int NQH, int NKH, int HD, float eps,
                             float* q_out, void* kc, void* vc, bool kv16, uint8_t* split, int ctx, cudaStream_t s) {
  if (T <= 0 || HD != PF_HD || (split && p0 + T > ctx)) return cudaErrorInvalidValue;
  uint16_t* ks = reinterpret_cast<uint16_t*>(split);
  if (kv16)
    return launch_pdl(pf_qk_kernel<false, true>, dim3(T), dim3(PF_THREADS), 0, s, part, splits, plane, q_norm, k_norm,
                      rope, p0, NQH, NKH, eps, q_out, (__nv_bfloat16*)kc, (__nv_bfloat16*)vc, nullptr, nullptr,
                      (size_t)0, ks, ctx);
  return launch_pdl(pf_qk_kernel<false, false>, dim3(T), dim3(PF_THREADS), 0, s, part, splits, plane, q_norm, k_norm,
                    rope, p0, NQH, NKH, eps, q_out, (float*)kc, (float*)vc, nullptr, nullptr, (size_t)0, ks, ctx);
}

size_t pf_attention_part_floats(int max_tokens, int ctx, int NQH, int NKH) {
  const int G = NQH / NKH, QT = PA_ROWS / G;
  const size_t nb = (size_t)(max_tokens + QT - 1) / QT, maxc = (size_t)(ctx + PA_KC - 1) / PA_KC;
  return nb * maxc * NKH * PA_PART;
}

size_t pf_kv_split_bytes(int ctx, int KVD) { return (size_t)4 * ctx * KVD * sizeof(uint16_t); }

cudaError_t pf_attention(const float* q, const void* kc, const void* vc, bool kv16, int T, int p0, int NQH, int NKH,
                         int HD, float scale, int window, float* part, uint8_t* split, int ctx, bool rows_split,
                         uint8_t* thi, uint8_t* tlo, cudaStream_t s) {
  if (T <= 0 || HD != PF_HD || NKH <= 0 || NQH % NKH || !split || p0 + T > ctx) return cudaErrorInvalidValue;
  const int G = NQH / NKH;
  if (G != 1 && G != 2 && G != 4 && G != 8 && G != 16) return cudaErrorInvalidValue;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    r = cudaFuncSetAttribute(pf_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TA_SMEM);
    if (r != cudaSuccess) return r;
    attr_set[dev] = true;
  }
  const int QT = PA_ROWS / G;
  const int nb = (T + QT - 1) / QT;
  const int maxc = (p0 + T - 1) / PA_KC + 1;
  if (maxc > 32) return cudaErrorInvalidValue;  // merge weights hold 32 key ranges (2048 positions)
  // bf16 hi / lo copies of the rows the chunk can see: [klo, p0 + T)
  const int KVD = NKH * PF_HD;
  // (rows p0.. when pf_qk_rope_store made their copies already)
  const int r0 = window > 0 ? max(0, p0 + 1 - window) / PA_KC * PA_KC : 0, r1 = rows_split ? p0 : p0 + T;
  uint16_t* khi = reinterpret_cast<uint16_t*>(split);
  uint16_t* klo = khi + (size_t)ctx * KVD;
  uint16_t* vhi = klo + (size_t)ctx * KVD;
  uint16_t* vlo = vhi + (size_t)ctx * KVD;
  const long long n8 = (long long)(r1 - r0) * (KVD / 8);
  const int sblocks = (int)std::min<long long>((n8 + 255) / 256, 148 * 8);
  if (n8 > 0) {  // none for a chunk at the start of the window whose own rows were split
    if (kv16)
      r = launch_pdl(pf_kv_split_kernel<true>, dim3(sblocks), dim3(256), 0, s, (const __nv_bfloat16*)kc,
                     (const __nv_bfloat16*)vc, r0, r1, KVD, khi, klo, vhi, vlo);
    else
      r = launch_pdl(pf_kv_split_kernel<false>, dim3(sblocks), dim3(256), 0, s, (const float*)kc, (const float*)vc, r0,
                     r1, KVD, khi, klo, vhi, vlo);
    if (r != cudaSuccess) return r;
  }
  const uint16_t* qhi = reinterpret_cast<const uint16_t*>(q);  // hi / lo halves from pf_qk_rope_store
  const uint16_t* qlo = qhi + (size_t)T * NQH * PF_HD;
  r = launch_pdl(pf_attn_tc_kernel, dim3(maxc, nb, NKH), dim3(TA_THREADS), TA_SMEM, s, qhi, qlo, (const uint16_t*)khi,
                 (const uint16_t*)klo, (const uint16_t*)vhi, (const uint16_t*)vlo, T, p0, NQH, NKH, scale, window, maxc,
                 part);
  if (r != cudaSuccess) return r;
  return launch_pdl(pf_attn_merge_kernel, dim3(nb, NKH, PF_HD / 64), dim3(PF_THREADS), 0, s, (const float*)part, T, p0,
                    NQH, NKH, window, maxc, thi, tlo);
}

size_t bd_attention_part_floats(int max_rows, int ctx) {
  return (size_t)max_rows * ((ctx + BD_KC - 1) / BD_KC) * BD_PART;
}

cudaError_t bd_attention(const float* qkv, int splits, long long plane, const float* q_norm, const float* k_norm,
                         const float2* rope, float eps, void* kc, void* vc, bool kv16, int B, const int32_t* pos,
                         const int32_t* seqs, size_t seq_stride, int max_pos, int NQH, int NKH, int HD, float scale,
                         int window, float* part, uint8_t* thi, uint8_t* tlo, cudaStream_t s) {
  if (B <= 0 || HD != PF_HD || NQH != BD_NH || NKH != 1) return cudaErrorInvalidValue;
  const int maxc = max_pos / BD_KC + 1;
  if (maxc > 32) return cudaErrorInvalidValue;  // merge weights hold 32 key ranges (2048 positions)
  cudaError_t r;
  if (kv16)
    r = launch_pdl(bd_attn_part_kernel<true>, dim3(maxc, B), dim3(BD_WARPS * 32), 0, s, qkv, splits, plane, q_norm, k_norm,
                   rope, eps, (__nv_bfloat16*)kc, (__nv_bfloat16*)vc, pos, seqs, seq_stride, scale, window, maxc, part);
  else
    r = launch_pdl(bd_attn_part_kernel<false>, dim3(maxc, B), dim3(BD_WARPS * 32), 0, s, qkv, splits, plane, q_norm,
                   k_norm, rope, eps, (float*)kc, (float*)vc, pos, seqs, seq_stride, scale, window, maxc, part);
  if (r != cudaSuccess) return r;
  return launch_pdl(bd_attn_merge_kernel, dim3(B), dim3(PF_THREADS), 0, s, (const float*)part, pos, window, maxc, thi,
                    tlo);
}

cudaError_t pf_geglu(const float* gu, int splits, long long plane, int T, int I, uint8_t* thi, uint8_t* tlo,
                     cudaStream_t s) {
  if (T <= 0 || I % 64 || splits < 1) return cudaErrorInvalidValue;
  const long long n = (long long)T * (I / 8);
  const int blocks = (int)((n + PF_THREADS - 1) / PF_THREADS < 148 * 8 ? (n + PF_THREADS - 1) / PF_THREADS : 148 * 8);
  return launch_pdl(pf_geglu_kernel, dim3(blocks), dim3(PF_THREADS), 0, s, gu, splits, plane, T, I, thi, tlo);
}
