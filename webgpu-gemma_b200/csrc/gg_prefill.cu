// gg_prefill.cu -- the kernels between the tensor-core GEMMs of a batched prefill.
//
// The reference prefills serially, one full forward per prompt token (engine.ts:923-928).
// Here a chunk of T prompt tokens moves through each layer together: the matrices become
// GEMMs over T rows (gg_gemm.cu), and the per-token work between them -- norms, residual adds,
// q/k norm + RoPE, the KV store, causal attention over the cache, GeGLU -- runs in the
// kernels below, one CTA per token row (or per 8 queries for attention). The math per token
// is the reference's (formulas of shaders.ts, f32 throughout); only the order of some sums
// differs, within f32 rounding.
#include "gg_gemm_dev.cuh"
#include "gg_prefill.h"

namespace gg {

constexpr int PF_THREADS = 256;
constexpr int PF_MAX_H = 4096;
constexpr int PF_QB = 8;   // queries per attention CTA (one warp each)
constexpr int PF_KB = 64;  // keys per attention block
constexpr int PF_HD = 256;
constexpr int PF_KS = PF_HD + 1;  // padded K row in shared memory (conflict-free column reads)
constexpr int PF_ATT_SMEM = (PF_QB * PF_HD + PF_KB * PF_KS + PF_KB * PF_HD + PF_QB * PF_KB + 2 * PF_QB) * 4;

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
  const int t = blockIdx.x;
  const uint8_t* row = embd + (size_t)ids[t] * rs;
  const float sq = sqrtf((float)H);
  for (int i = threadIdx.x; i < H; i += PF_THREADS) {
    const float d = __half2float(*reinterpret_cast<const __half*>(row + H + 2 * (i >> 5)));
    float v = (float)(int8_t)row[i] * d;
    hidden[(size_t)t * H + i] = v * sq;
  }
}

__global__ void __launch_bounds__(PF_THREADS)
    pf_addnorm_kernel(const float* __restrict__ part, int splits, long long plane, const float* __restrict__ w_post,
                      const float* rin, float* rout, const float* __restrict__ w_norm, uint8_t* thi, uint8_t* tlo,
                      int H, float eps) {
  __shared__ float row[PF_MAX_H];
  __shared__ float red[PF_THREADS / 32];
  const int t = blockIdx.x;
  const long long base = (long long)t * H;
  if (part) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += PF_THREADS) {
      float v = part[base + i];
      for (int z = 1; z < splits; z++) v += part[(long long)z * plane + base + i];
      row[i] = v;
      ss += v * v;
    }
    const float rms = sqrtf(block_sum256(ss, red) / (float)H + eps);
    for (int i = threadIdx.x; i < H; i += PF_THREADS) {
      const float r = rin[base + i] + row[i] * w_post[i] / rms;
      row[i] = r;
      if (rout) rout[base + i] = r;
    }
  } else {
    for (int i = threadIdx.x; i < H; i += PF_THREADS) {
      const float r = rin[base + i];
      row[i] = r;
      if (rout && rout != rin) rout[base + i] = r;
    }
  }
  if (!w_norm) return;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += PF_THREADS) ss += row[i] * row[i];
  const float rms = sqrtf(block_sum256(ss, red) / (float)H + eps);
  for (int c = threadIdx.x; c < H / 8; c += PF_THREADS) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = row[8 * c + j] * w_norm[8 * c + j] / rms;
    xtile_put8(thi, tlo, H / 64, t, 8 * c, v);
  }
}

__global__ void __launch_bounds__(PF_THREADS)
    pf_qk_kernel(const float* __restrict__ part, int splits, long long plane, const float* __restrict__ q_norm,
                 const float* __restrict__ k_norm, float theta, int p0, int NQH, int NKH, float eps,
                 float* __restrict__ q_out, float* __restrict__ kc, float* __restrict__ vc) {
  constexpr int NJ = PF_HD / 32;
  const int t = blockIdx.x, pos = p0 + t;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int QD = NQH * PF_HD, KVD = NKH * PF_HD, W = QD + 2 * KVD;
  const long long base = (long long)t * W;
  for (int h = warp; h < NQH + NKH; h += PF_THREADS / 32) {
    float v[NJ];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; j++) {
      const long long o = base + h * PF_HD + lane + 32 * j;
      float a = part[o];
      for (int z = 1; z < splits; z++) a += part[(long long)z * plane + o];
      v[j] = a;
      ss += a * a;
    }
    const float rms = sqrtf(warp_sum(ss) / (float)PF_HD + eps);
    const float* nw = h < NQH ? q_norm : k_norm;
#pragma unroll
    for (int j = 0; j < NJ; j++) v[j] = v[j] * nw[lane + 32 * j] / rms;
#pragma unroll
    for (int j = 0; j < NJ / 2; j++) {
      const int i = lane + 32 * j;
      const float freq = 1.0f / powf(theta, (float)(i * 2) / (float)PF_HD);
      const float ang = (float)pos * freq;
      const float cs = cosf(ang), sn = sinf(ang);
      const float x0 = v[j], x1 = v[j + NJ / 2];
      v[j] = x0 * cs - x1 * sn;
      v[j + NJ / 2] = x0 * sn + x1 * cs;
    }
#pragma unroll
    for (int j = 0; j < NJ; j++) {
      const int i = lane + 32 * j;
      if (h < NQH) q_out[(long long)t * QD + h * PF_HD + i] = v[j];
      else kc[(long long)pos * KVD + (h - NQH) * PF_HD + i] = v[j];
    }
  }
  for (int i = threadIdx.x; i < KVD; i += PF_THREADS) {
    const long long o = base + QD + KVD + i;
    float a = part[o];
    for (int z = 1; z < splits; z++) a += part[(long long)z * plane + o];
    vc[(long long)pos * KVD + i] = a;
  }
}

// Online-softmax attention: CTA = (8 consecutive queries, one q head); warp i scores query i
// against 64 keys at a time (lane -> keys lane, lane + 32); thread d accumulates output dim d.
__global__ void __launch_bounds__(PF_THREADS)
    pf_attn_kernel(const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc, int T,
                   int p0, int NQH, int NKH, float scale, uint8_t* thi, uint8_t* tlo) {
  extern __shared__ float sm[];
  float* qs = sm;                         // [QB][HD]
  float* ks = qs + PF_QB * PF_HD;         // [KB][KS]
  float* vs = ks + PF_KB * PF_KS;         // [KB][HD]
  float* ps = vs + PF_KB * PF_HD;         // [QB][KB]
  float* al = ps + PF_QB * PF_KB;         // [QB] rescale factors
  float* ls = al + PF_QB;                 // [QB] softmax denominators
  const int t0 = blockIdx.x * PF_QB, h = blockIdx.y, kvh = h * NKH / NQH;
  const int nq = min(PF_QB, T - t0);
  const int QD = NQH * PF_HD, KVD = NKH * PF_HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, d = threadIdx.x;
  for (int idx = threadIdx.x; idx < PF_QB * PF_HD; idx += PF_THREADS) {
    const int i = idx / PF_HD, dd = idx % PF_HD;
    qs[idx] = i < nq ? q[(long long)(t0 + i) * QD + h * PF_HD + dd] : 0.f;
  }
  const int kmax = p0 + t0 + nq - 1;
  const int qpos = p0 + t0 + warp;
  float m = -1e30f, l = 0.f;
  float o[PF_QB];
#pragma unroll
  for (int i = 0; i < PF_QB; i++) o[i] = 0.f;
  for (int j0 = 0; j0 <= kmax; j0 += PF_KB) {
    const int nk = min(PF_KB, kmax + 1 - j0);
    __syncthreads();
    for (int idx = threadIdx.x; idx < nk * PF_HD; idx += PF_THREADS) {
      const int j = idx / PF_HD, dd = idx % PF_HD;
      const long long g = (long long)(j0 + j) * KVD + kvh * PF_HD + dd;
      ks[j * PF_KS + dd] = kc[g];
      vs[j * PF_HD + dd] = vc[g];
    }
    __syncthreads();
    if (warp < nq) {
      const float* qr = qs + warp * PF_HD;
      const float* k0 = ks + lane * PF_KS;
      const float* k1 = ks + (lane + 32) * PF_KS;
      float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
      for (int dd = 0; dd < PF_HD; dd++) {
        const float qd = qr[dd];
        s0 = fmaf(qd, k0[dd], s0);
        s1 = fmaf(qd, k1[dd], s1);
      }
      const bool v0 = lane < nk && j0 + lane <= qpos, v1 = lane + 32 < nk && j0 + lane + 32 <= qpos;
      s0 = v0 ? s0 * scale : -INFINITY;
      s1 = v1 ? s1 * scale : -INFINITY;
      const float mnew = fmaxf(m, warp_max(fmaxf(s0, s1)));
      const float e0 = v0 ? expf(s0 - mnew) : 0.f, e1 = v1 ? expf(s1 - mnew) : 0.f;
      const float alpha = expf(m - mnew);
      l = l * alpha + warp_sum(e0 + e1);
      m = mnew;
      ps[warp * PF_KB + lane] = e0;
      ps[warp * PF_KB + lane + 32] = e1;
      if (lane == 0) al[warp] = alpha;
    } else if (lane == 0) {
      al[warp] = 1.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < PF_QB; i++) {
      if (i >= nq) break;
      float acc = o[i] * al[i];
      const float* pr = ps + i * PF_KB;
      for (int j = 0; j < nk; j++) acc = fmaf(pr[j], vs[j * PF_HD + d], acc);
      o[i] = acc;
    }
  }
  if (lane == 0 && warp < nq) ls[warp] = l;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < PF_QB; i++)
    if (i < nq) qs[i * PF_HD + d] = o[i] / ls[i];
  __syncthreads();
  const int i = threadIdx.x >> 5, c = threadIdx.x & 31;
  if (i < nq) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; j++) v[j] = qs[i * PF_HD + 8 * c + j];
    xtile_put8(thi, tlo, QD / 64, t0 + i, h * PF_HD + 8 * c, v);
  }
}

__global__ void __launch_bounds__(PF_THREADS) pf_geglu_kernel(const float* __restrict__ gu, int splits, long long plane,
                                                              int T, int I, uint8_t* thi, uint8_t* tlo) {
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

}  // namespace gg

using namespace gg;

cudaError_t pf_embed(const int32_t* ids, int T, const uint8_t* embd, int rs, int H, float* hidden, cudaStream_t s) {
  if (T <= 0) return cudaErrorInvalidValue;
  pf_embed_kernel<<<T, PF_THREADS, 0, s>>>(ids, embd, rs, H, hidden);
  return cudaGetLastError();
}

cudaError_t pf_addnorm(const float* part, int splits, long long plane, const float* w_post, const float* resid_in,
                       float* resid_out, const float* w_norm, uint8_t* thi, uint8_t* tlo, int T, int H, float eps,
                       cudaStream_t s) {
  if (T <= 0 || H > PF_MAX_H || H % 64) return cudaErrorInvalidValue;
  pf_addnorm_kernel<<<T, PF_THREADS, 0, s>>>(part, splits, plane, w_post, resid_in, resid_out, w_norm, thi, tlo, H, eps);
  return cudaGetLastError();
}

cudaError_t pf_qk_rope_store(const float* part, int splits, long long plane, const float* q_norm,
                             const float* k_norm, float theta, int T, int p0, int NQH, int NKH, int HD, float eps,
                             float* q_out, float* kc, float* vc, cudaStream_t s) {
  if (T <= 0 || HD != PF_HD) return cudaErrorInvalidValue;
  pf_qk_kernel<<<T, PF_THREADS, 0, s>>>(part, splits, plane, q_norm, k_norm, theta, p0, NQH, NKH, eps, q_out, kc, vc);
  return cudaGetLastError();
}

cudaError_t pf_attention(const float* q, const float* kc, const float* vc, int T, int p0, int NQH, int NKH, int HD,
                         float scale, uint8_t* thi, uint8_t* tlo, cudaStream_t s) {
  if (T <= 0 || HD != PF_HD) return cudaErrorInvalidValue;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    r = cudaFuncSetAttribute(pf_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PF_ATT_SMEM);
    if (r != cudaSuccess) return r;
    attr_set[dev] = true;
  }
  dim3 grid((T + PF_QB - 1) / PF_QB, NQH);
  pf_attn_kernel<<<grid, PF_THREADS, PF_ATT_SMEM, s>>>(q, kc, vc, T, p0, NQH, NKH, scale, thi, tlo);
  return cudaGetLastError();
}

cudaError_t pf_geglu(const float* gu, int splits, long long plane, int T, int I, uint8_t* thi, uint8_t* tlo,
                     cudaStream_t s) {
  if (T <= 0 || I % 64 || splits < 1) return cudaErrorInvalidValue;
  const long long n = (long long)T * (I / 8);
  const int blocks = (int)((n + PF_THREADS - 1) / PF_THREADS < 148 * 8 ? (n + PF_THREADS - 1) / PF_THREADS : 148 * 8);
  pf_geglu_kernel<<<blocks, PF_THREADS, 0, s>>>(gu, splits, plane, T, I, thi, tlo);
  return cudaGetLastError();
}
