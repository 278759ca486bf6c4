// gg_sample.cuh -- the end of a token step: the 256 per-lane (value, index) maxima of the logits
// (the reference's topk256 / argmax lanes) and the sampler that picks the next token from them.
// Shared by the step kernels, the batched sampler and the allocation-free sampler.
#pragma once
#include "gg_device.cuh"
#include "gg_model.h"

namespace gg {

// Key of an empty lane: (-1e30, index 0 in the inverted low word), the shaders' start value.
GG_DEV unsigned long long init_lane_key() {
  return ((unsigned long long)f32_order_key(-1e30f) << 32) | 0xffffffffull;
}

// The sampler's shared-memory workspace. The step kernel carves it from its weight ring, which is
// idle once the LM head is done; the other kernels declare one.
struct SampleScratch {
  double sv[256];
  double share[256];
  unsigned long long wk[8];
  double sum_all;
  int sl[256];
  uint32_t cid[256];
  float probs[256];
  int result;
};

// Run by every thread of one CTA (at least 256 threads). engine.ts:823-901.
GG_DEV int sample_token(const GGModelDev& m, GGState* st, SampleScratch& S) {
  double* sv = S.sv;
  int* sl = S.sl;
  int& result = S.result;
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
    unsigned long long* wk = S.wk;
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
  uint32_t* cid = S.cid;
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
  float* probs = S.probs;
  double* share = S.share;
  double& sum_all = S.sum_all;
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

}  // namespace gg
