// gg_gemm.cu -- Q8_0 x activations on the sm_100a tensor cores (tcgen05, TMEM accumulators).
//
// One CTA computes a 128-row x NT-token tile of Y over a K-slice:
//   warp 0      bulk copies of the activation tiles (bf16 hi and lo, NT x 64) into a ring;
//   warp 1      TMEM allocation and the MMA issue: per 64-wide K slab, 4 K-steps of three
//               MMAs (Whi*Xhi, Whi*Xlo, Wlo*Xhi), one f32 accumulator per term, summed in
//               the epilogue;
//   warps 2-9   dequantise: each lane reads one Q8_0 block (32 int8 + f16 scale) of a slab
//               from the tiled weight copy straight into registers, several slabs ahead,
//               turns it into exact f32 weights, splits them into bf16 hi/lo and writes them
//               in the swizzled operand layout; warps 2-5 then read the accumulators out of
//               TMEM.
// The weight products q*d are exact in f32 and hi + lo keeps 16 of their bits; with X split
// the same way the result matches an f32 dot product to ~1e-5 relative. This replaces the
// reference's linearQ8 shader (src/shaders.ts:92-151) for batched rows (prefill, batches).
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "gg_gemm.h"
#include "gg_gemm_dev.cuh"
#include "gg_launch.h"

namespace gg {

constexpr int GM_TW = 8;                          // dequantising warps (warps 2..9)
constexpr int GM_THREADS = 64 + 32 * GM_TW;
constexpr int GM_RAW_Q = 128 * 64;
constexpr int GM_PF = 4;                          // raw slabs each dequantising lane holds ahead
constexpr int GM_A_BYTES = 128 * 128;             // 128 rows x 64 bf16

// Two shared-memory rings: dequantised weight operands (hi, lo) and activation operands
// (hi, lo). Raw Q8_0 slabs travel global -> registers in the dequantising warps, GM_PF slabs
// ahead. NT = 64 fits two CTAs per SM, so one CTA's hand-offs overlap the other's work.
template <int NT>
struct GemmCfg {
  static constexpr int AS = 2;
  static constexpr int BS = NT == 128 ? 3 : 2;
  static constexpr int A_STAGE = 2 * GM_A_BYTES;
  static constexpr int B_BYTES = NT * 128;
  static constexpr int B_STAGE = 2 * B_BYTES;
  static constexpr int BAR_BYTES = 128;
  static constexpr int SMEM = 1024 + AS * A_STAGE + BS * B_STAGE + BAR_BYTES;
  static constexpr int NACC = 3;  // one f32 accumulator per product term, summed in the epilogue
  static constexpr int TMEM_COLS = NT == 128 ? 512 : 256;
  static constexpr int MIN_CTAS = NT == 128 ? 1 : 2;
};

struct GemmArgs {
  const uint8_t* wt;  // tiled weights
  const uint8_t* xhi;
  const uint8_t* xlo;
  float* y;
  uint8_t* ghi;  // dense kernel only: when set, gelu(gate) * up of row pairs (2j, 2j + 1) goes
  uint8_t* glo;  // to these activation tiles (M / 2 columns) instead of y
  long long ldy, split_stride;
  int M, K, T, KS, slabs_per_split, splits;
  uint32_t* err;
  uint64_t timeout_ns;
};

// Exact int8 -> f32 of byte b of wx = raw ^ 0x80808080 (2^23 + u with u = q + 128, minus 2^23 + 128).
GG_DEV float q8_at(uint32_t wx, int b) {
  return __int_as_float((int)__byte_perm(wx, 0x4B000000u, 0x7440u + (uint32_t)b)) - 8388736.0f;
}

GG_DEV uint4 ldg_nc16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}
GG_DEV uint32_t ldg_nc_u16(const void* p) {
  unsigned short v;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// One Q8_0 block (32 int8 in q0, q1; f16 scale d) of row r, block h of a 128 x 64 slab, into
// the swizzled bf16 operand tiles: w = q * d exactly in f32; hi = w truncated to bf16,
// lo = (w - hi) rounded to bf16, so hi + lo = w to 2^-16 relative.
GG_DEV void dequant_block32(uint4 q0, uint4 q1, float d, uint8_t* ahi, uint8_t* alo, int r, int h) {
  const uint32_t words[8] = {q0.x ^ 0x80808080u, q0.y ^ 0x80808080u, q0.z ^ 0x80808080u, q0.w ^ 0x80808080u,
                             q1.x ^ 0x80808080u, q1.y ^ 0x80808080u, q1.z ^ 0x80808080u, q1.w ^ 0x80808080u};
  const uint32_t rowoff = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
#pragma unroll
  for (int j = 0; j < 4; j++) {  // chunk 4h + j: weights 8j..8j+7 of this block
    uint32_t hw[4], lw[4];
#pragma unroll
    for (int p = 0; p < 4; p++) {
      const uint32_t wx = words[2 * j + (p >> 1)];
      const int b0 = (p & 1) * 2;
      const float w0 = q8_at(wx, b0) * d, w1 = q8_at(wx, b0 + 1) * d;
      const uint32_t u0 = __float_as_uint(w0) & 0xFFFF0000u, u1 = __float_as_uint(w1) & 0xFFFF0000u;
      hw[p] = __byte_perm(u0, u1, 0x7632u);
      const __nv_bfloat162 l2 = __floats2bfloat162_rn(w0 - __uint_as_float(u0), w1 - __uint_as_float(u1));
      lw[p] = *reinterpret_cast<const uint32_t*>(&l2);
    }
    const int c = h * 4 + j;
    const uint32_t off = rowoff + ((uint32_t)((c ^ (r & 7)) & 7) << 4);
    *reinterpret_cast<uint4*>(ahi + off) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    *reinterpret_cast<uint4*>(alo + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
  }
}

template <int NT>
__global__ void __launch_bounds__(GM_THREADS, GemmCfg<NT>::MIN_CTAS) gg_gemm_q8_kernel(const GemmArgs a) {
  using C = GemmCfg<NT>;
  constexpr int AS = C::AS, BS = C::BS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* aring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bring = aring + AS * C::A_STAGE;
  uint64_t* full_a = reinterpret_cast<uint64_t*>(bring + BS * C::B_STAGE);
  uint64_t* empty_a = full_a + AS;
  uint64_t* full_b = empty_a + AS;
  uint64_t* empty_b = full_b + BS;
  uint64_t* acc_bar = empty_b + BS;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int s0 = blockIdx.z * a.slabs_per_split;
  const int ns = min(a.slabs_per_split, a.KS - s0);
  const SpinCtl sc{a.err, a.timeout_ns};
  // Under programmatic dependent launch the weights (never written by any kernel) stream in
  // before pdl_wait(); the activation copies (warp 0) and the output writes wait for it.
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int i = 0; i < AS; i++) {
      mbar_init(&full_a[i], GM_TW);
      mbar_init(&empty_a[i], 1);
    }
    for (int i = 0; i < BS; i++) {
      mbar_init(&full_b[i], 1);
      mbar_init(&empty_b[i], 1);
    }
    mbar_init(acc_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // activation tiles
      pdl_wait();
      const size_t KS = (size_t)a.KS;
      int issued = 0;
      for (int i = 0; i < ns; i++) {
        const int o = i % BS;
        if (*abort_flag) break;
        if (i >= BS && !mbar_wait(&empty_b[o], ((i / BS) - 1) & 1, sc)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* dst = bring + o * C::B_STAGE;
        mbar_arrive_expect_tx(&full_b[o], C::B_STAGE);
#pragma unroll
        for (int h = 0; h < NT / 64; h++) {
          const size_t blk = ((size_t)(n_tile * (NT / 64) + h) * KS + (size_t)(s0 + i)) * 8192u;
          bulk_g2s_plain(dst + h * 8192, a.xhi + blk, 8192, &full_b[o]);
          bulk_g2s_plain(dst + C::B_BYTES + h * 8192, a.xlo + blk, 8192, &full_b[o]);
        }
        issued++;
      }
      for (int i = issued > BS ? issued - BS : 0; i < issued; i++) mbar_wait(&full_b[i % BS], (i / BS) & 1, sc);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issue
      // The stage's activation tiles are x_hi rows then x_lo rows: one operand of 2 NT rows, so
      // one MMA of N = 2 NT makes Whi*Xhi and Whi*Xlo (accumulators 0 and 1) at once. One thread
      // issues an MMA about every 80 cycles, so two MMAs per K step instead of three.
      const uint32_t idesc = umma_idesc_bf16_m128(NT), idesc2 = umma_idesc_bf16_m128(2 * NT);
      for (int i = 0; i < ns; i++) {
        const int ia = i % AS, ib = i % BS;
        if (!mbar_wait(&full_b[ib], (i / BS) & 1, sc) || !mbar_wait(&full_a[ia], (i / AS) & 1, sc)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t ahi = smem_u32(aring + ia * C::A_STAGE), alo = ahi + GM_A_BYTES;
        const uint32_t bhi = smem_u32(bring + ib * C::B_STAGE), blo = bhi + C::B_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint32_t off = kk * 32;
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          umma_bf16(tmem, umma_desc_sw128(ahi + off), umma_desc_sw128(bhi + off), idesc2, acc);
          umma_bf16(tmem + 2 * NT, umma_desc_sw128(alo + off), umma_desc_sw128(bhi + off), idesc, acc);
        }
        umma_commit(&empty_a[ia]);
        umma_commit(&empty_b[ib]);
      }
      umma_commit(acc_bar);  // arrives once every MMA issued above has completed
    }
  } else {
    // dequantise: lane -> (row r, block h) of each 128 x 64 slab; raw data GM_PF slabs ahead
    const int tw = warp - 2;
    const int r = tw * 16 + (lane >> 1), h = lane & 1;
    const uint8_t* wbase = a.wt + ((size_t)m_tile * a.KS + (size_t)s0) * GG_Q8_TILE_BYTES;
    const uint8_t* qoff = wbase + r * 64 + h * 32;
    const uint8_t* soff = wbase + GM_RAW_Q + r * 4 + h * 2;
    uint4 qa[GM_PF], qb[GM_PF];
    uint32_t sv[GM_PF];
#pragma unroll
    for (int u = 0; u < GM_PF; u++) {
      if (u < ns) {
        qa[u] = ldg_nc16(qoff + (size_t)u * GG_Q8_TILE_BYTES);
        qb[u] = ldg_nc16(qoff + (size_t)u * GG_Q8_TILE_BYTES + 16);
        sv[u] = ldg_nc_u16(soff + (size_t)u * GG_Q8_TILE_BYTES);
      }
    }
    bool stop = false;
    for (int i0 = 0; i0 < ns && !stop; i0 += GM_PF) {
#pragma unroll
      for (int u = 0; u < GM_PF; u++) {
        const int i = i0 + u;
        if (i >= ns) break;
        const int ia = i % AS;
        if (*abort_flag || (i >= AS && !mbar_wait(&empty_a[ia], ((i / AS) - 1) & 1, sc))) {
          *abort_flag = 1;
          stop = true;
          break;
        }
        const float d = __half2float(__ushort_as_half((unsigned short)sv[u]));
        const uint4 words0 = qa[u], words1 = qb[u];
        if (i + GM_PF < ns) {  // refill this slot with the slab GM_PF ahead
          qa[u] = ldg_nc16(qoff + (size_t)(i + GM_PF) * GG_Q8_TILE_BYTES);
          qb[u] = ldg_nc16(qoff + (size_t)(i + GM_PF) * GG_Q8_TILE_BYTES + 16);
          sv[u] = ldg_nc_u16(soff + (size_t)(i + GM_PF) * GG_Q8_TILE_BYTES);
        }
        uint8_t* ahi = aring + ia * C::A_STAGE;
        dequant_block32(words0, words1, d, ahi, ahi + GM_A_BYTES, r, h);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[ia]);
      }
    }
    if (tw < 4) {  // epilogue: warp w reads TMEM lanes 32*(w%4)..
      const int q = warp & 3;
      pdl_wait();
      const bool ok = mbar_wait(acc_bar, 0, sc);
      tc_fence_after();
      const int go = __shfl_sync(0xffffffffu, (ok && !*abort_flag) ? 1 : 0, 0);
      if (go) {
        const int m = m_tile * 128 + q * 32 + lane;
        float* yb = a.y + (long long)blockIdx.z * a.split_stride + m;
#pragma unroll 1
        for (int c = 0; c < NT; c += 16) {
          float v[16];
          tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c, v);
#pragma unroll 1
          for (int k = 1; k < C::NACC; k++) {
            float u[16];
            tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(k * NT + c), u);
#pragma unroll
            for (int j = 0; j < 16; j++) v[j] += u[j];
          }
#pragma unroll
          for (int j = 0; j < 16; j++) {
            const int t = n_tile * NT + c + j;
            if (t < a.T) yb[(long long)t * a.ldy] = v[j];
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- dense path
// For many activation rows (prompt chunks) the weights are dequantised once, at load, into
// bf16 (hi, lo) operand tiles in HBM (32 KB per 128 x 64 slab: hi then lo, swizzled as the
// tensor core reads them). The kernel is then only copies and MMAs:
//   warp 0     bulk copies of a slab's weight tile and the NT x 64 activation tile into a ring;
//   warp 1     TMEM allocation and the MMAs (three products per K step into two accumulators);
//   warps 2-5  epilogue.
constexpr int GD_THREADS = 192;
constexpr int GD_A_STAGE = 2 * GM_A_BYTES;  // hi, lo

template <int NT>
struct DenseCfg {
  static constexpr int B_BYTES = NT * 128;
  static constexpr int STAGE = GD_A_STAGE + 2 * B_BYTES;
  static constexpr int S = NT == 256 ? 2 : (NT == 64 ? 4 : 3);
  static constexpr int SMEM = 1024 + S * STAGE + 128;
  static constexpr int TMEM_COLS = NT == 256 ? 512 : 256;  // two accumulators of NT columns
};

constexpr int GD_EPI_FLOATS = 16 * 36;  // per epilogue warp: 16 tokens x 32 rows, rows padded to 36 floats

// Epilogue of one 128-row x NT-token tile whose two accumulators sit in TMEM columns
// [tacc, tacc + NT) and [tacc + NT, tacc + 2 NT) (warp q: TMEM lanes 32q..32q+31, so lane = row
// 32q + lane of the tile): their sum goes to y (+ split z's plane) as f32, or, with a.ghi set,
// through GeGLU (geluMul, shaders.ts:153-170) to activation tiles. For GeGLU the matrix
// interleaves gate (row 2j) and up (row 2j + 1), so a warp's 32 rows are output columns
// 16q'..16q'+15 (q' = 4 m_tile + q) as gate/up lane pairs; a block of 16 tokens x 32 rows goes
// through shared memory st (GD_EPI_FLOATS; rows of 36 floats keep the float4 reads
// conflict-free) and each lane turns one token's 8 pairs into one 8-column hi/lo chunk.
template <int NT>
GG_DEV void dense_epilogue(const GemmArgs& a, uint32_t tacc, int q, int lane, int n_tile, int m_tile, int z, float* st) {
  const uint32_t tl = tacc + ((uint32_t)(q * 32) << 16);
  if (a.ghi) {
    const int j0 = m_tile * 64 + q * 16, tt = lane & 15, hf = lane >> 4;
    const int KSo = a.M / 128;  // 64-column blocks of the M / 2 output columns
#pragma unroll 1
    for (int c = 0; c < NT; c += 16) {
      float v[16], u[16];
      tmem_ld16(tl + (uint32_t)c, v);
      tmem_ld16(tl + (uint32_t)(NT + c), u);
#pragma unroll
      for (int j = 0; j < 16; j++) st[j * 36 + lane] = v[j] + u[j];
      __syncwarp();
      const float4* r = reinterpret_cast<const float4*>(st + tt * 36 + 16 * hf);
      const float4 p0 = r[0], p1 = r[1], p2 = r[2], p3 = r[3];
      __syncwarp();
      const int t = n_tile * NT + c + tt;
      if (t < a.T) {
        const float o[8] = {gelu_tanh(p0.x) * p0.y, gelu_tanh(p0.z) * p0.w, gelu_tanh(p1.x) * p1.y,
                            gelu_tanh(p1.z) * p1.w, gelu_tanh(p2.x) * p2.y, gelu_tanh(p2.z) * p2.w,
                            gelu_tanh(p3.x) * p3.y, gelu_tanh(p3.z) * p3.w};
        xtile_put8(a.ghi, a.glo, KSo, t, j0 + 8 * hf, o);
      }
    }
  } else {
    float* yb = a.y + (long long)z * a.split_stride + m_tile * 128 + q * 32 + lane;
#pragma unroll 1
    for (int c = 0; c < NT; c += 16) {
      float v[16], u[16];
      tmem_ld16(tl + (uint32_t)c, v);
      tmem_ld16(tl + (uint32_t)(NT + c), u);
#pragma unroll
      for (int j = 0; j < 16; j++) {
        const int t = n_tile * NT + c + j;
        if (t < a.T) yb[(long long)t * a.ldy] = v[j] + u[j];
      }
    }
  }
}

template <int NT>
__global__ void __launch_bounds__(GD_THREADS, 1) gg_gemm_dense_kernel(const GemmArgs a) {
  using C = DenseCfg<NT>;
  constexpr int S = C::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S * C::STAGE);
  uint64_t* empty = full + S;
  uint64_t* acc_bar = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int s0 = blockIdx.z * a.slabs_per_split;
  const int ns = min(a.slabs_per_split, a.KS - s0);
  const SpinCtl sc{a.err, a.timeout_ns};
  pdl_trigger();  // weight tiles of the first stages load before pdl_wait(), activations after
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_bar, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {
      const size_t KS = (size_t)a.KS;
      const int pre = min(ns, S);  // stages whose weight tile is issued before the wait
      for (int i = 0; i < pre; i++) {
        mbar_arrive_expect_tx(&full[i], C::STAGE);
        bulk_g2s_plain(ring + i * C::STAGE, a.wt + ((size_t)m_tile * KS + (size_t)(s0 + i)) * GD_A_STAGE, GD_A_STAGE,
                       &full[i]);
      }
      pdl_wait();
      int issued = 0;
      for (int i = 0; i < ns; i++) {
        const int o = i % S;
        if (*abort_flag) break;
        if (i >= S && !mbar_wait(&empty[o], ((i / S) - 1) & 1, sc)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* dst = ring + o * C::STAGE;
        if (i >= pre) {
          mbar_arrive_expect_tx(&full[o], C::STAGE);
          bulk_g2s_plain(dst, a.wt + ((size_t)m_tile * KS + (size_t)(s0 + i)) * GD_A_STAGE, GD_A_STAGE, &full[o]);
        }
#pragma unroll
        for (int hh = 0; hh < NT / 64; hh++) {
          const size_t blk = ((size_t)(n_tile * (NT / 64) + hh) * KS + (size_t)(s0 + i)) * 8192u;
          bulk_g2s_plain(dst + GD_A_STAGE + hh * 8192, a.xhi + blk, 8192, &full[o]);
          bulk_g2s_plain(dst + GD_A_STAGE + C::B_BYTES + hh * 8192, a.xlo + blk, 8192, &full[o]);
        }
        issued++;
      }
      for (int i = issued > S ? issued - S : 0; i < issued; i++) mbar_wait(&full[i % S], (i / S) & 1, sc);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // x_hi and x_lo rows are one operand of 2 NT rows: for NT <= 128 one MMA of N = 2 NT makes
      // Whi*Xhi (accumulator 0) and Whi*Xlo (accumulator 1), then Wlo*Xhi adds into accumulator 1.
      const uint32_t idesc = umma_idesc_bf16_m128(NT), idesc2 = umma_idesc_bf16_m128(NT <= 128 ? 2 * NT : NT);
      for (int i = 0; i < ns; i++) {
        const int o = i % S;
        if (!mbar_wait(&full[o], (i / S) & 1, sc)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t ahi = smem_u32(ring + o * C::STAGE), alo = ahi + GM_A_BYTES;
        const uint32_t bhi = ahi + GD_A_STAGE, blo = bhi + C::B_BYTES;
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint32_t off = kk * 32;
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          if constexpr (NT <= 128) {
            umma_bf16(tmem, umma_desc_sw128(ahi + off), umma_desc_sw128(bhi + off), idesc2, acc);
          } else {
            umma_bf16(tmem, umma_desc_sw128(ahi + off), umma_desc_sw128(bhi + off), idesc, acc);
            umma_bf16(tmem + NT, umma_desc_sw128(ahi + off), umma_desc_sw128(blo + off), idesc, acc);
          }
          umma_bf16(tmem + NT, umma_desc_sw128(alo + off), umma_desc_sw128(bhi + off), idesc, 1u);
        }
        umma_commit(&empty[o]);
      }
      umma_commit(acc_bar);
    }
  } else {  // warps 2..5: epilogue (warp w reads TMEM lanes 32*(w%4)..)
    const int q = warp & 3;
    pdl_wait();
    const bool ok = mbar_wait(acc_bar, 0, sc);
    tc_fence_after();
    const int go = __shfl_sync(0xffffffffu, (ok && !*abort_flag) ? 1 : 0, 0);
    // the ring is idle once the accumulator is complete: its first bytes stage the GeGLU blocks
    if (go) {
      float* st = reinterpret_cast<float*>(ring) + q * GD_EPI_FLOATS;
      dense_epilogue<NT>(a, tmem, q, lane, n_tile, m_tile, blockIdx.z, st);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// The same GEMM as a persistent tile loop (NT = 64, 128): CTA c takes work items c, c + grid, ...
// (item = 128-row tile x NT-token tile x K split, token tiles fastest so the CTAs running at once
// share weight tiles in L2). The copy ring runs on across items, and TMEM holds two accumulator
// sets of 2 NT columns: while the epilogue warps drain item k from one set, the MMAs of item
// k + 1 fill the other, so the epilogue (and a GeGLU in it) is off the tensor pipe's path.
// Hand-offs: full / empty per ring stage (copies -> MMAs -> copies), accf[b] (the MMAs of an
// item in set b complete; one commit) and acce[b] (the four epilogue warps have read set b).
template <int NT>
struct DensePCfg {
  static constexpr int B_BYTES = NT * 128;
  static constexpr int STAGE = GD_A_STAGE + 2 * B_BYTES;
  static constexpr int S = NT == 64 ? 4 : 3;
  static constexpr int EPI = 4 * GD_EPI_FLOATS * 4;
  static constexpr int SMEM = 1024 + S * STAGE + EPI + 256;
  static constexpr int TMEM_COLS = 4 * NT;
};

struct DenseItem {
  int n_tile, m_tile, z, s0, ns;
};
GG_DEV DenseItem dense_item(const GemmArgs& a, int w, int ntt, int mt) {
  DenseItem d;
  d.n_tile = w % ntt;
  const int r = w / ntt;
  d.m_tile = r % mt;
  d.z = r / mt;
  d.s0 = d.z * a.slabs_per_split;
  d.ns = min(a.slabs_per_split, a.KS - d.s0);
  return d;
}

template <int NT>
__global__ void __launch_bounds__(GD_THREADS, 1) gg_gemm_dense_pk_kernel(const GemmArgs a) {
  static_assert(NT == 64 || NT == 128, "two accumulator sets of 2 NT columns in TMEM's 512");
  using C = DensePCfg<NT>;
  constexpr int S = C::S;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* epi = reinterpret_cast<float*>(ring + S * C::STAGE);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S * C::STAGE + C::EPI);
  uint64_t* empty = full + S;
  uint64_t* accf = empty + S;  // [2]
  uint64_t* acce = accf + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntt = (a.T + NT - 1) / NT, mt = a.M / 128;
  const int items = ntt * mt * a.splits;
  const SpinCtl sc{a.err, a.timeout_ns};
  pdl_trigger();  // weight tiles of the first stages load before pdl_wait(), activations after
  if (threadIdx.x == 0) {
    for (int i = 0; i < S; i++) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(&accf[b], 1);
      mbar_init(&acce[b], 4);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp == 0) {
    if (lane == 0) {
      const size_t KS = (size_t)a.KS;
      int pre = 0;  // stages of the first item whose weight tile is issued before the wait
      if ((int)blockIdx.x < items) {
        const DenseItem d = dense_item(a, blockIdx.x, ntt, mt);
        pre = min(d.ns, S);
        for (int i = 0; i < pre; i++) {
          mbar_arrive_expect_tx(&full[i], C::STAGE);
          bulk_g2s_plain(ring + i * C::STAGE, a.wt + ((size_t)d.m_tile * KS + (size_t)(d.s0 + i)) * GD_A_STAGE,
                         GD_A_STAGE, &full[i]);
        }
      }
      pdl_wait();
      int g = 0;  // stages issued (over all items)
      bool run = true;
      for (int w = blockIdx.x; w < items && run; w += gridDim.x) {
        const DenseItem d = dense_item(a, w, ntt, mt);
        for (int i = 0; i < d.ns; i++) {
          const int o = g % S;
          if (*abort_flag) {
            run = false;
            break;
          }
          if (g >= S && !mbar_wait(&empty[o], ((g / S) - 1) & 1, sc)) {
            *abort_flag = 1;
            run = false;
            break;
          }
          uint8_t* dst = ring + o * C::STAGE;
          if (g >= pre) {
            mbar_arrive_expect_tx(&full[o], C::STAGE);
            bulk_g2s_plain(dst, a.wt + ((size_t)d.m_tile * KS + (size_t)(d.s0 + i)) * GD_A_STAGE, GD_A_STAGE, &full[o]);
          }
#pragma unroll
          for (int hh = 0; hh < NT / 64; hh++) {
            const size_t blk = ((size_t)(d.n_tile * (NT / 64) + hh) * KS + (size_t)(d.s0 + i)) * 8192u;
            bulk_g2s_plain(dst + GD_A_STAGE + hh * 8192, a.xhi + blk, 8192, &full[o]);
            bulk_g2s_plain(dst + GD_A_STAGE + C::B_BYTES + hh * 8192, a.xlo + blk, 8192, &full[o]);
          }
          g++;
        }
      }
      for (int i = g > S ? g - S : 0; i < g; i++) mbar_wait(&full[i % S], (i / S) & 1, sc);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // x_hi and x_lo rows are one operand of 2 NT rows: one MMA of N = 2 NT makes Whi*Xhi
      // (columns 0..NT-1 of the set) and Whi*Xlo (NT..2NT-1), then Wlo*Xhi adds into the latter.
      const uint32_t idesc = umma_idesc_bf16_m128(NT), idesc2 = umma_idesc_bf16_m128(2 * NT);
      int g = 0, k = 0;
      for (int w = blockIdx.x; w < items; w += gridDim.x, k++) {
        if (*abort_flag) break;
        const DenseItem d = dense_item(a, w, ntt, mt);
        const int b = k & 1;
        if (k >= 2 && !mbar_wait(&acce[b], ((k >> 1) - 1) & 1, sc)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc0 = tmem + (uint32_t)(b * 2 * NT);
        bool run = true;
        for (int i = 0; i < d.ns; i++, g++) {
          const int o = g % S;
          if (!mbar_wait(&full[o], (g / S) & 1, sc)) {
            *abort_flag = 1;
            run = false;
            break;
          }
          tc_fence_after();
          const uint32_t ahi = smem_u32(ring + o * C::STAGE), alo = ahi + GM_A_BYTES;
          const uint32_t bhi = ahi + GD_A_STAGE;
#pragma unroll
          for (int kk = 0; kk < 4; kk++) {
            const uint32_t off = kk * 32;
            umma_bf16(acc0, umma_desc_sw128(ahi + off), umma_desc_sw128(bhi + off), idesc2, (i > 0 || kk > 0) ? 1u : 0u);
            umma_bf16(acc0 + NT, umma_desc_sw128(alo + off), umma_desc_sw128(bhi + off), idesc, 1u);
          }
          umma_commit(&empty[o]);
        }
        if (!run) break;
        umma_commit(&accf[b]);
      }
    }
  } else {  // warps 2..5: epilogue (warp w reads TMEM lanes 32*(w%4)..)
    const int q = warp & 3;
    float* st = epi + q * GD_EPI_FLOATS;
    pdl_wait();
    int k = 0;
    for (int w = blockIdx.x; w < items; w += gridDim.x, k++) {
      const int b = k & 1;
      const bool ok = mbar_wait(&accf[b], (k >> 1) & 1, sc);
      tc_fence_after();
      const int go = __shfl_sync(0xffffffffu, (ok && !*abort_flag) ? 1 : 0, 0);
      if (!go) {
        if (lane == 0) *abort_flag = 1;
        break;
      }
      const DenseItem d = dense_item(a, w, ntt, mt);
      dense_epilogue<NT>(a, tmem + (uint32_t)(b * 2 * NT), q, lane, d.n_tile, d.m_tile, d.z, st);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[b]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- block-scaled path
// The same product with the Q8_0 scale applied per 32-wide block after the MMAs, as the
// reference's linearQ8 does (acc += d * sum of q * x per block, shaders.ts:92-151). A
// persistent kernel: CTA c takes work items c, c + grid, ... (item = 128-row tile x NT-token
// tile x K split) and every role walks the same sequence of (item, slab) pairs, so the rings
// run on across item boundaries:
//   warp 0      bulk copies of the raw Q8_0 slabs (128 x 64 quants + scales, 8704 B) into a
//               ring (constant data: no wait for the previous kernel);
//   warp 2      bulk copies of each slab's activation tiles (bf16 hi, lo) into a second ring;
//   warps 3-6   convert the quants to bf16 (exact: |q| <= 128 has at most 8 significant bits)
//               into a swizzled operand ring, one weight row per thread, and copy the slab's
//               block scales (as f32) into a ring of their own;
//   warp 1      TMEM allocation and the MMAs: the stage's activation tiles are x_hi rows then
//               x_lo rows, one K-major operand of 2 NT rows, so one MMA of N = 2 NT makes both
//               products Q*Xhi and Q*Xlo (in adjacent column halves); per Q8_0 block (two K
//               steps of 16) two MMAs into its own TMEM accumulator, a slab's two blocks in one
//               of P buffer pairs, then one commit per slab;
//   warps 7..   per slab, read its two block accumulators (both halves) in TMEM round trips
//               of CH columns (warp w: TMEM lanes 32*(w%4).., CW of the NT columns) and add
//               d * (hi + lo) into f32 registers; at the end of an item write its tile.
// One thread issues a tcgen05.mma about every 80-90 cycles whatever its size, so the product
// is built from few wide MMAs: 4 per 128 x 64 slab. The MMAs of a slab complete well after
// they are issued; the 512 TMEM columns hold P = 128 / NT slabs of block accumulators, so that
// many slabs are in flight between the MMAs and the promotion. Two products per K step
// instead of three, and 1.0625 bytes per weight read instead of the dequantised copy's four.
// The products q * x_hi and q * x_lo are exact in f32 and x_hi + x_lo = x to 2^-17 relative.
constexpr int GS_CONV = 4;
constexpr int GS_WARP_CONV = 3;  // first converting warp
constexpr int GS_WARP_EPI = GS_WARP_CONV + GS_CONV;

template <int NT>
struct ScaledCfg {
  static constexpr int XROWS = NT < 64 ? NT : 64;               // rows copied from each 64-row tile block
  static constexpr int XB = NT * 128;                           // one activation operand (hi or lo) of a slab
  static constexpr int D = NT == 32 ? 6 : (NT == 64 ? 5 : 3);   // operand stages (activations + converted weights)
  static constexpr int RS = NT == 64 ? 6 : 8;                   // raw weight stages
  static constexpr int SS = 8;                                  // scale stages
  static constexpr int P = 128 / NT;                            // TMEM buffer pairs (512 columns: 4 NT each)
  static constexpr int EPI = NT == 128 ? 8 : NT / 8;            // promoting warps
  static constexpr int CW = NT * 4 / EPI;                       // columns per promoting warp
  static constexpr int CH = NT == 128 ? 8 : 16;                 // columns of each block half per TMEM round
  static constexpr int THREADS = 32 * (GS_WARP_EPI + EPI);
  static constexpr int TMEM_COLS = 512;
  static constexpr int A_OFF = D * 2 * XB;                      // after the 1 KB-aligned activation ring
  static constexpr int RAW_OFF = A_OFF + D * GM_A_BYTES;
  static constexpr int SC_OFF = RAW_OFF + RS * GG_Q8_TILE_BYTES;
  static constexpr int BAR_OFF = SC_OFF + SS * 128 * 8;
  static constexpr int R = P > D ? P : D;                        // slab-done barriers (see the kernel)
  static constexpr int NBAR = 2 * RS + 2 * D + R + P + 2 * SS + 1;
  static constexpr int SMEM = 1024 + BAR_OFF + NBAR * 8 + 16;
  static_assert(CW % CH == 0 && SMEM <= 232448, "fits one CTA per SM");
};

// 32 consecutive f32 columns of this thread's TMEM lane, without the wait (tmem_ld_wait()).
GG_DEV void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
GG_DEV void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
GG_DEV void tmem_ld8_nowait(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}
template <int N>
GG_DEV void tmem_ld_nowait(uint32_t taddr, uint32_t* r) {
  static_assert(N == 8 || N == 16 || N == 32, "x8, x16 or x32");
  if constexpr (N == 32)
    tmem_ld32_nowait(taddr, *reinterpret_cast<uint32_t(*)[32]>(r));
  else if constexpr (N == 16)
    tmem_ld16_nowait(taddr, *reinterpret_cast<uint32_t(*)[16]>(r));
  else
    tmem_ld8_nowait(taddr, *reinterpret_cast<uint32_t(*)[8]>(r));
}
GG_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Four int8 quants (one word) -> two words of bf16 pairs, exactly.
GG_DEV uint2 q8x4_to_bf16(uint32_t w) {
  const uint32_t wx = w ^ 0x80808080u;
  const uint32_t f0 = __float_as_uint(q8_at(wx, 0)), f1 = __float_as_uint(q8_at(wx, 1));
  const uint32_t f2 = __float_as_uint(q8_at(wx, 2)), f3 = __float_as_uint(q8_at(wx, 3));
  return make_uint2(__byte_perm(f0, f1, 0x7632u), __byte_perm(f2, f3, 0x7632u));
}

// Work item w of a launch: m tile fastest, then token tile, then K split.
struct ScaledItem {
  int mt, nt, s0, ns;
};
GG_DEV ScaledItem scaled_item(const GemmArgs& a, int w, int m_tiles, int n_tiles) {
  ScaledItem it;
  it.mt = w % m_tiles;
  const int r = w / m_tiles;
  it.nt = r % n_tiles;
  it.s0 = (r / n_tiles) * a.slabs_per_split;
  it.ns = min(a.slabs_per_split, a.KS - it.s0);
  return it;
}

template <int NT>
__global__ void __launch_bounds__(ScaledCfg<NT>::THREADS, 1) gg_gemm_q8s_kernel(const GemmArgs a) {
  using C = ScaledCfg<NT>;
  constexpr int D = C::D, RS = C::RS, SS = C::SS, P = C::P, R = C::R;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* xring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* aring = xring + C::A_OFF;
  uint8_t* rring = xring + C::RAW_OFF;
  float2* sring = reinterpret_cast<float2*>(xring + C::SC_OFF);  // [SS][128]: a row's two block scales
  uint64_t* full_r = reinterpret_cast<uint64_t*>(xring + C::BAR_OFF);
  uint64_t* empty_r = full_r + RS;  // raw slot converted
  uint64_t* full_x = empty_r + RS;  // activation stage landed
  uint64_t* full_a = full_x + D;    // weight operand converted (and the activations seen landed)
  // mdone_s[g % R]: the MMAs of slab g completed, so its block accumulators are complete and its
  // operand stages free. R >= P and R >= D keep every wait on it within one phase: the MMAs of
  // slab g + R need operand stage g + R (issued only after the activation producer and the
  // converters waited for slab g + R - D) and buffer pair g + R (released only after the
  // promotion consumed slab g + R - P).
  uint64_t* sdone = full_a + D;
  uint64_t* tempty = sdone + C::R;  // a slab's block accumulators read
  uint64_t* sfull = tempty + P;     // scales written
  uint64_t* sempty = sfull + SS;    // ... and read
  uint64_t* mdone = sempty + SS;    // every MMA issued has completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mdone + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_tiles = a.M / 128, n_tiles = (a.T + NT - 1) / NT;
  const int n_items = m_tiles * n_tiles * a.splits;
  const SpinCtl sc{a.err, a.timeout_ns};
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; i++) {
      mbar_init(&full_r[i], 1);
      mbar_init(&empty_r[i], GS_CONV);
    }
    for (int i = 0; i < D; i++) {
      mbar_init(&full_x[i], 1);
      mbar_init(&full_a[i], GS_CONV);
    }
    for (int i = 0; i < R; i++) mbar_init(&sdone[i], 1);
    for (int i = 0; i < P; i++) mbar_init(&tempty[i], C::EPI);
    for (int i = 0; i < SS; i++) {
      mbar_init(&sfull[i], GS_CONV);
      mbar_init(&sempty[i], C::EPI);
    }
    mbar_init(mdone, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // raw weight slabs (never written by any kernel: no PDL wait)
      uint32_t g = 0;
      bool stop = false;
      for (int w = blockIdx.x; w < n_items && !stop; w += gridDim.x) {
        const ScaledItem it = scaled_item(a, w, m_tiles, n_tiles);
        const uint8_t* src = a.wt + ((size_t)it.mt * a.KS + (size_t)it.s0) * GG_Q8_TILE_BYTES;
        for (int i = 0; i < it.ns; i++, g++) {
          const uint32_t o = g % RS;
          if (*abort_flag || (g >= (uint32_t)RS && !mbar_wait(&empty_r[o], ((g / RS) - 1) & 1, sc))) {
            *abort_flag = 1;
            stop = true;
            break;
          }
          mbar_arrive_expect_tx(&full_r[o], GG_Q8_TILE_BYTES);
          bulk_g2s_plain(rring + o * GG_Q8_TILE_BYTES, src + (size_t)i * GG_Q8_TILE_BYTES, GG_Q8_TILE_BYTES, &full_r[o]);
        }
      }
      // before exit: every copy issued has landed (none may still write this CTA's memory)
      for (uint32_t i = g > (uint32_t)RS ? g - RS : 0; i < g; i++) mbar_wait(&full_r[i % RS], (i / RS) & 1, sc);
    }
  } else if (warp == 2) {
    if (lane == 0) {  // activation tiles
      pdl_wait();
      uint32_t g = 0;
      bool stop = false;
      const size_t KS = (size_t)a.KS;
      for (int w = blockIdx.x; w < n_items && !stop; w += gridDim.x) {
        const ScaledItem it = scaled_item(a, w, m_tiles, n_tiles);
        for (int i = 0; i < it.ns; i++, g++) {
          const uint32_t o = g % D, u = g - D;  // the stage's previous slab
          if (*abort_flag || (g >= (uint32_t)D && !mbar_wait(&sdone[u % R], (u / R) & 1, sc))) {
            *abort_flag = 1;
            stop = true;
            break;
          }
          uint8_t* dst = xring + o * 2 * C::XB;
          mbar_arrive_expect_tx(&full_x[o], 2 * C::XB);
#pragma unroll
          for (int hh = 0; hh < (NT + 63) / 64; hh++) {
            // token rows NT*nt + 64*hh.. sit in 64-row tile block (NT*nt)/64 + hh, from row (NT*nt)%64
            const int tb = (NT * it.nt) / 64 + hh, r0 = (NT * it.nt) % 64;
            const size_t blk = ((size_t)tb * KS + (size_t)(it.s0 + i)) * 8192u + (size_t)r0 * 128;
            bulk_g2s_plain(dst + hh * 8192, a.xhi + blk, C::XROWS * 128, &full_x[o]);
            bulk_g2s_plain(dst + C::XB + hh * 8192, a.xlo + blk, C::XROWS * 128, &full_x[o]);
          }
        }
      }
      for (uint32_t i = g > (uint32_t)D ? g - D : 0; i < g; i++) mbar_wait(&full_x[i % D], (i / D) & 1, sc);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issue
      const uint32_t idesc = umma_idesc_bf16_m128(2 * NT);  // x_hi and x_lo rows together
      // Descriptors of stage 0; a stage, a K step or the lo half only moves the start address
      // (16-byte units in the low 14 bits, which no sum here carries out of: shared memory < 256 KB).
      const uint64_t a0 = umma_desc_sw128(smem_u32(aring)), b0 = umma_desc_sw128(smem_u32(xring));
      uint32_t g = 0;
      bool stop = false;
      for (int w = blockIdx.x; w < n_items && !stop; w += gridDim.x) {
        const ScaledItem it = scaled_item(a, w, m_tiles, n_tiles);
        for (int i = 0; i < it.ns; i++, g++) {
          const uint32_t o = g % D, p = g % P, u = g - P;  // u: the pair's previous slab
          if (!mbar_wait(&full_a[o], (g / D) & 1, sc) || (g >= (uint32_t)P && !mbar_wait(&tempty[p], (u / P) & 1, sc))) {
            stop = true;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a0 + (uint64_t)(o * (GM_A_BYTES >> 4));
          const uint64_t bx = b0 + (uint64_t)(o * ((2 * C::XB) >> 4));
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const uint32_t d = tmem + (uint32_t)((2 * p + h) * 2 * NT);
#pragma unroll
            for (int kk = 0; kk < 2; kk++) {
              const uint64_t off = (uint64_t)(2 * h + kk) * 2;  // 32 bytes per K step of 16
              umma_bf16(d, ad + off, bx + off, idesc, kk > 0 ? 1u : 0u);
            }
          }
          umma_commit(&sdone[g % R]);
        }
      }
      if (stop) *abort_flag = 1;
      umma_commit(mdone);  // no MMA may still write TMEM when it is freed
      mbar_wait(mdone, 0, sc);
    }
  } else if (warp < GS_WARP_EPI) {  // convert: thread r = weight row r of every slab
    const int r = (warp - GS_WARP_CONV) * 32 + lane;
    const uint32_t rowoff = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    uint32_t g = 0;
    bool stop = false;
    for (int w = blockIdx.x; w < n_items && !stop; w += gridDim.x) {
      const ScaledItem it = scaled_item(a, w, m_tiles, n_tiles);
      for (int i = 0; i < it.ns; i++, g++) {
        const uint32_t o = g % RS, oa = g % D, os = g % SS, u = g - D;
        if (*abort_flag || !mbar_wait(&full_r[o], (g / RS) & 1, sc) ||
            (g >= (uint32_t)D && !mbar_wait(&sdone[u % R], (u / R) & 1, sc)) ||
            (g >= (uint32_t)SS && !mbar_wait(&sempty[os], ((g / SS) - 1) & 1, sc))) {
          *abort_flag = 1;
          stop = true;
          break;
        }
        const uint8_t* raw = rring + o * GG_Q8_TILE_BYTES;
        const uint32_t s2 = *reinterpret_cast<const uint32_t*>(raw + GM_RAW_Q + r * 4);
        sring[os * 128 + r] = make_float2(__half2float(__ushort_as_half((unsigned short)(s2 & 0xffffu))),
                                          __half2float(__ushort_as_half((unsigned short)(s2 >> 16))));
        uint8_t* dst = aring + oa * GM_A_BYTES;
#pragma unroll
        for (int c = 0; c < 4; c++) {
          // chunk c ^ H[m] for lanes 2m, 2m + 1, with H[m] = 2m in GF(4) = (0, 2, 3, 1): both
          // H and H ^ m are permutations, so neither the 64-byte-strided loads nor the
          // swizzled stores of a quarter warp meet a bank twice
          const int cc = c ^ ((0x78 >> (2 * ((lane >> 1) & 3))) & 3);
          const uint4 q = *reinterpret_cast<const uint4*>(raw + r * 64 + cc * 16);
          const uint2 b0 = q8x4_to_bf16(q.x), b1 = q8x4_to_bf16(q.y), b2 = q8x4_to_bf16(q.z), b3 = q8x4_to_bf16(q.w);
          // weights 16cc..16cc+15 = operand chunks 2cc, 2cc + 1 (8 bf16 each) of row r
          *reinterpret_cast<uint4*>(dst + rowoff + ((uint32_t)(((2 * cc) ^ (r & 7)) & 7) << 4)) =
              make_uint4(b0.x, b0.y, b1.x, b1.y);
          *reinterpret_cast<uint4*>(dst + rowoff + ((uint32_t)(((2 * cc + 1) ^ (r & 7)) & 7) << 4)) =
              make_uint4(b2.x, b2.y, b3.x, b3.y);
        }
        fence_proxy_async_smem();
        // the stage's activations too have landed before the MMAs are told the stage is ready
        const bool xin = mbar_wait(&full_x[oa], (g / D) & 1, sc);
        __syncwarp();
        if (!xin) {
          *abort_flag = 1;
          stop = true;
          break;
        }
        if (lane == 0) {
          mbar_arrive(&sfull[os]);
          mbar_arrive(&full_a[oa]);
          mbar_arrive(&empty_r[o]);
        }
      }
    }
  } else {  // block promotion: thread = TMEM lane = weight row, columns cb..cb + CW - 1
    constexpr int CW = C::CW, CH = C::CH;
    const int q = warp & 3, rr = q * 32 + lane, cb = ((warp - GS_WARP_EPI) >> 2) * CW;
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)cb;
    uint32_t g = 0;  // slabs consumed, over all items
    bool ok = true, waited = false;
    for (int w = blockIdx.x; w < n_items && ok; w += gridDim.x) {
      const ScaledItem it = scaled_item(a, w, m_tiles, n_tiles);
      float acc[CW];
#pragma unroll
      for (int c = 0; c < CW; c++) acc[c] = 0.f;
      for (int i = 0; i < it.ns; i++, g++) {
        const uint32_t p = g % P, os = g % SS;
        if (*abort_flag || !mbar_wait(&sdone[g % R], (g / R) & 1, sc) || !mbar_wait(&sfull[os], (g / SS) & 1, sc)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float2 d = sring[os * 128 + rr];
        __syncwarp();
        if (lane == 0) mbar_arrive(&sempty[os]);
        const uint32_t t0 = tl + (uint32_t)(4 * p * NT), t1 = t0 + 2 * NT;  // the slab's two block accumulators
#pragma unroll
        for (int c0 = 0; c0 < CW; c0 += CH) {  // columns c0..c0 + CH of both halves of both blocks
          uint32_t v[4 * CH];
          tmem_ld_nowait<CH>(t0 + (uint32_t)c0, v);
          tmem_ld_nowait<CH>(t0 + (uint32_t)(NT + c0), v + CH);
          tmem_ld_nowait<CH>(t1 + (uint32_t)c0, v + 2 * CH);
          tmem_ld_nowait<CH>(t1 + (uint32_t)(NT + c0), v + 3 * CH);
          tmem_ld_wait();
          if (c0 + CH == CW) {  // this warp's columns of both blocks read: release them
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&tempty[p]);
          }
#pragma unroll
          for (int c = 0; c < CH; c++) {
            const float b0v = __uint_as_float(v[c]) + __uint_as_float(v[CH + c]);
            const float b1v = __uint_as_float(v[2 * CH + c]) + __uint_as_float(v[3 * CH + c]);
            acc[c0 + c] = fmaf(d.y, b1v, fmaf(d.x, b0v, acc[c0 + c]));
          }
        }
      }
      if (!ok) break;
      if (!waited) {  // before the first write to a buffer of the chain
        pdl_wait();
        waited = true;
      }
      const int z = w / (m_tiles * n_tiles);
      float* yb = a.y + (long long)z * a.split_stride + (it.mt * 128 + rr);
#pragma unroll
      for (int c = 0; c < CW; c++) {
        const int t = it.nt * NT + cb + c;
        if (t < a.T) yb[(long long)t * a.ldy] = acc[c];
      }
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------- one row
// y[m] = sum_b d[m][b] * (q[m][32b..32b+31] . x[32b..]) for a single activation row: the
// reference's linearQ8 (shaders.ts:92-151) at batch 1, read straight from the device rows. A
// warp per weight row; lane l takes the row's 16-byte chunks l, l + 32, ... (16 int8 weights,
// exact int8 -> f32 by the 2^23 magic-number trick, 16 FMAs, times the block scale). x sits in
// shared memory permuted so that the warp's four float4 reads of a step are each contiguous
// (quad i of chunk c at [i][c]): no bank conflicts.
constexpr int MV_THREADS = 256;
// R rows per warp at a time (their loads in flight together, x read once for all R): R = 4 when
// the matrix has rows enough for a CTA per SM that way, else 1.
template <int R>
__global__ void __launch_bounds__(MV_THREADS) gg_matvec_q8_kernel(const uint8_t* __restrict__ rows, int rs, int M,
                                                                int K, const float* __restrict__ x,
                                                                float* __restrict__ y) {
  pdl_trigger();
  extern __shared__ float4 xq[];  // [4][K / 16]
  const int nch = K / 16;
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  for (int qd = threadIdx.x; qd < K / 4; qd += MV_THREADS)
    xq[(qd & 3) * nch + (qd >> 2)] = reinterpret_cast<const float4*>(x)[qd];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ngroups = (M + R - 1) / R;
  for (int gi = blockIdx.x * (MV_THREADS / 32) + warp; gi < ngroups; gi += gridDim.x * (MV_THREADS / 32)) {
    const int m0 = gi * R;
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; r++) acc[r] = 0.f;
#pragma unroll(R == 1 ? 2 : 1)
    for (int c = lane; c < nch; c += 32) {
      uint4 w[R];
      float d[R];
#pragma unroll
      for (int r = 0; r < R; r++) {
        const uint8_t* row = rows + (size_t)min(m0 + r, M - 1) * rs;
        w[r] = ldg_nc16(row + 16 * c);
        d[r] = __half2float(__ushort_as_half((unsigned short)ldg_nc_u16(row + K + 2 * (c >> 1))));
      }
      float sum[R];
#pragma unroll
      for (int r = 0; r < R; r++) sum[r] = 0.f;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const float4 xv = xq[i * nch + c];
#pragma unroll
        for (int r = 0; r < R; r++) {
          const uint32_t wx = (i == 0 ? w[r].x : i == 1 ? w[r].y : i == 2 ? w[r].z : w[r].w) ^ 0x80808080u;
          sum[r] = fmaf(q8_at(wx, 0), xv.x, sum[r]);
          sum[r] = fmaf(q8_at(wx, 1), xv.y, sum[r]);
          sum[r] = fmaf(q8_at(wx, 2), xv.z, sum[r]);
          sum[r] = fmaf(q8_at(wx, 3), xv.w, sum[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < R; r++) acc[r] = fmaf(sum[r], d[r], acc[r]);
    }
#pragma unroll
    for (int r = 0; r < R; r++) {
      const float v = warp_sum(acc[r]);
      if (lane == 0 && m0 + r < M) y[m0 + r] = v;
    }
  }
}

// Tiled Q8_0 copy -> dense (hi, lo) operand tiles: one CTA per 128 x 64 slab, one thread per
// Q8_0 block (same dequantisation as the GEMM's dequantising warps).
__global__ void __launch_bounds__(256) gg_dense_tile_kernel(const uint8_t* __restrict__ q8tiles, uint8_t* __restrict__ dense) {
  const uint8_t* src = q8tiles + (size_t)blockIdx.x * GG_Q8_TILE_BYTES;
  uint8_t* dst = dense + (size_t)blockIdx.x * GD_A_STAGE;
  const int r = threadIdx.x >> 1, h = threadIdx.x & 1;
  const uint4 q0 = *reinterpret_cast<const uint4*>(src + r * 64 + h * 32);
  const uint4 q1 = *reinterpret_cast<const uint4*>(src + r * 64 + h * 32 + 16);
  const float d = __half2float(*reinterpret_cast<const __half*>(src + GM_RAW_Q + r * 4 + h * 2));
  dequant_block32(q0, q1, d, dst, dst + GM_A_BYTES, r, h);
}

// Device rows -> tiled copy: block (mt, s) = rows 128*mt.. x columns 64*s.. quants, then the two
// f16 scales of each row's blocks 2s, 2s+1.
__global__ void gg_q8_tile_kernel(const uint8_t* __restrict__ rows, int rs, int K, uint8_t* __restrict__ tiles) {
  const int KS = K / 64, t = blockIdx.x, mt = t / KS, sl = t % KS;
  uint8_t* dst = tiles + (size_t)t * GG_Q8_TILE_BYTES;
  for (int i = threadIdx.x; i < 128 * 4; i += blockDim.x) {
    const int r = i >> 2, c = i & 3;
    *reinterpret_cast<uint4*>(dst + r * 64 + c * 16) =
        *reinterpret_cast<const uint4*>(rows + (size_t)(mt * 128 + r) * rs + sl * 64 + c * 16);
  }
  for (int r = threadIdx.x; r < 128; r += blockDim.x)
    *reinterpret_cast<uint32_t*>(dst + GM_RAW_Q + r * 4) =
        *reinterpret_cast<const uint32_t*>(rows + (size_t)(mt * 128 + r) * rs + K + sl * 4);
}

// f32 rows -> activation tiles; one thread per 8 columns.
__global__ void gg_xtiles_kernel(const float* __restrict__ x, int T, int Tpad, int K, uint8_t* hi, uint8_t* lo) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  const int KS = K / 64, k8 = K / 8;
  const long long n = (long long)Tpad * k8;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / k8), k = (int)(i % k8) * 8;
    float v[8];
    if (t < T) {
      const float4 a = *reinterpret_cast<const float4*>(x + (long long)t * K + k);
      const float4 b = *reinterpret_cast<const float4*>(x + (long long)t * K + k + 4);
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
      for (int j = 0; j < 8; j++) v[j] = 0.f;
    }
    xtile_put8(hi, lo, KS, t, k, v);
  }
}

}  // namespace gg

using namespace gg;

size_t gg_xtiles_bytes(int T, int K) { return (size_t)((T + 255) / 256 * 256) * (size_t)K * 2; }

size_t gg_q8_tiles_bytes(int M, int K) { return (size_t)(M / 128) * (size_t)(K / 64) * GG_Q8_TILE_BYTES; }

cudaError_t gg_make_q8_tiles(GGQ8Map* out, const uint8_t* rows, int M, int K, uint8_t* tiles, cudaStream_t s) {
  if (M % 128 || K % 64 || M <= 0 || K <= 0) return cudaErrorInvalidValue;
  const int rs = ((K + (K / 32) * 2) + 15) / 16 * 16;
  const int ntiles = (M / 128) * (K / 64);
  gg_q8_tile_kernel<<<ntiles, 256, 0, s>>>(rows, rs, K, tiles);
  out->tiles = tiles;
  out->M = M;
  out->K = K;
  return cudaGetLastError();
}

size_t gg_dense_tiles_bytes(int M, int K) { return (size_t)(M / 128) * (size_t)(K / 64) * GD_A_STAGE; }

cudaError_t gg_make_dense_tiles(GGQ8Map* w, uint8_t* dense, cudaStream_t s) {
  if (!w->tiles) return cudaErrorInvalidValue;
  gg_dense_tile_kernel<<<(w->M / 128) * (w->K / 64), 256, 0, s>>>(w->tiles, dense);
  w->dense = dense;
  return cudaGetLastError();
}

cudaError_t gg_xtiles_from_f32(const float* x, int T, int K, uint8_t* xhi, uint8_t* xlo, cudaStream_t s) {
  if (T <= 0 || K % 64) return cudaErrorInvalidValue;
  const int Tpad = (T + 255) / 256 * 256;  // whole tiles of the widest (256-row) kernel
  const long long n = (long long)Tpad * (K / 8);
  const int blocks = (int)((n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8);
  cudaError_t r = launch_pdl(gg_xtiles_kernel, dim3(blocks), dim3(256), 0, s, x, T, Tpad, K, xhi, xlo);
  if (r != cudaSuccess) return r;
  return cudaGetLastError();
}

template <int NT>
static cudaError_t launch_nt(const GGQ8Map& w, const GemmArgs& a, int splits, cudaStream_t s) {
  static bool attr_set[64] = {};  // the attribute is per function and device
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    r = cudaFuncSetAttribute(gg_gemm_q8_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmCfg<NT>::SMEM);
    if (r != cudaSuccess) return r;
    attr_set[dev] = true;
  }
  dim3 grid((a.T + NT - 1) / NT, w.M / 128, splits);
  r = launch_pdl(gg_gemm_q8_kernel<NT>, grid, dim3(GM_THREADS), GemmCfg<NT>::SMEM, s, a);
  if (r != cudaSuccess) return r;
  return cudaGetLastError();
}

template <int NT>
static cudaError_t launch_dense(const GemmArgs& a, int m_tiles, int splits, cudaStream_t s) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    r = cudaFuncSetAttribute(gg_gemm_dense_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, DenseCfg<NT>::SMEM);
    if (r != cudaSuccess) return r;
    attr_set[dev] = true;
  }
  dim3 grid((a.T + NT - 1) / NT, m_tiles, splits);
  r = launch_pdl(gg_gemm_dense_kernel<NT>, grid, dim3(GD_THREADS), DenseCfg<NT>::SMEM, s, a);
  if (r != cudaSuccess) return r;
  return cudaGetLastError();
}

static cudaError_t device_sms(int dev, int* out) {
  static int sms[64] = {};
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!sms[dev]) {
    cudaError_t r = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (r != cudaSuccess) return r;
  }
  *out = sms[dev];
  return cudaSuccess;
}

// Persistent dense kernel: one CTA per SM at most, each walking work items blockIdx.x, + gridDim.x, ...
template <int NT>
static cudaError_t launch_dense_pk(const GemmArgs& a, int m_tiles, int splits, cudaStream_t s) {
  static bool attr_set[64] = {};
  int dev = 0, sms = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r == cudaSuccess) r = device_sms(dev, &sms);
  if (r != cudaSuccess) return r;
  if (!attr_set[dev]) {
    r = cudaFuncSetAttribute(gg_gemm_dense_pk_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, DensePCfg<NT>::SMEM);
    if (r != cudaSuccess) return r;
    attr_set[dev] = true;
  }
  const long long items = (long long)((a.T + NT - 1) / NT) * m_tiles * splits;
  dim3 grid((unsigned)std::min<long long>(items, sms), 1, 1);
  r = launch_pdl(gg_gemm_dense_pk_kernel<NT>, grid, dim3(GD_THREADS), DensePCfg<NT>::SMEM, s, a);
  if (r != cudaSuccess) return r;
  return cudaGetLastError();
}

template <int NT>
static cudaError_t launch_scaled(const GemmArgs& a, int m_tiles, int splits, cudaStream_t s) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    r = cudaFuncSetAttribute(gg_gemm_q8s_kernel<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, ScaledCfg<NT>::SMEM);
    if (r != cudaSuccess) return r;
    attr_set[dev] = true;
  }
  // persistent: one CTA per SM at most, each walking work items blockIdx.x, + gridDim.x, ...
  static int sms[64] = {};
  if (!sms[dev]) {
    r = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (r != cudaSuccess) return r;
  }
  const long long items = (long long)((a.T + NT - 1) / NT) * m_tiles * splits;
  dim3 grid((unsigned)std::min<long long>(items, sms[dev]), 1, 1);
  r = launch_pdl(gg_gemm_q8s_kernel<NT>, grid, dim3(ScaledCfg<NT>::THREADS), ScaledCfg<NT>::SMEM, s, a);
  if (r != cudaSuccess) return r;
  return cudaGetLastError();
}

static int g_gemm_path = GG_GEMM_DEQUANT;
void gg_gemm_set_path(int path) { g_gemm_path = path; }
int gg_gemm_path() { return g_gemm_path; }

// The dense (dequantised copy) kernel for T > 8 rows: the row tile width by T.
static cudaError_t dispatch_dense(const GGQ8Map& w, GemmArgs a, int splits, cudaStream_t s) {
  a.wt = w.dense;
  if (a.T <= 64) return launch_dense_pk<64>(a, w.M / 128, splits, s);
  // 256-row tiles halve the weight-tile reads, but only matrices wide enough to fill two waves
  // of 256-row tiles have tiles to spare (one and a half waves lose more than the reads save)
  const bool wide = a.T > 128 && (long long)((a.T + 255) / 256) * (w.M / 128) * splits >= 2 * 148;
  return wide ? launch_dense<256>(a, w.M / 128, splits, s) : launch_dense_pk<128>(a, w.M / 128, splits, s);
}

cudaError_t gg_gemm_q8(const GGQ8Map& w, const uint8_t* xhi, const uint8_t* xlo, int T, float* y, long long ldy,
                       int splits, long long split_stride, uint32_t* err, uint64_t timeout_ns, cudaStream_t s) {
  if (T <= 0 || splits <= 0) return cudaErrorInvalidValue;
  GemmArgs a{};
  a.wt = w.tiles;
  a.xhi = xhi;
  a.xlo = xlo;
  a.y = y;
  a.ldy = ldy;
  a.split_stride = split_stride;
  a.M = w.M;
  a.K = w.K;
  a.T = T;
  a.KS = w.K / 64;
  a.slabs_per_split = (a.KS + splits - 1) / splits;
  if ((long long)(splits - 1) * a.slabs_per_split >= a.KS) return cudaErrorInvalidValue;  // an empty split
  a.err = err;
  a.timeout_ns = timeout_ns;
  a.splits = splits;
  if (g_gemm_path == GG_GEMM_SCALED) {
    if (T <= 32) return launch_scaled<32>(a, w.M / 128, splits, s);
    return T <= 64 ? launch_scaled<64>(a, w.M / 128, splits, s) : launch_scaled<128>(a, w.M / 128, splits, s);
  }
  if (T > 8 && w.dense) return dispatch_dense(w, a, splits, s);  // dequantised copy: 4 B per weight read
  return T <= 64 ? launch_nt<64>(w, a, splits, s) : launch_nt<128>(w, a, splits, s);
}

bool gg_gemm_geglu_fusable(const GGQ8Map& w, int T, int splits) {
  return g_gemm_path == GG_GEMM_DEQUANT && T > 8 && w.dense != nullptr && splits == 1 && w.M % 128 == 0;
}

cudaError_t gg_gemm_q8_geglu(const GGQ8Map& w, const uint8_t* xhi, const uint8_t* xlo, int T, uint8_t* ghi,
                             uint8_t* glo, uint32_t* err, uint64_t timeout_ns, cudaStream_t s) {
  if (T <= 0 || !ghi || !glo || !gg_gemm_geglu_fusable(w, T, 1)) return cudaErrorInvalidValue;
  GemmArgs a{};
  a.xhi = xhi;
  a.xlo = xlo;
  a.ghi = ghi;
  a.glo = glo;
  a.M = w.M;
  a.K = w.K;
  a.T = T;
  a.KS = w.K / 64;
  a.slabs_per_split = a.KS;
  a.err = err;
  a.timeout_ns = timeout_ns;
  a.splits = 1;
  return dispatch_dense(w, a, 1, s);
}

cudaError_t gg_matvec_q8(const uint8_t* rows, int rs, int M, int K, const float* x, float* y, int sms,
                         cudaStream_t s) {
  if (M <= 0 || K <= 0 || K % 64 || K > 16384 || rs < K + K / 16) return cudaErrorInvalidValue;
  const size_t smem = (size_t)K * 4;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return r;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    r = cudaFuncSetAttribute(gg::gg_matvec_q8_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    if (r == cudaSuccess)
      r = cudaFuncSetAttribute(gg::gg_matvec_q8_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    if (r != cudaSuccess) return r;
    attr_set[dev] = true;
  }
  constexpr int WARPS = gg::MV_THREADS / 32;
  const int cap = sms * 8;  // CTAs: eight per SM of 8 warps
  if ((M + 4 * WARPS - 1) / (4 * WARPS) >= sms) {  // four rows per warp still fill every SM
    const int grid = std::min((M + 4 * WARPS - 1) / (4 * WARPS), cap);
    return gg::launch_pdl(gg::gg_matvec_q8_kernel<4>, dim3(grid), dim3(gg::MV_THREADS), smem, s, rows, rs, M, K, x, y);
  }
  const int grid = std::min((M + WARPS - 1) / WARPS, cap);
  return gg::launch_pdl(gg::gg_matvec_q8_kernel<1>, dim3(grid), dim3(gg::MV_THREADS), smem, s, rows, rs, M, K, x, y);
}
