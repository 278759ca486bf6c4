// gg_gemm.cu -- Q8_0 x activations on the sm_100a tensor cores (tcgen05, TMEM accumulators).
//
// One CTA computes a 128-row x NT-token tile of Y over a K-slice:
//   warp 0      TMA loads of the raw Q8_0 tile (128 rows x 64 quants + the 256-wide scale
//               window) into a ring;
//   warp 1      bulk copies of the activation tiles (bf16 hi and lo, NT x 64) into their
//               own ring, running ahead of the MMAs;
//   warp 2      TMEM allocation and the MMA issue: per 64-wide K slab, 4 K-steps of
//               three MMAs (Whi*Xhi + Whi*Xlo + Wlo*Xhi) into one f32 accumulator;
//   warps 3-10  dequantise: each lane turns one Q8_0 block (32 int8 x f16 scale) into exact
//               f32 weights, splits them into bf16 hi/lo and writes them in the swizzled
//               operand layout; warps 3-6 then read the accumulator out of TMEM.
// The weight products q*d are exact in f32 and hi + lo keeps 16 of their bits; with X split
// the same way the result matches an f32 dot product to ~1e-5 relative. This replaces the
// reference's linearQ8 shader (src/shaders.ts:92-151) for batched rows (prefill, batches).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "gg_gemm.h"
#include "gg_gemm_dev.cuh"

namespace gg {

constexpr int GM_THREADS = 352;
constexpr int GM_RAW_Q = 128 * 64;
constexpr int GM_RAW_S = 128 * 16;
constexpr int GM_RAW_BYTES = GM_RAW_Q + GM_RAW_S;
constexpr int GM_A_BYTES = 128 * 128;  // 128 rows x 64 bf16

// Three rings: raw Q8_0 tiles (TMA), dequantised weight operands (hi, lo), activation
// operands (hi, lo). The activation ring is separate so its loads run ahead of the MMAs.
template <int NT>
struct GemmCfg {
  static constexpr int RS = NT == 128 ? 5 : 6;
  static constexpr int AS = NT == 128 ? 2 : 3;
  static constexpr int BS = NT == 128 ? 3 : 4;
  static constexpr int A_STAGE = 2 * GM_A_BYTES;
  static constexpr int B_BYTES = NT * 128;
  static constexpr int B_STAGE = 2 * B_BYTES;
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = 1024 + AS * A_STAGE + BS * B_STAGE + RS * GM_RAW_BYTES + BAR_BYTES;
};

struct GemmArgs {
  const uint8_t* xhi;
  const uint8_t* xlo;
  float* y;
  long long ldy, split_stride;
  int M, K, T, KS, slabs_per_split;
  uint32_t* err;
  uint64_t timeout_ns;
};

// Exact int8 -> f32 of byte b of wx = raw ^ 0x80808080 (2^23 + u with u = q + 128, minus 2^23 + 128).
GG_DEV float q8_at(uint32_t wx, int b) {
  return __int_as_float((int)__byte_perm(wx, 0x4B000000u, 0x7440u + (uint32_t)b)) - 8388736.0f;
}

template <int NT>
__global__ void __launch_bounds__(GM_THREADS, 1)
    gg_gemm_q8_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap ts,
                      const GemmArgs a) {
  using C = GemmCfg<NT>;
  constexpr int RS = C::RS, AS = C::AS, BS = C::BS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* aring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bring = aring + AS * C::A_STAGE;
  uint8_t* raw = bring + BS * C::B_STAGE;
  uint64_t* full_raw = reinterpret_cast<uint64_t*>(raw + RS * GM_RAW_BYTES);
  uint64_t* empty_raw = full_raw + RS;
  uint64_t* full_a = empty_raw + RS;
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

  if (threadIdx.x == 0) {
    for (int i = 0; i < RS; i++) {
      mbar_init(&full_raw[i], 1);
      mbar_init(&empty_raw[i], 8);
    }
    for (int i = 0; i < AS; i++) {
      mbar_init(&full_a[i], 8);
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
  if (warp == 2) {
    tmem_alloc(tmem_slot, NT);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // raw Q8_0 tiles
      int issued = 0;
      for (int i = 0; i < ns; i++) {
        const int r = i % RS;
        if (*abort_flag) break;
        if (i >= RS && !mbar_wait(&empty_raw[r], ((i / RS) - 1) & 1, sc)) {
          *abort_flag = 1;
          break;
        }
        const int k0 = (s0 + i) * 64;
        mbar_arrive_expect_tx(&full_raw[r], GM_RAW_BYTES);
        tma_load_2d(raw + r * GM_RAW_BYTES, &tq, k0, m_tile * 128, &full_raw[r]);
        tma_load_2d(raw + r * GM_RAW_BYTES + GM_RAW_Q, &ts, a.K + (k0 >> 8) * 16, m_tile * 128, &full_raw[r]);
        issued++;
      }
      for (int i = issued > RS ? issued - RS : 0; i < issued; i++) mbar_wait(&full_raw[i % RS], (i / RS) & 1, sc);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // activation tiles
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
  } else if (warp == 2) {
    if (lane == 0) {  // MMA issue
      const uint32_t idesc = umma_idesc_bf16_m128(NT);
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
          umma_bf16(tmem, umma_desc_sw128(ahi + off), umma_desc_sw128(bhi + off), idesc, (i | kk) ? 1u : 0u);
          umma_bf16(tmem, umma_desc_sw128(ahi + off), umma_desc_sw128(blo + off), idesc, 1u);
          umma_bf16(tmem, umma_desc_sw128(alo + off), umma_desc_sw128(bhi + off), idesc, 1u);
        }
        umma_commit(&empty_a[ia]);
        umma_commit(&empty_b[ib]);
      }
      umma_commit(acc_bar);  // arrives once every MMA issued above has completed
    }
  } else {
    // dequantise: lane -> (row r, block half h) of the 128 x 64 slab
    const int tw = warp - 3;
    const int r = tw * 16 + (lane >> 1), h = lane & 1;
    const uint32_t rowoff = (uint32_t)((r >> 3) * 1024 + (r & 7) * 128);
    for (int i = 0; i < ns; i++) {
      const int rr = i % RS, ia = i % AS;
      if (*abort_flag) break;
      if (!mbar_wait(&full_raw[rr], (i / RS) & 1, sc)) {
        *abort_flag = 1;
        break;
      }
      const uint8_t* rq = raw + rr * GM_RAW_BYTES + r * 64 + h * 32;
      const uint4 q0 = *reinterpret_cast<const uint4*>(rq);
      const uint4 q1 = *reinterpret_cast<const uint4*>(rq + 16);
      const int k0 = (s0 + i) * 64;
      const __half dh =
          reinterpret_cast<const __half*>(raw + rr * GM_RAW_BYTES + GM_RAW_Q + r * 16)[((k0 & 255) >> 5) + h];
      const float d = __half2float(dh);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty_raw[rr]);
      if (i >= AS && !mbar_wait(&empty_a[ia], ((i / AS) - 1) & 1, sc)) {
        *abort_flag = 1;
        break;
      }
      uint8_t* ahi = aring + ia * C::A_STAGE;
      uint8_t* alo = ahi + GM_A_BYTES;
      const uint32_t words[8] = {q0.x ^ 0x80808080u, q0.y ^ 0x80808080u, q0.z ^ 0x80808080u, q0.w ^ 0x80808080u,
                                 q1.x ^ 0x80808080u, q1.y ^ 0x80808080u, q1.z ^ 0x80808080u, q1.w ^ 0x80808080u};
#pragma unroll
      for (int j = 0; j < 4; j++) {  // chunk j: weights 8j..8j+7 of this block
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int p = 0; p < 4; p++) {
          // w = q * d exactly in f32; hi = w truncated to bf16, lo = (w - hi) rounded to bf16:
          // hi + lo = w to 2^-16 relative.
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
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full_a[ia]);
    }
    if (tw < 4) {  // epilogue: warp w reads TMEM lanes 32*(w%4)..
      const int q = warp & 3;
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
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(tmem, NT);
  }
}

// f32 rows -> activation tiles; one thread per 8 columns.
__global__ void gg_xtiles_kernel(const float* __restrict__ x, int T, int Tpad, int K, uint8_t* hi, uint8_t* lo) {
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

size_t gg_xtiles_bytes(int T, int K) { return (size_t)((T + 127) / 128 * 128) * (size_t)K * 2; }

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::mutex g_encode_mu;

static cudaError_t get_encode() {
  std::lock_guard<std::mutex> g(g_encode_mu);
  if (g_encode) return cudaSuccess;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t r = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q);
  if (r != cudaSuccess) return r;
  if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return cudaSuccess;
}

cudaError_t gg_make_q8_map(GGQ8Map* out, const uint8_t* base, int M, int K) {
  if (M % 128 || K % 64 || M <= 0 || K <= 0) return cudaErrorInvalidValue;
  cudaError_t r = get_encode();
  if (r != cudaSuccess) return r;
  const int rs = ((K + (K / 32) * 2) + 15) / 16 * 16;
  out->base = base;
  out->M = M;
  out->K = K;
  out->rs = rs;
  cuuint64_t gdim[2] = {(cuuint64_t)rs, (cuuint64_t)M};
  cuuint64_t gstride[1] = {(cuuint64_t)rs};
  cuuint32_t estr[2] = {1, 1};
  cuuint32_t boxq[2] = {64, 128};
  cuuint32_t boxs[2] = {16, 128};
  CUresult c = g_encode(&out->q, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), gdim, gstride, boxq, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (c != CUDA_SUCCESS) return cudaErrorInvalidValue;
  c = g_encode(&out->s, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t*>(base), gdim, gstride, boxs, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (c != CUDA_SUCCESS) return cudaErrorInvalidValue;
  return cudaSuccess;
}

cudaError_t gg_xtiles_from_f32(const float* x, int T, int K, uint8_t* xhi, uint8_t* xlo, cudaStream_t s) {
  if (T <= 0 || K % 64) return cudaErrorInvalidValue;
  const int Tpad = (T + 127) / 128 * 128;
  const long long n = (long long)Tpad * (K / 8);
  const int blocks = (int)((n + 255) / 256 < 148 * 8 ? (n + 255) / 256 : 148 * 8);
  gg_xtiles_kernel<<<blocks, 256, 0, s>>>(x, T, Tpad, K, xhi, xlo);
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
  gg_gemm_q8_kernel<NT><<<grid, GM_THREADS, GemmCfg<NT>::SMEM, s>>>(w.q, w.s, a);
  return cudaGetLastError();
}

cudaError_t gg_gemm_q8(const GGQ8Map& w, const uint8_t* xhi, const uint8_t* xlo, int T, float* y, long long ldy,
                       int splits, long long split_stride, uint32_t* err, uint64_t timeout_ns, cudaStream_t s) {
  if (T <= 0 || splits <= 0) return cudaErrorInvalidValue;
  GemmArgs a{};
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
  return T <= 64 ? launch_nt<64>(w, a, splits, s) : launch_nt<128>(w, a, splits, s);
}
