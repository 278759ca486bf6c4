// gg_gemm.h -- host-side interface of the Q8_0 tensor-core GEMM (gg_gemm.cu).
//
// Y[t][m] = sum_k X[t][k] * W[m][k] for a Q8_0 weight matrix W in the device row format
// (K int8 quants, K/32 f16 scales, padded to 16 bytes) and T activation rows X.
// X is passed as two bf16 tile arrays (hi, lo; hi + lo = x to ~2^-17) written by
// gg_xtiles_from_f32 or by a producer kernel through xtile_put8 (gg_gemm_dev.cuh).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct GGQ8Map {
  CUtensorMap q;  // quants: box 64 B x 128 rows
  CUtensorMap s;  // scales: box 16 B (8 f16) x 128 rows
  const uint8_t* base;
  int M, K, rs;
};

// Bytes of one activation tile array for T rows of width K (T rounded up to 128).
size_t gg_xtiles_bytes(int T, int K);

// Tensor maps for a weight matrix. Returns cudaSuccess or an error (M % 128, K % 64 required).
cudaError_t gg_make_q8_map(GGQ8Map* out, const uint8_t* base, int M, int K);

// x [T][K] f32 -> tile arrays (rows T..round128(T)-1 zero).
cudaError_t gg_xtiles_from_f32(const float* x, int T, int K, uint8_t* xhi, uint8_t* xlo, cudaStream_t s);

// Y (+ split * split_stride) [t][m] with row stride ldy; K is cut into `splits` slices whose
// partial results land in consecutive split planes (the caller sums them).
cudaError_t gg_gemm_q8(const GGQ8Map& w, const uint8_t* xhi, const uint8_t* xlo, int T, float* y, long long ldy,
                       int splits, long long split_stride, uint32_t* err, uint64_t timeout_ns, cudaStream_t s);
