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

// A weight matrix as the GEMM reads it: a tiled copy of the device rows in which every
// 128-row x 64-column slab is one contiguous block of GG_Q8_TILE_BYTES (128 x 64 int8 quants,
// then the 128 x 2 f16 scales of its two Q8_0 blocks), blocks ordered (m_tile * K/64 + slab).
// One bulk copy then moves a whole slab.
#define GG_Q8_TILE_BYTES 8704
struct GGQ8Map {
  const uint8_t* tiles;
  int M, K;
  const uint8_t* dense = nullptr;  // optional: bf16 (hi, lo) operand tiles, 32 KB per slab
};

size_t gg_q8_tiles_bytes(int M, int K);

// Fill `tiles` (gg_q8_tiles_bytes(M, K) bytes) from a matrix in the device row format.
// M % 128 == 0 and K % 64 == 0 are required.
cudaError_t gg_make_q8_tiles(GGQ8Map* out, const uint8_t* rows, int M, int K, uint8_t* tiles, cudaStream_t s);

// Optional dequantised copy used for more than 64 activation rows (prompt chunks):
// gg_dense_tiles_bytes(M, K) bytes, built from the tiled Q8_0 copy.
size_t gg_dense_tiles_bytes(int M, int K);
cudaError_t gg_make_dense_tiles(GGQ8Map* w, uint8_t* dense, cudaStream_t s);

// Bytes of one activation tile array for T rows of width K (T rounded up to 256).
size_t gg_xtiles_bytes(int T, int K);

// x [T][K] f32 -> tile arrays (rows T..round256(T)-1 zero).
cudaError_t gg_xtiles_from_f32(const float* x, int T, int K, uint8_t* xhi, uint8_t* xlo, cudaStream_t s);

// One activation row: y[m] = row m of a Q8_0 matrix in the device row format (stride rs bytes)
// times x (K floats), f32 accumulation on the CUDA cores (the tensor-core tiles do not pay at
// batch 1). K % 64 == 0, K <= 16384.
cudaError_t gg_matvec_q8(const uint8_t* rows, int rs, int M, int K, const float* x, float* y, int sms,
                         cudaStream_t s);

// Kernel family behind gg_gemm_q8: GG_GEMM_DEQUANT (default) dequantises q * d in the kernel
// for up to 8 rows and reads the dequantised copy (when one was made) for more (three products
// per K step); GG_GEMM_SCALED converts the quants to bf16 and applies each Q8_0 block's scale
// after its MMAs (1.0625 B per weight read, two products per K step, one persistent CTA per SM).
#define GG_GEMM_DEQUANT 0
#define GG_GEMM_SCALED 1
void gg_gemm_set_path(int path);
int gg_gemm_path();

// Y (+ split * split_stride) [t][m] with row stride ldy; K is cut into `splits` slices whose
// partial results land in consecutive split planes (the caller sums them).
cudaError_t gg_gemm_q8(const GGQ8Map& w, const uint8_t* xhi, const uint8_t* xlo, int T, float* y, long long ldy,
                       int splits, long long split_stride, uint32_t* err, uint64_t timeout_ns, cudaStream_t s);

// The gate/up projection with GeGLU in the GEMM's epilogue: w's rows interleave gate (2j) and
// up (2j + 1); gelu(gate) * up for the T rows goes straight to activation tiles (ghi, glo) of
// K = M / 2 columns, which must not alias xhi / xlo. Only the dense single-split kernel has
// this epilogue: gg_gemm_geglu_fusable says whether gg_gemm_q8 with `splits` would take it.
bool gg_gemm_geglu_fusable(const GGQ8Map& w, int T, int splits);
cudaError_t gg_gemm_q8_geglu(const GGQ8Map& w, const uint8_t* xhi, const uint8_t* xlo, int T, uint8_t* ghi,
                             uint8_t* glo, uint32_t* err, uint64_t timeout_ns, cudaStream_t s);
