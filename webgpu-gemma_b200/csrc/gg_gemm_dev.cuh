// gg_gemm_dev.cuh -- device side of the activation tile format used by the Q8_0 GEMM.
//
// Activation rows are stored for the tensor core as bf16 (hi, lo) pairs in blocks of
// 64 rows x 64 columns (8 KB each, SW128 K-major, see gg_tc.cuh). Block (tb, s) holds rows
// 64*tb.. and columns 64*s..; blocks are ordered row-block major: ((tb * KS) + s) * 8192 bytes.
#pragma once
#include "gg_tc.cuh"

// Store columns k..k+7 (k % 8 == 0) of row t.
GG_DEV void xtile_put8(uint8_t* hi, uint8_t* lo, int KS, int t, int k, const float (&v)[8]) {
  const size_t blk = ((size_t)(t >> 6) * KS + (k >> 6)) * 8192u + sw128_offset(t & 63, k & 63);
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    __nv_bfloat16 h0, l0, h1, l1;
    split_bf16(v[2 * j], h0, l0);
    split_bf16(v[2 * j + 1], h1, l1);
    h[j] = pack_bf16x2(h0, h1);
    l[j] = pack_bf16x2(l0, l1);
  }
  *reinterpret_cast<uint4*>(hi + blk) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo + blk) = make_uint4(l[0], l[1], l[2], l[3]);
}
