// gg_prefill.h -- launchers of the batched prefill kernels (gg_prefill.cu).
//
// A prompt chunk of T tokens runs layer by layer over all T rows at once: the four Q8_0
// matrices go through the tensor-core GEMM (gg_gemm.h) and these kernels do what lies between
// them. Split-K GEMM results arrive as `splits` planes of `plane` floats that the next kernel
// sums in plane order.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

// (cos, sin) table [ctx][HD/2] of pos * theta^(-2i/HD) (the RoPE rotation of shaders.ts:420-467).
cudaError_t gg_rope_table(float theta, int HD, int ctx, float2* out, cudaStream_t s);

// hidden[t] = dequantised embedding row ids[t] * sqrt(H) (shaders.ts:2-23).
cudaError_t pf_embed(const int32_t* ids, int T, const uint8_t* embd, int rs, int H, float* hidden, cudaStream_t s);

// resid_out[t] = resid_in[t] + rmsnorm(sum of planes)[t] * w_post   (fusedNormAdd, shaders.ts:386-418;
//                skipped when part == nullptr: resid_out = resid_in)
// tiles[t]     = rmsnorm(resid_out[t]) * w_norm                      (rmsNorm, shaders.ts:25-56;
//                skipped when w_norm == nullptr)
// resid_out may alias resid_in.
cudaError_t pf_addnorm(const float* part, int splits, long long plane, const float* w_post, const float* resid_in,
                       float* resid_out, const float* w_norm, uint8_t* thi, uint8_t* tlo, int T, int H, float eps,
                       cudaStream_t s);

// Per token: sum the QKV planes, q/k per-head rmsNorm + RoPE at position p0 + t
// (shaders.ts:420-467), q -> q_out as bf16 hi / lo halves ([T][NQH*HD] hi, then [T][NQH*HD] lo,
// the operand form pf_attention reads), k and v -> rows p0.. of this layer's cache (f32
// elements, or bf16 rounded to nearest even when kv16). With `split` (pf_attention's scratch
// for a cache of ctx rows) the new rows' bf16 hi / lo copies are written there too, so
// pf_attention with rows_split = true splits only the rows before p0.
cudaError_t pf_qk_rope_store(const float* part, int splits, long long plane, const float* q_norm,
                             const float* k_norm, const float2* rope, int T, int p0, int NQH, int NKH, int HD, float eps,
                             float* q_out, void* kc, void* vc, bool kv16, uint8_t* split, int ctx, cudaStream_t s);

// Causal attention of the T queries (q as written by pf_qk_rope_store) at positions
// p0..p0+T-1 over cache rows 0..p0+t
// (shaders.ts:229-325), output written as activation tiles of width NQH*HD. `part` is scratch
// of pf_attention_part_floats(T, p0 + T, NQH, NKH) floats (partial results per key range).
size_t pf_attention_part_floats(int max_tokens, int ctx, int NQH, int NKH);
// window > 0: each query at position p sees only keys p-window+1..p (sliding-window layer).
// `split` is scratch of pf_kv_split_bytes(ctx, NKH * HD) bytes: bf16 hi / lo copies of the rows
// the chunk attends to, made once per call and read by every attention CTA.
size_t pf_kv_split_bytes(int ctx, int KVD);
cudaError_t pf_attention(const float* q, const void* kc, const void* vc, bool kv16, int T, int p0, int NQH, int NKH,
                         int HD, float scale, int window, float* part, uint8_t* split, int ctx, bool rows_split,
                         uint8_t* thi, uint8_t* tlo, cudaStream_t s);

// act[t][i] = gelu_tanh(gu[t][2i]) * gu[t][2i+1] (shaders.ts:153-170, gu = sum of planes) as
// activation tiles of width I.
cudaError_t pf_geglu(const float* gu, int splits, long long plane, int T, int I, uint8_t* thi, uint8_t* tlo,
                     cudaStream_t s);

// ---- batched decode: row b is one token of the sequence in KV slot seqs[b] at position pos[b]

// Attention of each row's query over its slot's cache rows 0..pos[b] (4 query heads sharing one
// KV head), written as activation tiles, with the q/k step fused in: q is normed and rotated from
// the q/k/v GEMM's split planes (qkv, splits, plane), and the new k and v are stored at pos[b]
// (kc/vc: this layer's rows of slot 0). max_pos >= every pos[b]; `part` holds
// bd_attention_part_floats(B, ctx) floats.
size_t bd_attention_part_floats(int max_rows, int ctx);
cudaError_t bd_attention(const float* qkv, int splits, long long plane, const float* q_norm, const float* k_norm,
                         const float2* rope, float eps, void* kc, void* vc, bool kv16, int B, const int32_t* pos,
                         const int32_t* seqs, size_t seq_stride, int max_pos, int NQH, int NKH, int HD, float scale,
                         int window, float* part, uint8_t* thi, uint8_t* tlo, cudaStream_t s);
