/*
 * gemma_b200.h -- C-ABI of libgemma_b200.so, the B200 (sm_100a) Gemma 3 Q8_0 token loop.
 *
 * This library replaces the WebGPU half of the reference's engine (svenflow/webgpu-gemma,
 * src/engine.ts: GemmaEngineImpl, lines 124-949 and 1039-1077). The reference's public
 * TypeScript surface (createGemmaEngine, GemmaEngine.addUserMessage/generate/
 * resetConversation/dispose), its GGUF parser and its tokenizer stay on the host side and
 * call these functions with plain pointers and sizes.
 *
 * Every function returns 0 on success and a negative GG_E_* code on failure;
 * gg_last_error() returns the message of the engine's most recent failure.
 * One engine is bound to one GPU and one CUDA stream and is not re-entrant: calls on the
 * same engine must be serialised by the caller (the reference awaits each step too).
 */
#ifndef GEMMA_B200_H
#define GEMMA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GG_OK 0
#define GG_E_ARG -1      /* bad argument (null pointer, size, name, range) */
#define GG_E_CUDA -2     /* a CUDA runtime call failed */
#define GG_E_STATE -3    /* call out of order (e.g. step before gg_finalize) */
#define GG_E_DEVICE -4   /* a kernel reported an error (bounded wait expired, bad input) */
#define GG_E_NOMEM -5    /* device allocation failed */

typedef struct gg_engine gg_engine;

/* gg_config.flags: prefill one token per launch, as the reference does (engine.ts:923-928).
 * Without it gg_prefill runs the prompt in chunks of up to 512 tokens through tensor-core
 * GEMMs (same math, f32 results within rounding of the serial path). */
#define GG_FLAG_SERIAL_PREFILL 1
/* gg_config.flags: keep the KV cache in bf16 (round to nearest even at the store) instead of
 * the reference's f32 (engine.ts:440-447): half the cache memory and half the attention bytes.
 * Attention reads the stored (rounded) rows, the current position's included. */
#define GG_FLAG_KV_BF16 2

/* Field-for-field the reference's GemmaConfig (src/types.ts:2-17), plus the number of
 * independent KV slots and option flags. */
typedef struct {
  int32_t hidden_size, q_dim, kv_dim, num_q_heads, num_kv_heads, head_dim, intermediate_size,
      vocab_size, num_layers, context_length;
  float rms_norm_eps, rope_theta_global, rope_theta_swa;
  int32_t swa_period;
  int32_t max_seqs; /* KV slots (sequences); 1 for the reference's single conversation */
  int32_t flags;    /* GG_FLAG_* bits */
  /* 0: every layer attends the whole prefix, as the reference does. W > 0: the sliding-window
   * layers (isSwaLayer, types.ts:38-40) attend only positions pos-W+1..pos, as Gemma 3 is
   * specified (W = 512 for the 270M and 1B models). */
  int32_t sliding_window;
} gg_config;

/* Sampling options of one step: GenerateOptions (src/types.ts:65-78). Doubles, as the
 * reference's sampler computes in JS numbers (engine.ts:868-899): 0.7, 0.9 and 1.2 reach the
 * kernel without an f32 rounding. */
typedef struct {
  double temperature; /* 0 = greedy */
  double top_p;
  double rep_penalty; /* 1.0 = none */
} gg_sample;

/* Replaces initWebGPU + createWorkBuffers (engine.ts:124-138, 402-448): binds the engine
 * to CUDA device `device`, allocates the KV caches and work buffers. */
int gg_create(const gg_config* cfg, int device, gg_engine** out);

/* Replaces the per-tensor upload of uploadWeightsStreaming / uploadWeightsFromBuffer
 * (engine.ts:219-400, with packQ8_0ForGPU gguf.ts:126-149 moved to the device). `bytes`
 * are the tensor's raw GGUF bytes (Q8_0 34-byte blocks, F32 or F16); `dims` are GGUF
 * dims (ne0 first). The caller keeps ownership of `bytes`. */
int gg_upload_tensor(gg_engine* eng, const char* name, int ggml_type, const void* bytes, size_t nbytes,
                     const uint64_t* dims, int n_dims);

/* Checks that every tensor is present and builds the step program (createBindGroups,
 * engine.ts:450-732). */
int gg_finalize(gg_engine* eng);

/* Replaces prefillBatched (engine.ts:923-928): runs the n tokens through all layers at
 * positions start_pos..start_pos+n-1 of KV slot `seq`, writing the KV cache. The ids are
 * also added to the slot's repetition-penalty set (allTokens, engine.ts:989). */
int gg_prefill(gg_engine* eng, int seq, const int32_t* ids, int n, int start_pos);

/* Replaces getFirstTokenAfterPrefill (engine.ts:941-949): LM head on the last prefilled
 * token of `seq` plus sampling. `uniform` replaces Math.random() (ignored when greedy). */
int gg_sample_last(gg_engine* eng, int seq, const gg_sample* s, double uniform, int32_t* out_token);

/* Replaces forwardPassAndGetToken (engine.ts:904-915): feeds `token` at `pos`, runs the
 * LM head and the sampler, returns the next token. */
int gg_step(gg_engine* eng, int seq, int32_t token, int pos, const gg_sample* s, double uniform,
            int32_t* out_token);

/* n chained steps on the device (the token loop of engine.ts:1003-1025 without stop
 * checks): step i feeds the token sampled by step i-1. uniforms may be NULL when greedy.
 * out_tokens receives the n sampled tokens. */
int gg_decode(gg_engine* eng, int seq, int32_t token, int pos, int n, const gg_sample* s,
              const double* uniforms, int32_t* out_tokens);

/* Logits of the last LM-head run (vocab_size floats): the reference's logits buffer
 * (engine.ts:432), for parity checks and teacher forcing. */
int gg_get_logits(gg_engine* eng, float* out);

/* Final-normed hidden state of the last step (hidden_size floats), engine.ts:797-801. */
int gg_get_hidden(gg_engine* eng, float* out);

/* One row of the KV cache (kv_dim floats, widened from bf16 under GG_FLAG_KV_BF16;
 * which = 0 for K, 1 for V). */
int gg_get_kv(gg_engine* eng, int seq, int layer, int pos, int which, float* out);

/* Debug/parity aid: copy `n` floats of an internal buffer of the last launch.
 * which: 0 fused QKV output, 1 attention output, 2 O projection, 3 GeGLU output,
 * 4 down projection (layer outputs hold the last layer's values), 5 hidden state,
 * 6 residual, 7 final-normed hidden, 8 logits. */
int gg_debug_read(gg_engine* eng, int which, float* out, int n);

/* Parity aid for the weight upload (packQ8_0ForGPU + f16ToF32, gguf.ts:95-149): the n = K
 * values of row `row` of one Q8_0 matrix as the device holds it, dequantised as f32(q) *
 * f32(d) -- the exact products every kernel multiplies. which: 0 fused Q|K|V, 1 O, 2 gate/up
 * (gate_i at row 2i, up_i at 2i+1), 3 down, 4 token_embd / tied LM head (layer ignored).
 * copy: 0 the row format the decode kernel streams, 1 the tiled copy the tensor-core GEMM
 * reads (GG_E_STATE when the model's shapes give it none). */
int gg_dequant_row(gg_engine* eng, int which, int layer, int row, int copy, float* out, int n);

/* Repetition-penalty set of `seq` (allTokens, engine.ts:989-994): reset / add ids. */
int gg_seen_reset(gg_engine* eng, int seq);
int gg_seen_add(gg_engine* eng, int seq, const int32_t* ids, int n);

/* resetKVCaches (engine.ts:930-939) for one slot. */
int gg_reset_kv(gg_engine* eng, int seq);

/* Tracing: when on, every CTA of each launch stamps the device global timer (ns) at its phase
 * boundaries: out[(cta * 512 + phase) * 4 + event], phase = 6*layer + k (k: 0 QKV, 1 attention,
 * 2 split combine, 3 O projection, 4 gate/up, 5 down), phase 6*L = LM head; event 0 = enter,
 * 1 = inputs arrived, 2 = done. gg_read_trace copies the first n stamps. */
int gg_set_trace(gg_engine* eng, int on);
/* Number of CTAs of the persistent step kernel (at most one per SM; 128 on a B200). */
int gg_grid(gg_engine* eng, int* out);
int gg_read_trace(gg_engine* eng, uint64_t* out, int n);

/* forwardPassAndGetToken (engine.ts:904-915) for n independent conversations at once, `steps`
 * times in a row: row i is KV slot seqs[i] (distinct), fed tokens[i] at position pos[i]; each
 * step samples row i with sp[i] and draw uniforms[k * n + i] (k = step), appends the token to
 * the slot's repetition-penalty set, and feeds it at the next position. out_tokens[k * n + i]
 * receives the token of step k. All layers and the LM head run as tensor-core GEMMs over the n
 * rows. Requires 4 query heads sharing one KV head; 1 <= n <= min(max_seqs, 128). */
int gg_decode_batch(gg_engine* eng, int n, const int32_t* seqs, const int32_t* tokens, const int32_t* pos, int steps,
                    const gg_sample* sp, const double* uniforms, int32_t* out_tokens);

/* linearQ8 (shaders.ts:92-151, dispatched per matrix at engine.ts:769-793, 817-821) on `batch`
 * activation rows at once, on the tensor cores: y[b][m] = sum_k x[b][k] * W[m][k] for one of
 * the engine's Q8_0 matrices. which: 0 fused Q|K|V rows, 1 O, 2 gate/up (gate_i at row 2i,
 * up_i at 2i+1), 3 down, 4 the tied LM head (layer ignored). x is [batch][K] and y [batch][M],
 * host arrays; 1 <= batch <= 4096. gg_last_device_ms gives the device time of the product
 * (the GEMM and, when K was split, the sum of the split planes). */
int gg_linear(gg_engine* eng, int which, int layer, const float* x, int batch, float* y);

/* Kernel family of the tensor-core Q8_0 products (gg_linear, batched prefill, gg_decode_batch),
 * process-wide: 0 (default) dequantises q * d into bf16 hi + lo operands (in the kernel for up
 * to 8 rows, else from a dequantised copy made at load: 4 B per weight read); 1 converts the
 * quants to bf16 exactly and applies each 32-wide block's f16 scale after that block's MMAs
 * (1.0625 B per weight read, no use of the dequantised copy; slower on B200 today). Returns
 * the previous value; kind -1 only queries. No counterpart in the reference, which has one
 * linearQ8 shader (shaders.ts:92-151). */
int gg_set_gemm_kernel(int kind);

/* Failure-detection self-test: a one-CTA kernel waits on a device flag that nothing sets,
 * with the same bounded wait the step kernel uses. Returns GG_E_DEVICE ("activation wait
 * timed out") after about timeout_ns; the engine stays usable afterwards. No counterpart in
 * the reference (its WebGPU device-lost handler, engine.ts:134-137, has no bounded waits). */
int gg_selftest_wait(gg_engine* eng, uint64_t timeout_ns);

/* Bounded-wait limit of the device spins, in nanoseconds (default 1e9). */
int gg_set_timeout(gg_engine* eng, uint64_t ns);

/* Device time of the last gg_step / gg_decode / gg_prefill call, in milliseconds. */
int gg_last_device_ms(gg_engine* eng, float* ms);

/* dispose (engine.ts:1039-1077). */
int gg_destroy(gg_engine* eng);

/* Message of the engine's last failure ("" if none). eng = NULL gives the calling thread's last
 * failure of a call without an engine (gg_create, gg_sample_logits_noalloc); that message is
 * kept per thread and stays valid until the same thread's next such failure. */
const char* gg_last_error(const gg_engine* eng);

/* Sampling from logits the caller already holds on the GPU, with no memory allocation.
 * It has no counterpart in the reference: it is the step kernel's last stage -- the 256
 * per-lane maxima of the logits and the sampler, with the same rules and results as
 * gg_sample_last -- offered on its own to callers that cannot call cudaMalloc: code that
 * runs while another allocator (a framework's caching allocator, a fixed arena) owns the
 * device memory, and latency-bound loops where cudaMalloc/cudaFree would stall on a
 * device-wide synchronisation.
 *   logits      device pointer, vocab f32 values, on the calling thread's current device
 *   vocab       1 .. 524288; larger values are rejected with GG_E_ARG
 *   seen_bits   device pointer or NULL: bit (t % 32) of word t / 32 marks token t for the
 *               repetition penalty (tokens generated this turn); NULL = no tokens
 *   sp, uniform sampling parameters and the draw, as for gg_sample_last
 *   out_token   device pointer, receives the sampled token
 *   stream      a cudaStream_t of the current device (another device's stream is rejected
 *               with GG_E_ARG), or NULL for the default stream
 * Asynchronous: *out_token is written when the stream reaches the kernel. Its scratch is one
 * static 256 KiB device array (held by every GPU that loads this library until the process
 * exits). The first call on a device -- and the first in a new context on it, e.g. after
 * cudaDeviceReset -- looks up that array's device address, so make it before any stream
 * capture on that device. All calls on a device share the array: calls that can run at the
 * same time on the GPU (different streams, or threads without ordering) race and must be
 * serialised by the caller. Errors: GG_E_ARG / GG_E_CUDA, message from gg_last_error(NULL),
 * which is kept per calling thread. */
int gg_sample_logits_noalloc(const float* logits, int vocab, const uint32_t* seen_bits, const gg_sample* sp,
                             double uniform, int32_t* out_token, void* stream);

/* ---- Tokenizer (host only; no GPU involved). Replaces src/tokenizer.ts: the greedy
 * longest-match encoder the reference runs in JavaScript, with its UTF-16 code-unit semantics
 * (lengths, prefix search and the skip over unknown input count UTF-16 units). Strings cross
 * the boundary as UTF-8. */
typedef struct gg_tokenizer gg_tokenizer;

/* extractFromGGUF + buildTokenIndex + initFunctionTokens (tokenizer.ts:26-68): the vocabulary
 * as n UTF-8 strings (tokens[i], lens[i] bytes; the GGUF tokenizer.ggml.tokens array). The
 * caller keeps ownership of the strings. */
int gg_tokenizer_create(const char* const* tokens, const size_t* lens, int n, gg_tokenizer** out);

/* encode (tokenizer.ts:106-126): <bos> first, then the text split on the special-token names,
 * each piece greedily matched. *n_out receives the number of ids; at most cap are written. */
int gg_tokenizer_encode(const gg_tokenizer* tk, const char* text, size_t len, int32_t* ids, int cap, int* n_out);

/* decodeTokens (tokenizer.ts:128-141) as UTF-8: '\u2581' becomes a space, unknown ids
 * "<unk:ID>". *len_out receives the byte length; at most cap bytes are written (no NUL). */
int gg_tokenizer_decode(const gg_tokenizer* tk, const int32_t* ids, int n, char* text, size_t cap, size_t* len_out);

/* Id of a token text (tokenByText lookup, first id wins), or -1 (e.g. "<end_function_call>"
 * for the stop check of engine.ts:1014-1019). */
int gg_tokenizer_token_id(const gg_tokenizer* tk, const char* name, int32_t* id);

void gg_tokenizer_destroy(gg_tokenizer* tk);

/* Library build identifier (sm_100a kernels, compiled-in limits). */
const char* gg_version(void);

#ifdef __cplusplus
}
#endif
#endif /* GEMMA_B200_H */
