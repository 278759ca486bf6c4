// gg_model.h -- descriptors shared by the host engine and the sm_100a kernels.
//
// Device weight layout ("row format"): a Q8_0 matrix with M rows of K inputs is stored as
// M rows of `row_stride(K)` bytes: K int8 quants, then K/32 f16 scales, then zero padding to
// a 16-byte multiple. A CTA's rows are contiguous, so one cp.async.bulk moves a whole stage.
// The reference's GPU layout is 36-byte {f32 scale, 8 x u32} blocks (src/gguf.ts:126-149);
// this layout keeps the GGUF's 34 bytes per 32 weights (f16 scale) and separates quants from
// scales so every lane reads 16 quant bytes with one 128-bit load.
#pragma once
#include <stdint.h>
#include <stddef.h>

#define GG_MAX_LAYERS 64
#define GG_HEAD_DIM 256                // Gemma 3 head size (compile-time for the attention phase)
#define GG_POS_PER_SPLIT 8             // KV positions per attention split
#define GG_TRACE_PHASES 512            // phases traced per CTA by GG_TRACE launches (4 stamps each)
#define GG_STEP_GRID 148               // step kernel: CTAs, one per SM of the B200 (a compile-time divisor: / and % by it become a multiply and shift)
#define GG_STEP_NCW 15                 // step kernel: consumer warps per CTA (+ one producer warp: 4 warps per SM sub-partition, 128 registers a thread)
#define GG_STEP_STAGES 9               // step kernel: weight ring stages
#define GG_STEP_STAGE_BYTES 20480      // step kernel: bytes per ring stage (16 rows of 1,152 Q8_0 weights)

static inline int gg_row_stride(int K) { return ((K + (K / 32) * 2) + 15) / 16 * 16; }

struct GGLayerW {
  const uint8_t* wqkv;   // Q+2KV rows (q rows, then k, then v), K = H
  const uint8_t* wo;     // H rows, K = Q
  const uint8_t* wgu;    // 2I rows, gate_i at row 2i and up_i at row 2i+1, K = H
  const uint8_t* wdown;  // H rows, K = I
  const float* attn_norm;
  const float* ffn_norm;
  const float* q_norm;
  const float* k_norm;
  const float* post_attn_norm;
  const float* post_ffw_norm;
  float theta;
  int window;  // 0: attend the whole prefix; W: only positions pos-W+1..pos (sliding-window layer)
  const float2* rope;  // [CTX][HD/2] (cos, sin) of pos * theta^(-2i/HD) for this layer's theta
  // The O projection by column slices for the step kernel: slice u (attention dims 8u..8u+7) is
  // H x 8 int8 quants (row r at 8r) then the H f16 scales of their Q8_0 block (row r at 8H + 2r),
  // H * 10 bytes per slice.
  const uint8_t* wo_cols;
};

// u64 words from one accumulator quad to the next: one 128-byte L2 line per quad.
#define GG_ACC_QUAD_WORDS 16

struct GGModelDev {
  int H, Q, KV, NQH, NKH, HD, I, V, L, CTX;
  float eps, attn_scale;
  int rs_h, rs_q, rs_i;  // row strides (bytes) for K = H, Q, I
  int grid;              // CTAs of the persistent kernel (one per SM)
  int stage_bytes, nstages;
  int pos_per_split, max_splits, ncomb, dims_per_comb;  // attention splits; merge units of 8 dims
  int xs0, xs1;     // x-plane buffer sizes (elements, multiples of 64): xs0 >= H, xs1 >= max(Q, I)
  int tmp_floats;   // attention scratch (q | k | v)
  int smem_bytes;
  const uint8_t* embd;   // V rows, K = H (tied LM head)
  const float* out_norm;
  uint8_t* kcache;  // [seq][L][CTX][KV] elements of kv_es bytes: f32, or bf16 (GG_FLAG_KV_BF16)
  uint8_t* vcache;
  size_t kv_seq_stride;  // elements per sequence
  // tagged activation exchange (value | tag << 32)
  // (each CTA's outputs of a phase in its own slot of sl_* words; see the step kernel)
  uint64_t* t_qkv;  // [grid][sl_qkv] q | k | v rows
  uint64_t* t_o;    // [max_splits][att_slot] attention split partials (o, max, sum per head)
  uint64_t* t_att;  // Q merged attention output (8 dims per merge unit, contiguous)
  uint64_t* t_act;  // [grid][sl_i] GeGLU outputs
  uint64_t* t_down; // [grid][sl_h] down projection rows
  float* logits;                    // V
  unsigned long long* lane_keys;    // 256 per-lane (value, index) maxima of the LM head
  float* dbg_hidden;    // H: hidden state after the last finished layer (CTA 0 writes)
  float* dbg_residual;  // H
  float* dbg_normed;    // H: final-normed hidden state (input of the LM head)
  uint8_t* seen;        // [max_seqs][ceil(V/8)] this turn's tokens (repetition penalty)
  int seen_stride;
  int32_t* seen_cnt;    // [max_seqs] tokens added to each slot's seen set since its last reset
  int max_seqs;
  unsigned long long* trace;  // [grid][GG_TRACE_PHASES][4] globaltimer stamps
  int kv_es;  // bytes per KV cache element: 4 (f32), or 2 (bf16)
  // Step kernel. Rows per ring stage for K = H, I, and for row pairs of K = H (even); words per
  // CTA slot of the exchange buffers (whole quads: the CTA's outputs start on a 32-byte sector)
  // of the Q+2KV, H and I (pair) outputs; words per attention split (NQH x (HD + 4): o, max, sum).
  int rps_h, rps_i, rps_gu;
  int sl_qkv, sl_h, sl_i;
  // ceil(2^40 / nq) for the quad counts of those outputs ((Q + 2KV) / 4, H / 4, I / 4): the owner
  // of quad q is ((q + 1) * G - 1) * mq >> 40 (exact while that product's factors stay below 2^40)
  unsigned long long mq_qkv, mq_h, mq_i;
  int att_slot;
  int lm_rows;  // most LM-head rows of one CTA (its logits are staged in shared memory)
  // Step kernel shared-memory layout: byte offsets from the dynamic shared-memory base (after the
  // ring and its mbarriers). The attention scratch (q | k | v) and the LM-head logits share the
  // O / down plane buffer when they fit: none of the three is live while another is.
  int sm_xa, sm_xb, sm_hid, sm_res, sm_tmp, sm_lmv, sm_scal, sm_red, sm_flag, sm_rows;
  // K-split reductions of the step kernel (the O projection: every merge unit adds its 8 columns'
  // products): per launch parity and layer, acc_stride u64 accumulators holding the sum of the
  // 2^-32 fixed-point partials shifted left by 8 plus, in the low byte, the number of
  // contributions (exact and order-independent; a reader waits for the full count). Each quad
  // of four rows sits alone in a 128-byte L2 line (GG_ACC_QUAD_WORDS words apart): all CTAs add
  // into every row, and the atomic updates of one line are applied one after another.
  unsigned long long* acc;  // [2][L][acc_stride]
  int acc_stride;           // (H / 4) * GG_ACC_QUAD_WORDS: row r at word (r / 4) * GG_ACC_QUAD_WORDS + r % 4
  int wo_rows_per_stage;    // most rows of a Wo column slice (10 bytes each) that one ring stage holds
  // The step kernel keeps a copy of this descriptor up to layers[L - 1] in shared memory at
  // sm_model (GG_MODEL_BYTES(L) bytes), so its parameter reads never wait on L2.
  int sm_model;
  GGLayerW layers[GG_MAX_LAYERS];  // last member: a copy of the first L entries is a valid prefix
};

#define GG_MODEL_BYTES(L) (offsetof(GGModelDev, layers) + (size_t)(L) * sizeof(GGLayerW))

// Launch-mode bits.
enum : int {
  GG_RUN_LAYERS = 1,  // embedding + all transformer layers for st->token at st->pos
  GG_RUN_LM = 2,      // final norm + LM head (+ per-lane maxima)
  GG_RUN_SAMPLE = 4,  // sampler on the lane maxima -> st->out_token
  GG_PREFILL_ADVANCE = 8,  // after the launch: token = ids[++i], pos += 1 (serial prefill)
  GG_TRACE = 16,           // every CTA stamps its phase boundaries into GGModelDev::trace
};

// Per-engine device state. The prefix up to `epoch` is written by the host at the start of a
// chain of launches; the device advances token/pos/prefill_ids/uniforms/step_index itself.
// Sampling parameters of one sequence (the C-ABI's gg_sample).
struct GGSampleDev {
  double temperature, top_p, rep_penalty;
};

struct GGState {
  int32_t token;   // token fed at `pos`
  int32_t pos;     // its position
  int32_t seq;     // KV slot
  int32_t mode;    // GG_RUN_* bits
  double temperature, top_p, rep_penalty;
  int32_t step_index;        // incremented per sampled token
  int32_t pad0_;
  double uniform;            // the draw replacing Math.random() when `uniforms` is null
  const double* uniforms;    // per-step draws, advanced by one per sampled token
  uint64_t timeout_ns;       // bounded-wait limit
  const int32_t* prefill_ids;  // serial prefill: ids still to feed
  int32_t prefill_left;
  int32_t ring_len;
  int32_t* token_ring;       // sampled tokens at [step_index % ring_len]
  // ---- owned by the device (and reset by dedicated host calls)
  uint32_t epoch;     // tag base; advanced by the last CTA of each launch
  uint32_t done;      // end-of-launch ticket
  uint32_t error;     // GG_ERR_* bits
  int32_t out_token;  // sampled token
  int32_t seen_count; // > 0 once this turn has tokens in the seen set
  uint32_t parity;    // accumulator set of the next launch (flipped by the last CTA of each)
  int32_t pad_[2];
};
