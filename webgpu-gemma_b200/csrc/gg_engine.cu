// gg_engine.cu -- host engine behind the C-ABI of include/gemma_b200.h.
//
// Owns one GPU's copy of the model (repacked on the device from raw GGUF bytes), the KV
// caches, the tagged activation buffers and the step state; launches the persistent decode
// kernel (gg_decode.cu) cooperatively, one launch per token.
#include <cuda_runtime.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/gemma_b200.h"
#include "gg_device.cuh"
#include "gg_model.h"
#include "gg_gemm.h"
#include "gg_launch.h"
#include "gg_prefill.h"

namespace gg {
extern "C" __global__ void gg_step_kernel(const GGModelDev* __restrict__ mp, GGState* __restrict__ st, const GGState in,
                                          int use_in, GGState* host_st);
extern "C" __global__ void gg_step_kernel_kv16(const GGModelDev* __restrict__ mp, GGState* __restrict__ st,
                                               const GGState in, int use_in, GGState* host_st);
}

// The persistent step kernel built for the engine's KV element type.
using DecodeFn = void (*)(const GGModelDev*, GGState*, const GGState, int, GGState*);
static DecodeFn decode_fn(const GGModelDev& m) { return m.kv_es == 2 ? gg::gg_step_kernel_kv16 : gg::gg_step_kernel; }
constexpr int GG_STEP_THREADS = (GG_STEP_NCW + 1) * 32;

// ------------------------------------------------------------------------------ utility kernels

// Raw GGUF Q8_0 blocks (34 B: f16 d, 32 x int8) of an M x K tensor -> row format rows
// dst_row0 + r * dst_step. Replaces packQ8_0ForGPU (src/gguf.ts:126-149) on the device.
__global__ void gg_repack_q8_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, long long nblocks,
                                    int K, int rs, long long dst_row0, int dst_step) {
  long long b = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const int bpr = K / 32;
  long long r = b / bpr;
  int j = (int)(b % bpr);
  const uint8_t* s = src + b * 34;
  uint8_t* row = dst + (dst_row0 + r * dst_step) * (long long)rs;
  for (int k = 0; k < 32; k++) row[32 * j + k] = s[2 + k];
  row[K + 2 * j] = s[0];
  row[K + 2 * j + 1] = s[1];
}

// F16 -> F32 (dequantizeF16, src/gguf.ts:151-158). IEEE binary16 conversion is exact.
__global__ void gg_f16_to_f32_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst, long long n) {
  long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = __half2float(__ushort_as_half(src[i]));
}

// Wo (H rows of the row format, K = Q) -> Q / 8 column slices for the step kernel: slice u holds
// the 8 quants of columns 8u..8u+7 of every row (row r at 8r), then the f16 scales of their block
// (row r at 8H + 2r).
__global__ void gg_wo_cols_kernel(const uint8_t* __restrict__ wo, int H, int Q, int rs, uint8_t* __restrict__ out) {
  const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // u * H + r
  if (i >= (long long)(Q / 8) * H) return;
  const int u = (int)(i / H), r = (int)(i % H);
  const uint8_t* row = wo + (size_t)r * rs;
  uint8_t* slice = out + (size_t)u * H * 10;
  *reinterpret_cast<uint2*>(slice + 8 * (size_t)r) =
      make_uint2(*reinterpret_cast<const uint32_t*>(row + 8 * u), *reinterpret_cast<const uint32_t*>(row + 8 * u + 4));
  *reinterpret_cast<uint16_t*>(slice + 8 * (size_t)H + 2 * (size_t)r) = *reinterpret_cast<const uint16_t*>(row + Q + 2 * ((8 * u) / 32));
}

// Fixed-point accumulators ((2^-32 units << 8) + contribution count, two's complement u64) -> f32.
__global__ void gg_fixed_to_f32_kernel(const unsigned long long* __restrict__ src, float* __restrict__ dst, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n)  // row i's word (padded quads); the value bits sit above the 8-bit count
    dst[i] = (float)((long long)src[(i >> 2) * GG_ACC_QUAD_WORDS + (i & 3)] >> 8) * 0x1p-32f;
}

__global__ void gg_init_keys_kernel(unsigned long long* keys) {
  int i = threadIdx.x;
  if (i < 256) keys[i] = ((unsigned long long)f32_order_key(-1e30f) << 32) | 0xffffffffull;
}

__global__ void gg_seen_add_kernel(uint8_t* seen, const int32_t* ids, int n, int V, GGState* st, int32_t* slot_cnt) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    int t = ids[i];
    if (t >= 0 && t < V) atomicOr(reinterpret_cast<unsigned int*>(seen) + (t >> 5), 1u << (t & 31));
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    atomicAdd(&st->seen_count, n);
    atomicAdd(slot_cnt, n);
  }
}

// Self-test of the bounded waits: waits (with the decode kernel's tag_wait) for a tagged
// word that nothing writes, so the wait runs out and sets the error word.
__global__ void gg_wait_probe_kernel(const uint64_t* word, uint32_t* err, uint64_t timeout_ns) {
  SpinCtl sc{err, timeout_ns};
  if (threadIdx.x == 0) (void)tag_wait(word, 0x80000001u, sc);
}

// ------------------------------------------------------------------------------ engine

struct gg_engine {
  gg_config cfg{};
  int device = 0;
  int sm_count = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  GGModelDev md{};
  GGModelDev* d_md = nullptr;
  GGState* d_st = nullptr;
  GGState* h_st = nullptr;  // pinned
  std::vector<void*> allocs;
  // weights
  std::vector<uint8_t*> wqkv, wo, wgu, wdown;
  std::vector<uint8_t*> wo_cols;  // the step kernel's Wo column slices
  std::vector<float*> norms[6];  // attn_norm, ffn_norm, q_norm, k_norm, post_attn_norm, post_ffw_norm
  uint8_t* embd = nullptr;
  float* out_norm = nullptr;
  std::vector<uint32_t> have;  // per layer bitmask of uploaded tensors
  bool have_embd = false, have_out_norm = false;
  bool finalized = false;
  uint8_t* staging = nullptr;
  size_t staging_cap = 0;
  int32_t* d_ids = nullptr;
  int ids_cap = 0;
  double* d_unif = nullptr;
  int unif_cap = 0;
  int32_t* d_ring = nullptr;
  int ring_cap = 0;
  int32_t* h_ring = nullptr;  // pinned
  int last_hidden_seq = -1;
  int trace_on = 0;
  uint64_t timeout_ns = 1000000000ull;
  float last_ms = 0.f;
  std::string err;
  // tensor-core GEMM: tensor maps per weight matrix ([layer][0 qkv, 1 o, 2 gu, 3 down]), LM head
  std::vector<GGQ8Map> qmaps;
  GGQ8Map lm_map{};
  bool gemm_ok = false;
  float* lin_x = nullptr;
  uint8_t* lin_tiles = nullptr;
  float* lin_y = nullptr;
  size_t lin_x_cap = 0, lin_tiles_cap = 0, lin_y_cap = 0;
  // batched prefill buffers (one chunk of up to GG_PF_CHUNK prompt tokens)
  float* pf_hidden = nullptr;
  float* pf_res = nullptr;
  float* pf_q = nullptr;
  float* pf_y = nullptr;
  float* pf_att = nullptr;  // attention partials per key range
  uint8_t* pf_tiles = nullptr;
  size_t pf_tiles_half = 0;
  uint8_t* pf_gtiles = nullptr;  // GeGLU output tiles written by the gate/up GEMM's epilogue
  size_t pf_gtiles_half = 0;
  uint8_t* pf_kvsplit = nullptr;  // bf16 hi / lo copies of the K and V rows a chunk attends to
  // batched decode: one token for each of up to bd_max sequences per step
  int bd_max = 0;
  float* bd_logits = nullptr;            // [bd_max][V]
  float* bd_att = nullptr;               // attention partials
  unsigned long long* bd_keys = nullptr; // [bd_max][256] lane maxima
  int32_t* bd_seq = nullptr;
  int32_t* bd_tok = nullptr;
  int32_t* bd_pos = nullptr;
  GGSampleDev* bd_sp = nullptr;
  double* bd_unif = nullptr;
  int32_t* bd_out = nullptr;
  int32_t* bd_out_h = nullptr;  // pinned
  size_t bd_io_cap = 0;         // entries of bd_unif / bd_out / bd_out_h
};

constexpr int GG_BATCH_MAX = 128;  // sequences per batched step
static_assert(sizeof(GGSampleDev) == sizeof(gg_sample), "gg_sample layout");

constexpr int GG_PF_CHUNK = 512;  // prompt tokens per batched-prefill chunk

// Failures of calls that have no engine (gg_create, gg_sample_logits_noalloc) land here, one
// message per calling thread (as errno): threads that fail at the same time do not overwrite
// each other's message, and the pointer gg_last_error(NULL) returns stays valid until the same
// thread's next failure.
static thread_local std::string g_create_err;

void gg_set_engineless_error(const char* msg) { g_create_err = msg; }

static int fail(gg_engine* e, int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  if (e) e->err = buf;
  else g_create_err = buf;
  return code;
}

#define GG_CUDA(e, call)                                                                      \
  do {                                                                                        \
    cudaError_t _r = (call);                                                                  \
    if (_r != cudaSuccess) return fail((e), GG_E_CUDA, "%s: %s", #call, cudaGetErrorString(_r)); \
  } while (0)

template <class T>
static int dalloc(gg_engine* e, T** p, size_t bytes) {
  void* q = nullptr;
  cudaError_t r = cudaMalloc(&q, bytes ? bytes : 16);
  if (r != cudaSuccess) return fail(e, GG_E_NOMEM, "cudaMalloc(%zu): %s", bytes, cudaGetErrorString(r));
  // Stream-ordered zeroing: the engine's stream does not synchronise with the legacy stream.
  r = cudaMemsetAsync(q, 0, bytes ? bytes : 16, e->stream);
  if (r == cudaSuccess) r = cudaStreamSynchronize(e->stream);
  if (r != cudaSuccess) return fail(e, GG_E_CUDA, "cudaMemset: %s", cudaGetErrorString(r));
  e->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return GG_OK;
}
#define GG_TRY(x)          \
  do {                     \
    int _c = (x);          \
    if (_c != GG_OK) return _c; \
  } while (0)

enum { T_Q = 0, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN, T_ATTN_NORM, T_FFN_NORM, T_Q_NORM, T_K_NORM, T_POST_ATTN, T_POST_FFW, T_COUNT };
static const char* kLayerNames[T_COUNT] = {"attn_q",    "attn_k",   "attn_v",      "attn_output",  "ffn_gate",
                                           "ffn_up",    "ffn_down", "attn_norm",   "ffn_norm",     "attn_q_norm",
                                           "attn_k_norm", "post_attention_norm", "post_ffw_norm"};

extern "C" int gg_create(const gg_config* cfg, int device, gg_engine** out) {
  if (!cfg || !out) return fail(nullptr, GG_E_ARG, "null argument");
  *out = nullptr;
  const gg_config& c = *cfg;
  if (c.hidden_size <= 0 || c.hidden_size % 32 || c.num_layers <= 0 || c.num_layers > GG_MAX_LAYERS ||
      c.num_q_heads <= 0 || c.num_kv_heads <= 0 || c.num_q_heads % c.num_kv_heads || c.head_dim <= 0 ||
      c.head_dim % 32 || c.head_dim > 1024 || c.q_dim != c.num_q_heads * c.head_dim ||
      c.kv_dim != c.num_kv_heads * c.head_dim || c.intermediate_size <= 0 || c.intermediate_size % 32 ||
      c.vocab_size < 256 || c.context_length <= 0 || c.max_seqs <= 0 || c.q_dim % 32)
    return fail(nullptr, GG_E_ARG, "unsupported config (dims must be positive multiples of 32, q_dim = heads*head_dim)");
  if (c.swa_period < 1 || c.sliding_window < 0)
    return fail(nullptr, GG_E_ARG, "unsupported config (swa_period >= 1, sliding_window >= 0)");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev)
    return fail(nullptr, GG_E_CUDA, "no CUDA device %d", device);
  gg_engine* e = new gg_engine();
  e->cfg = c;
  e->device = device;
  auto bail = [&](int code) {
    g_create_err = e->err;
    gg_destroy(e);
    return code;
  };
  if (cudaSetDevice(device) != cudaSuccess) { fail(e, GG_E_CUDA, "cudaSetDevice"); return bail(GG_E_CUDA); }
  cudaDeviceProp prop;
  cudaGetDeviceProperties(&prop, device);
  if (prop.major < 10) { fail(e, GG_E_CUDA, "device %d is sm_%d%d; this library is built for sm_100a", device, prop.major, prop.minor); return bail(GG_E_CUDA); }
  e->sm_count = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreate(&e->ev0) != cudaSuccess || cudaEventCreate(&e->ev1) != cudaSuccess) {
    fail(e, GG_E_CUDA, "stream/event creation failed");
    return bail(GG_E_CUDA);
  }
  const int H = c.hidden_size, Q = c.q_dim, KV = c.kv_dim, I = c.intermediate_size, V = c.vocab_size, L = c.num_layers;
  GGModelDev& m = e->md;
  m.H = H; m.Q = Q; m.KV = KV; m.NQH = c.num_q_heads; m.NKH = c.num_kv_heads; m.HD = c.head_dim;
  m.I = I; m.V = V; m.L = L; m.CTX = c.context_length;
  m.eps = c.rms_norm_eps;
  m.attn_scale = (float)(1.0 / sqrt((double)c.head_dim));  // engine.ts:200
  m.rs_h = gg_row_stride(H); m.rs_q = gg_row_stride(Q); m.rs_i = gg_row_stride(I);
  m.max_seqs = c.max_seqs;
  int rc = GG_OK;
  e->wqkv.resize(L); e->wo.resize(L); e->wgu.resize(L); e->wdown.resize(L);
  for (auto& v : e->norms) v.resize(L);
  e->have.assign(L, 0u);
  for (int l = 0; l < L && rc == GG_OK; l++) {
    rc = dalloc(e, &e->wqkv[l], (size_t)(Q + 2 * KV) * m.rs_h);
    if (rc == GG_OK) rc = dalloc(e, &e->wo[l], (size_t)H * m.rs_q);
    if (rc == GG_OK) rc = dalloc(e, &e->wgu[l], (size_t)2 * I * m.rs_h);
    if (rc == GG_OK) rc = dalloc(e, &e->wdown[l], (size_t)H * m.rs_i);
    const int nlen[6] = {H, H, c.head_dim, c.head_dim, H, H};
    for (int k = 0; k < 6 && rc == GG_OK; k++) rc = dalloc(e, &e->norms[k][l], (size_t)nlen[k] * 4);
  }
  if (rc == GG_OK) rc = dalloc(e, &e->embd, (size_t)V * m.rs_h);
  if (rc == GG_OK) rc = dalloc(e, &e->out_norm, (size_t)H * 4);
  m.kv_seq_stride = (size_t)L * m.CTX * KV;
  m.kv_es = (c.flags & GG_FLAG_KV_BF16) ? 2 : 4;
  if (rc == GG_OK) rc = dalloc(e, &m.kcache, m.kv_seq_stride * m.kv_es * c.max_seqs);
  if (rc == GG_OK) rc = dalloc(e, &m.vcache, m.kv_seq_stride * m.kv_es * c.max_seqs);
  if (rc != GG_OK) return bail(rc);
  return (*out = e, GG_OK);
}

static int schedule(gg_engine* e) {
  GGModelDev& m = e->md;
  // One CTA per B200 SM: 148 CTAs split the 1B model's row sets into whole quads of near-equal
  // size (2-3 q/k/v quads, 1-2 quads of O and down rows, 11-12 quads of gate/up pairs, 442-443
  // quads of LM-head rows); 2.3 % faster per token than a power-of-two grid of 128.
  if (e->sm_count < GG_STEP_GRID)
    return fail(e, GG_E_ARG, "the step kernel needs %d SMs (device has %d)", GG_STEP_GRID, e->sm_count);
  m.grid = GG_STEP_GRID;
  const int G = m.grid;
  // the step kernel splits quads as c * nq / G in 32-bit arithmetic
  if ((long long)(G + 1) * (m.V / 4 + 1) >= (1ll << 31)) return fail(e, GG_E_ARG, "vocabulary too large for the step kernel's row split");
  if (m.HD != GG_HEAD_DIM) return fail(e, GG_E_ARG, "head_dim must be %d (Gemma 3)", GG_HEAD_DIM);
  if (m.H / 4 > 32 * GG_STEP_NCW) return fail(e, GG_E_ARG, "hidden_size above %d", 128 * GG_STEP_NCW);
  if (m.I / 4 > 4 * 32 * GG_STEP_NCW || m.Q / 4 > 4 * 32 * GG_STEP_NCW)
    return fail(e, GG_E_ARG, "intermediate_size and q_dim must be at most %d", 512 * GG_STEP_NCW);
  const int SB = GG_STEP_STAGE_BYTES;
  if (m.rs_i > SB || m.rs_q > SB || 2 * m.rs_h > SB) return fail(e, GG_E_ARG, "rows too wide for a %d-byte ring stage", SB);
  m.stage_bytes = SB;
  m.rps_h = SB / m.rs_h;
  m.rps_i = SB / m.rs_i;
  m.rps_gu = (SB / m.rs_h) & ~1;
  const auto slot = [&](int nq) { return 4 * ((nq + G - 1) / G); };
  m.sl_qkv = slot((m.Q + 2 * m.KV) / 4);
  m.sl_h = slot(m.H / 4);
  m.sl_i = slot(m.I / 4);
  const auto magic = [](int nq) { return ((1ull << 40) + (unsigned long long)nq - 1) / (unsigned long long)nq; };
  m.mq_qkv = magic((m.Q + 2 * m.KV) / 4);
  m.mq_h = magic(m.H / 4);
  m.mq_i = magic(m.I / 4);
  m.lm_rows = slot(m.V / 4);
  // the q/k/v, O and down rows of a CTA are computed one per consumer warp
  if (m.sl_qkv > GG_STEP_NCW || m.sl_h > GG_STEP_NCW)
    return fail(e, GG_E_ARG, "the step kernel needs at most %d q/k/v and hidden rows per CTA (grid %d)", GG_STEP_NCW, G);
  // rows of one phase per CTA: at most one per consumer warp and ring stage group (matvec)
  m.pos_per_split = GG_POS_PER_SPLIT;
  if (2 * GG_POS_PER_SPLIT * m.KV * 4 > SB) return fail(e, GG_E_ARG, "kv_dim too large for a ring stage");
  m.max_splits = (m.CTX + m.pos_per_split - 1) / m.pos_per_split;
  if ((m.max_splits + G - 1) / G > GG_STEP_NCW / m.NQH)
    return fail(e, GG_E_ARG, "context too long for the step kernel's %d attention splits per CTA", GG_STEP_NCW / m.NQH);
  m.att_slot = m.NQH * (m.HD + 4);
  // the small phases (q/k/v, O, down rows of a CTA) keep all their ring stages resident at once
  {
    const int rq = SB / m.rs_h, ro = SB / m.rs_q, rd = SB / m.rs_i;
    const int nst = std::max({(m.sl_qkv + std::min(rq, m.sl_qkv) - 1) / std::min(rq, m.sl_qkv),
                              (m.sl_h + std::min(ro, m.sl_h) - 1) / std::min(ro, m.sl_h),
                              (m.sl_h + std::min(rd, m.sl_h) - 1) / std::min(rd, m.sl_h)});
    const int nst_gu = (m.sl_i + m.rps_gu / 2 - 1) / (m.rps_gu / 2);  // gate/up stages (one waiting warp each)
    if (nst >= GG_STEP_STAGES || nst_gu >= GG_STEP_STAGES || nst_gu > GG_STEP_NCW)
      return fail(e, GG_E_ARG, "rows too wide: a phase needs %d ring stages at once", std::max(nst, nst_gu));
  }
  m.dims_per_comb = 8;
  m.ncomb = m.Q / 8;
  if (m.ncomb > G) return fail(e, GG_E_ARG, "q_dim / 8 = %d attention merge units exceed the grid (%d)", m.ncomb, G);
  // the merge units apply their 8 columns of Wo: H rows of 10 bytes in one ring stage
  m.wo_rows_per_stage = SB / 10;
  if (m.H > m.wo_rows_per_stage || m.H % 8)
    return fail(e, GG_E_ARG, "hidden_size must be a multiple of 8 and at most %d (one ring stage of O columns)", m.wo_rows_per_stage);
  m.acc_stride = (m.H + 3) / 4 * GG_ACC_QUAD_WORDS;
  m.xs0 = (m.H + 63) / 64 * 64;
  m.xs1 = (std::max(m.Q, m.I) + 63) / 64 * 64;
  m.tmp_floats = m.Q + 2 * m.KV;
  m.nstages = GG_STEP_STAGES;
  // keep in step with the carve at the top of step_body (gg_step.cu)
  // shared-memory layout of the step kernel (carved the same way at the top of step_body)
  {
    size_t off = (size_t)GG_STEP_STAGES * SB + 16 * (size_t)GG_STEP_STAGES;  // ring + full/empty mbarriers
    const auto take = [&](size_t bytes) {
      const size_t o = off;
      off = (off + bytes + 15) / 16 * 16;
      return (int)o;
    };
    const size_t xb_bytes = (size_t)3 * m.xs1 + m.xs1 / 4;
    m.sm_xa = take((size_t)3 * m.xs0 + m.xs0 / 4);
    m.sm_xb = take(xb_bytes);
    // q | k | v (attention) and the LM-head logits reuse the O / down planes when they fit
    m.sm_tmp = 4 * (size_t)m.tmp_floats <= xb_bytes ? m.sm_xb : take(4 * (size_t)m.tmp_floats);
    m.sm_lmv = 4 * (size_t)m.lm_rows <= xb_bytes ? m.sm_xb : take(4 * (size_t)m.lm_rows);
    m.sm_hid = take(4 * (size_t)m.H);
    m.sm_res = take(4 * (size_t)m.H);
    m.sm_scal = take(16 * 4 * GG_STEP_NCW);
    m.sm_red = take(4 * 16 * GG_STEP_NCW);
    m.sm_flag = take(16);
    m.sm_rows = take(32);
    m.sm_model = take(GG_MODEL_BYTES(m.L));
    m.smem_bytes = (int)off;
  }
  cudaFuncAttributes fa;
  GG_CUDA(e, cudaFuncGetAttributes(&fa, decode_fn(m)));
  int optin = 0;
  GG_CUDA(e, cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, e->device));
  if ((long)m.smem_bytes + (long)fa.sharedSizeBytes > (long)optin)
    return fail(e, GG_E_ARG, "step kernel needs %d + %d bytes of shared memory, the device offers %d", m.smem_bytes,
                (int)fa.sharedSizeBytes, optin);
  GG_CUDA(e, cudaFuncSetAttribute(decode_fn(m), cudaFuncAttributeMaxDynamicSharedMemorySize, m.smem_bytes));
  int nb = 0;
  GG_CUDA(e, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, decode_fn(m), GG_STEP_THREADS, m.smem_bytes));
  if (nb < 1) return fail(e, GG_E_CUDA, "step kernel cannot be resident (smem %d)", m.smem_bytes);
  return GG_OK;
}

extern "C" int gg_upload_tensor(gg_engine* e, const char* name, int type, const void* bytes, size_t nbytes,
                                const uint64_t* dims, int n_dims) {
  if (!e || !name || !bytes || !dims || n_dims < 1 || n_dims > 4) return fail(e, GG_E_ARG, "null or bad argument");
  if (e->finalized) return fail(e, GG_E_STATE, "gg_upload_tensor after gg_finalize");
  GG_CUDA(e, cudaSetDevice(e->device));
  const gg_config& c = e->cfg;
  const GGModelDev& m = e->md;
  uint64_t nel = 1;
  for (int i = 0; i < n_dims; i++) nel *= dims[i];
  const uint64_t ne0 = dims[0], ne1 = n_dims > 1 ? nel / dims[0] : 1;
  // classify
  int layer = -1, kind = -1;
  bool is_embd = !strcmp(name, "token_embd.weight"), is_out = !strcmp(name, "output_norm.weight");
  if (!is_embd && !is_out) {
    char key[64];
    int il = -1;
    if (sscanf(name, "blk.%d.%63[^.].weight", &il, key) != 2 || il < 0 || il >= c.num_layers)
      return fail(e, GG_E_ARG, "unknown tensor '%s'", name);
    for (int k = 0; k < T_COUNT; k++)
      if (!strcmp(key, kLayerNames[k])) kind = k;
    if (kind < 0) return fail(e, GG_E_ARG, "unknown tensor '%s'", name);
    layer = il;
  }
  const bool q8 = is_embd || (kind >= 0 && kind <= T_DOWN);
  if (q8) {
    if (type != 8) return fail(e, GG_E_ARG, "%s: expected Q8_0 (type 8), got %d", name, type);
    uint64_t expK, expM;
    uint8_t* dst;
    long long row0 = 0;
    int step = 1, rs;
    if (is_embd) { expK = c.hidden_size; expM = c.vocab_size; dst = e->embd; rs = m.rs_h; }
    else switch (kind) {
      case T_Q: expK = c.hidden_size; expM = c.q_dim; dst = e->wqkv[layer]; rs = m.rs_h; break;
      case T_K: expK = c.hidden_size; expM = c.kv_dim; dst = e->wqkv[layer]; rs = m.rs_h; row0 = c.q_dim; break;
      case T_V: expK = c.hidden_size; expM = c.kv_dim; dst = e->wqkv[layer]; rs = m.rs_h; row0 = c.q_dim + c.kv_dim; break;
      case T_O: expK = c.q_dim; expM = c.hidden_size; dst = e->wo[layer]; rs = m.rs_q; break;
      case T_GATE: expK = c.hidden_size; expM = c.intermediate_size; dst = e->wgu[layer]; rs = m.rs_h; step = 2; break;
      case T_UP: expK = c.hidden_size; expM = c.intermediate_size; dst = e->wgu[layer]; rs = m.rs_h; step = 2; row0 = 1; break;
      default: expK = c.intermediate_size; expM = c.hidden_size; dst = e->wdown[layer]; rs = m.rs_i; break;
    }
    if (ne0 != expK || ne1 != expM)
      return fail(e, GG_E_ARG, "%s: dims [%llu, %llu], expected [%llu, %llu]", name, (unsigned long long)ne0,
                  (unsigned long long)ne1, (unsigned long long)expK, (unsigned long long)expM);
    const size_t need = (size_t)(nel / 32) * 34;  // tensorByteSize (gguf.ts:181-187)
    if (nbytes != need) return fail(e, GG_E_ARG, "%s: %zu bytes, expected %zu", name, nbytes, need);
    if (e->staging_cap < need) {
      if (e->staging) cudaFree(e->staging);
      e->staging = nullptr;
      e->staging_cap = 0;
      GG_CUDA(e, cudaMalloc(&e->staging, need));
      e->staging_cap = need;
    }
    // A pageable cudaMemcpy may return before its DMA lands; order the copy on our stream.
    GG_CUDA(e, cudaMemcpyAsync(e->staging, bytes, need, cudaMemcpyHostToDevice, e->stream));
    long long nb = (long long)(nel / 32);
    gg_repack_q8_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, e->stream>>>(e->staging, dst, nb, (int)expK, rs, row0, step);
    GG_CUDA(e, cudaGetLastError());
    GG_CUDA(e, cudaStreamSynchronize(e->stream));
  } else {
    uint64_t expN = c.hidden_size;
    float* dst = nullptr;
    if (is_out) dst = e->out_norm;
    else {
      if (kind == T_Q_NORM || kind == T_K_NORM) expN = c.head_dim;
      dst = e->norms[kind - T_ATTN_NORM][layer];
    }
    if (nel != expN) return fail(e, GG_E_ARG, "%s: %llu elements, expected %llu", name, (unsigned long long)nel, (unsigned long long)expN);
    if (type == 0) {
      if (nbytes != nel * 4) return fail(e, GG_E_ARG, "%s: %zu bytes, expected %llu", name, nbytes, (unsigned long long)(nel * 4));
      GG_CUDA(e, cudaMemcpyAsync(dst, bytes, nel * 4, cudaMemcpyHostToDevice, e->stream));
      GG_CUDA(e, cudaStreamSynchronize(e->stream));
    } else if (type == 1) {
      if (nbytes != nel * 2) return fail(e, GG_E_ARG, "%s: %zu bytes, expected %llu", name, nbytes, (unsigned long long)(nel * 2));
      if (e->staging_cap < nbytes) {
        if (e->staging) cudaFree(e->staging);
        e->staging = nullptr;
        e->staging_cap = 0;
        GG_CUDA(e, cudaMalloc(&e->staging, nbytes));
        e->staging_cap = nbytes;
      }
      GG_CUDA(e, cudaMemcpyAsync(e->staging, bytes, nbytes, cudaMemcpyHostToDevice, e->stream));
      gg_f16_to_f32_kernel<<<(unsigned)((nel + 255) / 256), 256, 0, e->stream>>>((const uint16_t*)e->staging, dst, (long long)nel);
      GG_CUDA(e, cudaGetLastError());
      GG_CUDA(e, cudaStreamSynchronize(e->stream));
    } else {
      return fail(e, GG_E_ARG, "%s: unsupported type %d (F32 or F16 expected)", name, type);
    }
  }
  if (is_embd) e->have_embd = true;
  else if (is_out) e->have_out_norm = true;
  else e->have[layer] |= 1u << kind;
  return GG_OK;
}

extern "C" int gg_finalize(gg_engine* e) {
  if (!e) return fail(e, GG_E_ARG, "null engine");
  if (e->finalized) return GG_OK;
  GG_CUDA(e, cudaSetDevice(e->device));
  const gg_config& c = e->cfg;
  if (!e->have_embd) return fail(e, GG_E_STATE, "missing token_embd.weight");
  if (!e->have_out_norm) return fail(e, GG_E_STATE, "missing output_norm.weight");
  for (int l = 0; l < c.num_layers; l++)
    for (int k = 0; k < T_COUNT; k++)
      if (!(e->have[l] & (1u << k))) return fail(e, GG_E_STATE, "missing blk.%d.%s.weight", l, kLayerNames[k]);
  GGModelDev& m = e->md;
  GG_TRY(schedule(e));
  m.embd = e->embd;
  m.out_norm = e->out_norm;
  e->wo_cols.assign(c.num_layers, nullptr);
  for (int l = 0; l < c.num_layers; l++) {
    const long long n = (long long)(m.Q / 8) * m.H;
    GG_TRY(dalloc(e, &e->wo_cols[l], 10 * (size_t)n));
    gg_wo_cols_kernel<<<(unsigned)((n + 255) / 256), 256, 0, e->stream>>>(e->wo[l], m.H, m.Q, m.rs_q, e->wo_cols[l]);
    GG_CUDA(e, cudaGetLastError());
  }
  GG_TRY(dalloc(e, &m.acc, 8 * (size_t)2 * c.num_layers * m.acc_stride));
  GG_CUDA(e, cudaMemsetAsync(m.acc, 0, 8 * (size_t)2 * c.num_layers * m.acc_stride, e->stream));
  for (int l = 0; l < c.num_layers; l++) {
    GGLayerW& w = m.layers[l];
    w.wqkv = e->wqkv[l]; w.wo = e->wo[l]; w.wgu = e->wgu[l]; w.wdown = e->wdown[l];
    w.wo_cols = e->wo_cols[l];
    w.attn_norm = e->norms[0][l]; w.ffn_norm = e->norms[1][l]; w.q_norm = e->norms[2][l];
    w.k_norm = e->norms[3][l]; w.post_attn_norm = e->norms[4][l]; w.post_ffw_norm = e->norms[5][l];
    // getRopeTheta (types.ts:38-44)
    bool swa = (l % c.swa_period) < (c.swa_period - 1);
    w.theta = swa ? c.rope_theta_swa : c.rope_theta_global;
    w.window = (swa && c.sliding_window > 0) ? c.sliding_window : 0;
  }
  // RoPE tables, one per distinct theta
  {
    std::vector<std::pair<float, float2*>> tabs;
    for (int l = 0; l < c.num_layers; l++) {
      GGLayerW& w = m.layers[l];
      float2* tab = nullptr;
      for (auto& t : tabs)
        if (t.first == w.theta) tab = t.second;
      if (!tab) {
        GG_TRY(dalloc(e, &tab, sizeof(float2) * (size_t)m.CTX * (m.HD / 2)));
        GG_CUDA(e, gg_rope_table(w.theta, m.HD, m.CTX, tab, e->stream));
        tabs.push_back({w.theta, tab});
      }
      w.rope = tab;
    }
  }
  // Tiled weight copies for the batched (tensor-core) path; unusable shapes leave it off.
  e->gemm_ok = (m.H % 128 == 0) && (m.Q % 64 == 0) && ((m.Q + 2 * m.KV) % 128 == 0) && (m.I % 64 == 0) &&
               ((2 * m.I) % 128 == 0) && (m.V % 128 == 0) && (m.H % 64 == 0);
  e->qmaps.resize((size_t)c.num_layers * 4);
  for (int l = 0; l < c.num_layers && e->gemm_ok; l++) {
    const uint8_t* ptr[4] = {e->wqkv[l], e->wo[l], e->wgu[l], e->wdown[l]};
    const int M[4] = {m.Q + 2 * m.KV, m.H, 2 * m.I, m.H}, K[4] = {m.H, m.Q, m.H, m.I};
    for (int j = 0; j < 4; j++) {
      uint8_t* t = nullptr;
      GG_TRY(dalloc(e, &t, gg_q8_tiles_bytes(M[j], K[j])));
      GG_CUDA(e, gg_make_q8_tiles(&e->qmaps[(size_t)l * 4 + j], ptr[j], M[j], K[j], t, e->stream));
      uint8_t* dt = nullptr;  // dequantised copy for prompt chunks
      GG_TRY(dalloc(e, &dt, gg_dense_tiles_bytes(M[j], K[j])));
      GG_CUDA(e, gg_make_dense_tiles(&e->qmaps[(size_t)l * 4 + j], dt, e->stream));
    }
  }
  if (e->gemm_ok) {
    uint8_t* t = nullptr;
    GG_TRY(dalloc(e, &t, gg_q8_tiles_bytes(m.V, m.H)));
    GG_CUDA(e, gg_make_q8_tiles(&e->lm_map, e->embd, m.V, m.H, t, e->stream));
  }
  cudaGetLastError();
  if (e->gemm_ok) {
    const size_t TC = GG_PF_CHUNK;
    const int maxM = std::max(std::max(2 * m.I, m.Q + 2 * m.KV), m.H);
    const size_t yfl = std::max(TC * (size_t)maxM, (size_t)e->sm_count * 128 * 128);
    e->pf_tiles_half = gg_xtiles_bytes((int)TC, std::max(std::max(m.H, m.Q), m.I));
    GG_TRY(dalloc(e, &e->pf_hidden, 4 * TC * m.H));
    GG_TRY(dalloc(e, &e->pf_res, 4 * TC * m.H));
    GG_TRY(dalloc(e, &e->pf_q, 4 * TC * m.Q));
    GG_TRY(dalloc(e, &e->pf_y, 4 * yfl));
    GG_TRY(dalloc(e, &e->pf_att, 4 * pf_attention_part_floats((int)TC, m.CTX, m.NQH, m.NKH)));
    GG_TRY(dalloc(e, &e->pf_tiles, 2 * e->pf_tiles_half));
    e->pf_gtiles_half = gg_xtiles_bytes((int)TC, m.I);
    GG_TRY(dalloc(e, &e->pf_gtiles, 2 * e->pf_gtiles_half));
    GG_TRY(dalloc(e, &e->pf_kvsplit, pf_kv_split_bytes(m.CTX, m.KV)));
  }
  // exchange buffers of the step kernel (tagged words; one slot per CTA, or per attention split)
  GG_TRY(dalloc(e, &m.t_qkv, 8 * (size_t)m.grid * m.sl_qkv));
  GG_TRY(dalloc(e, &m.t_o, 8 * (size_t)m.max_splits * m.att_slot));
  GG_TRY(dalloc(e, &m.t_att, 8 * (size_t)m.Q));
  GG_TRY(dalloc(e, &m.t_act, 8 * (size_t)m.grid * m.sl_i));
  GG_TRY(dalloc(e, &m.t_down, 8 * (size_t)m.grid * m.sl_h));
  GG_TRY(dalloc(e, &m.logits, 4 * (size_t)m.V));
  GG_TRY(dalloc(e, &m.lane_keys, 8 * 256));
  GG_TRY(dalloc(e, &m.dbg_hidden, 4 * (size_t)m.H));
  GG_TRY(dalloc(e, &m.dbg_residual, 4 * (size_t)m.H));
  GG_TRY(dalloc(e, &m.dbg_normed, 4 * (size_t)m.H));
  m.seen_stride = ((m.V + 31) / 32) * 4;
  GG_TRY(dalloc(e, &m.seen, (size_t)m.seen_stride * c.max_seqs));
  GG_TRY(dalloc(e, &m.seen_cnt, sizeof(int32_t) * (size_t)c.max_seqs));
  GG_TRY(dalloc(e, &m.trace, 8 * (size_t)m.grid * GG_TRACE_PHASES * 4));
  GG_TRY(dalloc(e, &e->d_md, sizeof(GGModelDev)));
  GG_TRY(dalloc(e, &e->d_st, sizeof(GGState)));
  GG_CUDA(e, cudaHostAlloc(&e->h_st, sizeof(GGState), cudaHostAllocMapped));  // gg_step's kernel writes its tail here
  memset(e->h_st, 0, sizeof(GGState));
  GG_CUDA(e, cudaMemcpyAsync(e->d_md, &m, sizeof(GGModelDev), cudaMemcpyHostToDevice, e->stream));
  GGState s0{};
  s0.epoch = 1;
  s0.timeout_ns = e->timeout_ns;
  GG_CUDA(e, cudaMemcpyAsync(e->d_st, &s0, sizeof(GGState), cudaMemcpyHostToDevice, e->stream));
  gg_init_keys_kernel<<<1, 256, 0, e->stream>>>(m.lane_keys);
  GG_CUDA(e, cudaGetLastError());
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  if (e->staging) { cudaFree(e->staging); e->staging = nullptr; e->staging_cap = 0; }
  e->finalized = true;
  return GG_OK;
}

// ------------------------------------------------------------------------------ launches

static int ready(gg_engine* e, int seq) {
  if (!e) return fail(e, GG_E_ARG, "null engine");
  if (!e->finalized) return fail(e, GG_E_STATE, "engine not finalized");
  if (seq < 0 || seq >= e->cfg.max_seqs) return fail(e, GG_E_ARG, "seq %d out of range", seq);
  cudaError_t r = cudaSetDevice(e->device);
  if (r != cudaSuccess) return fail(e, GG_E_CUDA, "cudaSetDevice: %s", cudaGetErrorString(r));
  return GG_OK;
}

// Write the host-owned prefix of the state (everything before `epoch`).
static int put_inputs(gg_engine* e, const GGState& in) {
  *e->h_st = in;
  GG_CUDA(e, cudaMemcpyAsync(e->d_st, e->h_st, offsetof(GGState, epoch), cudaMemcpyHostToDevice, e->stream));
  return GG_OK;
}

// One token-kernel launch. in != nullptr: the host inputs travel as a launch parameter and the
// last CTA writes the device-owned tail into the mapped pinned state (no copies either way).
static int launch(gg_engine* e, const GGState* in = nullptr) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(e->md.grid);
  lc.blockDim = dim3(GG_STEP_THREADS);
  lc.dynamicSmemBytes = e->md.smem_bytes;
  lc.stream = e->stream;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  lc.attrs = at;
  lc.numAttrs = 1;
  const GGState in_v = in ? *in : GGState{};
  GG_CUDA(e, cudaLaunchKernelEx(&lc, decode_fn(e->md), (const GGModelDev*)e->d_md, e->d_st, in_v, in ? 1 : 0,
                                in ? e->h_st : (GGState*)nullptr));
  return GG_OK;
}

// Read back error/out_token, synchronise, and turn device error bits into a status.
static int finish_synced(gg_engine* e, int32_t* out_token);
static int finish(gg_engine* e, int32_t* out_token) {
  GG_CUDA(e, cudaMemcpyAsync(&e->h_st->epoch, &e->d_st->epoch, sizeof(GGState) - offsetof(GGState, epoch),
                             cudaMemcpyDeviceToHost, e->stream));
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  return finish_synced(e, out_token);
}
// After the stream has drained the launch and the state copy back: timing, error bits, token.
static int finish_synced(gg_engine* e, int32_t* out_token) {
  if (cudaEventElapsedTime(&e->last_ms, e->ev0, e->ev1) != cudaSuccess) {
    e->last_ms = 0.f;
    cudaGetLastError();  // no pending error left for a later call to pick up
  }
  uint32_t err = e->h_st->error;
  if (err) {
    cudaMemsetAsync(&e->d_st->error, 0, 4, e->stream);
    cudaStreamSynchronize(e->stream);
    return fail(e, GG_E_DEVICE, "device reported error 0x%x (%s%s%s)", err, (err & GG_ERR_WAIT_FLAG) ? "activation wait timed out " : "",
                (err & GG_ERR_WAIT_MBAR) ? "ring wait timed out " : "", (err & GG_ERR_BAD_INPUT) ? "token/pos/seq out of range" : "");
  }
  if (out_token) *out_token = e->h_st->out_token;
  return GG_OK;
}

static GGState base_inputs(gg_engine* e, int seq, int mode) {
  GGState s{};
  s.seq = seq;
  s.mode = mode;
  s.timeout_ns = e->timeout_ns;
  s.rep_penalty = 1.0;
  if (e->trace_on) s.mode |= GG_TRACE;
  return s;
}

static void set_sampling(GGState& s, const gg_sample* sp, double u) {
  if (sp) {
    s.temperature = sp->temperature;
    s.top_p = sp->top_p;
    s.rep_penalty = sp->rep_penalty;
  }
  s.uniform = u;
}

static int pick_splits(int tiles, int KS, int slots);

static int gemm_tiles(int T, int M) { return (T <= 64 ? 1 : (T + 127) / 128) * (M / 128); }
// CTA slots of the GEMM that gg_gemm_q8 picks for T rows: the block-scaled kernel runs one CTA
// per SM; of the dequantising kernels the Q8 one (T <= 8, or no dense copy) fits two.
static int gemm_slots(const gg_engine* e, int T) {
  if (gg_gemm_path() == GG_GEMM_SCALED) return e->sm_count;
  return e->sm_count * (T <= 8 || !e->gemm_ok ? 2 : 1);
}

// Batched prefill of ids already in e->d_ids: chunks of up to GG_PF_CHUNK tokens, each layer
// as four tensor-core GEMMs over the chunk's rows and the kernels of gg_prefill.cu between them.
static int prefill_batched(gg_engine* e, int seq, int n, int start_pos) {
  const GGModelDev& m = e->md;
  cudaStream_t s = e->stream;
  uint8_t* thi = e->pf_tiles;
  uint8_t* tlo = e->pf_tiles + e->pf_tiles_half;
  uint8_t* ghi = e->pf_gtiles;
  uint8_t* glo = e->pf_gtiles + e->pf_gtiles_half;
  uint32_t* err = &e->d_st->error;
  const uint64_t to = e->timeout_ns;
  const int QKV = m.Q + 2 * m.KV;
  int T = 0;
  for (int c0 = 0; c0 < n; c0 += GG_PF_CHUNK) {
    T = std::min(GG_PF_CHUNK, n - c0);
    const int p0 = start_pos + c0;
    GG_CUDA(e, pf_embed(e->d_ids + c0, T, m.embd, m.rs_h, m.H, e->pf_hidden, s));
    GG_CUDA(e, pf_addnorm(nullptr, 0, 0, nullptr, e->pf_hidden, e->pf_hidden, m.layers[0].attn_norm, thi, tlo, T, m.H,
                          m.eps, s));
    for (int l = 0; l < m.L; l++) {
      const GGLayerW& w = m.layers[l];
      const GGQ8Map* mp = &e->qmaps[(size_t)l * 4];
      const size_t kvo = ((size_t)seq * m.kv_seq_stride + (size_t)l * m.CTX * m.KV) * m.kv_es;
      uint8_t* kc = m.kcache + kvo;
      uint8_t* vc = m.vcache + kvo;
      int sp = pick_splits(gemm_tiles(T, QKV), m.H / 64, gemm_slots(e, T));
      long long plane = (long long)T * QKV;
      GG_CUDA(e, gg_gemm_q8(mp[0], thi, tlo, T, e->pf_y, QKV, sp, plane, err, to, s));
      GG_CUDA(e, pf_qk_rope_store(e->pf_y, sp, plane, w.q_norm, w.k_norm, w.rope, T, p0, m.NQH, m.NKH, m.HD, m.eps,
                                  e->pf_q, kc, vc, m.kv_es == 2, e->pf_kvsplit, m.CTX, s));
      GG_CUDA(e, pf_attention(e->pf_q, kc, vc, m.kv_es == 2, T, p0, m.NQH, m.NKH, m.HD, m.attn_scale, w.window,
                              e->pf_att, e->pf_kvsplit, m.CTX, true, thi, tlo, s));
      sp = pick_splits(gemm_tiles(T, m.H), m.Q / 64, gemm_slots(e, T));
      plane = (long long)T * m.H;
      GG_CUDA(e, gg_gemm_q8(mp[1], thi, tlo, T, e->pf_y, m.H, sp, plane, err, to, s));
      GG_CUDA(e, pf_addnorm(e->pf_y, sp, plane, w.post_attn_norm, e->pf_hidden, e->pf_res, w.ffn_norm, thi, tlo, T,
                            m.H, m.eps, s));
      sp = pick_splits(gemm_tiles(T, 2 * m.I), m.H / 64, gemm_slots(e, T));
      const bool fuse = gg_gemm_geglu_fusable(mp[2], T, sp);
      if (fuse) {
        GG_CUDA(e, gg_gemm_q8_geglu(mp[2], thi, tlo, T, ghi, glo, err, to, s));
      } else {
        plane = (long long)T * 2 * m.I;
        GG_CUDA(e, gg_gemm_q8(mp[2], thi, tlo, T, e->pf_y, 2 * m.I, sp, plane, err, to, s));
        GG_CUDA(e, pf_geglu(e->pf_y, sp, plane, T, m.I, thi, tlo, s));
      }
      sp = pick_splits(gemm_tiles(T, m.H), m.I / 64, gemm_slots(e, T));
      plane = (long long)T * m.H;
      GG_CUDA(e, gg_gemm_q8(mp[3], fuse ? ghi : thi, fuse ? glo : tlo, T, e->pf_y, m.H, sp, plane, err, to, s));
      const float* next_norm = l + 1 < m.L ? m.layers[l + 1].attn_norm : nullptr;
      GG_CUDA(e, pf_addnorm(e->pf_y, sp, plane, w.post_ffw_norm, e->pf_res, e->pf_hidden, next_norm, thi, tlo, T, m.H,
                            m.eps, s));
    }
  }
  // the LM-head launch of gg_sample_last reads the last token's hidden state from here
  GG_CUDA(e, cudaMemcpyAsync(m.dbg_hidden, e->pf_hidden + (size_t)(T - 1) * m.H, 4 * (size_t)m.H,
                             cudaMemcpyDeviceToDevice, s));
  return GG_OK;
}

cudaError_t gg_batch_sample(const float* logits, int B, int V, const int32_t* seqs, const GGSampleDev* sp,
                            const double* unif, uint8_t* seen, int seen_stride, int32_t* seen_cnt,
                            unsigned long long* keys, int32_t* tokens, int32_t* pos, int32_t* out, cudaStream_t s);

// One batched decode step for the B sequences in bd_seq / bd_tok / bd_pos (device arrays):
// all layers on the tensor-core path, LM head as a GEMM, one sampler CTA per row. Leaves the
// sampled tokens in d_out and in bd_tok, and advances bd_pos.
static int batch_step(gg_engine* e, int B, int max_pos, const double* d_unif, int32_t* d_out) {
  const GGModelDev& m = e->md;
  cudaStream_t s = e->stream;
  uint8_t* thi = e->pf_tiles;
  uint8_t* tlo = e->pf_tiles + e->pf_tiles_half;
  uint8_t* ghi = e->pf_gtiles;
  uint8_t* glo = e->pf_gtiles + e->pf_gtiles_half;
  uint32_t* err = &e->d_st->error;
  const uint64_t to = e->timeout_ns;
  const int QKV = m.Q + 2 * m.KV;
  GG_CUDA(e, pf_embed(e->bd_tok, B, m.embd, m.rs_h, m.H, e->pf_hidden, s));
  GG_CUDA(e, pf_addnorm(nullptr, 0, 0, nullptr, e->pf_hidden, e->pf_hidden, m.layers[0].attn_norm, thi, tlo, B, m.H,
                        m.eps, s));
  for (int l = 0; l < m.L; l++) {
    const GGLayerW& w = m.layers[l];
    const GGQ8Map* mp = &e->qmaps[(size_t)l * 4];
    uint8_t* kc = m.kcache + (size_t)l * m.CTX * m.KV * m.kv_es;
    uint8_t* vc = m.vcache + (size_t)l * m.CTX * m.KV * m.kv_es;
    int sp = pick_splits(gemm_tiles(B, QKV), m.H / 64, gemm_slots(e, B));
    long long plane = (long long)B * QKV;
    GG_CUDA(e, gg_gemm_q8(mp[0], thi, tlo, B, e->pf_y, QKV, sp, plane, err, to, s));
    GG_CUDA(e, bd_attention(e->pf_y, sp, plane, w.q_norm, w.k_norm, w.rope, m.eps, kc, vc, m.kv_es == 2, B, e->bd_pos,
                            e->bd_seq, m.kv_seq_stride, max_pos, m.NQH, m.NKH, m.HD,
                            m.attn_scale, w.window, e->bd_att, thi, tlo, s));
    sp = pick_splits(gemm_tiles(B, m.H), m.Q / 64, gemm_slots(e, B));
    plane = (long long)B * m.H;
    GG_CUDA(e, gg_gemm_q8(mp[1], thi, tlo, B, e->pf_y, m.H, sp, plane, err, to, s));
    GG_CUDA(e, pf_addnorm(e->pf_y, sp, plane, w.post_attn_norm, e->pf_hidden, e->pf_res, w.ffn_norm, thi, tlo, B, m.H,
                          m.eps, s));
    sp = pick_splits(gemm_tiles(B, 2 * m.I), m.H / 64, gemm_slots(e, B));
    const bool fuse = gg_gemm_geglu_fusable(mp[2], B, sp);
    if (fuse) {
      GG_CUDA(e, gg_gemm_q8_geglu(mp[2], thi, tlo, B, ghi, glo, err, to, s));
    } else {
      plane = (long long)B * 2 * m.I;
      GG_CUDA(e, gg_gemm_q8(mp[2], thi, tlo, B, e->pf_y, 2 * m.I, sp, plane, err, to, s));
      GG_CUDA(e, pf_geglu(e->pf_y, sp, plane, B, m.I, thi, tlo, s));
    }
    sp = pick_splits(gemm_tiles(B, m.H), m.I / 64, gemm_slots(e, B));
    plane = (long long)B * m.H;
    GG_CUDA(e, gg_gemm_q8(mp[3], fuse ? ghi : thi, fuse ? glo : tlo, B, e->pf_y, m.H, sp, plane, err, to, s));
    // the last layer's output goes through the final norm (output_norm) into the LM-head tiles
    const float* next_norm = l + 1 < m.L ? m.layers[l + 1].attn_norm : m.out_norm;
    GG_CUDA(e, pf_addnorm(e->pf_y, sp, plane, w.post_ffw_norm, e->pf_res, e->pf_hidden, next_norm, thi, tlo, B, m.H,
                          m.eps, s));
  }
  GG_CUDA(e, gg_gemm_q8(e->lm_map, thi, tlo, B, e->bd_logits, m.V, 1, 0, err, to, s));
  GG_CUDA(e, gg_batch_sample(e->bd_logits, B, m.V, e->bd_seq, e->bd_sp, d_unif, m.seen, m.seen_stride, m.seen_cnt,
                             e->bd_keys, e->bd_tok, e->bd_pos, d_out, s));
  return GG_OK;
}

extern "C" int gg_decode_batch(gg_engine* e, int n, const int32_t* seqs, const int32_t* tokens, const int32_t* pos,
                               int steps, const gg_sample* sp, const double* uniforms, int32_t* out_tokens) {
  GG_TRY(ready(e, 0));
  const gg_config& c = e->cfg;
  const GGModelDev& m = e->md;
  if (!e->gemm_ok || m.NQH != 4 || m.NKH != 1)
    return fail(e, GG_E_STATE, "batched decode needs the tensor-core path and 4 query heads sharing 1 KV head");
  if (n < 1 || n > std::min(c.max_seqs, GG_BATCH_MAX)) return fail(e, GG_E_ARG, "batch of %d sequences (1..%d)", n, std::min(c.max_seqs, GG_BATCH_MAX));
  if (steps < 1 || !seqs || !tokens || !pos || !sp || !uniforms || !out_tokens) return fail(e, GG_E_ARG, "bad arguments");
  int max_pos = 0;
  std::vector<char> used(c.max_seqs, 0);
  for (int i = 0; i < n; i++) {
    if (seqs[i] < 0 || seqs[i] >= c.max_seqs) return fail(e, GG_E_ARG, "seq %d out of range", seqs[i]);
    if (used[seqs[i]]++) return fail(e, GG_E_ARG, "seq %d appears twice in one batch", seqs[i]);
    if (tokens[i] < 0 || tokens[i] >= c.vocab_size) return fail(e, GG_E_ARG, "token %d out of range", tokens[i]);
    if (pos[i] < 0 || pos[i] + steps > c.context_length)
      return fail(e, GG_E_ARG, "positions %d..%d exceed context %d", pos[i], pos[i] + steps - 1, c.context_length);
    max_pos = std::max(max_pos, pos[i]);
  }
  if (e->bd_max == 0) {  // first batched call: buffers for up to bd_max rows
    const int bm = std::min(c.max_seqs, GG_BATCH_MAX);
    GG_TRY(dalloc(e, &e->bd_logits, sizeof(float) * (size_t)bm * m.V));
    GG_TRY(dalloc(e, &e->bd_att, sizeof(float) * bd_attention_part_floats(bm, m.CTX)));
    GG_TRY(dalloc(e, &e->bd_keys, 8 * (size_t)bm * 256));
    GG_TRY(dalloc(e, &e->bd_seq, 4 * (size_t)bm));
    GG_TRY(dalloc(e, &e->bd_tok, 4 * (size_t)bm));
    GG_TRY(dalloc(e, &e->bd_pos, 4 * (size_t)bm));
    GG_TRY(dalloc(e, &e->bd_sp, sizeof(GGSampleDev) * (size_t)bm));
    e->bd_max = bm;
  }
  const size_t io = (size_t)steps * n;
  if (e->bd_io_cap < io) {
    if (e->bd_unif) cudaFree(e->bd_unif);
    if (e->bd_out) cudaFree(e->bd_out);
    if (e->bd_out_h) cudaFreeHost(e->bd_out_h);
    e->bd_unif = nullptr;
    e->bd_out = nullptr;
    e->bd_out_h = nullptr;
    e->bd_io_cap = 0;
    GG_CUDA(e, cudaMalloc(&e->bd_unif, sizeof(double) * io));
    GG_CUDA(e, cudaMalloc(&e->bd_out, sizeof(int32_t) * io));
    GG_CUDA(e, cudaMallocHost(&e->bd_out_h, sizeof(int32_t) * io));
    e->bd_io_cap = io;
  }
  cudaStream_t s = e->stream;
  GG_CUDA(e, cudaMemcpyAsync(e->bd_seq, seqs, 4 * (size_t)n, cudaMemcpyHostToDevice, s));
  GG_CUDA(e, cudaMemcpyAsync(e->bd_tok, tokens, 4 * (size_t)n, cudaMemcpyHostToDevice, s));
  GG_CUDA(e, cudaMemcpyAsync(e->bd_pos, pos, 4 * (size_t)n, cudaMemcpyHostToDevice, s));
  GG_CUDA(e, cudaMemcpyAsync(e->bd_sp, sp, sizeof(GGSampleDev) * (size_t)n, cudaMemcpyHostToDevice, s));
  GG_CUDA(e, cudaMemcpyAsync(e->bd_unif, uniforms, sizeof(double) * io, cudaMemcpyHostToDevice, s));
  GG_CUDA(e, cudaEventRecord(e->ev0, s));
  for (int k = 0; k < steps; k++) GG_TRY(batch_step(e, n, max_pos + k, e->bd_unif + (size_t)k * n, e->bd_out + (size_t)k * n));
  GG_CUDA(e, cudaEventRecord(e->ev1, s));
  GG_CUDA(e, cudaMemcpyAsync(e->bd_out_h, e->bd_out, sizeof(int32_t) * io, cudaMemcpyDeviceToHost, s));
  GG_TRY(finish(e, nullptr));
  memcpy(out_tokens, e->bd_out_h, sizeof(int32_t) * io);
  return GG_OK;
}

extern "C" int gg_prefill(gg_engine* e, int seq, const int32_t* ids, int n, int start_pos) {
  GG_TRY(ready(e, seq));
  if (n <= 0 || !ids) return fail(e, GG_E_ARG, "empty prefill");
  if (start_pos < 0 || start_pos + n > e->cfg.context_length)
    return fail(e, GG_E_ARG, "positions %d..%d exceed context %d", start_pos, start_pos + n - 1, e->cfg.context_length);
  for (int i = 0; i < n; i++)
    if (ids[i] < 0 || ids[i] >= e->cfg.vocab_size) return fail(e, GG_E_ARG, "token id %d out of range", ids[i]);
  if (e->ids_cap < n) {
    if (e->d_ids) cudaFree(e->d_ids);
    e->d_ids = nullptr;
    e->ids_cap = 0;
    GG_CUDA(e, cudaMalloc(&e->d_ids, sizeof(int32_t) * n));
    e->ids_cap = n;
  }
  GG_CUDA(e, cudaMemcpyAsync(e->d_ids, ids, sizeof(int32_t) * n, cudaMemcpyHostToDevice, e->stream));
  gg_seen_add_kernel<<<(n + 255) / 256, 256, 0, e->stream>>>(e->md.seen + (size_t)seq * e->md.seen_stride, e->d_ids, n,
                                                             e->cfg.vocab_size, e->d_st, e->md.seen_cnt + seq);
  GG_CUDA(e, cudaGetLastError());
  if (e->gemm_ok && !(e->cfg.flags & GG_FLAG_SERIAL_PREFILL)) {
    GG_CUDA(e, cudaEventRecord(e->ev0, e->stream));
    GG_TRY(prefill_batched(e, seq, n, start_pos));
    GG_CUDA(e, cudaEventRecord(e->ev1, e->stream));
    GG_TRY(finish(e, nullptr));
    e->last_hidden_seq = seq;
    return GG_OK;
  }
  GGState s = base_inputs(e, seq, GG_RUN_LAYERS | GG_PREFILL_ADVANCE);
  s.token = ids[0];
  s.pos = start_pos;
  s.prefill_ids = e->d_ids + 1;
  s.prefill_left = n - 1;
  GG_TRY(put_inputs(e, s));
  GG_CUDA(e, cudaEventRecord(e->ev0, e->stream));
  for (int i = 0; i < n; i++) GG_TRY(launch(e));
  GG_CUDA(e, cudaEventRecord(e->ev1, e->stream));
  GG_TRY(finish(e, nullptr));
  e->last_hidden_seq = seq;
  return GG_OK;
}

extern "C" int gg_sample_last(gg_engine* e, int seq, const gg_sample* sp, double uniform, int32_t* out_token) {
  GG_TRY(ready(e, seq));
  if (!out_token) return fail(e, GG_E_ARG, "null out_token");
  if (e->last_hidden_seq != seq) return fail(e, GG_E_STATE, "gg_sample_last(seq %d) must follow gg_prefill of that seq", seq);
  GGState s = base_inputs(e, seq, GG_RUN_LM | GG_RUN_SAMPLE);
  set_sampling(s, sp, uniform);
  GG_TRY(put_inputs(e, s));
  GG_CUDA(e, cudaEventRecord(e->ev0, e->stream));
  GG_TRY(launch(e));
  GG_CUDA(e, cudaEventRecord(e->ev1, e->stream));
  return finish(e, out_token);
}

extern "C" int gg_step(gg_engine* e, int seq, int32_t token, int pos, const gg_sample* sp, double uniform,
                       int32_t* out_token) {
  GG_TRY(ready(e, seq));
  if (!out_token) return fail(e, GG_E_ARG, "null out_token");
  if (token < 0 || token >= e->cfg.vocab_size) return fail(e, GG_E_ARG, "token %d out of range", token);
  if (pos < 0 || pos >= e->cfg.context_length) return fail(e, GG_E_ARG, "pos %d out of range", pos);
  GGState s = base_inputs(e, seq, GG_RUN_LAYERS | GG_RUN_LM | GG_RUN_SAMPLE);
  s.token = token;
  s.pos = pos;
  set_sampling(s, sp, uniform);
  // inputs as a launch parameter, the result written by the kernel into the mapped pinned state:
  // the only host <-> device traffic is the launch and those writes
  GG_CUDA(e, cudaEventRecord(e->ev0, e->stream));
  GG_TRY(launch(e, &s));
  GG_CUDA(e, cudaEventRecord(e->ev1, e->stream));
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  GG_TRY(finish_synced(e, out_token));
  e->last_hidden_seq = seq;
  return GG_OK;
}

extern "C" int gg_decode(gg_engine* e, int seq, int32_t token, int pos, int n, const gg_sample* sp,
                         const double* uniforms, int32_t* out_tokens) {
  GG_TRY(ready(e, seq));
  if (n <= 0 || !out_tokens) return fail(e, GG_E_ARG, "bad n / out_tokens");
  if (token < 0 || token >= e->cfg.vocab_size) return fail(e, GG_E_ARG, "token %d out of range", token);
  if (pos < 0 || pos + n > e->cfg.context_length) return fail(e, GG_E_ARG, "positions %d..%d exceed context", pos, pos + n - 1);
  if (e->ring_cap < n) {
    if (e->d_ring) cudaFree(e->d_ring);
    if (e->h_ring) cudaFreeHost(e->h_ring);
    e->d_ring = nullptr; e->h_ring = nullptr; e->ring_cap = 0;
    GG_CUDA(e, cudaMalloc(&e->d_ring, sizeof(int32_t) * n));
    GG_CUDA(e, cudaMallocHost(&e->h_ring, sizeof(int32_t) * n));
    e->ring_cap = n;
  }
  GGState s = base_inputs(e, seq, GG_RUN_LAYERS | GG_RUN_LM | GG_RUN_SAMPLE);
  s.token = token;
  s.pos = pos;
  set_sampling(s, sp, 0.0);
  const bool greedy = !sp || sp->temperature == 0.0;
  if (!greedy) {
    if (!uniforms) return fail(e, GG_E_ARG, "uniforms required when temperature > 0");
    if (e->unif_cap < n) {
      if (e->d_unif) cudaFree(e->d_unif);
      e->d_unif = nullptr; e->unif_cap = 0;
      GG_CUDA(e, cudaMalloc(&e->d_unif, sizeof(double) * n));
      e->unif_cap = n;
    }
    GG_CUDA(e, cudaMemcpyAsync(e->d_unif, uniforms, sizeof(double) * n, cudaMemcpyHostToDevice, e->stream));
    s.uniforms = e->d_unif;
  }
  s.token_ring = e->d_ring;
  s.ring_len = n;
  s.step_index = 0;
  GG_TRY(put_inputs(e, s));
  GG_CUDA(e, cudaEventRecord(e->ev0, e->stream));
  for (int i = 0; i < n; i++) GG_TRY(launch(e));
  GG_CUDA(e, cudaEventRecord(e->ev1, e->stream));
  GG_CUDA(e, cudaMemcpyAsync(e->h_ring, e->d_ring, sizeof(int32_t) * n, cudaMemcpyDeviceToHost, e->stream));
  GG_TRY(finish(e, nullptr));
  memcpy(out_tokens, e->h_ring, sizeof(int32_t) * n);
  e->last_hidden_seq = seq;
  return GG_OK;
}

extern "C" int gg_get_logits(gg_engine* e, float* out) {
  GG_TRY(ready(e, 0));
  if (!out) return fail(e, GG_E_ARG, "null out");
  GG_CUDA(e, cudaMemcpyAsync(out, e->md.logits, 4 * (size_t)e->md.V, cudaMemcpyDeviceToHost, e->stream));
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  return GG_OK;
}

extern "C" int gg_get_hidden(gg_engine* e, float* out) {
  GG_TRY(ready(e, 0));
  if (!out) return fail(e, GG_E_ARG, "null out");
  GG_CUDA(e, cudaMemcpyAsync(out, e->md.dbg_normed, 4 * (size_t)e->md.H, cudaMemcpyDeviceToHost, e->stream));
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  return GG_OK;
}

extern "C" int gg_get_kv(gg_engine* e, int seq, int layer, int pos, int which, float* out) {
  GG_TRY(ready(e, seq));
  if (!out || layer < 0 || layer >= e->cfg.num_layers || pos < 0 || pos >= e->cfg.context_length)
    return fail(e, GG_E_ARG, "bad layer/pos");
  const uint8_t* base = which ? e->md.vcache : e->md.kcache;
  const int es = e->md.kv_es, KV = e->md.KV;
  size_t off = ((size_t)seq * e->md.kv_seq_stride + ((size_t)layer * e->md.CTX + pos) * KV) * es;
  std::vector<uint16_t> raw(es == 2 ? KV : 0);
  void* dst = es == 2 ? (void*)raw.data() : (void*)out;
  GG_CUDA(e, cudaMemcpyAsync(dst, base + off, (size_t)es * KV, cudaMemcpyDeviceToHost, e->stream));
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  for (int i = 0; es == 2 && i < KV; i++) {  // bf16 -> f32: the upper half of the f32 pattern
    const uint32_t u = (uint32_t)raw[i] << 16;
    std::memcpy(out + i, &u, 4);
  }
  return GG_OK;
}

// Element i of a tagged exchange buffer, to f32. sl > 0: the buffer holds one slot of sl words
// per CTA, and quad q = i / 4 of the nq quads lives in the slot of the CTA that owns it (the
// step kernel's quad partition q in [c * nq / G, (c + 1) * nq / G)).
__global__ void gg_untag_kernel(const uint64_t* src, float* dst, int n, int nq, int G, int sl) {
  int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  size_t w = (size_t)i;
  if (sl > 0) {
    const uint32_t q = (uint32_t)i >> 2;
    const uint32_t c = ((q + 1u) * (uint32_t)G - 1u) / (uint32_t)nq;
    const uint32_t qb = (c * (uint32_t)nq) / (uint32_t)G;
    w = (size_t)c * sl + 4 * (q - qb) + (i & 3);
  }
  dst[i] = __uint_as_float((uint32_t)src[w]);
}

// One weight row dequantised from what the device holds: f32(int8 q) * f32(f16 d), the exact
// values every matvec and GEMM of this library multiplies (the reference's packQ8_0ForGPU +
// f16ToF32, src/gguf.ts:95-149, and the shader's q * d). tiled = 0 reads the row format, 1 the
// GEMM's tiled copy (row r of 128-row tile r / 128, 64-column slabs).
__global__ void gg_dequant_row_kernel(const uint8_t* __restrict__ base, int K, int tiled, int r, float* __restrict__ out) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= K) return;
  const uint8_t *qp, *dp;
  if (!tiled) {
    qp = base + k;
    dp = base + K + 2 * (k >> 5);
  } else {
    const uint8_t* t = base + ((size_t)(r >> 7) * (K / 64) + (k >> 6)) * GG_Q8_TILE_BYTES;
    qp = t + (r & 127) * 64 + (k & 63);
    dp = t + 128 * 64 + (r & 127) * 4 + ((k >> 5) & 1) * 2;
  }
  out[k] = (float)(int8_t)*qp * __half2float(*reinterpret_cast<const __half*>(dp));
}

extern "C" int gg_dequant_row(gg_engine* e, int which, int layer, int row, int copy, float* out, int n) {
  GG_TRY(ready(e, 0));
  const GGModelDev& m = e->md;
  if (!out || which < 0 || which > 4 || copy < 0 || copy > 1) return fail(e, GG_E_ARG, "bad matrix %d or copy %d", which, copy);
  if (which < 4 && (layer < 0 || layer >= m.L)) return fail(e, GG_E_ARG, "layer %d outside 0..%d", layer, m.L - 1);
  const int M[5] = {m.Q + 2 * m.KV, m.H, 2 * m.I, m.H, m.V}, K[5] = {m.H, m.Q, m.H, m.I, m.H};
  const int rs[5] = {m.rs_h, m.rs_q, m.rs_h, m.rs_i, m.rs_h};
  if (row < 0 || row >= M[which]) return fail(e, GG_E_ARG, "row %d outside 0..%d", row, M[which] - 1);
  if (n != K[which]) return fail(e, GG_E_ARG, "n=%d, the row has %d values", n, K[which]);
  const uint8_t* base;
  if (copy == 0) {
    const uint8_t* rows[4] = {e->wqkv[layer < 0 ? 0 : layer], e->wo[layer < 0 ? 0 : layer], e->wgu[layer < 0 ? 0 : layer],
                              e->wdown[layer < 0 ? 0 : layer]};
    base = (which == 4 ? e->embd : rows[which]) + (size_t)row * rs[which];
  } else {
    if (!e->gemm_ok) return fail(e, GG_E_STATE, "this model has no tiled copy (shapes not multiples of 128 x 64)");
    base = (which == 4 ? e->lm_map : e->qmaps[(size_t)layer * 4 + which]).tiles;
  }
  float* tmp = nullptr;
  GG_CUDA(e, cudaMalloc(&tmp, 4 * (size_t)n));
  gg_dequant_row_kernel<<<(n + 255) / 256, 256, 0, e->stream>>>(base, n, copy, row, tmp);
  cudaError_t r = cudaGetLastError();
  if (r == cudaSuccess) r = cudaMemcpyAsync(out, tmp, 4 * (size_t)n, cudaMemcpyDeviceToHost, e->stream);
  cudaError_t r2 = cudaStreamSynchronize(e->stream);
  cudaFree(tmp);
  if (r == cudaSuccess) r = r2;
  if (r != cudaSuccess) return fail(e, GG_E_CUDA, "dequant row: %s", cudaGetErrorString(r));
  return GG_OK;
}

extern "C" int gg_debug_read(gg_engine* e, int which, float* out, int n) {
  GG_TRY(ready(e, 0));
  const GGModelDev& m = e->md;
  const uint64_t* tagged[5] = {m.t_qkv, m.t_att, nullptr, m.t_act, m.t_down};
  const int tlen[5] = {m.Q + 2 * m.KV, m.Q, m.H, m.I, m.H};
  const float* plain[4] = {m.dbg_hidden, m.dbg_residual, m.dbg_normed, m.logits};
  const int plen[4] = {m.H, m.H, m.H, m.V};
  if (!out || which < 0 || which > 8) return fail(e, GG_E_ARG, "bad buffer id %d", which);
  int cap = which < 5 ? tlen[which] : plen[which - 5];
  if (n <= 0 || n > cap) return fail(e, GG_E_ARG, "n=%d outside 1..%d", n, cap);
  if (which == 2) {  // O projection: fixed-point sums of the last launch (parity flipped after it)
    uint32_t par = 0;
    GG_CUDA(e, cudaMemcpyAsync(&par, &e->d_st->parity, 4, cudaMemcpyDeviceToHost, e->stream));
    GG_CUDA(e, cudaStreamSynchronize(e->stream));
    const unsigned long long* src = m.acc + ((size_t)((par ^ 1u) & 1u) * m.L + (m.L - 1)) * m.acc_stride;
    float* tmp = nullptr;
    GG_CUDA(e, cudaMalloc(&tmp, 4 * (size_t)n));
    gg_fixed_to_f32_kernel<<<(n + 255) / 256, 256, 0, e->stream>>>(src, tmp, n);
    cudaError_t r = cudaMemcpyAsync(out, tmp, 4 * (size_t)n, cudaMemcpyDeviceToHost, e->stream);
    cudaStreamSynchronize(e->stream);
    cudaFree(tmp);
    if (r != cudaSuccess) return fail(e, GG_E_CUDA, "debug read: %s", cudaGetErrorString(r));
  } else if (which < 5) {
    float* tmp = nullptr;
    GG_CUDA(e, cudaMalloc(&tmp, 4 * (size_t)n));
    const int nq[5] = {(m.Q + 2 * m.KV) / 4, m.Q / 4, m.H / 4, m.I / 4, m.H / 4};
    const int sl[5] = {m.sl_qkv, 0, m.sl_h, m.sl_i, m.sl_h};
    gg_untag_kernel<<<(n + 255) / 256, 256, 0, e->stream>>>(tagged[which], tmp, n, nq[which], m.grid, sl[which]);
    cudaError_t r = cudaMemcpyAsync(out, tmp, 4 * (size_t)n, cudaMemcpyDeviceToHost, e->stream);
    cudaStreamSynchronize(e->stream);
    cudaFree(tmp);
    if (r != cudaSuccess) return fail(e, GG_E_CUDA, "debug read: %s", cudaGetErrorString(r));
  } else {
    GG_CUDA(e, cudaMemcpyAsync(out, plain[which - 5], 4 * (size_t)n, cudaMemcpyDeviceToHost, e->stream));
    GG_CUDA(e, cudaStreamSynchronize(e->stream));
  }
  return GG_OK;
}

extern "C" int gg_seen_reset(gg_engine* e, int seq) {
  GG_TRY(ready(e, seq));
  GG_CUDA(e, cudaMemsetAsync(e->md.seen + (size_t)seq * e->md.seen_stride, 0, e->md.seen_stride, e->stream));
  GG_CUDA(e, cudaMemsetAsync(&e->d_st->seen_count, 0, sizeof(int32_t), e->stream));
  GG_CUDA(e, cudaMemsetAsync(e->md.seen_cnt + seq, 0, sizeof(int32_t), e->stream));
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  return GG_OK;
}

extern "C" int gg_seen_add(gg_engine* e, int seq, const int32_t* ids, int n) {
  GG_TRY(ready(e, seq));
  if (n <= 0) return GG_OK;
  if (!ids) return fail(e, GG_E_ARG, "null ids");
  if (e->ids_cap < n) {
    if (e->d_ids) cudaFree(e->d_ids);
    e->d_ids = nullptr; e->ids_cap = 0;
    GG_CUDA(e, cudaMalloc(&e->d_ids, sizeof(int32_t) * n));
    e->ids_cap = n;
  }
  GG_CUDA(e, cudaMemcpyAsync(e->d_ids, ids, sizeof(int32_t) * n, cudaMemcpyHostToDevice, e->stream));
  gg_seen_add_kernel<<<(n + 255) / 256, 256, 0, e->stream>>>(e->md.seen + (size_t)seq * e->md.seen_stride, e->d_ids, n,
                                                             e->cfg.vocab_size, e->d_st, e->md.seen_cnt + seq);
  GG_CUDA(e, cudaGetLastError());
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  return GG_OK;
}

extern "C" int gg_reset_kv(gg_engine* e, int seq) {
  GG_TRY(ready(e, seq));
  size_t n = e->md.kv_seq_stride * e->md.kv_es;
  GG_CUDA(e, cudaMemsetAsync(e->md.kcache + (size_t)seq * n, 0, n, e->stream));
  GG_CUDA(e, cudaMemsetAsync(e->md.vcache + (size_t)seq * n, 0, n, e->stream));
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  return GG_OK;
}

extern "C" int gg_grid(gg_engine* e, int* out) {
  if (!e || !out) return fail(e, GG_E_ARG, "null argument");
  *out = e->md.grid ? e->md.grid : e->sm_count;
  return GG_OK;
}

extern "C" int gg_set_trace(gg_engine* e, int on) {
  if (!e) return fail(e, GG_E_ARG, "null engine");
  e->trace_on = on ? 1 : 0;
  return GG_OK;
}

extern "C" int gg_read_trace(gg_engine* e, uint64_t* out, int n) {
  GG_TRY(ready(e, 0));
  const int cap = e->md.grid * GG_TRACE_PHASES * 4;
  if (!out || n <= 0 || n > cap) return fail(e, GG_E_ARG, "n must be 1..%d", cap);
  GG_CUDA(e, cudaMemcpyAsync(out, e->md.trace, 8 * (size_t)n, cudaMemcpyDeviceToHost, e->stream));
  GG_CUDA(e, cudaStreamSynchronize(e->stream));
  return GG_OK;
}

extern "C" int gg_set_gemm_kernel(int kind) {
  const int prev = gg_gemm_path();
  if (kind == GG_GEMM_SCALED || kind == GG_GEMM_DEQUANT) gg_gemm_set_path(kind);
  else if (kind != -1) return GG_E_ARG;
  return prev;
}

extern "C" int gg_selftest_wait(gg_engine* e, uint64_t timeout_ns) {
  GG_TRY(ready(e, 0));
  if (timeout_ns < 1000 || timeout_ns > 10000000000ull) return fail(e, GG_E_ARG, "timeout out of range");
  uint64_t* word = nullptr;
  GG_CUDA(e, cudaMalloc(&word, 64));
  cudaMemsetAsync(word, 0, 64, e->stream);
  cudaEventRecord(e->ev0, e->stream);  // finish() reads the ev0 -> ev1 time
  gg_wait_probe_kernel<<<1, 32, 0, e->stream>>>(word, &e->d_st->error, timeout_ns);
  cudaEventRecord(e->ev1, e->stream);
  cudaError_t r = cudaGetLastError();
  if (r == cudaSuccess) r = cudaStreamSynchronize(e->stream);
  cudaFree(word);
  if (r != cudaSuccess) return fail(e, GG_E_CUDA, "wait probe: %s", cudaGetErrorString(r));
  return finish(e, nullptr);  // reads and clears the error word, GG_E_DEVICE if it is set
}

// Sum of `splits` consecutive planes of n floats, in plane order.
__global__ void gg_sum_splits_kernel(const float* __restrict__ p, int splits, long long n, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    float s = p[i];
    for (int z = 1; z < splits; z++) s += p[(long long)z * n + i];
    out[i] = s;
  }
}

// K-splits so that the tiles of one GEMM fill the CTA slots without an empty split (at most 16,
// at least 3 K slabs each). Tiles of up to 64 rows run two CTAs per SM.
static int pick_splits(int tiles, int KS, int slots) {
  int s = 1;
  while (s < 16 && tiles * (s + 1) <= slots && KS / (s + 1) >= 2) s++;  // at least two K slabs per split
  while (s > 1 && (long long)(s - 1) * ((KS + s - 1) / s) >= KS) s--;
  return s;
}

static int grow(gg_engine* e, void** p, size_t* cap, size_t need) {
  if (*cap >= need) return GG_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  cudaError_t r = cudaMalloc(p, need);
  if (r != cudaSuccess) return fail(e, GG_E_NOMEM, "cudaMalloc(%zu): %s", need, cudaGetErrorString(r));
  *cap = need;
  return GG_OK;
}

extern "C" int gg_linear(gg_engine* e, int which, int layer, const float* x, int batch, float* y) {
  GG_TRY(ready(e, 0));
  if (!e->gemm_ok) return fail(e, GG_E_STATE, "tensor-core path unavailable for this model's shapes");
  if (!x || !y || batch < 1 || batch > 4096) return fail(e, GG_E_ARG, "bad x/y/batch");
  if (which < 0 || which > 4) return fail(e, GG_E_ARG, "matrix %d not in 0..4", which);
  if (which < 4 && (layer < 0 || layer >= e->cfg.num_layers)) return fail(e, GG_E_ARG, "layer %d out of range", layer);
  const GGQ8Map& w = which == 4 ? e->lm_map : e->qmaps[(size_t)layer * 4 + which];
  const int M = w.M, K = w.K, T = batch;
  if (T == 1) {  // a single row: the CUDA-core matvec over the device rows
    const uint8_t* rows[5] = {which < 4 ? e->wqkv[layer] : nullptr, which < 4 ? e->wo[layer] : nullptr,
                              which < 4 ? e->wgu[layer] : nullptr, which < 4 ? e->wdown[layer] : nullptr, e->embd};
    const int rs[5] = {e->md.rs_h, e->md.rs_q, e->md.rs_h, e->md.rs_i, e->md.rs_h};
    GG_TRY(grow(e, (void**)&e->lin_x, &e->lin_x_cap, sizeof(float) * (size_t)K));
    GG_TRY(grow(e, (void**)&e->lin_y, &e->lin_y_cap, sizeof(float) * (size_t)M));
    GG_CUDA(e, cudaMemcpyAsync(e->lin_x, x, sizeof(float) * (size_t)K, cudaMemcpyHostToDevice, e->stream));
    GG_CUDA(e, cudaEventRecord(e->ev0, e->stream));
    GG_CUDA(e, gg_matvec_q8(rows[which], rs[which], M, K, e->lin_x, e->lin_y, e->sm_count, e->stream));
    GG_CUDA(e, cudaEventRecord(e->ev1, e->stream));
    GG_CUDA(e, cudaMemcpyAsync(y, e->lin_y, sizeof(float) * (size_t)M, cudaMemcpyDeviceToHost, e->stream));
    return finish(e, nullptr);
  }
  const int splits = pick_splits(gemm_tiles(T, M), K / 64, gemm_slots(e, T));
  const size_t tb = gg_xtiles_bytes(T, K);
  GG_TRY(grow(e, (void**)&e->lin_x, &e->lin_x_cap, sizeof(float) * (size_t)T * K));
  GG_TRY(grow(e, (void**)&e->lin_tiles, &e->lin_tiles_cap, 2 * tb));
  GG_TRY(grow(e, (void**)&e->lin_y, &e->lin_y_cap, sizeof(float) * (size_t)T * M * (splits + 1)));
  GG_CUDA(e, cudaMemcpyAsync(e->lin_x, x, sizeof(float) * (size_t)T * K, cudaMemcpyHostToDevice, e->stream));
  GG_CUDA(e, gg_xtiles_from_f32(e->lin_x, T, K, e->lin_tiles, e->lin_tiles + tb, e->stream));
  GG_CUDA(e, cudaEventRecord(e->ev0, e->stream));  // times the product (+ split sum) only
  const long long plane = (long long)T * M;
  float* out = e->lin_y;
  if (splits == 1) {
    GG_CUDA(e, gg_gemm_q8(w, e->lin_tiles, e->lin_tiles + tb, T, out, M, 1, 0, &e->d_st->error, e->timeout_ns, e->stream));
  } else {
    float* part = e->lin_y + plane;
    GG_CUDA(e, gg_gemm_q8(w, e->lin_tiles, e->lin_tiles + tb, T, part, M, splits, plane, &e->d_st->error, e->timeout_ns,
                          e->stream));
    GG_CUDA(e, gg::launch_pdl(gg_sum_splits_kernel, dim3(e->sm_count * 4), dim3(256), 0, e->stream, (const float*)part,
                              splits, (long long)plane, out));
  }
  GG_CUDA(e, cudaEventRecord(e->ev1, e->stream));
  GG_CUDA(e, cudaMemcpyAsync(y, out, sizeof(float) * (size_t)plane, cudaMemcpyDeviceToHost, e->stream));
  return finish(e, nullptr);
}

extern "C" int gg_set_timeout(gg_engine* e, uint64_t ns) {
  if (!e) return fail(e, GG_E_ARG, "null engine");
  if (ns < 1000) return fail(e, GG_E_ARG, "timeout must be >= 1 us");
  e->timeout_ns = ns;
  return GG_OK;
}

extern "C" int gg_last_device_ms(gg_engine* e, float* ms) {
  if (!e || !ms) return fail(e, GG_E_ARG, "null argument");
  *ms = e->last_ms;
  return GG_OK;
}

extern "C" int gg_destroy(gg_engine* e) {
  if (!e) return GG_OK;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (void* p : e->allocs) cudaFree(p);
  if (e->staging) cudaFree(e->staging);
  if (e->d_ids) cudaFree(e->d_ids);
  if (e->d_unif) cudaFree(e->d_unif);
  if (e->d_ring) cudaFree(e->d_ring);
  if (e->h_ring) cudaFreeHost(e->h_ring);
  if (e->h_st) cudaFreeHost(e->h_st);
  if (e->bd_unif) cudaFree(e->bd_unif);
  if (e->bd_out) cudaFree(e->bd_out);
  if (e->bd_out_h) cudaFreeHost(e->bd_out_h);
  if (e->lin_x) cudaFree(e->lin_x);
  if (e->lin_tiles) cudaFree(e->lin_tiles);
  if (e->lin_y) cudaFree(e->lin_y);
  if (e->ev0) cudaEventDestroy(e->ev0);
  if (e->ev1) cudaEventDestroy(e->ev1);
  if (e->stream) cudaStreamDestroy(e->stream);
  delete e;
  return GG_OK;
}

extern "C" const char* gg_last_error(const gg_engine* e) { return e ? e->err.c_str() : g_create_err.c_str(); }

extern "C" const char* gg_version(void) { return "gemma_b200 0.1 (sm_100a, persistent decode kernel, ncw=16)"; }
