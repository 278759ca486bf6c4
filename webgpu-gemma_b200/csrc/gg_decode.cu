// gg_decode.cu -- sampling kernels outside the step kernel: the batched sampler of gg_decode_batch
// (one CTA per row of a logits matrix) and the allocation-free sampler behind
// gg_sample_logits_noalloc. Both end in sample_token (gg_sample.cuh), the same sampler the step
// kernel's last CTA runs (src/engine.ts:823-901).
#include "gg_device.cuh"
#include "gg_launch.h"
#include "gg_model.h"
#include "gg_sample.cuh"

namespace gg {

// ---------------------------------------------------------------------- batched sampling

// One CTA per row of a [B][V] logits matrix: the 256 lane maxima of the row, then the sampler
// (sample_token, engine.ts:823-901) with that row's parameters, draw and KV slot's seen set.
// The sampled token is added to the slot's seen set, becomes the row's next input token, and
// the row's position advances.
__global__ void __launch_bounds__(512)
    gg_batch_sample_kernel(const float* __restrict__ logits, int V, const int32_t* __restrict__ seqs,
                           const GGSampleDev* __restrict__ sp, const double* __restrict__ unif, uint8_t* seen,
                           int seen_stride, int32_t* seen_cnt, unsigned long long* keys, int32_t* tokens,
                           int32_t* pos, int32_t* out) {
  pdl_trigger();
  pdl_wait();  // before touching any buffer shared with the other kernels of the chain
  __shared__ GGModelDev sm;
  __shared__ GGState ss;
  __shared__ unsigned long long sk[8][256];
  const int b = blockIdx.x, t = threadIdx.x;
  const float* row = logits + (size_t)b * V;
  const unsigned long long ik = init_lane_key();
  // Element i belongs to lane i % 256. Thread t reads 16-byte groups c = t, t + 512, ... (eight
  // loads in flight): elements 4c..4c+3 are lanes 4 (c % 64) + j, shared by the eight threads
  // t % 64 + 64 k.
  unsigned long long best[4] = {ik, ik, ik, ik};
  const int n4 = V >> 2;
  auto take = [&](const float4 f, int c) {
    const float fv[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      float v = fv[j];
      if (!isnan(v)) {
        if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal under '>': key them alike
        const uint32_t i = 4u * (uint32_t)c + j;
        const unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - i);
        best[j] = k > best[j] ? k : best[j];
      }
    }
  };
  const float4* row4 = reinterpret_cast<const float4*>(row);
  int c = t;
  for (; c + 7 * 512 < n4; c += 8 * 512) {
    float4 f[8];
#pragma unroll
    for (int u = 0; u < 8; u++) f[u] = __ldcs(row4 + c + u * 512);
#pragma unroll
    for (int u = 0; u < 8; u++) take(f[u], c + u * 512);
  }
  for (; c < n4; c += 512) take(__ldcs(row4 + c), c);
#pragma unroll
  for (int j = 0; j < 4; j++) sk[t >> 6][4 * (t & 63) + j] = best[j];
  __syncthreads();
  unsigned long long kb = ik;
  if (t < 256) {
#pragma unroll
    for (int q = 0; q < 8; q++) kb = sk[q][t] > kb ? sk[q][t] : kb;
    for (int i = 4 * n4; i < V; i++) {  // tail when V % 4 != 0 (< 4 elements): lane i % 256
      if ((i & 255) != t) continue;
      float v = row[i];
      if (!isnan(v)) {
        if (v == 0.0f) v = 0.0f;
        const unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - (uint32_t)i);
        kb = k > kb ? k : kb;
      }
    }
  }
  unsigned long long* rk = keys + (size_t)b * 256;
  if (t < 256) rk[t] = kb;
  const int seq = seqs[b];
  if (t == 0) {
    sm.lane_keys = rk;
    sm.seen = seen;
    sm.seen_stride = seen_stride;
    sm.V = V;
    ss.seq = seq;
    ss.temperature = sp[b].temperature;
    ss.top_p = sp[b].top_p;
    ss.rep_penalty = sp[b].rep_penalty;
    ss.uniform = unif[b];
    ss.uniforms = nullptr;
    ss.seen_count = seen_cnt[seq];
  }
  __threadfence_block();
  __syncthreads();
  __shared__ SampleScratch sscr;
  const int tok = sample_token(sm, &ss, sscr);
  if (t == 0) {
    out[b] = tok;
    if (tok >= 0 && tok < V) {
      atomicOr(reinterpret_cast<unsigned int*>(seen + (size_t)seq * seen_stride) + (tok >> 5), 1u << (tok & 31));
      seen_cnt[seq] += 1;
    }
    tokens[b] = tok;
    pos[b] += 1;
  }
}

}  // namespace gg

cudaError_t gg_batch_sample(const float* logits, int B, int V, const int32_t* seqs, const GGSampleDev* sp,
                            const double* unif, uint8_t* seen, int seen_stride, int32_t* seen_cnt,
                            unsigned long long* keys, int32_t* tokens, int32_t* pos, int32_t* out, cudaStream_t s) {
  if (B <= 0) return cudaErrorInvalidValue;
  return gg::launch_pdl(gg::gg_batch_sample_kernel, dim3(B), dim3(512), 0, s, logits, V, seqs, sp, unif, seen,
                        seen_stride, seen_cnt, keys, tokens, pos, out);
}

// ------------------------------------------------------------------ sampling without allocation
//
// gg_sample_logits_noalloc: the step kernel's last stage -- the 256 per-lane maxima of the
// logits (shaders.ts:363-384) and the sampler (engine.ts:823-901) -- as a kernel of its own over
// logits the caller already holds on the device. Its scratch (per-CTA lane maxima and an
// end-of-launch ticket) lives in a static device array, so a call allocates no memory.

#include <cuda.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "gemma_b200.h"

namespace gg {

constexpr int SL_THREADS = 256;                                   // thread t owns top-256 lane t
constexpr int SL_ROWS_PER_THREAD = 16;
constexpr int SL_ROWS_PER_CTA = SL_THREADS * SL_ROWS_PER_THREAD;  // 4096 logits per CTA
constexpr int SL_MAX_CTAS = 128;
constexpr int SL_MAX_VOCAB = SL_MAX_CTAS * SL_ROWS_PER_CTA;       // 524,288 (Gemma 3: 262,144)
constexpr int SL_KEYS_OFF = 32;  // word 0: ticket; from word 32: SL_MAX_CTAS x 256 lane keys
constexpr size_t SL_SCRATCH_WORDS = SL_KEYS_OFF + (size_t)SL_MAX_CTAS * SL_THREADS;

// 262,400 bytes on every GPU that loads the library, held until the process exits. Shared by
// all calls: the ticket (word 0) must be zero when a launch starts and is cleared by the host
// before each launch; every CTA overwrites its own lane-key slot before anything reads it.
static __device__ __align__(256) unsigned long long g_sample_scratch[SL_SCRATCH_WORDS];

__global__ void __launch_bounds__(SL_THREADS)
    gg_sample_logits_kernel(const float* __restrict__ logits, int V, const uint32_t* __restrict__ seen_bits,
                            double temperature, double top_p, double rep_penalty, double uniform,
                            int32_t* __restrict__ out_token, unsigned long long* __restrict__ scratch) {
  __shared__ int is_last;
  __shared__ GGModelDev sm;
  __shared__ GGState ss;
  const int t = threadIdx.x;
  unsigned long long* keys = scratch + SL_KEYS_OFF;
  // Rows base + t + 256 j all fall in lane t: (value, lowest row) maximum, strict '>' from
  // (-1e30, 0), NaN never taken; -0 is keyed as +0 since the two compare equal.
  const unsigned long long ik = init_lane_key();
  unsigned long long best = ik;
  const int base = blockIdx.x * SL_ROWS_PER_CTA;
#pragma unroll 4
  for (int j = 0; j < SL_ROWS_PER_THREAD; j++) {
    const int row = base + t + j * SL_THREADS;
    if (row < V) {
      float v = __ldg(logits + row);
      if (!isnan(v)) {
        if (v == 0.0f) v = 0.0f;
        const unsigned long long k = ((unsigned long long)f32_order_key(v) << 32) | (0xffffffffu - (uint32_t)row);
        best = k > best ? k : best;
      }
    }
  }
  keys[(size_t)blockIdx.x * SL_THREADS + t] = best;
  __threadfence();
  __syncthreads();
  if (t == 0) is_last = atomicAdd(scratch, 1ull) == (unsigned long long)(gridDim.x - 1);
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  unsigned long long k = ik;
  for (int c = 0; c < (int)gridDim.x; c++) {
    const unsigned long long o = __ldcg(keys + (size_t)c * SL_THREADS + t);
    k = o > k ? o : k;
  }
  keys[t] = k;  // slot 0 now holds the merged maxima; thread t reads back only its own lane
  if (t == 0) {
    sm.lane_keys = keys;
    sm.seen = reinterpret_cast<uint8_t*>(const_cast<uint32_t*>(seen_bits));
    sm.seen_stride = 0;
    sm.V = V;
    ss.seq = 0;
    ss.temperature = temperature;
    ss.top_p = top_p;
    ss.rep_penalty = rep_penalty;
    ss.uniform = uniform;
    ss.uniforms = nullptr;
    ss.seen_count = seen_bits ? 1 : 0;
  }
  __threadfence_block();
  __syncthreads();
  __shared__ SampleScratch sscr;
  const int tok = sample_token(sm, &ss, sscr);
  if (t == 0) *out_token = tok;
}

}  // namespace gg

void gg_set_engineless_error(const char* msg);  // gg_engine.cu: the message gg_last_error(NULL) returns

namespace {

constexpr int SL_MAX_DEVICES = 64;
std::mutex g_sl_mu;
// Device address of the array per device, with the id of the context it was looked up in: a
// context that replaced that one (after cudaDeviceReset, or another context made current) has
// its own copy of the array at a possibly different address, so the lookup is redone there.
struct SlSlot {
  unsigned long long ctx_id = 0;
  unsigned long long* addr = nullptr;
};
SlSlot g_sl_scratch[SL_MAX_DEVICES];

typedef CUresult (*PfnCtxGetCurrent)(CUcontext*);
typedef CUresult (*PfnCtxGetId)(CUcontext, unsigned long long*);

// Unique id (for the life of the process) of the calling thread's current context, or 0.
unsigned long long current_ctx_id() {
  static PfnCtxGetCurrent get_cur = nullptr;
  static PfnCtxGetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_cur = reinterpret_cast<PfnCtxGetCurrent>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<PfnCtxGetId>(f);
  });
  CUcontext c = nullptr;
  unsigned long long id = 0;
  if (!get_cur || !get_id || get_cur(&c) != CUDA_SUCCESS || !c || get_id(c, &id) != CUDA_SUCCESS) return 0;
  return id;
}

int sl_fail(int code, const char* fmt, ...) {
  char buf[320];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  gg_set_engineless_error(buf);
  return code;
}

}  // namespace

extern "C" int gg_sample_logits_noalloc(const float* logits, int vocab, const uint32_t* seen_bits,
                                        const gg_sample* sp, double uniform, int32_t* out_token, void* stream) {
  using namespace gg;
  if (!logits || !sp || !out_token) return sl_fail(GG_E_ARG, "gg_sample_logits_noalloc: null logits, sample or out_token");
  if (vocab < 1 || vocab > SL_MAX_VOCAB)
    return sl_fail(GG_E_ARG,
                   "gg_sample_logits_noalloc: vocab %d outside 1..%d (its static scratch holds the lane maxima "
                   "of %d blocks of %d logits)", vocab, SL_MAX_VOCAB, SL_MAX_CTAS, SL_ROWS_PER_CTA);
  int dev = -1;
  cudaError_t r = cudaGetDevice(&dev);
  if (r != cudaSuccess) return sl_fail(GG_E_CUDA, "gg_sample_logits_noalloc: cudaGetDevice: %s", cudaGetErrorString(r));
  if (dev < 0 || dev >= SL_MAX_DEVICES) return sl_fail(GG_E_ARG, "gg_sample_logits_noalloc: device %d >= %d", dev, SL_MAX_DEVICES);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (s) {  // the kernel and the memset run on the current device: the stream must belong to it
    int sdev = -1;
    r = cudaStreamGetDevice(s, &sdev);
    if (r != cudaSuccess) return sl_fail(GG_E_ARG, "gg_sample_logits_noalloc: cudaStreamGetDevice: %s", cudaGetErrorString(r));
    if (sdev != dev)
      return sl_fail(GG_E_ARG, "gg_sample_logits_noalloc: stream belongs to device %d, the current device is %d", sdev, dev);
  }
  unsigned long long* scratch = nullptr;
  {
    // First call on a device (or in a new context on it): look up the array's device address
    // with that device current. The host-side name g_sample_scratch is not a device address and
    // is never passed to a kernel.
    std::lock_guard<std::mutex> g(g_sl_mu);
    SlSlot& slot = g_sl_scratch[dev];
    const unsigned long long ctx = current_ctx_id();  // 0 before the runtime made a context current
    if (!slot.addr || ctx == 0 || slot.ctx_id != ctx) {
      void* p = nullptr;
      r = cudaGetSymbolAddress(&p, g_sample_scratch);  // also makes the primary context current
      if (r != cudaSuccess || !p)
        return sl_fail(GG_E_CUDA, "gg_sample_logits_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                       cudaGetErrorString(r));
      slot.addr = static_cast<unsigned long long*>(p);
      slot.ctx_id = current_ctx_id();
    }
    scratch = slot.addr;
  }
  r = cudaMemsetAsync(scratch, 0, sizeof(unsigned long long), s);  // the ticket starts at zero
  if (r != cudaSuccess) return sl_fail(GG_E_CUDA, "gg_sample_logits_noalloc: clearing the ticket: %s", cudaGetErrorString(r));
  const int grid = (vocab + SL_ROWS_PER_CTA - 1) / SL_ROWS_PER_CTA;
  gg_sample_logits_kernel<<<grid, SL_THREADS, 0, s>>>(logits, vocab, seen_bits, sp->temperature, sp->top_p,
                                                      sp->rep_penalty, uniform, out_token, scratch);
  r = cudaGetLastError();
  if (r != cudaSuccess) return sl_fail(GG_E_CUDA, "gg_sample_logits_noalloc: launch: %s", cudaGetErrorString(r));
  return GG_OK;
}
