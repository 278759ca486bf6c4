// gg_device.cuh -- device-side building blocks for the sm_100a Gemma 3 token loop.
//
// mbarrier + cp.async.bulk (TMA bulk copy) helpers for the weight-streaming ring,
// tagged 64-bit words ("value | epoch << 32") used to pass activations between CTAs,
// bounded spins that raise an error word instead of hanging, and the exact int8 -> f32
// conversion used by the Q8_0 dot products.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <type_traits>

#define GG_DEV __device__ __forceinline__

// Error bits written to GGState::error by a kernel that gave up waiting.
enum : uint32_t {
  GG_ERR_WAIT_FLAG = 1u,   // a tagged activation word never arrived
  GG_ERR_WAIT_MBAR = 2u,   // a shared-memory ring slot never filled / drained
  GG_ERR_BAD_INPUT = 4u,   // token / position out of range at kernel start
};

GG_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Shared-memory accesses by 32-bit shared-window address (ld/st.shared): the hot loops read
// planes and ring stages through these, never through generic pointers.
GG_DEV uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
GG_DEV uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
GG_DEV float ldsf(uint32_t a) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
  return v;
}
GG_DEV float lds_half(uint32_t a) {  // an f16 value, widened
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return __half2float(__ushort_as_half(v));
}
GG_DEV void sts32(uint32_t a, uint32_t v) { asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory"); }

GG_DEV uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier / bulk copy

GG_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
GG_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

GG_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
GG_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
// `count` arrivals at once.
GG_DEV void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
GG_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// L2 eviction policy for data read exactly once per step (weights): evict first, so the
// small activations and KV rows keep their L2 lines.
GG_DEV uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// One bulk copy global -> this CTA's shared memory, completing on `bar` (complete_tx).
// dst/src 16-byte aligned, bytes a multiple of 16. No multicast.
GG_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------- tagged words

// A tagged word carries one f32 and the epoch of the phase that produced it. Readers spin
// until the tag matches, so the data word is its own ready flag (no separate barrier).
GG_DEV void tag_store(uint64_t* p, float v, uint32_t tag) {
  uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// Four consecutive tagged words (p 32-byte aligned: one sector) in one 32-byte store. Each 8-byte
// word still carries its own tag, so a reader that polls word by word sees whole words either
// way; a quarter of the store instructions and sector writes of four tag_store calls.
GG_DEV void tag_store4(uint64_t* p, float v0, float v1, float v2, float v3, uint32_t tag) {
  const uint64_t t = (uint64_t)tag << 32;
  asm volatile("st.relaxed.gpu.global.v4.b64 [%0], {%1, %2, %3, %4};" ::"l"(p), "l"(t | __float_as_uint(v0)),
               "l"(t | __float_as_uint(v1)), "l"(t | __float_as_uint(v2)), "l"(t | __float_as_uint(v3))
               : "memory");
}
GG_DEV uint64_t tag_load(const uint64_t* p) {
  uint64_t w;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Four consecutive words (p 32-byte aligned: one sector) with one load at gpu scope (served by
// L2: always sees the latest store of another SM).
GG_DEV void ld4_relaxed(const uint64_t* p, uint64_t (&w)[4]) {
  asm volatile("ld.relaxed.gpu.global.v4.u64 {%0, %1, %2, %3}, [%4];"
               : "=l"(w[0]), "=l"(w[1]), "=l"(w[2]), "=l"(w[3])
               : "l"(p)
               : "memory");
}

struct SpinCtl {
  uint32_t* err;        // global error word (GGState::error)
  uint64_t timeout_ns;  // give up after this long
};

// How long a wait spins before it starts looking at the global error word. Normal waits are
// far shorter; reading one global word from every waiting warp of every SM would turn that
// word's L2 line into a hot spot.
#define GG_QUIET_SPIN_NS 20000ull

// Wait for a tagged word; on timeout (or an error raised elsewhere) return 0.0f and set err.
// Polls without a back-off: a sleep between polls adds its length to every hand-over.
GG_DEV float tag_wait(const uint64_t* p, uint32_t tag, const SpinCtl& sc) {
  uint64_t w = tag_load(p);
  if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
  for (int it = 0; it < 512; ++it) {  // fast path: polls only, no clock reads
    w = tag_load(p);
    if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
  }
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    w = tag_load(p);
    if ((uint32_t)(w >> 32) == tag) return __uint_as_float((uint32_t)w);
    if ((it & 15u) == 0) {
      const uint64_t dt = global_timer_ns() - t0;
      if (dt > GG_QUIET_SPIN_NS) {
        if (*(volatile uint32_t*)sc.err) return 0.0f;
        if (dt > sc.timeout_ns) {
          atomicOr(sc.err, GG_ERR_WAIT_FLAG);
          return 0.0f;
        }
      }
    }
  }
}

// Bounded wait on an mbarrier phase for a thread that is not on the critical path: each try
// may suspend the thread (up to 200 ns, woken when the phase completes) instead of spinning, so
// it takes no issue slots from the warps that work meanwhile. Returns false (and sets err) on
// timeout.
GG_DEV bool mbar_wait_suspend(uint64_t* bar, uint32_t parity, const SpinCtl& sc) {
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity), "r"(200u)
        : "memory");
    if (done) return true;
    const uint64_t dt = global_timer_ns() - t0;
    if (dt > GG_QUIET_SPIN_NS && *(volatile uint32_t*)sc.err) return false;
    if (dt > sc.timeout_ns) {
      atomicOr(sc.err, GG_ERR_WAIT_MBAR);
      return false;
    }
  }
}

// Bounded wait on an mbarrier phase. Returns false (and sets err) on timeout.
GG_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, const SpinCtl& sc) {
  // Fast path without reading the clock; the timed loop below bounds the wait. Not unrolled:
  // every copy of a wait loop costs instruction-cache space on the critical path.
#pragma unroll 1
  for (int it = 0; it < 64; ++it)
    if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
#pragma unroll 1
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0) {
      const uint64_t dt = global_timer_ns() - t0;
      if (dt > GG_QUIET_SPIN_NS) {
        if (*(volatile uint32_t*)sc.err) return false;
        if (dt > sc.timeout_ns) {
          atomicOr(sc.err, GG_ERR_WAIT_MBAR);
          return false;
        }
      }
    }
  }
}

// ---------------------------------------------------------------- math helpers

// Exact int8 -> f32 for byte `b` of word `wx` (wx = raw ^ 0x80808080): the byte is placed in
// the mantissa of 2^23 (0x4B0000xx = 2^23 + u) and the bias 2^23 + 128 removed. Both steps
// are exact in f32.
template <int B>
GG_DEV float q8_byte(uint32_t wx) {
  return __int_as_float((int)__byte_perm(wx, 0x4B000000u, 0x7440u + B)) - 8388736.0f;
}

// Sum over the 16 int8 of `w` times x[0..15] (fp32 fused multiply-adds, in element order).
GG_DEV float dot16(uint4 w, float4 a, float4 b, float4 c, float4 d) {
  uint32_t w0 = w.x ^ 0x80808080u, w1 = w.y ^ 0x80808080u, w2 = w.z ^ 0x80808080u, w3 = w.w ^ 0x80808080u;
  float s = q8_byte<0>(w0) * a.x;
  s = fmaf(q8_byte<1>(w0), a.y, s);
  s = fmaf(q8_byte<2>(w0), a.z, s);
  s = fmaf(q8_byte<3>(w0), a.w, s);
  s = fmaf(q8_byte<0>(w1), b.x, s);
  s = fmaf(q8_byte<1>(w1), b.y, s);
  s = fmaf(q8_byte<2>(w1), b.z, s);
  s = fmaf(q8_byte<3>(w1), b.w, s);
  s = fmaf(q8_byte<0>(w2), c.x, s);
  s = fmaf(q8_byte<1>(w2), c.y, s);
  s = fmaf(q8_byte<2>(w2), c.z, s);
  s = fmaf(q8_byte<3>(w2), c.w, s);
  s = fmaf(q8_byte<0>(w3), d.x, s);
  s = fmaf(q8_byte<1>(w3), d.y, s);
  s = fmaf(q8_byte<2>(w3), d.z, s);
  s = fmaf(q8_byte<3>(w3), d.w, s);
  return s;
}

// GELU with the tanh approximation and the argument clamp of shaders.ts:153-170.
GG_DEV float gelu_tanh(float x) {
  const float S = 0.7978845608028654f, A = 0.044715f;
  float t = S * x * (1.0f + A * x * x);
  t = fminf(fmaxf(t, -15.0f), 15.0f);
  return 0.5f * x * (1.0f + tanhf(t));
}

// KV cache elements: f32 (the reference's layout) or bf16 (GG_FLAG_KV_BF16; stored rounded to
// nearest even, widened exactly when read).
template <bool KV16>
using kv_t = typename std::conditional<KV16, __nv_bfloat16, float>::type;
GG_DEV float kv_widen(float v) { return v; }
GG_DEV float kv_widen(__nv_bfloat16 v) { return __bfloat162float(v); }
template <bool KV16>
GG_DEV kv_t<KV16> kv_narrow(float v) {
  if constexpr (KV16) return __float2bfloat16_rn(v);
  else return v;
}
// The value a bf16 cache holds for v (rounded to nearest even), as f32.
GG_DEV float bf16_rne(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
// Eight bf16 (one 16-byte load) widened to f32: each is the upper half of its f32 pattern.
GG_DEV void bf16x8_widen(const uint4 w, float* f) {
  const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; i++) {
    f[2 * i] = __uint_as_float(u[i] << 16);
    f[2 * i + 1] = __uint_as_float(u[i] & 0xffff0000u);
  }
}

// Programmatic dependent launch (see gg_launch.h): let the next kernel of the stream become
// resident now / wait until the kernels this one depends on have completed and their writes
// are visible. Both are no-ops in a kernel launched without the attribute.
GG_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
GG_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

GG_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
GG_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Warp totals of 16 values at once: afterwards every lane holds v[i] summed over the warp, for
// all i. A butterfly reduce-scatter (8 + 4 + 2 + 1 shuffles, 1 more to finish each lane pair)
// leaves lane L with the total of value 8*L4 + 4*L3 + 2*L2 + L1 (Lk = bit k of L), then 16
// shuffles broadcast the totals: 32 shuffles instead of 16 separate 5-step reductions.
GG_DEV void warp_sum16(float (&v)[16]) {
  const int lane = threadIdx.x & 31;
  float a8[8], a4[4], a2[2];
  const bool u16 = lane & 16, u8 = lane & 8, u4 = lane & 4, u2 = lane & 2;
#pragma unroll
  for (int i = 0; i < 8; i++)
    a8[i] = (u16 ? v[i + 8] : v[i]) + __shfl_xor_sync(0xffffffffu, u16 ? v[i] : v[i + 8], 16);
#pragma unroll
  for (int i = 0; i < 4; i++)
    a4[i] = (u8 ? a8[i + 4] : a8[i]) + __shfl_xor_sync(0xffffffffu, u8 ? a8[i] : a8[i + 4], 8);
#pragma unroll
  for (int i = 0; i < 2; i++)
    a2[i] = (u4 ? a4[i + 2] : a4[i]) + __shfl_xor_sync(0xffffffffu, u4 ? a4[i] : a4[i + 2], 4);
  float a1 = (u2 ? a2[1] : a2[0]) + __shfl_xor_sync(0xffffffffu, u2 ? a2[0] : a2[1], 2);
  a1 += __shfl_xor_sync(0xffffffffu, a1, 1);
#pragma unroll
  for (int j = 0; j < 16; j++)
    v[j] = __shfl_sync(0xffffffffu, a1, 16 * ((j >> 3) & 1) + 8 * ((j >> 2) & 1) + 4 * ((j >> 1) & 1) + 2 * (j & 1));
}

// Order-preserving map f32 -> u32 (larger float => larger key); NaN is never produced here.
GG_DEV uint32_t f32_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
GG_DEV float f32_from_order_key(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// dp4a with a signed first operand and a signed / unsigned second operand.
GG_DEV int dp4a_ss(int a, int b, int c) {
  int d;
  asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
GG_DEV int dp4a_su(int a, int b, int c) {
  int d;
  asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// Swizzled float4 slot of logical x element chunk c (16 elements = 4 float4), sub-slot i.
// Eight consecutive chunks read their i-th float4 from eight distinct 16-byte bank groups.
GG_DEV int xswz(int c, int i) { return 4 * c + ((i + (c >> 1)) & 3); }
