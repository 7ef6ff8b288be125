// Shared device helpers for the hot/cold sparse-FFN kernels (sm_100a only).
//
// Format constants restate the reference's cold-record layout
// (splitter.py:57-76): hidden 4096, INT4 group 128, 6400-byte records of
// [u16 nid][gate 2048 B][up 2048 B][down 2048 B][3 x 32 fp16 scales][pad].
#pragma once

#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hotcold.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "hotcold kernels are written for sm_100a only"
#endif

namespace hc {

constexpr int H = 4096;                  // hidden dim (splitter.py:59)
constexpr int VEC_BYTES = H / 2;         // 2048 B of INT4 per vector (splitter.py:69)
constexpr int GROUP = 128;               // INT4 group (splitter.py:70)
constexpr int NGROUPS = H / GROUP;       // 32 (splitter.py:71)
constexpr int REC_BYTES = 6400;          // NEURON_RECORD_BYTES (splitter.py:76)
constexpr int REC_COPY = 6352;           // 6338 payload bytes rounded up to 16
constexpr int SCALE_OFF = 2 + 3 * VEC_BYTES;   // 6146: first fp16 scale
constexpr int SECTION_HEADER = 16;       // '<HHIq' (splitter.py:230)
constexpr int TABLE_SIZE = 65536;        // u16 neuron ids

// ----------------------------------------------------------------------------
// address / memory helpers
// ----------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ----------------------------------------------------------------------------
// mbarrier + bulk copy (TMA engine, 1-D form: 16-B aligned, size % 16 == 0)
// ----------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// non-blocking probe of the phase with parity `parity`
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// blocking probe that suspends the thread for at most ~hint_ns
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase completed, false once `limit_ns` passed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// global -> shared bulk copy completing on `bar` (transaction bytes).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// fire-and-forget L2 prefetch of [src, src + bytes) (16-B aligned, size % 16 == 0)
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2_range(const void* src, size_t bytes) {
  const char* p = static_cast<const char*>(src);
  for (size_t off = 0; off < bytes; off += 32768) {
    const size_t n = bytes - off < 32768 ? bytes - off : 32768;
    prefetch_l2(p + off, static_cast<uint32_t>(n));
  }
}

// named barrier among `nthreads` threads (id 0 is __syncthreads)
__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ----------------------------------------------------------------------------
// element decoders
// ----------------------------------------------------------------------------
// 8 packed signed INT4 (element 2i in the low nibble of byte i) -> fp32.
// Arithmetic shift sign-extends the nibble: 8..15 -> -8..-1 (splitter.py:119-120).
__device__ __forceinline__ void int4x8_to_f32(uint32_t w, float f[8]) {
#pragma unroll
  for (int e = 0; e < 8; ++e) f[e] = static_cast<float>(static_cast<int32_t>(w << (28 - 4 * e)) >> 28);
}

// e4m3x2 (low byte -> low half) -> f16x2, exact
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t w16) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(static_cast<unsigned short>(w16 & 0xFFFFu)));
  return r;
}

// y0 += lo(h2) * b, y1 += hi(h2) * b: f16 x f16 products (exact in fp32), fp32 accumulate
__device__ __forceinline__ void fma2_f16_f32(float& y0, float& y1, uint32_t h2, unsigned short b) {
  asm("{\n\t.reg .f16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\t"
      "fma.rn.f32.f16 %0, lo, %3, %0;\n\tfma.rn.f32.f16 %1, hi, %3, %1;\n\t}"
      : "+f"(y0), "+f"(y1)
      : "r"(h2), "h"(b));
}

// a += lo(w) * lo(x), b += hi(w) * hi(x): f16 x f16 products, fp32 accumulate
__device__ __forceinline__ void fma2_f16f16_f32(float& a, float& b, uint32_t w, uint32_t x) {
  asm("{\n\t.reg .f16 wl, wh, xl, xh;\n\tmov.b32 {wl, wh}, %2;\n\tmov.b32 {xl, xh}, %3;\n\t"
      "fma.rn.f32.f16 %0, wl, xl, %0;\n\tfma.rn.f32.f16 %1, wh, xh, %1;\n\t}"
      : "+f"(a), "+f"(b)
      : "r"(w), "r"(x));
}

// bytes [2 .. 6) of the 8-byte pair (a, b): the 2-byte shift every record field has
__device__ __forceinline__ uint32_t shift2(uint32_t a, uint32_t b) { return __funnelshift_r(a, b, 16); }

// 4-way byte dot products with 32-bit accumulate: a unsigned bytes, b signed / unsigned bytes
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ uint32_t dp4a_uu(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// ----------------------------------------------------------------------------
// activation (engine.py:163-170)
// ----------------------------------------------------------------------------
__device__ __forceinline__ float act_one(float v, int relu) {
  return relu ? fmaxf(v, 0.0f) : v / (1.0f + __expf(-v));
}
__device__ __forceinline__ float gated(float g, float u, int relu, int both) {
  return both ? act_one(g, relu) * act_one(u, relu) : act_one(g, relu) * u;
}

// ----------------------------------------------------------------------------
// warp reduction of V values at once: afterwards lane L holds the warp sum of
// value (L >> (5 - log2 V)); V - 1 + 5 - log2(V) shuffles instead of 5 V.
// ----------------------------------------------------------------------------
template <int V>
__device__ __forceinline__ float warp_reduce_multi(float (&v)[V]) {
  static_assert(V >= 1 && V <= 32 && (V & (V - 1)) == 0, "V must be a power of two <= 32");
  const int lane = threadIdx.x & 31;
  int n = V;
#pragma unroll
  for (int o = 16; o >= 1 && n > 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
    const int h = n >> 1;
#pragma unroll
    for (int i = 0; i < V / 2; ++i) {
      if (i < h) {
        const float keep = upper ? v[i + h] : v[i];
        const float send = upper ? v[i] : v[i + h];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
      }
    }
    n = h;
  }
  float r = v[0];
  constexpr int LOGV = (V >= 32) ? 5 : (V >= 16) ? 4 : (V >= 8) ? 3 : (V >= 4) ? 2 : (V >= 2) ? 1 : 0;
#pragma unroll
  for (int o = (16 >> LOGV); o >= 1; o >>= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

}  // namespace hc
