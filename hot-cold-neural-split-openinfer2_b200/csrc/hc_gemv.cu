// Batch-1 FP8 GEMV for the decode step's attention projections (the
// reference stores q/k/v/o FP8 at rest and casts them to fp16 for every
// F.linear, engine.py:77-82, :100-123): y = W x with W [rows][4096] e4m3
// read directly (half the bytes of the fp16 copy), x [4096] fp16, fp32
// accumulation, fp16 output (optionally times a per-row fp32 scale).
//
// HBM-bound: every weight byte is read once.  Each warp keeps x in
// registers (128 elements per lane as f16 pairs) and walks rows
// gw, gw + W, ... (W = warps in the grid) two at a time, every lane loading
// 16 contiguous bytes of each row per step (8 steps per row), so a warp has
// 4 KB of each of two rows in flight.  e4m3 pairs convert exactly to f16
// pairs; products are f16 x f16 (exact in fp32), sums fp32.
#include "hc_common.cuh"

namespace hcg {
using namespace hc;

constexpr int GEMV_K = 4096;
constexpr int STEPS = GEMV_K / 512;        // 16 bytes per lane per step
constexpr int GEMV_THREADS = 256;

__device__ __forceinline__ float dot16(const uint4 w, const uint32_t (&xp)[8]) {
  const uint32_t v[4] = {w.x, w.y, w.z, w.w};
  float a = 0.0f, b = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    fma2_f16f16_f32(a, b, e4m3x2_to_f16x2(v[i]), xp[2 * i]);
    fma2_f16f16_f32(a, b, e4m3x2_to_f16x2(v[i] >> 16), xp[2 * i + 1]);
  }
  return a + b;
}

// With `norm_w`, x is RMS-normalised first (torch.nn.RMSNorm: x / sqrt(mean(x^2)
// + eps) times the weight): every warp loads all of x anyway, so it sums the
// squares itself (no block synchronisation) and uses f16(x * w) as the
// operand, applying the scalar 1 / rms to its fp32 sums.  With `residual`,
// y = residual + W x in one fp16 rounding (the decoder layer's x + attention(x)).
template <bool NORM>
__global__ void __launch_bounds__(GEMV_THREADS, 2) fp8_gemv_kernel(const uint8_t* __restrict__ w,
                                                                 const float* __restrict__ row_scale, int64_t rows,
                                                                 const __half* __restrict__ x,
                                                                 const __half* __restrict__ norm_w, float eps,
                                                                 const __half* __restrict__ residual,
                                                                 __half* __restrict__ y) {
  const int lane = threadIdx.x & 31;
  const int64_t gw = (int64_t)blockIdx.x * (GEMV_THREADS / 32) + (threadIdx.x >> 5);
  const int64_t nw = (int64_t)gridDim.x * (GEMV_THREADS / 32);
  // x elements [512 s + 16 lane, +16) for s = 0..7, as f16 pairs
  uint32_t xp[STEPS][8];
  float ss = 0.0f;
#pragma unroll
  for (int s = 0; s < STEPS; ++s) {
    const uint4* src = reinterpret_cast<const uint4*>(x + 512 * s + 16 * lane);
    const uint4 a = __ldg(src), b = __ldg(src + 1);
    xp[s][0] = a.x; xp[s][1] = a.y; xp[s][2] = a.z; xp[s][3] = a.w;
    xp[s][4] = b.x; xp[s][5] = b.y; xp[s][6] = b.z; xp[s][7] = b.w;
    if constexpr (NORM) {
      const uint4* wsrc = reinterpret_cast<const uint4*>(norm_w + 512 * s + 16 * lane);
      const uint4 c = __ldg(wsrc), d = __ldg(wsrc + 1);
      const uint32_t wv[8] = {c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&xp[s][i]));
        const float2 wf = __half22float2(*reinterpret_cast<const __half2*>(&wv[i]));
        ss = fmaf(xf.x, xf.x, fmaf(xf.y, xf.y, ss));
        const __half2 z = __floats2half2_rn(xf.x * wf.x, xf.y * wf.y);
        xp[s][i] = *reinterpret_cast<const uint32_t*>(&z);
      }
    }
  }
  float rstd = 1.0f;
  if constexpr (NORM) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    rstd = rsqrtf(ss / (float)GEMV_K + eps);
  }
  for (int64_t r = gw * 2; r < rows; r += nw * 2) {
    const bool two = r + 1 < rows;
    const uint4* w0 = reinterpret_cast<const uint4*>(w + r * GEMV_K) + lane;
    const uint4* w1 = reinterpret_cast<const uint4*>(w + (two ? r + 1 : r) * GEMV_K) + lane;
    uint4 a[STEPS], b[STEPS];
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      a[s] = __ldcs(w0 + 32 * s);            // streamed once: evict-first
      b[s] = __ldcs(w1 + 32 * s);
    }
    float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      s0 += dot16(a[s], xp[s]);
      s1 += dot16(b[s], xp[s]);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if (lane == 0) {
      float y0 = (row_scale ? s0 * __ldg(row_scale + r) : s0) * rstd;
      if (residual) y0 += __half2float(residual[r]);
      y[r] = __float2half_rn(y0);
      if (two) {
        float y1 = (row_scale ? s1 * __ldg(row_scale + r + 1) : s1) * rstd;
        if (residual) y1 += __half2float(residual[r + 1]);
        y[r + 1] = __float2half_rn(y1);
      }
    }
  }
}

}  // namespace hcg

using namespace hcg;

extern "C" int hc_fp8_gemv_ex(const uint8_t* w, const float* row_scale, int64_t rows, int32_t cols, const void* x,
                              const void* norm_w, float eps, const void* residual, void* y, hc_stream_t stream) {
  if (!w || !x || !y || rows <= 0 || cols != GEMV_K) return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(y) & 1) || (reinterpret_cast<uintptr_t>(norm_w) & 15) ||
      (reinterpret_cast<uintptr_t>(residual) & 1))
    return HC_ERR_ARG;
  if (norm_w && !(eps >= 0.0f)) return HC_ERR_ARG;
  // the residual is read after the products: it must not be overwritten by another row of y
  if (residual && residual != y) {
    const char* r0 = static_cast<const char*>(residual);
    const char* y0 = static_cast<const char*>(y);
    if (r0 < y0 + 2 * rows && y0 < r0 + 2 * rows) return HC_ERR_ARG;
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return HC_ERR_CUDA;
  // two rows per warp per pass; two CTAs (16 warps, ~127 registers a thread) fit an SM
  const int64_t warps_needed = (rows + 1) / 2;
  int64_t grid = (warps_needed + GEMV_THREADS / 32 - 1) / (GEMV_THREADS / 32);
  if (grid > 2LL * sms) grid = 2LL * sms;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* xh = static_cast<const __half*>(x);
  const __half* rh = static_cast<const __half*>(residual);
  __half* yh = static_cast<__half*>(y);
  if (norm_w)
    fp8_gemv_kernel<true><<<(int)grid, GEMV_THREADS, 0, s>>>(w, row_scale, rows, xh,
                                                              static_cast<const __half*>(norm_w), eps, rh, yh);
  else
    fp8_gemv_kernel<false><<<(int)grid, GEMV_THREADS, 0, s>>>(w, row_scale, rows, xh, nullptr, 0.0f, rh, yh);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_fp8_gemv(const uint8_t* w, const float* row_scale, int64_t rows, int32_t cols, const void* x,
                           void* y, hc_stream_t stream) {
  return hc_fp8_gemv_ex(w, row_scale, rows, cols, x, nullptr, 0.0f, nullptr, y, stream);
}
