// Batch-1 FP8 GEMV for the decode step's attention projections (the
// reference stores q/k/v/o FP8 at rest and casts them to fp16 for every
// F.linear, engine.py:77-82, :100-123): y = W x with W [rows][4096] e4m3
// read directly (half the bytes of the fp16 copy), x [4096] fp16, fp32
// accumulation, fp16 output (optionally times a per-row fp32 scale).
//
// HBM-bound: every weight byte is read once.  A CTA stages x (normalised when
// asked) once in shared memory; each warp then walks groups of R consecutive
// rows, every lane loading 16 contiguous bytes of each row per step (8 steps
// per row, all R x 8 loads in flight before the math) and reading its 16 x
// values of the step from shared memory.  R = 2 or 3 is chosen so that one
// wave of resident warps covers all rows.  e4m3 pairs convert exactly to f16
// pairs; products are f16 x f16 (exact in fp32), sums fp32.
#include "hc_common.cuh"

namespace hcg {
using namespace hc;

constexpr int GEMV_K = 4096;
constexpr int STEPS = GEMV_K / 512;        // 16 bytes per lane per step
constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;

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
// + eps) times the weight): the operand is f16(x * w) and the scalar 1 / rms
// multiplies the fp32 sums.  With `residual`, y = residual + W x in one fp16
// rounding (the decoder layer's x + attention(x)); a row's residual is read
// and its y written by the same lane, so residual may be y itself.
template <bool NORM, int R>
__global__ void __launch_bounds__(GEMV_THREADS, 2) fp8_gemv_kernel(const uint8_t* __restrict__ w,
                                                                 const float* __restrict__ row_scale, int64_t rows,
                                                                 const __half* __restrict__ x,
                                                                 const __half* __restrict__ norm_w, float eps,
                                                                 const __half* residual, __half* y) {
  __shared__ __align__(16) uint32_t xs[GEMV_K / 2];     // the operand as f16 pairs
  __shared__ float red[GEMV_WARPS];
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  // thread t stages elements [16t, 16t + 16)
  {
    const uint4* src = reinterpret_cast<const uint4*>(x + 16 * t);
    const uint4 xa = __ldg(src), xb = __ldg(src + 1);
    uint32_t v[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    float ss = 0.0f;
    if constexpr (NORM) {
      const uint4* wsrc = reinterpret_cast<const uint4*>(norm_w + 16 * t);
      const uint4 c = __ldg(wsrc), d = __ldg(wsrc + 1);
      const uint32_t wv[8] = {c.x, c.y, c.z, c.w, d.x, d.y, d.z, d.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 xf = __half22float2(*reinterpret_cast<const __half2*>(&v[i]));
        const float2 wf = __half22float2(*reinterpret_cast<const __half2*>(&wv[i]));
        ss = fmaf(xf.x, xf.x, fmaf(xf.y, xf.y, ss));
        const __half2 z = __floats2half2_rn(xf.x * wf.x, xf.y * wf.y);
        v[i] = *reinterpret_cast<const uint32_t*>(&z);
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) red[warp] = ss;
    }
    uint4* dst = reinterpret_cast<uint4*>(xs + 8 * t);
    dst[0] = make_uint4(v[0], v[1], v[2], v[3]);
    dst[1] = make_uint4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();
  float rstd = 1.0f;
  if constexpr (NORM) {
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < GEMV_WARPS; ++k) ss += red[k];
    rstd = rsqrtf(ss / (float)GEMV_K + eps);
  }
  const int64_t gw = (int64_t)blockIdx.x * GEMV_WARPS + warp;
  const int64_t nw = (int64_t)gridDim.x * GEMV_WARPS;
  for (int64_t r = gw * R; r < rows; r += nw * R) {
    uint4 a[R][STEPS];
#pragma unroll
    for (int k = 0; k < R; ++k) {
      const int64_t rk = r + k < rows ? r + k : rows - 1;      // a short last group re-reads its last row
      const uint4* wk = reinterpret_cast<const uint4*>(w + rk * GEMV_K) + lane;
#pragma unroll
      for (int s = 0; s < STEPS; ++s) a[k][s] = __ldcs(wk + 32 * s);   // streamed once: evict-first
    }
    float acc[R];
#pragma unroll
    for (int k = 0; k < R; ++k) acc[k] = 0.0f;
#pragma unroll
    for (int s = 0; s < STEPS; ++s) {
      // x elements [512 s + 16 lane, +16) as f16 pairs
      const uint4* xv = reinterpret_cast<const uint4*>(xs + 256 * s + 8 * lane);
      const uint4 p = xv[0], q = xv[1];
      const uint32_t xp[8] = {p.x, p.y, p.z, p.w, q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < R; ++k) acc[k] += dot16(a[k][s], xp);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1)
#pragma unroll
      for (int k = 0; k < R; ++k) acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
    if (lane < R && r + lane < rows) {
      float sum = acc[0];
#pragma unroll
      for (int k = 1; k < R; ++k)
        if (lane == k) sum = acc[k];
      const int64_t rr = r + lane;
      float yv = (row_scale ? sum * __ldg(row_scale + rr) : sum) * rstd;
      if (residual) yv += __half2float(residual[rr]);
      y[rr] = __float2half_rn(yv);
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
  // two CTAs (16 warps) fit an SM; R rows per warp so that one wave covers the rows
  const int64_t resident = 2LL * sms * GEMV_WARPS;
  const int R = rows > 2 * resident ? 3 : 2;
  const int64_t warps_needed = (rows + R - 1) / R;
  int64_t grid = (warps_needed + GEMV_WARPS - 1) / GEMV_WARPS;
  if (grid > 2LL * sms) grid = 2LL * sms;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const __half* xh = static_cast<const __half*>(x);
  const __half* rh = static_cast<const __half*>(residual);
  const __half* nh = static_cast<const __half*>(norm_w);
  __half* yh = static_cast<__half*>(y);
  const int g = (int)grid;
  if (norm_w && R == 3)
    fp8_gemv_kernel<true, 3><<<g, GEMV_THREADS, 0, s>>>(w, row_scale, rows, xh, nh, eps, rh, yh);
  else if (norm_w)
    fp8_gemv_kernel<true, 2><<<g, GEMV_THREADS, 0, s>>>(w, row_scale, rows, xh, nh, eps, rh, yh);
  else if (R == 3)
    fp8_gemv_kernel<false, 3><<<g, GEMV_THREADS, 0, s>>>(w, row_scale, rows, xh, nullptr, 0.0f, rh, yh);
  else
    fp8_gemv_kernel<false, 2><<<g, GEMV_THREADS, 0, s>>>(w, row_scale, rows, xh, nullptr, 0.0f, rh, yh);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_fp8_gemv(const uint8_t* w, const float* row_scale, int64_t rows, int32_t cols, const void* x,
                           void* y, hc_stream_t stream) {
  return hc_fp8_gemv_ex(w, row_scale, rows, cols, x, nullptr, 0.0f, nullptr, y, stream);
}
