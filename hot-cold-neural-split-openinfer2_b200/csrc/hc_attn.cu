// One-token decode attention of one layer: RoPE on q and the new k, the new
// k / v written into the KV cache, and causal softmax attention of every query
// head over positions 0..pos of its key-value head (grouped-query attention:
// query head h reads key-value head h / g, the reference's repeat_interleave,
// engine.py:100-125, rotary embedding engine.py:130-158).
//
// The sequence is split over SPLIT CTAs per key-value head (flash-decoding):
// CTA (h, s) covers positions [s c, (s+1) c) with c = ceil((pos + 1) / SPLIT)
// for the g query heads of key-value head h, keeping a running max, sum and
// weighted value sum per head (online softmax in fp32), and writes them to the
// workspace.  The CTA that finishes last for a key-value head (an atomic
// counter; nothing waits) combines the SPLIT partials and writes the heads'
// outputs.  The CTA whose range holds `pos` writes the new k / v into the
// cache first and reads them back like every other position: no other CTA
// reads that position.
//
// The position is read from device memory, so a captured CUDA graph replays
// the step as the position advances.  HBM-bound: 2 x (pos + 1) x 256 bytes of
// cache per key-value head.
#include "hc_common.cuh"

namespace hca {
using namespace hc;

constexpr int D = 128;              // head dimension (the kernel's only one)
constexpr int GMAX = 8;             // query heads per key-value head
constexpr int SPLIT = 16;           // CTAs per key-value head
constexpr int THREADS = 128;        // 4 warps; thread t owns dimension t in the prologue and the combines
constexpr int WARPS = THREADS / 32;
constexpr int PART = D + 2;         // per head: weighted value sum [D], running max, running sum

struct AttnParams {
  const __half* qkv;      // [nq D + 2 nkv D]: q, k, v of the token, before RoPE
  const float* cos_t;     // [cap][D / 2]
  const float* sin_t;
  const int64_t* pos;     // device scalar: the token's position
  __half* kc;             // [nkv][cap][D] this layer's key cache
  __half* vc;
  int cap, nq, nkv, g;
  float scale;            // 1 / sqrt(D)
  __half* out;            // [nq D]
  float* part;            // [nkv][SPLIT][g][PART]
  uint32_t* count;        // [nkv], zero between launches
  int32_t* status;
};

__global__ void __launch_bounds__(THREADS) attn_decode_kernel(const AttnParams p) {
  __shared__ float qs[GMAX][D];
  __shared__ float wm[WARPS][GMAX], wl[WARPS][GMAX];
  __shared__ float wo[WARPS][GMAX][D];
  __shared__ int last_s;
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int h = blockIdx.x / SPLIT, s = blockIdx.x % SPLIT;
  const int g = p.g;
  const int64_t pos64 = *p.pos;
  if (pos64 < 0 || pos64 >= p.cap) {        // every CTA sees the same position: all stop here
    if (t == 0 && blockIdx.x == 0) atomicOr(p.status, HC_ERR_RANGE);
    return;
  }
  const int pos = (int)pos64;
  const int n = pos + 1, chunk = (n + SPLIT - 1) / SPLIT;
  const int j0 = min(n, s * chunk), j1 = min(n, j0 + chunk);

  // RoPE: pairs (d, d + D/2) rotated by the position's angle, in fp32
  if (t < D / 2) {
    const float c = __ldg(p.cos_t + (size_t)pos * (D / 2) + t), sn = __ldg(p.sin_t + (size_t)pos * (D / 2) + t);
    for (int i = 0; i < g; ++i) {
      const __half* q = p.qkv + (size_t)(h * g + i) * D;
      const float a = __half2float(q[t]), b = __half2float(q[t + D / 2]);
      qs[i][t] = (a * c - b * sn) * p.scale;
      qs[i][t + D / 2] = (a * sn + b * c) * p.scale;
    }
    if (j0 <= pos && pos < j1) {            // this CTA holds the new position: cache its k (rotated) and v
      const __half* k = p.qkv + (size_t)p.nq * D + (size_t)h * D;
      const float a = __half2float(k[t]), b = __half2float(k[t + D / 2]);
      __half* kd = p.kc + ((size_t)h * p.cap + pos) * D;
      kd[t] = __float2half_rn(a * c - b * sn);
      kd[t + D / 2] = __float2half_rn(a * sn + b * c);
    }
  }
  if (j0 <= pos && pos < j1) {
    const __half* v = p.qkv + (size_t)(p.nq + p.nkv) * D + (size_t)h * D;
    p.vc[((size_t)h * p.cap + pos) * D + t] = v[t];
  }
  __syncthreads();

  // warp w takes positions j0 + w, j0 + w + WARPS, ...; lane owns dimensions [4 lane, 4 lane + 4)
  float qv[GMAX][4];
#pragma unroll
  for (int i = 0; i < GMAX; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) qv[i][e] = i < g ? qs[i][4 * lane + e] : 0.0f;
  float m[GMAX], l[GMAX], o[GMAX][4];
#pragma unroll
  for (int i = 0; i < GMAX; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.0f;
  }
  const __half* kbase = p.kc + (size_t)h * p.cap * D + 4 * lane;
  const __half* vbase = p.vc + (size_t)h * p.cap * D + 4 * lane;
  for (int j = j0 + w; j < j1; j += WARPS) {
    const uint2 kr = __ldcg(reinterpret_cast<const uint2*>(kbase + (size_t)j * D));
    const uint2 vr = __ldcg(reinterpret_cast<const uint2*>(vbase + (size_t)j * D));
    const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kr.x));
    const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kr.y));
    const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vr.x));
    const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vr.y));
    float sc[GMAX];
#pragma unroll
    for (int i = 0; i < GMAX; ++i)
      sc[i] = fmaf(qv[i][0], k01.x, fmaf(qv[i][1], k01.y, fmaf(qv[i][2], k23.x, qv[i][3] * k23.y)));
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
      for (int i = 0; i < GMAX; ++i)
        if (i < g) sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], off);
#pragma unroll
    for (int i = 0; i < GMAX; ++i) {
      if (i >= g) continue;
      const float mn = fmaxf(m[i], sc[i]);
      const float keep = __expf(m[i] - mn), pj = __expf(sc[i] - mn);
      m[i] = mn;
      l[i] = fmaf(l[i], keep, pj);
      o[i][0] = fmaf(o[i][0], keep, pj * v01.x);
      o[i][1] = fmaf(o[i][1], keep, pj * v01.y);
      o[i][2] = fmaf(o[i][2], keep, pj * v23.x);
      o[i][3] = fmaf(o[i][3], keep, pj * v23.y);
    }
  }
  // the CTA's partial: the four warps' running values combined
#pragma unroll
  for (int i = 0; i < GMAX; ++i) {
    if (i >= g) continue;
    if (lane == 0) {
      wm[w][i] = m[i];
      wl[w][i] = l[i];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) wo[w][i][4 * lane + e] = o[i][e];
  }
  __syncthreads();
  float* mine = p.part + ((size_t)h * SPLIT + s) * g * PART;
  for (int i = 0; i < g; ++i) {
    float M = -INFINITY;
    for (int k = 0; k < WARPS; ++k) M = fmaxf(M, wm[k][i]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
      for (int k = 0; k < WARPS; ++k) {
        const float f = __expf(wm[k][i] - M);      // 0 for a warp without positions
        L = fmaf(wl[k][i], f, L);
        O = fmaf(wo[k][i][t], f, O);
      }
    }
    mine[i * PART + t] = O;
    if (t == 0) {
      mine[i * PART + D] = M;
      mine[i * PART + D + 1] = L;
    }
  }
  // the last CTA of this key-value head combines the SPLIT partials
  __threadfence();
  __syncthreads();
  if (t == 0) last_s = atomicAdd(p.count + h, 1u) == (uint32_t)SPLIT - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();
  const float* all = p.part + (size_t)h * SPLIT * g * PART;
  for (int i = 0; i < g; ++i) {
    float M = -INFINITY;
    for (int k = 0; k < SPLIT; ++k) M = fmaxf(M, __ldcg(all + ((size_t)k * g + i) * PART + D));
    float L = 0.0f, O = 0.0f;
    for (int k = 0; k < SPLIT; ++k) {
      const float mk = __ldcg(all + ((size_t)k * g + i) * PART + D);
      if (mk == -INFINITY) continue;                 // a CTA whose range was empty
      const float f = __expf(mk - M);
      L = fmaf(__ldcg(all + ((size_t)k * g + i) * PART + D + 1), f, L);
      O = fmaf(__ldcg(all + ((size_t)k * g + i) * PART + t), f, O);
    }
    p.out[(size_t)(h * g + i) * D + t] = __float2half_rn(O / L);
  }
  if (t == 0) p.count[h] = 0u;                      // ready for the next launch (stream order)
}

}  // namespace hca

using namespace hca;

extern "C" int64_t hc_attn_decode_workspace_bytes(int32_t n_q_heads, int32_t n_kv_heads) {
  if (n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads || n_q_heads / n_kv_heads > GMAX) return -1;
  const int64_t g = n_q_heads / n_kv_heads;
  return 256 + (int64_t)sizeof(float) * n_kv_heads * SPLIT * g * PART;
}

extern "C" int hc_attn_decode(const void* qkv, const float* cos_t, const float* sin_t, const int64_t* pos,
                              void* k_cache, void* v_cache, int32_t capacity, int32_t n_q_heads,
                              int32_t n_kv_heads, int32_t head_dim, void* out, void* workspace, int32_t* status,
                              hc_stream_t stream) {
  if (!qkv || !cos_t || !sin_t || !pos || !k_cache || !v_cache || !out || !workspace || !status) return HC_ERR_ARG;
  if (head_dim != D || capacity <= 0 || hc_attn_decode_workspace_bytes(n_q_heads, n_kv_heads) < 0)
    return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15) || (reinterpret_cast<uintptr_t>(qkv) & 1) ||
      (reinterpret_cast<uintptr_t>(out) & 1))
    return HC_ERR_ARG;
  AttnParams p;
  p.qkv = static_cast<const __half*>(qkv);
  p.cos_t = cos_t;
  p.sin_t = sin_t;
  p.pos = pos;
  p.kc = static_cast<__half*>(k_cache);
  p.vc = static_cast<__half*>(v_cache);
  p.cap = capacity;
  p.nq = n_q_heads;
  p.nkv = n_kv_heads;
  p.g = n_q_heads / n_kv_heads;
  p.scale = 1.0f / sqrtf((float)D);
  p.out = static_cast<__half*>(out);
  p.count = static_cast<uint32_t*>(workspace);                            // first 256 bytes: counters
  p.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + 256);
  p.status = status;
  if (n_kv_heads > 64) return HC_ERR_UNSUPPORTED;                         // the counters' 256 bytes
  attn_decode_kernel<<<n_kv_heads * SPLIT, THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}
