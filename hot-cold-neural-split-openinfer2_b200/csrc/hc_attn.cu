// One-token decode attention of one layer: RoPE on q and the new k, the new
// k / v written into the KV cache, and causal softmax attention of every query
// head over positions 0..pos of its key-value head (grouped-query attention:
// query head h reads key-value head h / g, the reference's repeat_interleave,
// engine.py:100-125, rotary embedding engine.py:130-158).
//
// One thread-block cluster of CL CTAs per key-value head splits the sequence
// (flash-decoding): CTA r covers positions [r c, (r+1) c), c = ceil((pos+1)/CL),
// for the g query heads of the key-value head, keeping a running max, sum and
// weighted value sum per head (online softmax in fp32).  The CTAs' partials
// are combined through distributed shared memory after a cluster barrier (the
// hardware keeps a cluster's CTAs co-resident, so the barrier cannot wait on a
// CTA that is not running); each CTA then writes its share of the heads'
// outputs.  The CTA whose range holds `pos` writes the new k / v into the
// cache and uses them from shared memory; no other CTA reads that position.
//
// The position is read from device memory, so a captured CUDA graph replays
// the step as the position advances.  HBM-bound: 2 x (pos + 1) x 256 bytes of
// cache per key-value head.  Cached rows are loaded a round ahead of their
// math (in-order issue would otherwise pay one memory round trip per round).
#include <cooperative_groups.h>

#include "hc_common.cuh"

namespace hca {
using namespace hc;
namespace cg = cooperative_groups;

constexpr int D = 128;              // head dimension (the kernel's only one)
constexpr int GLIM = 8;             // query heads per key-value head, at most
constexpr int CL = 8;               // CTAs per key-value head (one cluster, a portable size)
constexpr int U = 8;                // positions a warp loads per round
constexpr int THREADS = 256;
constexpr int WARPS = THREADS / 32;

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
  int32_t* status;
};

template <int GM>
struct Smem {
  float qs[GM][D];                  // rotated, scaled q of the g heads
  float wm[WARPS][GM], wl[WARPS][GM];
  float wo[WARPS][GM][D];           // per-warp running values
  float pm[GM], pl[GM];             // this CTA's partial (read by the cluster)
  float po[GM][D];
  __align__(16) __half knew[D];
  __align__(16) __half vnew[D];
};

// GM: the largest group size the instance handles (g <= GM)
template <int GM>
__global__ void __launch_bounds__(THREADS) attn_decode_kernel(const AttnParams p) {
  constexpr int GMAX = GM;
  __shared__ Smem<GM> sm;
  cg::cluster_group cluster = cg::this_cluster();
  const int t = threadIdx.x, lane = t & 31, w = t >> 5;
  const int r = (int)cluster.block_rank();
  const int h = blockIdx.x / CL;
  const int g = p.g;

  // the token's q (and new k) pairs this thread rotates: loaded before anything
  // that depends on the position
  float qa[GMAX], qb[GMAX], ka = 0.0f, kb = 0.0f;
#pragma unroll
  for (int i = 0; i < GMAX; ++i) {
    qa[i] = 0.0f;
    qb[i] = 0.0f;
  }
  if (t < D / 2) {
#pragma unroll
    for (int i = 0; i < GMAX; ++i) {
      if (i < g) {
        const __half* q = p.qkv + (size_t)(h * g + i) * D;
        qa[i] = __half2float(q[t]);
        qb[i] = __half2float(q[t + D / 2]);
      }
    }
    const __half* k = p.qkv + (size_t)p.nq * D + (size_t)h * D;
    ka = __half2float(k[t]);
    kb = __half2float(k[t + D / 2]);
  }
  const int64_t pos64 = *p.pos;
  const bool bad = pos64 < 0 || pos64 >= p.cap;    // every CTA sees the same position
  if (bad && t == 0 && blockIdx.x == 0) atomicOr(p.status, HC_ERR_RANGE);
  const int pos = bad ? 0 : (int)pos64;
  const int n = bad ? 0 : pos + 1, chunk = (n + CL - 1) / CL;
  const int j0 = min(n, r * chunk), j1 = min(n, j0 + chunk);
  const bool holds = !bad && j0 <= pos && pos < j1;

  const __half* kbase = p.kc + (size_t)h * p.cap * D + 4 * lane;
  const __half* vbase = p.vc + (size_t)h * p.cap * D + 4 * lane;
  // warp w takes positions j0 + w, j0 + w + WARPS, ... in rounds of U; lane owns
  // dimensions [4 lane, 4 lane + 4)
  auto load_round = [&](int jb, uint2 (&kr)[U], uint2 (&vr)[U]) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = jb + u * WARPS;
      kr[u] = make_uint2(0u, 0u);
      vr[u] = make_uint2(0u, 0u);
      if (j < j1 && j != pos) {
        kr[u] = __ldcg(reinterpret_cast<const uint2*>(kbase + (size_t)j * D));
        vr[u] = __ldcg(reinterpret_cast<const uint2*>(vbase + (size_t)j * D));
      }
    }
  };
  uint2 kr[U], vr[U];
  load_round(j0 + w, kr, vr);

  // RoPE: pairs (d, d + D/2) rotated by the position's angle, in fp32
  if (t < D / 2 && !bad) {
    const float c = __ldg(p.cos_t + (size_t)pos * (D / 2) + t), sn = __ldg(p.sin_t + (size_t)pos * (D / 2) + t);
#pragma unroll
    for (int i = 0; i < GMAX; ++i) {
      if (i >= g) continue;
      sm.qs[i][t] = (qa[i] * c - qb[i] * sn) * p.scale;
      sm.qs[i][t + D / 2] = (qa[i] * sn + qb[i] * c) * p.scale;
    }
    if (holds) {                            // cache the new k (rotated)
      const __half k0 = __float2half_rn(ka * c - kb * sn), k1 = __float2half_rn(ka * sn + kb * c);
      __half* kd = p.kc + ((size_t)h * p.cap + pos) * D;
      kd[t] = k0;
      kd[t + D / 2] = k1;
      sm.knew[t] = k0;
      sm.knew[t + D / 2] = k1;
    }
  }
  if (holds && t < D) {                     // and v
    const __half v = p.qkv[(size_t)(p.nq + p.nkv) * D + (size_t)h * D + t];
    p.vc[((size_t)h * p.cap + pos) * D + t] = v;
    sm.vnew[t] = v;
  }
  __syncthreads();

  float qv[GMAX][4];
#pragma unroll
  for (int i = 0; i < GMAX; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) qv[i][e] = i < g ? sm.qs[i][4 * lane + e] : 0.0f;
  float m[GMAX], l[GMAX], o[GMAX][4];
#pragma unroll
  for (int i = 0; i < GMAX; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.0f;
  }
  for (int jb = j0 + w; jb < j1; jb += WARPS * U) {
    uint2 kn[U], vn[U];
    load_round(jb + WARPS * U, kn, vn);           // the next round's rows in flight during this one's math
    if (holds) {
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (jb + u * WARPS == pos) {
          kr[u] = *reinterpret_cast<const uint2*>(sm.knew + 4 * lane);
          vr[u] = *reinterpret_cast<const uint2*>(sm.vnew + 4 * lane);
        }
    }
    float sc[U][GMAX];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&kr[u].x));
      const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&kr[u].y));
#pragma unroll
      for (int i = 0; i < GMAX; ++i)
        sc[u][i] = fmaf(qv[i][0], k01.x, fmaf(qv[i][1], k01.y, fmaf(qv[i][2], k23.x, qv[i][3] * k23.y)));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1)
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int i = 0; i < GMAX; ++i)
          if (i < g) sc[u][i] += __shfl_xor_sync(0xffffffffu, sc[u][i], off);
#pragma unroll
    for (int i = 0; i < GMAX; ++i) {
      if (i >= g) continue;
      float mx = m[i];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (jb + u * WARPS < j1) mx = fmaxf(mx, sc[u][i]);
      const float keep = __expf(m[i] - mx);      // 0 on the first round (m = -inf)
      m[i] = mx;
      l[i] *= keep;
#pragma unroll
      for (int e = 0; e < 4; ++e) o[i][e] *= keep;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (jb + u * WARPS >= j1) continue;
        const float pj = __expf(sc[u][i] - mx);
        const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vr[u].x));
        const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vr[u].y));
        l[i] += pj;
        o[i][0] = fmaf(pj, v01.x, o[i][0]);
        o[i][1] = fmaf(pj, v01.y, o[i][1]);
        o[i][2] = fmaf(pj, v23.x, o[i][2]);
        o[i][3] = fmaf(pj, v23.y, o[i][3]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      kr[u] = kn[u];
      vr[u] = vn[u];
    }
  }

  // this CTA's partial: its warps' running values combined in shared memory
#pragma unroll
  for (int i = 0; i < GMAX; ++i) {
    if (i >= g) continue;
    if (lane == 0) {
      sm.wm[w][i] = m[i];
      sm.wl[w][i] = l[i];
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) sm.wo[w][i][4 * lane + e] = o[i][e];
  }
  __syncthreads();
  for (int item = t; item < g * D; item += THREADS) {
    const int i = item / D, d = item % D;
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < WARPS; ++k) M = fmaxf(M, sm.wm[k][i]);
    float L = 0.0f, O = 0.0f;
    if (M != -INFINITY) {
#pragma unroll
      for (int k = 0; k < WARPS; ++k) {
        const float f = __expf(sm.wm[k][i] - M);    // 0 for a warp without positions
        L = fmaf(sm.wl[k][i], f, L);
        O = fmaf(sm.wo[k][i][d], f, O);
      }
    }
    sm.po[i][d] = O;
    if (d == 0) {
      sm.pm[i] = M;
      sm.pl[i] = L;
    }
  }
  // every CTA's partial is complete and visible to the cluster
  cluster.sync();
  if (!bad) {
    // CTA r writes outputs [r (g D) / CL, (r+1) (g D) / CL), reading the CL partials
    const int lo = r * (g * D) / CL, hi = (r + 1) * (g * D) / CL;
    for (int item = lo + t; item < hi; item += THREADS) {
      const int i = item / D, d = item % D;
      float mk[CL];
      float M = -INFINITY;
#pragma unroll
      for (int k = 0; k < CL; ++k) {
        const Smem<GM>* rs = cluster.map_shared_rank(&sm, k);
        mk[k] = rs->pm[i];
        M = fmaxf(M, mk[k]);
      }
      float L = 0.0f, O = 0.0f;
#pragma unroll
      for (int k = 0; k < CL; ++k) {
        if (mk[k] == -INFINITY) continue;            // a CTA whose range was empty
        const Smem<GM>* rs = cluster.map_shared_rank(&sm, k);
        const float f = __expf(mk[k] - M);
        L = fmaf(rs->pl[i], f, L);
        O = fmaf(rs->po[i][d], f, O);
      }
      p.out[(size_t)(h * g + i) * D + d] = __float2half_rn(O / L);
    }
  }
  // no CTA leaves (its shared memory) while another may still read it
  cluster.sync();
}

}  // namespace hca

using namespace hca;

extern "C" int hc_attn_decode(const void* qkv, const float* cos_t, const float* sin_t, const int64_t* pos,
                              void* k_cache, void* v_cache, int32_t capacity, int32_t n_q_heads,
                              int32_t n_kv_heads, int32_t head_dim, void* out, int32_t* status, hc_stream_t stream) {
  if (!qkv || !cos_t || !sin_t || !pos || !k_cache || !v_cache || !out || !status) return HC_ERR_ARG;
  if (head_dim != D || capacity <= 0 || n_q_heads <= 0 || n_kv_heads <= 0 || n_q_heads % n_kv_heads ||
      n_q_heads / n_kv_heads > GLIM || n_kv_heads > 65535 / CL)
    return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15) ||
      (reinterpret_cast<uintptr_t>(qkv) & 1) || (reinterpret_cast<uintptr_t>(out) & 1))
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
  p.status = status;
  const int g = p.g;
  void (*kern)(AttnParams) = g <= 1 ? attn_decode_kernel<1>
                           : g <= 2 ? attn_decode_kernel<2>
                           : g <= 4 ? attn_decode_kernel<4>
                                    : attn_decode_kernel<8>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(n_kv_heads * CL);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, p) == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}
