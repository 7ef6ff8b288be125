// Fused low-rank activation predictor (predictor.py:55-96 NeuronPredictor,
// :435-456 PredictorRegistry.predict) and the cold-id selection of
// SparseFFNLayer._cold_ids_for (engine.py:274-283).
//
//   z      = W_down x                (rank x 4096, fp32)
//   logit  = W_up z + b              (inter x rank)
//   mask   = logit >= logit_threshold  (== sigmoid(logit) >= threshold, the
//            host derives the logit threshold from torch's own sigmoid)
//   ids    = ascending ids of mask & fetch_bits   (nonzero() minus hot ids,
//            minus ids without a record -- read_neurons skips those)
//
// Two launches, no host synchronisation:
//   1. pred_down_kernel: one CTA per 128-wide K chunk writes partial z; the
//      last CTA to finish sums the partials in fixed order into z.
//   2. pred_up_kernel:  one thread per neuron computes the logit, ballots the
//      mask word; the last CTA compacts row 0 into the ordered id list.
#include "hc_common.cuh"

#include <cuda.h>

#include <mutex>

namespace hc {

constexpr int PRED_KCHUNK = 128;
constexpr int PRED_MAX_RANK = 128;
constexpr int PRED_MAX_BATCH = 64;

struct PredWs {
  uint32_t* done_down;   // last-block counter of kernel 1
  uint32_t* done_up;     // last-block counter of kernel 2
  float* zpart;          // [H / 128][batch][rank]
  float* z;              // [batch][rank]
};

__host__ __device__ inline PredWs pred_ws(void* base, int batch, int rank) {
  PredWs w;
  char* p = static_cast<char*>(base);
  w.done_down = reinterpret_cast<uint32_t*>(p);
  w.done_up = reinterpret_cast<uint32_t*>(p + 128);
  w.zpart = reinterpret_cast<float*>(p + 256);
  w.z = w.zpart + (size_t)(H / PRED_KCHUNK) * batch * rank;
  return w;
}

__global__ void __launch_bounds__(256) pred_down_kernel(const float* __restrict__ x, int batch,
                                                        const float* __restrict__ norm_w, float eps,
                                                        const float* __restrict__ w_down, int rank, PredWs ws) {
  __shared__ float xs[PRED_MAX_BATCH][PRED_KCHUNK];
  __shared__ float rstd[PRED_MAX_BATCH];
  __shared__ bool last;
  const int chunk = blockIdx.x;
  const int k0 = chunk * PRED_KCHUNK;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (norm_w != nullptr) {
    // RMSNorm of every row (torch.nn.RMSNorm: x * rsqrt(mean(x^2) + eps) * w),
    // recomputed by each CTA over the full row
    for (int b = warp; b < batch; b += 8) {
      const float4* row = reinterpret_cast<const float4*>(x + (size_t)b * H);
      float ss = 0.0f;
      for (int i = lane; i < H / 4; i += 32) {
        const float4 v = __ldg(row + i);
        ss = fmaf(v.x, v.x, ss); ss = fmaf(v.y, v.y, ss); ss = fmaf(v.z, v.z, ss); ss = fmaf(v.w, v.w, ss);
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) rstd[b] = rsqrtf(ss / (float)H + eps);
    }
    __syncthreads();
  }
  for (int i = tid; i < batch * PRED_KCHUNK; i += 256) {
    const int b = i / PRED_KCHUNK, kk = i % PRED_KCHUNK;
    float v = x[(size_t)b * H + k0 + kk];
    if (norm_w != nullptr) v = v * rstd[b] * __ldg(norm_w + k0 + kk);
    xs[b][kk] = v;
  }
  __syncthreads();
  // warp per rank row: lane covers k0 + 4*lane .. +3 (one float4)
  for (int r = warp; r < rank; r += 8) {
    const float4 w = __ldg(reinterpret_cast<const float4*>(w_down + (size_t)r * H + k0) + lane);
    for (int b = 0; b < batch; ++b) {
      const float* xb = &xs[b][4 * lane];
      float acc = w.x * xb[0];
      acc = fmaf(w.y, xb[1], acc);
      acc = fmaf(w.z, xb[2], acc);
      acc = fmaf(w.w, xb[3], acc);
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) ws.zpart[((size_t)chunk * batch + b) * rank + r] = acc;
    }
  }
  // last CTA reduces the partials in chunk order (deterministic)
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(ws.done_down, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int i = tid; i < batch * rank; i += 256) {
    float s = 0.0f;
    for (int c = 0; c < (int)gridDim.x; ++c) s += __ldcg(ws.zpart + (size_t)c * batch * rank + i);
    ws.z[i] = s;
  }
  if (tid == 0) *ws.done_down = 0;
}

__global__ void __launch_bounds__(256) pred_up_kernel(int batch, const float* __restrict__ w_up,
                                                      const float* __restrict__ b_up, int rank, int inter,
                                                      float thr, uint32_t* __restrict__ mask_out,
                                                      float* __restrict__ probs_out, float* __restrict__ logits_out,
                                                      const uint32_t* __restrict__ fetch_bits,
                                                      const int32_t* __restrict__ table, int32_t* __restrict__ ids_out,
                                                      int32_t* __restrict__ rec_out, int32_t* __restrict__ count_out,
                                                      PredWs ws) {
  __shared__ float zs[PRED_MAX_RANK * 8];
  __shared__ bool last;
  __shared__ int wtot[8];
  __shared__ int base_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = blockIdx.x * 256 + tid;
  const int words = (inter + 31) / 32;
  const float bias = (n < inter) ? __ldg(b_up + n) : 0.0f;
  for (int b0 = 0; b0 < batch; b0 += 8) {
    const int nb = min(8, batch - b0);
    __syncthreads();
    for (int i = tid; i < nb * rank; i += 256) zs[i] = __ldcg(ws.z + (size_t)b0 * rank + i);
    __syncthreads();
    float acc[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[b] = 0.0f;
    if (n < inter) {
      const float4* row = reinterpret_cast<const float4*>(w_up + (size_t)n * rank);
      for (int r4 = 0; r4 < rank / 4; ++r4) {
        const float4 w = __ldg(row + r4);
#pragma unroll
        for (int b = 0; b < 8; ++b) {
          if (b < nb) {
            const float* zb = zs + b * rank + 4 * r4;
            acc[b] = fmaf(w.x, zb[0], acc[b]);
            acc[b] = fmaf(w.y, zb[1], acc[b]);
            acc[b] = fmaf(w.z, zb[2], acc[b]);
            acc[b] = fmaf(w.w, zb[3], acc[b]);
          }
        }
      }
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (b < nb) {
        const float lg = acc[b] + bias;
        const bool on = (n < inter) && (lg >= thr);
        const unsigned bits = __ballot_sync(0xffffffffu, on);
        const int word = n >> 5;
        if (lane == 0 && word < words) mask_out[(size_t)(b0 + b) * words + word] = bits;
        if (n < inter) {
          if (logits_out) logits_out[(size_t)(b0 + b) * inter + n] = lg;
          if (probs_out) probs_out[(size_t)(b0 + b) * inter + n] = 1.0f / (1.0f + expf(-lg));
        }
      }
    }
  }
  if (fetch_bits == nullptr) return;
  // last CTA: ordered compaction of row 0 (ascending id == nonzero() order)
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(ws.done_up, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (tid == 0) base_s = 0;
  __syncthreads();
  for (int w0 = 0; w0 < words; w0 += 256) {
    const int w = w0 + tid;
    const uint32_t bits = (w < words) ? (__ldcg(mask_out + w) & __ldg(fetch_bits + w)) : 0u;
    const int c = __popc(bits);
    int incl = c;
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) wtot[warp] = incl;
    __syncthreads();
    int wbase = base_s;
    for (int i = 0; i < warp; ++i) wbase += wtot[i];
    int pos = wbase + incl - c;
    uint32_t m = bits;
    while (m) {
      const int bit = __ffs(m) - 1;
      m &= m - 1;
      const int id = w * 32 + bit;
      ids_out[pos] = id;
      if (rec_out) rec_out[pos] = table ? table[id] : -1;
      ++pos;
    }
    __syncthreads();
    if (tid == 0) {
      int tot = 0;
      for (int i = 0; i < 8; ++i) tot += wtot[i];
      base_s += tot;
    }
    __syncthreads();
  }
  if (tid == 0) {
    *count_out = base_s;
    *ws.done_up = 0;
  }
}

}  // namespace hc

using namespace hc;

extern "C" int64_t hc_predictor_workspace_bytes(int32_t batch, int32_t rank, int32_t inter) {
  (void)inter;
  if (batch <= 0 || rank <= 0) return -1;
  return 256 + (int64_t)sizeof(float) * ((H / PRED_KCHUNK) * batch * rank + batch * rank);
}

namespace hc {
// Host-side argument checks shared by both entry points (HC_OK or HC_ERR_ARG),
// done before anything is enqueued.
static int pred_check_args(const float* x, int32_t batch, const float* w_down, const float* w_up, const float* b_up,
                           int32_t rank, int32_t inter, const uint32_t* mask_out, const uint32_t* fetch_bits,
                           const int32_t* ids_out, const int32_t* count_out) {
  if (!x || !w_down || !w_up || !b_up || !mask_out) return HC_ERR_ARG;
  if (batch <= 0 || batch > PRED_MAX_BATCH || rank <= 0 || rank > PRED_MAX_RANK || (rank & 3) != 0 ||
      inter <= 0 || inter > TABLE_SIZE)
    return HC_ERR_ARG;
  if (fetch_bits && (!ids_out || !count_out)) return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(w_down) & 15) || (reinterpret_cast<uintptr_t>(w_up) & 15) ||
      (reinterpret_cast<uintptr_t>(x) & 15))
    return HC_ERR_ARG;
  return HC_OK;
}
}  // namespace hc

extern "C" int hc_predictor_forward(const float* x, int32_t batch, const float* norm_w, float eps,
                                    const float* w_down, const float* w_up,
                                    const float* b_up, int32_t rank, int32_t inter, float logit_threshold,
                                    uint32_t* mask_out, float* probs_out, float* logits_out,
                                    const uint32_t* fetch_bits, const int32_t* table, int32_t* ids_out,
                                    int32_t* rec_out, int32_t* count_out, void* workspace, int32_t* status,
                                    hc_stream_t stream) {
  (void)status;
  const int chk = pred_check_args(x, batch, w_down, w_up, b_up, rank, inter, mask_out, fetch_bits, ids_out, count_out);
  if (chk != HC_OK) return chk;
  if (!workspace || (reinterpret_cast<uintptr_t>(workspace) & 15)) return HC_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  PredWs ws = pred_ws(workspace, batch, rank);
  pred_down_kernel<<<H / PRED_KCHUNK, 256, 0, s>>>(x, batch, norm_w, eps, w_down, rank, ws);
  if (cudaGetLastError() != cudaSuccess) return HC_ERR_CUDA;
  pred_up_kernel<<<(inter + 255) / 256, 256, 0, s>>>(batch, w_up, b_up, rank, inter, logit_threshold, mask_out,
                                                      probs_out, logits_out, fetch_bits, table, ids_out, rec_out,
                                                      count_out, ws);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

// --------------------------------------------------------------------------
// Allocation-free variant.  Some callers cannot allocate device memory at
// all: code that runs inside a fixed memory budget set up once at start (a
// serving process whose allocator is frozen after warm-up, an embedded
// runtime, a plugin host that owns every allocation and exposes none to its
// plugins).  For them the predictor's scratch lives in this file-scope
// device array instead of a caller workspace.  Every GPU that loads the
// library holds it until the process exits.
// --------------------------------------------------------------------------
namespace hc {
constexpr int STATIC_PRED_MAX_BR = 512;   // batch * rank the static scratch holds
constexpr size_t STATIC_PRED_BYTES =
    256 + sizeof(float) * ((size_t)(H / PRED_KCHUNK) * STATIC_PRED_MAX_BR + STATIC_PRED_MAX_BR);
static __device__ __align__(256) unsigned char g_pred_scratch[STATIC_PRED_BYTES];

// The array's device address, looked up once per device and context: a new
// context on the same ordinal (after cudaDeviceReset) loads the module again,
// so the cached address is keyed on the driver's unique context id.
constexpr int MAX_DEVICES = 64;
struct ScratchAddr {
  void* ptr = nullptr;
  unsigned long long ctx_id = 0;
};
static ScratchAddr g_pred_scratch_addr[MAX_DEVICES];
static std::mutex g_pred_scratch_mu;
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// Unique id of the calling thread's current context (0 when it cannot be read).
static unsigned long long current_ctx_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static bool looked_up = false;
  if (!looked_up) {
    void* f1 = nullptr;
    void* f2 = nullptr;
    cudaDriverEntryPointQueryResult q1, q2;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) == cudaSuccess &&
        q1 == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) == cudaSuccess &&
        q2 == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(f2);
    looked_up = true;
  }
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}
}  // namespace hc

extern "C" int hc_predictor_forward_static(const float* x, int32_t batch, const float* norm_w, float eps,
                                           const float* w_down, const float* w_up, const float* b_up, int32_t rank,
                                           int32_t inter, float logit_threshold, uint32_t* mask_out,
                                           float* probs_out, float* logits_out, const uint32_t* fetch_bits,
                                           const int32_t* table, int32_t* ids_out, int32_t* rec_out,
                                           int32_t* count_out, int32_t* status, hc_stream_t stream) {
  // every argument is checked before the shared array is touched
  const int chk = pred_check_args(x, batch, w_down, w_up, b_up, rank, inter, mask_out, fetch_bits, ids_out, count_out);
  if (chk != HC_OK) return chk;
  if ((int64_t)batch * rank > STATIC_PRED_MAX_BR) return HC_ERR_UNSUPPORTED;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return HC_ERR_CUDA;
  void* ws = nullptr;
  {
    // first call on this device (and context): resolve the array's device address
    const unsigned long long ctx = current_ctx_id();
    std::lock_guard<std::mutex> lock(g_pred_scratch_mu);
    ScratchAddr& a = g_pred_scratch_addr[dev];
    if (a.ptr == nullptr || ctx == 0 || a.ctx_id != ctx) {
      if (cudaGetSymbolAddress(&ws, g_pred_scratch) != cudaSuccess || ws == nullptr) return HC_ERR_CUDA;
      a.ptr = ws;
      a.ctx_id = current_ctx_id();     // the lookup made the device's context current
    }
    ws = a.ptr;
  }
  // the array keeps the previous call's contents: restart the two completion counters at zero
  if (cudaMemsetAsync(ws, 0, 256, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return HC_ERR_CUDA;
  return hc_predictor_forward(x, batch, norm_w, eps, w_down, w_up, b_up, rank, inter, logit_threshold, mask_out,
                              probs_out, logits_out, fetch_bits, table, ids_out, rec_out, count_out, ws, status,
                              stream);
}
