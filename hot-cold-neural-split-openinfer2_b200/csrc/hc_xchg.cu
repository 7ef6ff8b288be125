// Sum of every GPU's partial output, for the neuron-sharded batched decode.
//
// down_proj is linear in the neuron dimension (engine.py:184-188), so when
// each GPU computes a layer over its share of the neurons, the layer's output
// is the sum of the GPUs' partials.  This is that one exchange per layer,
// done with plain NVLink stores into the peers' exchange buffers (CUDA IPC
// mappings) instead of a library collective, so that it is an ordinary kernel
// that a CUDA graph can hold and whose waits are bounded:
//
//   1. CTA c stores its slice of this GPU's partial into every peer's buffer
//      (slot seq % 3, sender row = this GPU), then issues one system-scope
//      release and adds 1 to every peer's arrival counter;
//   2. it waits (bounded) until its own counter shows every peer's CTAs;
//   3. it adds, for its slice, the partials of all GPUs in GPU order to `out`,
//      so every GPU computes bit-identical sums.
//
// Buffer layout: [256 B header][3 slots][size senders][n max floats].  The
// header (64 words) holds the arrival counter (word 0, added to by the peers),
// this GPU's count of finished exchanges (word 32) and an exit counter (word
// 48); the arrival counter has its 128-byte line to itself.  The
// arrival counter only grows: after exchange q it holds q (size - 1) x 128
// (every exchange runs 128 CTAs).  The exchange number is read from the
// buffer, not passed in, so a captured CUDA graph can replay the exchange.
#include "hc_common.cuh"

namespace hcx {
using namespace hc;

constexpr size_t HDR = 256;
constexpr int SLOTS = 3;
constexpr int THREADS = 256;
constexpr int MAX_SIZE = 8;
constexpr int GRID = 128;            // CTAs of every exchange (the counter arithmetic relies on it)
constexpr int W_ARRIVE = 0, W_SEQ = 32, W_EXIT = 48;    // header words (HDR / 4 = 64 of them)
static_assert(W_EXIT < (int)(HDR / 4), "header words must stay inside the header");
constexpr uint64_t DEFAULT_WAIT_NS = 2000000000ull;

__device__ __forceinline__ float4* slot_row(void* buf, int slot, int sender, int size, int64_t cap) {
  return reinterpret_cast<float4*>(static_cast<char*>(buf) + HDR) + ((int64_t)slot * size + sender) * (cap / 4);
}

struct XParams {
  const float4* part;
  float4* out;
  int64_t n4;          // float4s to exchange
  int64_t cap;         // floats per sender row of the buffers
  void* const* peer_buf;
  int size, rank;
  uint64_t wait_ns;
  int32_t* status;
};
__device__ __forceinline__ uint32_t* hdr_word(void* buf, int w) { return static_cast<uint32_t*>(buf) + w; }

__global__ void __launch_bounds__(THREADS) xchg_sum_kernel(XParams p) {
  __shared__ int ok_s;
  __shared__ uint32_t seq_s;
  const int t = threadIdx.x, c = blockIdx.x, G = gridDim.x;
  void* own = p.peer_buf[p.rank];
  if (t == 0) seq_s = __ldcg(hdr_word(own, W_SEQ));    // exchanges finished here so far
  __syncthreads();
  const uint32_t seq = seq_s;
  const int slot = (int)(seq % SLOTS);
  const int64_t lo = c * p.n4 / G, hi = (c + 1) * p.n4 / G;
  for (int64_t i = lo + t; i < hi; i += THREADS) {
    const float4 v = p.part[i];
    for (int s = 0; s < p.size; ++s) {
      if (s == p.rank) continue;
      slot_row(p.peer_buf[s], slot, p.rank, p.size, p.cap)[i] = v;
    }
  }
  __syncthreads();
  if (t == 0) {
    // one release, cumulative over the CTA's stores above (ordered by the barrier)
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int s = 0; s < p.size; ++s) {
      if (s == p.rank) continue;
      asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(hdr_word(p.peer_buf[s], W_ARRIVE)) : "memory");
    }
    const uint32_t* f = hdr_word(own, W_ARRIVE);
    const uint32_t want = (seq + 1u) * (uint32_t)(p.size - 1) * (uint32_t)G;
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    for (uint32_t k = 0;; ++k) {
      uint32_t v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
      if ((int32_t)(v - want) >= 0) break;
      if ((k & 63) == 63 && globaltimer_ns() - t0 > p.wait_ns) {
        ok = false;
        break;
      }
      __nanosleep(64);
    }
    if (!ok) atomicOr(p.status, HC_ERR_TIMEOUT);
    ok_s = ok;
  }
  __syncthreads();
  if (ok_s) {                        // else a peer is missing: out stays untouched (status says why)
    for (int64_t i = lo + t; i < hi; i += THREADS) {
      float4 a = p.out[i];
      for (int s = 0; s < p.size; ++s) {
        const float4 v = (s == p.rank) ? p.part[i] : __ldcg(slot_row(own, slot, s, p.size, p.cap) + i);
        a.x += v.x; a.y += v.y; a.z += v.z; a.w += v.w;
      }
      p.out[i] = a;
    }
  }
  // the last CTA to leave counts the exchange (read by the next launch, stream-ordered)
  if (t == 0) {
    __threadfence();
    if (atomicAdd(hdr_word(own, W_EXIT), 1u) == (uint32_t)G - 1) {
      *hdr_word(own, W_EXIT) = 0u;
      *hdr_word(own, W_SEQ) = seq + 1u;
      __threadfence();
    }
  }
}

}  // namespace hcx

using namespace hcx;

extern "C" int64_t hc_xchg_buffer_bytes(int32_t size, int64_t max_floats) {
  if (size < 2 || size > MAX_SIZE || max_floats <= 0 || (max_floats & 3)) return -1;
  return (int64_t)(HDR + sizeof(float) * (size_t)SLOTS * size * max_floats);
}

extern "C" int hc_xchg_sum(const float* part, int64_t n, float* out, int64_t max_floats, const hc_tp_desc* tp,
                           int32_t* status, hc_stream_t stream) {
  if (!part || !out || !tp || !tp->peer_buf || !status || n <= 0 || (n & 3) || n > max_floats || (max_floats & 3))
    return HC_ERR_ARG;
  if (tp->size < 2 || tp->size > MAX_SIZE || tp->rank < 0 || tp->rank >= tp->size) return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(part) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return HC_ERR_ARG;
  XParams p;
  p.part = reinterpret_cast<const float4*>(part);
  p.out = reinterpret_cast<float4*>(out);
  p.n4 = n / 4;
  p.cap = max_floats;
  p.peer_buf = tp->peer_buf;
  p.size = tp->size;
  p.rank = tp->rank;
  p.wait_ns = tp->wait_ns > 0 ? tp->wait_ns : DEFAULT_WAIT_NS;
  p.status = status;
  // a fixed grid: the arrival counter advances by (size - 1) x GRID per exchange
  xchg_sum_kernel<<<GRID, THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(p);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}
