// Fused hot/cold sparse FFN over a stack of layers (batch-1 decode).
//
// Per layer l this computes what SparseFFNLayer.forward does
// (engine.py:292-312): x_{l+1} = x_l + sparse_ffn(RMSNorm(x_l)), where
// sparse_ffn (engine.py:173-209) is the hot FP8 neurons plus the cold INT4
// neurons selected by the predictor, summed in-kernel (exact by linearity of
// down_proj in the neuron dimension, engine.py:184-188).  The next layer's
// predictor runs on this layer's input, as DesdemonaEngine.forward's
// lookahead prefetch does (engine.py:421-438).
//
// One persistent cooperative launch, one CTA per SM:
//  * warp 8 (producer) streams this CTA's share of every layer's weights into
//    a ring of 14 shared-memory slots with 1-D bulk copies (TMA engine),
//    completing on per-slot mbarriers.  Weights never depend on activations,
//    so it runs ahead across the grid barriers and keeps HBM busy while the
//    consumers wait.
//  * warps 0-7 (consumers) own 16 consecutive elements each: thread t holds
//    x[16t, 16t+16) in registers for the gate/up dot products and accumulates
//    y[16t, 16t+16) for the down projection, so the down-projection is local
//    and only the per-neuron dot products need a CTA reduction (batched over
//    4 neurons per round).
//
// Phases of layer l (two grid barriers):
//   A: hot neurons (even split), W_down tiles of predictor l+1, the CTA's
//      share of the active cold records (ordered list split evenly);
//      partial y -> workspace                                  [barrier 2l]
//   B: column-slice reduction of the partials + residual -> x_{l+1};
//      z = sum of W_down partials; W_up tiles -> mask word of layer l+1
//                                                              [barrier 2l+1]
// Every wait (slot, grid barrier, mask readiness) is bounded by a time limit;
// on expiry the kernel ORs HC_ERR_TIMEOUT into the status word, drains its
// own copies in flight and returns.
#include "hc_common.cuh"

namespace hc {

constexpr int CONS_THREADS = 256;
constexpr int STACK_THREADS = CONS_THREADS + 32;
constexpr int SLOT_BYTES = 12800;     // one hot neuron (12288) or two cold records (2 x 6352)
constexpr int NSLOTS = 14;
constexpr int NB = 4;                 // neurons per reduction round
constexpr int WD_ROWS = 32;           // W_down tile: 32 k-rows x rank
constexpr int WU_ROWS = 32;           // W_up tile: 32 neurons x rank (+ bias) == one mask word
constexpr int COLD_WIN = 64;          // producer cold-list window (even)
constexpr int HOT_BYTES = 3 * H;      // 12288
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;   // 2 s

struct StackSmem {
  alignas(128) uint8_t ring[NSLOTS][SLOT_BYTES];
  float xs[H];                      // predictor input of layer l+1
  float z[128];
  float red[8][2 * NB];
  float act[NB];
  float zred[256];
  int32_t cold_list[COLD_WIN];
  uint32_t ballot_word;
  int32_t flag;                     // 1 = ok, 0 = abort (broadcast)
  int32_t abort;                    // sticky abort for the producer
  int32_t n_act;
  uint32_t cons_k;                  // slots consumed (for the drain)
  alignas(8) uint64_t full[NSLOTS];
  alignas(8) uint64_t empty[NSLOTS];
};

struct StackParams {
  const hc_layer_desc* layers;
  int n_layers;
  int inter;
  int words;                 // ceil(inter / 32)
  const float* x_in;
  uint32_t* masks;           // [n_layers][words]
  int masks_given;
  float* x_out;
  float* x_hist;
  float eps;
  int relu;
  int both;
  float thr;
  uint32_t* bar_count;
  uint32_t* exit_count;
  float* ypart;              // [G][H]
  float* zpart;              // [H / WD_ROWS][128]
  float* xbuf;               // [2][H]
  int32_t* status;
};

__host__ __device__ inline size_t stack_ws_offset_ypart() { return 256; }
__host__ __device__ inline size_t stack_ws_offset_zpart(int grid) {
  return 256 + sizeof(float) * (size_t)grid * H;
}
__host__ __device__ inline size_t stack_ws_offset_xbuf(int grid) {
  return stack_ws_offset_zpart(grid) + sizeof(float) * (H / WD_ROWS) * 128;
}
__host__ __device__ inline size_t stack_ws_bytes(int grid) { return stack_ws_offset_xbuf(grid) + sizeof(float) * 2 * H; }

__device__ __forceinline__ int64_t split_lo(int64_t n, int c, int G) { return n * c / G; }
// predictor tiles must fit a slot and split evenly over 8 lanes
__device__ __forceinline__ bool rank_ok(int r) { return r > 0 && r <= 96 && (r & 7) == 0; }

// --------------------------------------------------------------------------
// consumer math
// --------------------------------------------------------------------------
__device__ __forceinline__ float dot16_e4m3(uint4 w, const float (&x)[16]) {
  float f[4];
  float acc = 0.0f;
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    e4m3x4_to_f32(ws[i], f);
#pragma unroll
    for (int j = 0; j < 4; ++j) acc = fmaf(f[j], x[4 * i + j], acc);
  }
  return acc;
}
__device__ __forceinline__ void axpy16_e4m3(uint4 w, float a, float (&y)[16]) {
  float f[4];
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    e4m3x4_to_f32(ws[i], f);
#pragma unroll
    for (int j = 0; j < 4; ++j) y[4 * i + j] = fmaf(a, f[j], y[4 * i + j]);
  }
}
// 16 INT4 elements starting 2 bytes after `p8` (p8 is 8-byte aligned)
__device__ __forceinline__ void load_int4x16(const uint8_t* p8, uint32_t& o0, uint32_t& o1) {
  const uint2 a = *reinterpret_cast<const uint2*>(p8);
  const uint32_t b = *reinterpret_cast<const uint32_t*>(p8 + 8);
  o0 = shift2(a.x, a.y);
  o1 = shift2(a.y, b);
}
__device__ __forceinline__ float dot16_int4(uint32_t o0, uint32_t o1, const float (&x)[16]) {
  float q[8];
  float acc = 0.0f;
  int4x8_to_f32(o0, q);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc = fmaf(q[j], x[j], acc);
  int4x8_to_f32(o1, q);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc = fmaf(q[j], x[8 + j], acc);
  return acc;
}
__device__ __forceinline__ void axpy16_int4(uint32_t o0, uint32_t o1, float a, float (&y)[16]) {
  float q[8];
  int4x8_to_f32(o0, q);
#pragma unroll
  for (int j = 0; j < 8; ++j) y[j] = fmaf(a, q[j], y[j]);
  int4x8_to_f32(o1, q);
#pragma unroll
  for (int j = 0; j < 8; ++j) y[8 + j] = fmaf(a, q[j], y[8 + j]);
}
__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(*reinterpret_cast<const __half*>(p));
}

// consumer-wide broadcast of a decision taken by consumer thread 0
__device__ __forceinline__ bool cons_broadcast(StackSmem& sm, bool ok0) {
  if (threadIdx.x == 0) sm.flag = ok0 ? 1 : 0;
  named_bar(1, CONS_THREADS);
  const bool ok = sm.flag != 0;
  return ok;
}

// Wait (bounded, thread 0) for `n` consecutive ring fills starting at k, then
// let every consumer thread observe the completed phases itself.
__device__ __forceinline__ bool cons_acquire(StackSmem& sm, uint32_t k, int n) {
  bool ok0 = true;
  if (threadIdx.x == 0) {
    for (int i = 0; i < n && ok0; ++i) {
      const uint32_t f = k + i;
      ok0 = mbar_wait(&sm.full[f % NSLOTS], (f / NSLOTS) & 1u, WAIT_LIMIT_NS);
    }
    if (!ok0) sm.abort = 1;
  }
  const bool ok = cons_broadcast(sm, ok0);
  if (ok) {
    for (int i = 0; i < n; ++i) {
      const uint32_t f = k + i;
      while (!mbar_try_wait(&sm.full[f % NSLOTS], (f / NSLOTS) & 1u)) {
      }
    }
  }
  return ok;
}
__device__ __forceinline__ void cons_release(StackSmem& sm, uint32_t k, int n) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0)
    for (int i = 0; i < n; ++i) mbar_arrive(&sm.empty[(k + i) % NSLOTS]);
}

// grid-wide barrier among the consumer groups of all CTAs (bounded)
__device__ bool grid_barrier(StackSmem& sm, const StackParams& p, uint32_t target) {
  named_bar(1, CONS_THREADS);
  bool ok0 = true;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.bar_count, 1u);
    if (ld_acquire_u32(p.bar_count) < target) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_u32(p.bar_count) < target) {
        if ((++spins & 255) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
          ok0 = false;
          break;
        }
        __nanosleep(32);
      }
    }
    __threadfence();
    if (!ok0) {
      sm.abort = 1;
      atomicOr(p.status, HC_ERR_TIMEOUT);
    }
  }
  return cons_broadcast(sm, ok0);
}

// block reduction over the 256 consumer threads (result to all)
__device__ __forceinline__ float cons_sum(StackSmem& sm, float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5;
  named_bar(1, CONS_THREADS);
  if ((threadIdx.x & 31) == 0) sm.zred[warp] = v;
  named_bar(1, CONS_THREADS);
  float s = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) s += sm.zred[w];
  return s;
}

// reduce the 2*NB per-thread partials and form the NB activations in sm.act
// (scale_* == nullptr: cold path, scales already applied per thread)
__device__ __forceinline__ void cons_reduce_act(StackSmem& sm, float (&v)[2 * NB], int nb, const float* hot_scale,
                                                int64_t hot_first, const StackParams& p) {
  const float r = warp_reduce_multi<2 * NB>(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int SH = 5 - (NB == 4 ? 3 : NB == 8 ? 4 : NB == 2 ? 2 : 1);
  if ((lane & ((1 << SH) - 1)) == 0) sm.red[warp][lane >> SH] = r;
  named_bar(1, CONS_THREADS);
  if (threadIdx.x < nb) {
    const int j = threadIdx.x;
    float g = 0.0f, u = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      g += sm.red[w][j];
      u += sm.red[w][NB + j];
    }
    float sd = 1.0f;
    if (hot_scale != nullptr) {
      const float* s3 = hot_scale + (hot_first + j) * 3;
      g *= __ldg(s3 + 0);
      u *= __ldg(s3 + 1);
      sd = __ldg(s3 + 2);
    }
    sm.act[j] = gated(g, u, p.relu, p.both) * sd;
  }
  named_bar(1, CONS_THREADS);
}

// --------------------------------------------------------------------------
// producer helpers
// --------------------------------------------------------------------------
struct Producer {
  uint32_t k = 0;       // fills issued
  uint64_t pol = 0;
  bool ok = true;
};

// lane 0 only: take the next slot (bounded wait for it to be empty)
__device__ __forceinline__ uint8_t* prod_slot(StackSmem& sm, Producer& pr, uint32_t bytes) {
  const uint32_t s = pr.k % NSLOTS;
  const uint32_t round = pr.k / NSLOTS;
  if (round > 0) {
    if (!mbar_wait(&sm.empty[s], (round - 1) & 1u, WAIT_LIMIT_NS)) {
      pr.ok = false;
      return nullptr;
    }
  }
  mbar_arrive_expect_tx(&sm.full[s], bytes);
  return sm.ring[s];
}

__device__ __forceinline__ void consumer_layer_hot(StackSmem& sm, const StackParams& p, const hc_layer_desc& d,
                                                   int64_t h0, int64_t h1, uint32_t& ck, const float (&xn)[16],
                                                   float (&y)[16], bool& ok) {
  const int t = threadIdx.x;
  for (int64_t i = h0; i < h1 && ok; i += NB) {
    const int nb = (int)(h1 - i < NB ? (int64_t)(h1 - i) : (int64_t)NB);
    ok = cons_acquire(sm, ck, nb);
    if (!ok) break;
    float v[2 * NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      v[j] = 0.0f;
      v[NB + j] = 0.0f;
      if (j < nb) {
        const uint8_t* slot = sm.ring[(ck + j) % NSLOTS];
        const uint4 g = *reinterpret_cast<const uint4*>(slot + 16 * t);
        const uint4 u = *reinterpret_cast<const uint4*>(slot + H + 16 * t);
        v[j] = dot16_e4m3(g, xn);
        v[NB + j] = dot16_e4m3(u, xn);
      }
    }
    cons_reduce_act(sm, v, nb, d.hot_scale, i, p);
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      if (j < nb) {
        const uint8_t* slot = sm.ring[(ck + j) % NSLOTS];
        const uint4 dw = *reinterpret_cast<const uint4*>(slot + 2 * H + 16 * t);
        axpy16_e4m3(dw, sm.act[j], y);
      }
    }
    cons_release(sm, ck, nb);
    ck += nb;
  }
}

__device__ __forceinline__ void consumer_layer_cold(StackSmem& sm, const StackParams& p, int64_t c0, int64_t c1,
                                                    uint32_t& ck, const float (&xn)[16], float (&y)[16], bool& ok) {
  const int t = threadIdx.x;
  const int g8 = t >> 3;   // INT4 group of this thread's elements
  for (int64_t i = c0; i < c1 && ok; i += NB) {
    const int nb = (int)(c1 - i < NB ? (int64_t)(c1 - i) : (int64_t)NB);
    const int nslots = (nb + 1) >> 1;
    ok = cons_acquire(sm, ck, nslots);
    if (!ok) break;
    float v[2 * NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      v[j] = 0.0f;
      v[NB + j] = 0.0f;
      if (j < nb) {
        const uint8_t* rec = sm.ring[(ck + (j >> 1)) % NSLOTS] + (j & 1) * REC_COPY;
        uint32_t o0, o1;
        load_int4x16(rec + 8 * t, o0, o1);
        v[j] = dot16_int4(o0, o1, xn) * ld_half(rec + SCALE_OFF + 2 * g8);
        load_int4x16(rec + VEC_BYTES + 8 * t, o0, o1);
        v[NB + j] = dot16_int4(o0, o1, xn) * ld_half(rec + SCALE_OFF + 2 * NGROUPS + 2 * g8);
      }
    }
    cons_reduce_act(sm, v, nb, nullptr, 0, p);
#pragma unroll
    for (int j = 0; j < NB; ++j) {
      if (j < nb) {
        const uint8_t* rec = sm.ring[(ck + (j >> 1)) % NSLOTS] + (j & 1) * REC_COPY;
        uint32_t o0, o1;
        load_int4x16(rec + 2 * VEC_BYTES + 8 * t, o0, o1);
        const float c = sm.act[j] * ld_half(rec + SCALE_OFF + 4 * NGROUPS + 2 * g8);
        axpy16_int4(o0, o1, c, y);
      }
    }
    cons_release(sm, ck, nslots);
    ck += nslots;
  }
}

// --------------------------------------------------------------------------
// the kernel
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(STACK_THREADS, 1) ffn_stack_kernel(StackParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  StackSmem& sm = *reinterpret_cast<StackSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int G = gridDim.x;
  const int c = blockIdx.x;

  if (tid == 0) {
    for (int s = 0; s < NSLOTS; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], CONS_THREADS / 32);
    }
    sm.abort = 0;
    sm.flag = 1;
    sm.cons_k = 0;
    sm.ballot_word = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (tid >= CONS_THREADS) {
    // ============================ producer warp ============================
    const int lane = tid & 31;
    Producer pr;
    if (lane == 0) pr.pol = l2_evict_first_policy();
    for (int l = 0; l < p.n_layers; ++l) {
      const hc_layer_desc d = p.layers[l];
      const bool has_next = (l + 1 < p.n_layers) && !p.masks_given;
      const hc_layer_desc* dn = has_next ? &p.layers[l + 1] : nullptr;
      const bool pred_next = has_next && dn->pred_w_up != nullptr && rank_ok(dn->rank);
      const int rank_n = pred_next ? dn->rank : 0;
      bool ok = true;
      // hot neurons
      if (lane == 0) {
        const int64_t h0 = split_lo(d.n_hot, c, G), h1 = split_lo(d.n_hot, c + 1, G);
        for (int64_t i = h0; i < h1 && pr.ok; ++i) {
          uint8_t* dst = prod_slot(sm, pr, HOT_BYTES);
          if (!dst) break;
          bulk_g2s(dst, d.hot + i * HOT_BYTES, HOT_BYTES, &sm.full[pr.k % NSLOTS], pr.pol);
          ++pr.k;
        }
        // W_down tiles of the next layer's predictor
        if (pred_next && pr.ok) {
          const int nd = H / WD_ROWS;
          const int u0 = (int)split_lo(nd, c, G), u1 = (int)split_lo(nd, c + 1, G);
          const uint32_t bytes = WD_ROWS * rank_n * 4;
          for (int u = u0; u < u1 && pr.ok; ++u) {
            uint8_t* dst = prod_slot(sm, pr, bytes);
            if (!dst) break;
            bulk_g2s(dst, dn->pred_w_down_t + (size_t)u * WD_ROWS * rank_n, bytes, &sm.full[pr.k % NSLOTS], pr.pol);
            ++pr.k;
          }
        }
        ok = pr.ok;
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // wait until this layer's mask is complete (written before barrier 2l-1)
      if (ok && l > 0 && !p.masks_given) {
        if (lane == 0) {
          const uint32_t target = (uint32_t)(2 * l) * G;
          const uint64_t t0 = globaltimer_ns();
          uint32_t spins = 0;
          while (ld_acquire_u32(p.bar_count) < target) {
            if ((++spins & 255) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
              ok = false;
              break;
            }
            __nanosleep(64);
          }
          if (!ok) pr.ok = false;
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      if (!ok) break;
      // cold records: this CTA's slice [c0, c1) of the ordered active list
      {
        const uint32_t* mk = p.masks + (size_t)l * p.words;
        const int wpl = (p.words + 31) / 32;
        const int wb = lane * wpl, we = min(p.words, wb + wpl);
        int mycnt = 0;
        for (int w = wb; w < we; ++w) mycnt += __popc(__ldcg(mk + w) & __ldg(d.fetch_bits + w));
        int incl = mycnt;
        for (int o = 1; o < 32; o <<= 1) {
          const int u = __shfl_up_sync(0xffffffffu, incl, o);
          if (lane >= o) incl += u;
        }
        const int n_act = __shfl_sync(0xffffffffu, incl, 31);
        const int mybase = incl - mycnt;
        const int64_t c0 = split_lo(n_act, c, G), c1 = split_lo(n_act, c + 1, G);
        for (int64_t ws = c0; ws < c1 && ok; ws += COLD_WIN) {
          const int64_t we2 = (ws + COLD_WIN < c1 ? ws + COLD_WIN : c1);
          if (mybase < we2 && mybase + mycnt > ws) {
            int rank = mybase;
            for (int w = wb; w < we && rank < we2; ++w) {
              uint32_t m = __ldcg(mk + w) & __ldg(d.fetch_bits + w);
              while (m) {
                const int bit = __ffs(m) - 1;
                m &= m - 1;
                if (rank >= ws && rank < we2) {
                  const int nid = w * 32 + bit;
                  int rec = d.table[nid];
                  if (rec < 0 || rec >= d.n_records) {
                    atomicOr(p.status, HC_ERR_RANGE);
                    rec = 0;
                  }
                  sm.cold_list[rank - ws] = rec;
                }
                ++rank;
              }
            }
          }
          __syncwarp();
          if (lane == 0) {
            const int cnt = (int)(we2 - ws);
            for (int j = 0; j < cnt && pr.ok; j += 2) {
              const int two = (j + 1 < cnt) ? 2 : 1;
              uint8_t* dst = prod_slot(sm, pr, two * REC_COPY);
              if (!dst) break;
              uint64_t* bar = &sm.full[pr.k % NSLOTS];
              bulk_g2s(dst, d.cold_records + (size_t)sm.cold_list[j] * REC_BYTES, REC_COPY, bar, pr.pol);
              if (two == 2)
                bulk_g2s(dst + REC_COPY, d.cold_records + (size_t)sm.cold_list[j + 1] * REC_BYTES, REC_COPY, bar,
                         pr.pol);
              ++pr.k;
            }
            ok = pr.ok;
          }
          ok = __shfl_sync(0xffffffffu, ok, 0);
          __syncwarp();
        }
      }
      if (!ok) break;
      // W_up tiles of the next layer's predictor (phase B)
      if (lane == 0 && pred_next) {
        const int nu = (p.inter + WU_ROWS - 1) / WU_ROWS;
        const int u0 = (int)split_lo(nu, c, G), u1 = (int)split_lo(nu, c + 1, G);
        for (int u = u0; u < u1 && pr.ok; ++u) {
          const int rows = min(WU_ROWS, p.inter - u * WU_ROWS);
          const uint32_t wbytes = rows * rank_n * 4, bbytes = rows * 4;
          uint8_t* dst = prod_slot(sm, pr, wbytes + bbytes);
          if (!dst) break;
          uint64_t* bar = &sm.full[pr.k % NSLOTS];
          bulk_g2s(dst, dn->pred_w_up + (size_t)u * WU_ROWS * rank_n, wbytes, bar, pr.pol);
          bulk_g2s(dst + WU_ROWS * rank_n * 4, dn->pred_b_up + (size_t)u * WU_ROWS, bbytes, bar, pr.pol);
          ++pr.k;
        }
      }
      ok = __shfl_sync(0xffffffffu, lane == 0 ? pr.ok : true, 0);
      if (!ok) break;
    }
    if (lane == 0 && !pr.ok) {
      sm.abort = 1;
      atomicOr(p.status, HC_ERR_TIMEOUT);
    }
    __syncwarp();
    __syncthreads();
    // drain: every issued copy must have landed before the CTA exits
    if (lane == 0) {
      for (uint32_t f = sm.cons_k; f < pr.k; ++f)
        if (!mbar_wait(&sm.full[f % NSLOTS], (f / NSLOTS) & 1u, WAIT_LIMIT_NS)) {
          atomicOr(p.status, HC_ERR_TIMEOUT);
          break;
        }
    }
  } else {
    // ============================ consumer warps ===========================
    const int t = tid;
    uint32_t ck = 0;
    bool ok = true;
    for (int l = 0; l < p.n_layers && ok; ++l) {
      const hc_layer_desc d = p.layers[l];
      const bool has_next = (l + 1 < p.n_layers) && !p.masks_given;
      const hc_layer_desc* dn = has_next ? &p.layers[l + 1] : nullptr;
      const bool pred_next = has_next && dn->pred_w_up != nullptr && rank_ok(dn->rank);
      if (has_next && dn->pred_w_up != nullptr && !rank_ok(dn->rank) && t == 0 && c == 0)
        atomicOr(p.status, HC_ERR_UNSUPPORTED);
      const int rank_n = pred_next ? dn->rank : 0;
      const float* xl = (l == 0) ? p.x_in : p.xbuf + (size_t)(l & 1) * H;

      // ---- RMSNorm (engine.py:295; torch.nn.RMSNorm)
      float x[16], xn[16], y[16];
      {
        const float4* src = reinterpret_cast<const float4*>(xl + 16 * t);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float4 q = __ldcg(src + i);
          x[4 * i] = q.x; x[4 * i + 1] = q.y; x[4 * i + 2] = q.z; x[4 * i + 3] = q.w;
        }
      }
      float ss = 0.0f;
#pragma unroll
      for (int i = 0; i < 16; ++i) ss = fmaf(x[i], x[i], ss);
      ss = cons_sum(sm, ss);
      const float rstd = rsqrtf(ss / (float)H + p.eps);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float w = d.norm_w ? __ldg(d.norm_w + 16 * t + i) : 1.0f;
        xn[i] = x[i] * rstd * w;
        y[i] = 0.0f;
      }
      if (pred_next) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float w = dn->norm_w ? __ldg(dn->norm_w + 16 * t + i) : 1.0f;
          sm.xs[16 * t + i] = x[i] * rstd * w;
        }
      }
      // active cold count of this layer
      int cnt = 0;
      {
        const uint32_t* mk = p.masks + (size_t)l * p.words;
        for (int w = t; w < p.words; w += CONS_THREADS) cnt += __popc(__ldcg(mk + w) & __ldg(d.fetch_bits + w));
      }
      const int n_act = (int)(cons_sum(sm, (float)cnt) + 0.5f);   // exact: < 2^24

      // ---- phase A: hot neurons
      consumer_layer_hot(sm, p, d, split_lo(d.n_hot, c, G), split_lo(d.n_hot, c + 1, G), ck, xn, y, ok);
      // ---- phase A: W_down tiles -> z partials of predictor l+1
      if (ok && pred_next) {
        const int nd = H / WD_ROWS;
        const int u0 = (int)split_lo(nd, c, G), u1 = (int)split_lo(nd, c + 1, G);
        for (int u = u0; u < u1 && ok; ++u) {
          ok = cons_acquire(sm, ck, 1);
          if (!ok) break;
          const float* tile = reinterpret_cast<const float*>(sm.ring[ck % NSLOTS]);
          // thread -> (r, part): parts of the 32 rows
          const int parts = CONS_THREADS / rank_n;
          float acc = 0.0f;
          const int r = t % rank_n, part = t / rank_n;
          if (part < parts) {
            for (int row = part; row < WD_ROWS; row += parts)
              acc = fmaf(tile[row * rank_n + r], sm.xs[u * WD_ROWS + row], acc);
          }
          sm.zred[t] = acc;
          named_bar(1, CONS_THREADS);
          if (t < rank_n) {
            float s = 0.0f;
            for (int q = 0; q < parts; ++q) s += sm.zred[q * rank_n + t];
            p.zpart[(size_t)u * 128 + t] = s;
          }
          named_bar(1, CONS_THREADS);
          cons_release(sm, ck, 1);
          ck += 1;
        }
      }
      // ---- phase A: cold records
      if (ok) consumer_layer_cold(sm, p, split_lo(n_act, c, G), split_lo(n_act, c + 1, G), ck, xn, y, ok);
      if (!ok) break;
      {
        float4* dst = reinterpret_cast<float4*>(p.ypart + (size_t)c * H + 16 * t);
#pragma unroll
        for (int i = 0; i < 4; ++i) dst[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
      }
      ok = grid_barrier(sm, p, (uint32_t)(2 * l + 1) * G);
      if (!ok) break;

      // ---- phase B: reduce partial columns + residual
      {
        const int q0 = (int)split_lo(H / 4, c, G), q1 = (int)split_lo(H / 4, c + 1, G);
        const int warp = t >> 5, lane = t & 31;
        float* xnext = (l + 1 == p.n_layers) ? p.x_out : p.xbuf + (size_t)((l + 1) & 1) * H;
        for (int q = q0 + warp; q < q1; q += 8) {
          float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int r = lane; r < G; r += 32) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(p.ypart + (size_t)r * H) + q);
            s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
          }
#pragma unroll
          for (int o = 16; o >= 1; o >>= 1) {
            s.x += __shfl_xor_sync(0xffffffffu, s.x, o);
            s.y += __shfl_xor_sync(0xffffffffu, s.y, o);
            s.z += __shfl_xor_sync(0xffffffffu, s.z, o);
            s.w += __shfl_xor_sync(0xffffffffu, s.w, o);
          }
          if (lane == 0) {
            const float4 xv = __ldcg(reinterpret_cast<const float4*>(xl) + q);
            const float4 o = make_float4(xv.x + s.x, xv.y + s.y, xv.z + s.z, xv.w + s.w);
            reinterpret_cast<float4*>(xnext)[q] = o;
            if (p.x_hist) reinterpret_cast<float4*>(p.x_hist + (size_t)l * H)[q] = o;
          }
        }
      }
      // ---- phase B: predictor l+1 logits -> mask words
      if (has_next) {
        uint32_t* mk_next = p.masks + (size_t)(l + 1) * p.words;
        if (!pred_next) {
          // no predictor: fetch every cold neuron (engine.py:282-283)
          for (int w = (int)split_lo(p.words, c, G) + t; w < (int)split_lo(p.words, c + 1, G); w += CONS_THREADS) {
            const int valid = min(32, p.inter - 32 * w);
            mk_next[w] = valid >= 32 ? 0xffffffffu : ((1u << valid) - 1u);
          }
        } else {
          const int nu = (p.inter + WU_ROWS - 1) / WU_ROWS;
          const int u0 = (int)split_lo(nu, c, G), u1 = (int)split_lo(nu, c + 1, G);
          if (u1 > u0) {
            // z = sum of the W_down partials in tile order (deterministic)
            const int nd = H / WD_ROWS;
            const int parts = CONS_THREADS / rank_n;
            const int r = t % rank_n, part = t / rank_n;
            float acc = 0.0f;
            if (part < parts)
              for (int u = part; u < nd; u += parts) acc += __ldcg(p.zpart + (size_t)u * 128 + r);
            sm.zred[t] = acc;
            named_bar(1, CONS_THREADS);
            if (t < rank_n) {
              float s = 0.0f;
              for (int q = 0; q < parts; ++q) s += sm.zred[q * rank_n + t];
              sm.z[t] = s;
            }
            named_bar(1, CONS_THREADS);
          }
          for (int u = u0; u < u1 && ok; ++u) {
            ok = cons_acquire(sm, ck, 1);
            if (!ok) break;
            const float* tile = reinterpret_cast<const float*>(sm.ring[ck % NSLOTS]);
            const int rows = min(WU_ROWS, p.inter - u * WU_ROWS);
            const int j = t >> 3, part = t & 7;
            const int per = rank_n / 8;
            float acc = 0.0f;
            if (j < rows)
              for (int i = 0; i < per; ++i) acc = fmaf(tile[j * rank_n + part * per + i], sm.z[part * per + i], acc);
            acc += __shfl_xor_sync(0xffffffffu, acc, 4);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            const float lg = acc + ((j < rows) ? tile[WU_ROWS * rank_n + j] : 0.0f);
            const bool on = (j < rows) && (lg >= p.thr);
            const unsigned b = __ballot_sync(0xffffffffu, on && part == 0);
            if ((t & 31) == 0) {
              const uint32_t nib = ((b >> 0) & 1u) | (((b >> 8) & 1u) << 1) | (((b >> 16) & 1u) << 2) |
                                   (((b >> 24) & 1u) << 3);
              atomicOr(&sm.ballot_word, nib << (4 * (t >> 5)));
            }
            named_bar(1, CONS_THREADS);
            if (t == 0) {
              mk_next[u] = sm.ballot_word;
              sm.ballot_word = 0;
            }
            cons_release(sm, ck, 1);
            ck += 1;
          }
        }
      }
      if (!ok) break;
      // x_{l+1} (and mask l+1) must be complete before layer l+1 reads them
      if (l + 1 < p.n_layers) ok = grid_barrier(sm, p, (uint32_t)(2 * l + 2) * G);
    }
    if (t == 0) {
      sm.cons_k = ck;
      if (!ok) atomicOr(p.status, HC_ERR_TIMEOUT);
    }
    __syncthreads();
  }

  // reset the barrier counters once every CTA is past its last barrier
  if (tid == 0) {
    __threadfence();
    const uint32_t prev = atomicAdd(p.exit_count, 1u);
    if (prev == (uint32_t)G - 1) {
      *p.bar_count = 0;
      *p.exit_count = 0;
      __threadfence();
    }
  }
}

}  // namespace hc

using namespace hc;

extern "C" int hc_ffn_stack_grid(void) {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
  return sms;
}

extern "C" int64_t hc_ffn_stack_workspace_bytes(int32_t grid, int32_t inter) {
  (void)inter;
  if (grid <= 0) return -1;
  return (int64_t)stack_ws_bytes(grid);
}

extern "C" int hc_ffn_stack(const hc_layer_desc* layers, int32_t n_layers, int32_t inter, const float* x_in,
                            uint32_t* masks, int32_t masks_given, float* x_out, float* x_hist, float eps,
                            int32_t act, int32_t act_on_both, float logit_threshold, int32_t grid, void* workspace,
                            int32_t* status, hc_stream_t stream) {
  if (!layers || n_layers <= 0 || !x_in || !masks || !x_out || !workspace || !status) return HC_ERR_ARG;
  if (inter <= 0 || inter > TABLE_SIZE || (inter & 3) != 0 || (act != HC_ACT_SILU && act != HC_ACT_RELU))
    return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x_in) & 15) || (reinterpret_cast<uintptr_t>(x_out) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15) || (x_hist && (reinterpret_cast<uintptr_t>(x_hist) & 15)))
    return HC_ERR_ARG;
  int G = grid > 0 ? grid : hc_ffn_stack_grid();
  if (G <= 0) return HC_ERR_CUDA;
  static bool attr_set = false;
  const int smem = (int)sizeof(StackSmem);
  if (!attr_set) {
    if (cudaFuncSetAttribute(ffn_stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return HC_ERR_CUDA;
    attr_set = true;
  }
  StackParams p;
  p.layers = layers;
  p.n_layers = n_layers;
  p.inter = inter;
  p.words = (inter + 31) / 32;
  p.x_in = x_in;
  p.masks = masks;
  p.masks_given = masks_given;
  p.x_out = x_out;
  p.x_hist = x_hist;
  p.eps = eps;
  p.relu = act == HC_ACT_RELU;
  p.both = act_on_both != 0;
  p.thr = logit_threshold;
  char* ws = static_cast<char*>(workspace);
  p.bar_count = reinterpret_cast<uint32_t*>(ws);
  p.exit_count = reinterpret_cast<uint32_t*>(ws + 128);
  p.ypart = reinterpret_cast<float*>(ws + stack_ws_offset_ypart());
  p.zpart = reinterpret_cast<float*>(ws + stack_ws_offset_zpart(G));
  p.xbuf = reinterpret_cast<float*>(ws + stack_ws_offset_xbuf(G));
  p.status = status;
  void* args[] = {&p};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(ffn_stack_kernel), dim3(G),
                                              dim3(STACK_THREADS), args, smem, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}
