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

constexpr int CONS_THREADS = 512;      // 16 consumer warps, 8 elements of x / y per thread
constexpr int NWARPS = CONS_THREADS / 32;
constexpr int EPT = H / CONS_THREADS;  // elements per consumer thread (8)
constexpr int STACK_THREADS = CONS_THREADS + 64;   // + issuer warp + planner warp
constexpr int SLOT_BYTES = 12800;     // one hot neuron (12288) or two cold records (2 x 6352)
constexpr int NSLOTS = 15;
constexpr int REC_SLOT_OFF = 6352;    // second cold record in a slot
constexpr int NB = 8;                 // cold records per reduction round
constexpr int NB_HOT = 4;             // hot neurons per reduction round
constexpr int WD_ROWS = 32;           // W_down tile: 32 k-rows x rank
constexpr int WU_ROWS = 32;           // W_up tile: 32 neurons x rank (+ bias) == one mask word
constexpr int COLD_LIST = 1024;       // max cold records one CTA handles per layer
constexpr int MAX_WORDS = 1024;       // mask words (inter <= 32768)
constexpr int HOT_BYTES = 3 * H;      // 12288
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;   // 2 s
static_assert(SLOT_BYTES % 16 == 0 && REC_SLOT_OFF % 16 == 0, "bulk copies need 16-byte aligned slots");
static_assert(HOT_BYTES <= SLOT_BYTES && REC_SLOT_OFF + REC_COPY <= SLOT_BYTES, "slot too small");
static_assert(REC_SLOT_OFF >= REC_COPY, "cold records overlap");
static_assert(32 * 96 * 4 + 32 * 4 <= SLOT_BYTES, "predictor tiles must fit a slot");


struct StackSmem {
  alignas(128) uint8_t ring[NSLOTS][SLOT_BYTES];
  float xs[H];                      // predictor input of layer l+1
  float red[2][NWARPS][2 * NB];     // per-warp partial (gate, up) dots, double buffered
  float z[128];
  float zred[CONS_THREADS];
  uint32_t cmask[MAX_WORDS];        // mask & fetch_bits of the layer being planned
  int32_t plan_list[COLD_LIST];     // nids, then record indices, of this CTA's cold slice
  int32_t plan_n;                   // cold records in this CTA's slice
  uint32_t ballot_word;
  int32_t flag;                     // 1 = ok, 0 = abort (broadcast)
  int32_t abort;                    // sticky abort
  uint32_t cons_k;                  // slots consumed (for the drain)
  alignas(8) uint64_t full[NSLOTS];
  alignas(8) uint64_t empty[NSLOTS];
  alignas(8) uint64_t plan_full;    // planner -> issuer/consumers: list of layer l ready
  alignas(8) uint64_t plan_empty;   // issuer + consumers -> planner: list consumed
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
  uint64_t* trace;           // optional [n_layers][G][TRACE_EVENTS] globaltimer stamps
};

constexpr int TRACE_EVENTS = 24;
__device__ __forceinline__ void trace_ev(const StackParams& p, int l, int ev) {
  if (p.trace != nullptr)
    p.trace[((size_t)l * gridDim.x + blockIdx.x) * TRACE_EVENTS + ev] = globaltimer_ns();
}
__device__ __forceinline__ void trace_add(const StackParams& p, int l, int ev, uint64_t v) {
  if (p.trace != nullptr) p.trace[((size_t)l * gridDim.x + blockIdx.x) * TRACE_EVENTS + ev] += v;
}

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
// consumer helpers
// --------------------------------------------------------------------------
__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(*reinterpret_cast<const __half*>(p));
}
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

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
// Every thread waits (bounded) for the group's fills itself; a thread whose
// wait expires flags the abort, which all threads read after the group's
// barrier, so control flow stays uniform across the named barriers.
__device__ __forceinline__ void cons_wait_group(StackSmem& sm, uint32_t k, int n, uint64_t* waited = nullptr) {
  const uint64_t t0 = (waited != nullptr) ? globaltimer_ns() : 0;
  for (int i = 0; i < n; ++i) {
    const uint32_t f = k + i;
    if (!mbar_wait(&sm.full[f % NSLOTS], (f / NSLOTS) & 1u, WAIT_LIMIT_NS)) {
      sm.abort = 1;
      return;
    }
  }
  if (waited != nullptr) *waited += globaltimer_ns() - t0;
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

// block reduction (sum of a, max of b) over the 256 consumer threads
__device__ __forceinline__ void cons_sum_max(StackSmem& sm, float& a, float& b) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b = fmaxf(b, __shfl_xor_sync(0xffffffffu, b, o));
  }
  const int warp = threadIdx.x >> 5;
  named_bar(1, CONS_THREADS);
  if ((threadIdx.x & 31) == 0) {
    sm.zred[warp] = a;
    sm.zred[NWARPS + warp] = b;
  }
  named_bar(1, CONS_THREADS);
  a = 0.0f;
  b = 0.0f;
#pragma unroll
  for (int w = 0; w < NWARPS; ++w) {
    a += sm.zred[w];
    b = fmaxf(b, sm.zred[NWARPS + w]);
  }
}

// Thread t of the consumer group owns elements [8t, 8t+8) of x and y.  Its
// x is kept in registers as f16 pairs in the orders the decoders produce:
// xf8[i] = (x[2i], x[2i+1]) for FP8 rows; for an INT4 word xi4 = {(x0,x4),
// (x1,x5), (x2,x6), (x3,x7)}, and xoff = 1032*(x0+x2+x4+x6) + 72*(x1+x3+x5+x7)
// removes the decoding bias (see int4_pairs).
struct XRegs {
  uint32_t xf8[4];
  uint32_t xi4[4];
  float xoff;
};

// CTA reduction of 2*NBM per-thread partials (values: gate 0..NBM-1, then up
// 0..NBM-1): a warp-level multi-value reduction, one barrier, then lanes
// j < 2*NBM of every warp sum the NWARPS warp partials of value j.
template <int NBM>
__device__ __forceinline__ float group_reduce(StackSmem& sm, int buf, float (&v)[2 * NBM], bool& abort_seen) {
  constexpr int V = 2 * NBM;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float r = warp_reduce_multi<V>(v);
  constexpr int SH = 5 - (V == 16 ? 4 : V == 8 ? 3 : V == 4 ? 2 : 1);
  if ((lane & ((1 << SH) - 1)) == 0) sm.red[buf][warp][lane >> SH] = r;
  named_bar(1, CONS_THREADS);
  abort_seen = sm.abort != 0;      // sampled right after the barrier: identical in every thread
  float s = 0.0f;
  if (lane < V) {
#pragma unroll
    for (int w = 0; w < NWARPS; ++w) s += sm.red[buf][w][lane];
  }
  return s;
}

// 8 FP8 weights (one uint2) dotted with the thread's x: two fp32 chains
__device__ __forceinline__ float dot8_fp8(uint2 w, const XRegs& x) {
  float a = 0.0f, b = 0.0f;
  fma2_f16f16_f32(a, b, e4m3x2_to_f16x2(w.x), x.xf8[0]);
  fma2_f16f16_f32(a, b, e4m3x2_to_f16x2(w.x >> 16), x.xf8[1]);
  fma2_f16f16_f32(a, b, e4m3x2_to_f16x2(w.y), x.xf8[2]);
  fma2_f16f16_f32(a, b, e4m3x2_to_f16x2(w.y >> 16), x.xf8[3]);
  return a + b;
}

// One packed INT4 word (8 signed nibbles, element i in bits 4i..4i+3) as four
// f16 pairs with a bias, using one shift and four LOP3s (the sign flip is
// folded into the LOP3 constant):
//   h[0] = (1032+q0, 1032+q4)  h[1] = (1152+16q1, 1152+16q5)
//   h[2] = (1032+q2, 1032+q6)  h[3] = (1152+16q3, 1152+16q7)
__device__ __forceinline__ void int4_pairs(uint32_t w, uint32_t (&h)[4]) {
  const uint32_t w8 = w >> 8;
  h[0] = (w & 0x000F000Fu) ^ 0x64086408u;
  h[1] = (w & 0x00F000F0u) ^ 0x64806480u;
  h[2] = (w8 & 0x000F000Fu) ^ 0x64086408u;
  h[3] = (w8 & 0x00F000F0u) ^ 0x64806480u;
}
// sum over the word of q_i * x_i (bias removed with x.xoff)
__device__ __forceinline__ float dot8_int4(uint32_t w, const XRegs& x) {
  uint32_t h[4];
  int4_pairs(w, h);
  float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
  fma2_f16f16_f32(a0, a1, h[0], x.xi4[0]);
  fma2_f16f16_f32(b0, b1, h[1], x.xi4[1]);
  fma2_f16f16_f32(a0, a1, h[2], x.xi4[2]);
  fma2_f16f16_f32(b0, b1, h[3], x.xi4[3]);
  return fmaf(b0 + b1, 0.0625f, a0 + a1) - x.xoff;
}
// the thread's 8 INT4 elements of a record field: bytes [2 + 4t, 6 + 4t)
__device__ __forceinline__ uint32_t ld_int4x8(const uint8_t* field4t) {
  return shift2(ld_u32(field4t), ld_u32(field4t + 4));
}

// Hot group: nb (<= NB_HOT) FP8 neurons in ring fills ck .. ck+nb-1.
__device__ __forceinline__ bool hot_group(StackSmem& sm, const StackParams& p, const float* hot_scale,
                                          int64_t h_first, int nb, uint32_t ck, int buf, const XRegs& x,
                                          float (&y)[EPT], uint64_t* waited) {
  const int t = threadIdx.x, lane = t & 31;
  float sg = 1.0f, su = 1.0f, sd = 1.0f;
  if (hot_scale != nullptr && lane < nb) {
    const float* s3 = hot_scale + (h_first + lane) * 3;
    sg = __ldg(s3);
    su = __ldg(s3 + 1);
    sd = __ldg(s3 + 2);
  }
  cons_wait_group(sm, ck, nb, waited);
  float v[2 * NB_HOT];
#pragma unroll
  for (int j = 0; j < NB_HOT; ++j) {
    v[j] = 0.0f;
    v[NB_HOT + j] = 0.0f;
    if (j < nb) {
      const uint8_t* slot = sm.ring[(ck + j) % NSLOTS];
      v[j] = dot8_fp8(*reinterpret_cast<const uint2*>(slot + EPT * t), x);
      v[NB_HOT + j] = dot8_fp8(*reinterpret_cast<const uint2*>(slot + H + EPT * t), x);
    }
  }
  bool abort_seen;
  const float s = group_reduce<NB_HOT>(sm, buf, v, abort_seen);
  if (abort_seen) return true;
  const float uu = __shfl_down_sync(0xffffffffu, s, NB_HOT);   // lane j < nb: gate j, lane NB_HOT + j: up j
  float a = 0.0f;
  if (lane < nb) a = gated(s * sg, uu * su, p.relu, p.both) * sd;
#pragma unroll
  for (int n = 0; n < NB_HOT; ++n) {
    const float an = __shfl_sync(0xffffffffu, a, n);
    if (n < nb) {
      const unsigned short a16 = __half_as_ushort(__float2half_rn(an));
      const uint2 dw = *reinterpret_cast<const uint2*>(sm.ring[(ck + n) % NSLOTS] + 2 * H + EPT * t);
      fma2_f16_f32(y[0], y[1], e4m3x2_to_f16x2(dw.x), a16);
      fma2_f16_f32(y[2], y[3], e4m3x2_to_f16x2(dw.x >> 16), a16);
      fma2_f16_f32(y[4], y[5], e4m3x2_to_f16x2(dw.y), a16);
      fma2_f16_f32(y[6], y[7], e4m3x2_to_f16x2(dw.y >> 16), a16);
    }
  }
  cons_release(sm, ck, nb);
  return false;
}

// Cold group: nb (<= NB) INT4 records, two per ring fill.
__device__ __forceinline__ bool cold_group(StackSmem& sm, const StackParams& p, int nb, uint32_t ck, int buf,
                                           const XRegs& x, float (&y)[EPT], uint64_t* waited) {
  const int t = threadIdx.x, lane = t & 31;
  const int gs = 2 * (t >> 4);   // byte offset of this thread's INT4 group scale
  const int nslots = (nb + 1) >> 1;
  cons_wait_group(sm, ck, nslots, waited);
  float v[2 * NB];
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    v[j] = 0.0f;
    v[NB + j] = 0.0f;
    if (j < nb) {
      const uint8_t* rec = sm.ring[(ck + (j >> 1)) % NSLOTS] + (j & 1) * REC_SLOT_OFF;
      v[j] = dot8_int4(ld_int4x8(rec + 4 * t), x) * ld_half(rec + SCALE_OFF + gs);
      v[NB + j] = dot8_int4(ld_int4x8(rec + VEC_BYTES + 4 * t), x) * ld_half(rec + SCALE_OFF + 2 * NGROUPS + gs);
    }
  }
  bool abort_seen;
  const float s = group_reduce<NB>(sm, buf, v, abort_seen);
  if (abort_seen) return true;
  const float uu = __shfl_down_sync(0xffffffffu, s, NB);
  float a = 0.0f;
  if (lane < nb) a = gated(s, uu, p.relu, p.both);
  float csa = 0.0f, csb = 0.0f;   // sums of the f16 coefficients (the down rows carry a decoding bias)
#pragma unroll
  for (int n = 0; n < NB; ++n) {
    const float an = __shfl_sync(0xffffffffu, a, n);
    if (n < nb) {
      const uint8_t* rn = sm.ring[(ck + (n >> 1)) % NSLOTS] + (n & 1) * REC_SLOT_OFF;
      const __half c16 = __float2half_rn(an * ld_half(rn + SCALE_OFF + 4 * NGROUPS + gs));
      const __half c16s = __hmul(c16, __float2half(0.0625f));    // exact: power of two
      csa += __half2float(c16);
      csb += __half2float(c16s);
      uint32_t h[4];
      int4_pairs(ld_int4x8(rn + 2 * VEC_BYTES + 4 * t), h);
      const unsigned short cb = __half_as_ushort(c16), cs = __half_as_ushort(c16s);
      fma2_f16_f32(y[0], y[4], h[0], cb);   // (1032 + q) * c
      fma2_f16_f32(y[1], y[5], h[1], cs);   // (1152 + 16 q) * c / 16
      fma2_f16_f32(y[2], y[6], h[2], cb);
      fma2_f16_f32(y[3], y[7], h[3], cs);
    }
  }
  // remove the decoding bias: 1032 * c for even elements, 1152 * (c / 16) for odd ones
#pragma unroll
  for (int j = 0; j < EPT; ++j) y[j] = (j & 1) ? fmaf(-1152.0f, csb, y[j]) : fmaf(-1032.0f, csa, y[j]);
  cons_release(sm, ck, nslots);
  return false;
}

// --------------------------------------------------------------------------
// producer helpers
// --------------------------------------------------------------------------
struct Producer {
  uint32_t k = 0;       // fills issued
  uint64_t pol = 0;
  bool ok = true;
};

// issuer lane 0: take the next slot (bounded wait for it to be empty)
__device__ __forceinline__ uint8_t* prod_slot(StackSmem& sm, Producer& pr, uint32_t bytes,
                                              uint64_t* waited = nullptr) {
  const uint32_t s = pr.k % NSLOTS;
  const uint32_t round = pr.k / NSLOTS;
  if (round > 0) {
    const uint64_t t0 = (waited != nullptr) ? globaltimer_ns() : 0;
    if (!mbar_wait(&sm.empty[s], (round - 1) & 1u, WAIT_LIMIT_NS)) {
      pr.ok = false;
      return nullptr;
    }
    if (waited != nullptr) *waited += globaltimer_ns() - t0;
  }
  mbar_arrive_expect_tx(&sm.full[s], bytes);
  return sm.ring[s];
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
    mbar_init(&sm.plan_full, 1);
    mbar_init(&sm.plan_empty, 2);
    sm.abort = 0;
    sm.flag = 1;
    sm.cons_k = 0;
    sm.ballot_word = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (tid >= CONS_THREADS + 32) {
    // ============================ planner warp =============================
    // For each layer: wait until its mask is complete, stage mask & fetch_bits
    // in shared memory, count the active cold ids, and resolve this CTA's
    // slice [c0, c1) of the ascending active list to record indices.  All
    // global loads are issued in batches so the list costs a few latencies.
    const int lane = tid & 31;
    bool ok = true;
    for (int l = 0; l < p.n_layers && ok; ++l) {
      const hc_layer_desc d = p.layers[l];
      if (l > 0) {
        if (lane == 0) ok = mbar_wait(&sm.plan_empty, (uint32_t)(l - 1) & 1u, WAIT_LIMIT_NS);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
      if (l > 0 && !p.masks_given) {
        if (lane == 0) {
          const uint32_t target = (uint32_t)(2 * l) * G;
          const uint64_t t0 = globaltimer_ns();
          uint32_t spins = 0;
          while (ld_acquire_u32(p.bar_count) < target) {
            if ((++spins & 255) == 0 && globaltimer_ns() - t0 > WAIT_LIMIT_NS) {
              ok = false;
              break;
            }
            __nanosleep(32);
          }
        }
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
      const uint32_t* mk = p.masks + (size_t)l * p.words;
      for (int w0 = 0; w0 < p.words; w0 += 32 * 8) {
        uint32_t v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int w = w0 + k * 32 + lane;
          v[k] = (w < p.words) ? (__ldcg(mk + w) & __ldg(d.fetch_bits + w)) : 0u;
        }
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int w = w0 + k * 32 + lane;
          if (w < p.words) sm.cmask[w] = v[k];
        }
      }
      __syncwarp();
      const int wpl = (p.words + 31) / 32;
      const int wb = lane * wpl, we = min(p.words, wb + wpl);
      int mycnt = 0;
      for (int w = wb; w < we; ++w) mycnt += __popc(sm.cmask[w]);
      int incl = mycnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      const int n_act = __shfl_sync(0xffffffffu, incl, 31);
      const int c0 = (int)split_lo(n_act, c, G), c1 = (int)split_lo(n_act, c + 1, G);
      int cnt = c1 - c0;
      if (cnt > COLD_LIST) {
        if (lane == 0) atomicOr(p.status, HC_ERR_UNSUPPORTED);
        cnt = COLD_LIST;
      }
      int rank = incl - mycnt;
      if (rank < c0 + cnt && incl > c0) {
        for (int w = wb; w < we && rank < c0 + cnt; ++w) {
          uint32_t m = sm.cmask[w];
          while (m) {
            const int bit = __ffs(m) - 1;
            m &= m - 1;
            if (rank >= c0 && rank < c0 + cnt) sm.plan_list[rank - c0] = w * 32 + bit;
            ++rank;
          }
        }
      }
      __syncwarp();
      for (int i0 = 0; i0 < cnt; i0 += 32 * 4) {
        int r[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int i = i0 + k * 32 + lane;
          r[k] = (i < cnt) ? __ldg(d.table + sm.plan_list[i]) : 0;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int i = i0 + k * 32 + lane;
          if (i < cnt) {
            if (r[k] < 0 || r[k] >= d.n_records) {
              atomicOr(p.status, HC_ERR_RANGE);
              r[k] = 0;
            }
            sm.plan_list[i] = r[k];
            prefetch_l2(d.cold_records + (size_t)r[k] * REC_BYTES, REC_COPY);
          }
        }
      }
      if (lane == 0) sm.plan_n = cnt;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&sm.plan_full);
        trace_ev(p, l, 20);
      }
    }
    if (lane == 0 && !ok) {
      sm.abort = 1;
      atomicOr(p.status, HC_ERR_TIMEOUT);
    }
    __syncwarp();
    __syncthreads();
  } else if (tid >= CONS_THREADS) {
    // ============================ issuer warp ==============================
    // Lane 0 streams this CTA's units of every layer through the ring in the
    // consumers' order: hot neurons, W_down tiles (predictor l+1), the cold
    // records of the planner's list, W_up tiles (predictor l+1).  At each
    // layer start it also prefetches the layer's static ranges into L2 so
    // HBM keeps streaming while the consumers sit at a grid barrier.
    const int lane = tid & 31;
    Producer pr;
    if (lane == 0) {
      pr.pol = l2_evict_first_policy();
      for (int l = 0; l < p.n_layers && pr.ok; ++l) {
        const hc_layer_desc d = p.layers[l];
        const bool has_next = (l + 1 < p.n_layers) && !p.masks_given;
        const hc_layer_desc* dn = has_next ? &p.layers[l + 1] : nullptr;
        const bool pred_next = has_next && dn->pred_w_up != nullptr && rank_ok(dn->rank);
        const int rank_n = pred_next ? dn->rank : 0;
        const int64_t h0 = split_lo(d.n_hot, c, G), h1 = split_lo(d.n_hot, c + 1, G);
        const int nd = H / WD_ROWS;
        const int d0 = pred_next ? (int)split_lo(nd, c, G) : 0, d1 = pred_next ? (int)split_lo(nd, c + 1, G) : 0;
        const int nu = (p.inter + WU_ROWS - 1) / WU_ROWS;
        const int u0 = pred_next ? (int)split_lo(nu, c, G) : 0, u1 = pred_next ? (int)split_lo(nu, c + 1, G) : 0;
        // L2 prefetch of the layer's static bytes
        trace_ev(p, l, 10);
        if (h1 > h0) prefetch_l2_range(d.hot + h0 * HOT_BYTES, (size_t)(h1 - h0) * HOT_BYTES);
        if (d1 > d0)
          prefetch_l2_range(dn->pred_w_down_t + (size_t)d0 * WD_ROWS * rank_n, (size_t)(d1 - d0) * WD_ROWS * rank_n * 4);
        if (u1 > u0) {
          const int rows = min(u1 * WU_ROWS, p.inter) - u0 * WU_ROWS;
          prefetch_l2_range(dn->pred_w_up + (size_t)u0 * WU_ROWS * rank_n, (size_t)rows * rank_n * 4);
        }
        // hot neurons
        uint64_t iw_hot = 0, iw_cold = 0;
        for (int64_t i = h0; i < h1 && pr.ok; ++i) {
          uint8_t* dst = prod_slot(sm, pr, HOT_BYTES, p.trace ? &iw_hot : nullptr);
          if (!dst) break;
          bulk_g2s(dst, d.hot + i * HOT_BYTES, HOT_BYTES, &sm.full[pr.k % NSLOTS], pr.pol);
          ++pr.k;
        }
        trace_ev(p, l, 11);
        // W_down tiles of the next layer's predictor
        for (int u = d0; u < d1 && pr.ok; ++u) {
          const uint32_t bytes = WD_ROWS * rank_n * 4;
          uint8_t* dst = prod_slot(sm, pr, bytes);
          if (!dst) break;
          bulk_g2s(dst, dn->pred_w_down_t + (size_t)u * WD_ROWS * rank_n, bytes, &sm.full[pr.k % NSLOTS], pr.pol);
          ++pr.k;
        }
        if (!pr.ok) break;
        // cold records of the planner's list, two per slot
        trace_ev(p, l, 12);
        if (!mbar_wait(&sm.plan_full, (uint32_t)l & 1u, WAIT_LIMIT_NS)) {
          pr.ok = false;
          break;
        }
        trace_ev(p, l, 13);
        const int cnt = sm.plan_n;
        for (int j = 0; j < cnt && pr.ok; j += 2) {
          const int two = (j + 1 < cnt) ? 2 : 1;
          uint8_t* dst = prod_slot(sm, pr, two * REC_COPY, p.trace ? &iw_cold : nullptr);
          if (!dst) break;
          uint64_t* bar = &sm.full[pr.k % NSLOTS];
          bulk_g2s(dst, d.cold_records + (size_t)sm.plan_list[j] * REC_BYTES, REC_COPY, bar, pr.pol);
          if (two == 2)
            bulk_g2s(dst + REC_SLOT_OFF, d.cold_records + (size_t)sm.plan_list[j + 1] * REC_BYTES, REC_COPY, bar,
                     pr.pol);
          ++pr.k;
        }
        mbar_arrive(&sm.plan_empty);
        trace_ev(p, l, 14);
        trace_add(p, l, 18, iw_hot);
        trace_add(p, l, 19, iw_cold);
        if (!pr.ok) break;
        // W_up tiles of the next layer's predictor (phase B)
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
      if (!pr.ok) {
        sm.abort = 1;
        atomicOr(p.status, HC_ERR_TIMEOUT);
      }
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
    int gbuf = 0;
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
      if (t == 0) trace_ev(p, l, 0);
      uint64_t w_hot = 0, w_cold = 0;

      // ---- RMSNorm (engine.py:295; torch.nn.RMSNorm); x kept in registers as f16 pairs
      float y[EPT];
      XRegs xr;
      {
        float x[EPT], nw[EPT];
        const float4* src = reinterpret_cast<const float4*>(xl + EPT * t);
        const float4 q0 = __ldcg(src), q1 = __ldcg(src + 1);
        x[0] = q0.x; x[1] = q0.y; x[2] = q0.z; x[3] = q0.w; x[4] = q1.x; x[5] = q1.y; x[6] = q1.z; x[7] = q1.w;
        if (d.norm_w) {
          const float4* wsrc = reinterpret_cast<const float4*>(d.norm_w + EPT * t);
          const float4 w0 = __ldg(wsrc), w1 = __ldg(wsrc + 1);
          nw[0] = w0.x; nw[1] = w0.y; nw[2] = w0.z; nw[3] = w0.w; nw[4] = w1.x; nw[5] = w1.y; nw[6] = w1.z; nw[7] = w1.w;
        } else {
#pragma unroll
          for (int i = 0; i < EPT; ++i) nw[i] = 1.0f;
        }
        float ss = 0.0f, mx = 0.0f;
#pragma unroll
        for (int i = 0; i < EPT; ++i) ss = fmaf(x[i], x[i], ss);
        cons_sum_max(sm, ss, mx);
        const float rstd = rsqrtf(ss / (float)H + p.eps);
        __half xh[EPT];
        float xe = 0.0f, xo = 0.0f;
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
          xh[i] = __float2half_rn(x[i] * rstd * nw[i]);
          if (i & 1) xo += __half2float(xh[i]);
          else xe += __half2float(xh[i]);
        }
        xr.xoff = 1032.0f * xe + 72.0f * xo;
        auto pk = [](__half lo, __half hi) {
          return (uint32_t)__half_as_ushort(lo) | ((uint32_t)__half_as_ushort(hi) << 16);
        };
        xr.xf8[0] = pk(xh[0], xh[1]); xr.xf8[1] = pk(xh[2], xh[3]);
        xr.xf8[2] = pk(xh[4], xh[5]); xr.xf8[3] = pk(xh[6], xh[7]);
        xr.xi4[0] = pk(xh[0], xh[4]); xr.xi4[1] = pk(xh[1], xh[5]);
        xr.xi4[2] = pk(xh[2], xh[6]); xr.xi4[3] = pk(xh[3], xh[7]);
        if (pred_next) {
#pragma unroll
          for (int i = 0; i < EPT; ++i) {
            const float w = dn->norm_w ? __ldg(dn->norm_w + EPT * t + i) : 1.0f;
            sm.xs[EPT * t + i] = x[i] * rstd * w;
          }
        }
#pragma unroll
        for (int i = 0; i < EPT; ++i) y[i] = 0.0f;
      }
      if (t == 0) trace_ev(p, l, 1);
      // ---- phase A: hot neurons, groups of NB
      {
        const int64_t h0 = split_lo(d.n_hot, c, G), h1 = split_lo(d.n_hot, c + 1, G);
        for (int64_t i = h0; i < h1; i += NB_HOT) {
          const int nb = (int)(h1 - i < NB_HOT ? h1 - i : NB_HOT);
          if (hot_group(sm, p, d.hot_scale, i, nb, ck, gbuf, xr, y, (t == 0 && p.trace) ? &w_hot : nullptr)) {
            ok = false;
            break;
          }
          ck += nb;
          gbuf ^= 1;
        }
      }
      if (t == 0) trace_ev(p, l, 2);
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
      if (t == 0) trace_ev(p, l, 3);
      // ---- phase A: cold records (the planner's slice of the ordered list)
      if (ok) {
        bool ok0 = true;
        if (t == 0) ok0 = mbar_wait(&sm.plan_full, (uint32_t)l & 1u, WAIT_LIMIT_NS);
        ok = cons_broadcast(sm, ok0);
        if (ok) {
          while (!mbar_try_wait(&sm.plan_full, (uint32_t)l & 1u)) {
          }
          const int cnt = sm.plan_n;
          named_bar(1, CONS_THREADS);
          if (t == 0) {
            mbar_arrive(&sm.plan_empty);
            trace_ev(p, l, 4);
          }
          for (int i = 0; i < cnt; i += NB) {
            const int nb = cnt - i < NB ? cnt - i : NB;
            if (cold_group(sm, p, nb, ck, gbuf, xr, y, (t == 0 && p.trace) ? &w_cold : nullptr)) {
              ok = false;
              break;
            }
            ck += (nb + 1) >> 1;
            gbuf ^= 1;
          }
        }
      }
      if (!ok) break;
      {
        float4* dst = reinterpret_cast<float4*>(p.ypart + (size_t)c * H + EPT * t);
        dst[0] = make_float4(y[0], y[1], y[2], y[3]);
        dst[1] = make_float4(y[4], y[5], y[6], y[7]);
      }
      if (t == 0) {
        trace_ev(p, l, 5);
        trace_add(p, l, 15, w_hot);
        trace_add(p, l, 16, w_cold);
      }
      ok = grid_barrier(sm, p, (uint32_t)(2 * l + 1) * G);
      if (!ok) break;

      if (t == 0) trace_ev(p, l, 6);
      // ---- phase B: reduce partial columns + residual
      {
        const int q0 = (int)split_lo(H / 4, c, G), q1 = (int)split_lo(H / 4, c + 1, G);
        const int warp = t >> 5, lane = t & 31;
        float* xnext = (l + 1 == p.n_layers) ? p.x_out : p.xbuf + (size_t)((l + 1) & 1) * H;
        for (int q = q0 + warp; q < q1; q += NWARPS) {
          float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int r0 = 0; r0 < G; r0 += 32 * 8) {
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int r = r0 + 32 * k + lane;
              v[k] = (r < G) ? __ldcg(reinterpret_cast<const float4*>(p.ypart + (size_t)r * H) + q)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              s.x += v[k].x; s.y += v[k].y; s.z += v[k].z; s.w += v[k].w;
            }
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
      if (t == 0) trace_ev(p, l, 7);
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
            if (part < parts) {
              for (int u0 = part; u0 < nd; u0 += parts * 16) {
                float v[16];
#pragma unroll
                for (int k = 0; k < 16; ++k) {
                  const int u = u0 + k * parts;
                  v[k] = (u < nd) ? __ldcg(p.zpart + (size_t)u * 128 + r) : 0.0f;
                }
#pragma unroll
                for (int k = 0; k < 16; ++k) acc += v[k];
              }
            }
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
            const int j = (t < 256) ? (t >> 3) : WU_ROWS, part = t & 7;   // 256 threads: 32 neurons x 8
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
            if ((t & 31) == 0 && t < 256) {
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
      if (t == 0) trace_ev(p, l, 8);
      if (l + 1 < p.n_layers) ok = grid_barrier(sm, p, (uint32_t)(2 * l + 2) * G);
      if (t == 0) trace_ev(p, l, 9);
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
                            int32_t* status, uint64_t* trace, hc_stream_t stream) {
  if (!layers || n_layers <= 0 || !x_in || !masks || !x_out || !workspace || !status) return HC_ERR_ARG;
  if (inter <= 0 || inter > 32 * MAX_WORDS || (inter & 3) != 0 || (act != HC_ACT_SILU && act != HC_ACT_RELU))
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
  p.trace = trace;
  void* args[] = {&p};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(ffn_stack_kernel), dim3(G),
                                              dim3(STACK_THREADS), args, smem, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}
