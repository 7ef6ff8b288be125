// Fused hot/cold sparse FFN over a stack of layers (batch-1 decode).
//
// Per layer l this computes what SparseFFNLayer.forward does
// (engine.py:292-312): x_{l+1} = x_l + sparse_ffn(RMSNorm(x_l)), where
// sparse_ffn (engine.py:173-209) is the hot FP8 neurons plus the cold INT4
// neurons selected by the predictor, summed in-kernel (exact by linearity of
// down_proj in the neuron dimension, engine.py:184-188).  Layer l+1's
// predictor runs on layer l's input, as DesdemonaEngine.forward's lookahead
// prefetch does (engine.py:421-438).
//
// One persistent cooperative launch, one CTA per SM, one grid barrier per
// layer.  CTA c owns a slice of the hot neurons, a contiguous neuron-id range
// (for the predictor logits and the cold records in it) and a slice of the
// next predictor's W_down rows.  Warp roles:
//  * issuer warp: streams the CTA's units through a ring of 15 shared-memory
//    slots with 1-D bulk copies (TMA engine) completing on mbarriers, and
//    prefetches each layer's static weights into L2 one phase ahead;
//  * planner warp: turns the CTA's predicted-mask words into the ascending
//    list of active cold records (ColdWeightStore's id -> record lookup) and
//    prefetches those records into L2;
//  * 16 consumer warps: thread t owns x[8t, 8t+8) (f16 pairs in registers)
//    and y[8t, 8t+8); per group of neurons: partial gate/up dots, one CTA
//    reduction, activation, down-projection into y.
// Layer boundary: every CTA adds its partial y into a per-layer accumulator
// with vector atomics (and the next predictor's z partials likewise), arrives
// at the grid barrier, and after it reads x_{l+1} = x_l + y_l; the three
// accumulators rotate and are cleared two layers ahead.  The float atomics
// make the summation order, and so the last bits, vary between runs.
// Every wait (slot, mbarrier, grid barrier) is bounded by a time limit; on
// expiry the kernel ORs HC_ERR_TIMEOUT into the status word, drains its own
// copies in flight and returns.
#include "hc_common.cuh"

namespace hc {

constexpr int CONS_THREADS = 512;       // 16 consumer warps, 8 elements of x / y per thread
constexpr int NWARPS = CONS_THREADS / 32;
constexpr int EPT = H / CONS_THREADS;   // elements per consumer thread (8)
constexpr int STACK_THREADS = CONS_THREADS + 64;   // + issuer warp + planner warp
constexpr int SLOT_BYTES = 12800;       // one hot neuron (12288) or two cold records (2 x 6352)
constexpr int NSLOTS = 15;
constexpr int REC_SLOT_OFF = 6352;      // second cold record in a slot
constexpr int NB = 8;                   // cold records per reduction round
constexpr int NB_HOT = 4;               // hot neurons per reduction round
constexpr int WD_ROWS = 32;             // W_down tile: 32 k-rows x rank
constexpr int WU_ROWS = 32;             // W_up tile: 32 neurons x rank (+ bias) == one mask word
constexpr int COLD_LIST = 1024;         // max cold records one CTA handles per layer
constexpr int MAX_WORDS = 1024;         // mask words (inter <= 32768)
constexpr int HOT_BYTES = 3 * H;        // 12288
constexpr int NACC = 3;                 // rotating y / z accumulators
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;   // 2 s
static_assert(SLOT_BYTES % 16 == 0 && REC_SLOT_OFF % 16 == 0, "bulk copies need 16-byte aligned slots");
static_assert(HOT_BYTES <= SLOT_BYTES && REC_SLOT_OFF + REC_COPY <= SLOT_BYTES, "slot too small");
static_assert(32 * 96 * 4 + 32 * 4 <= SLOT_BYTES, "predictor tiles must fit a slot");
static_assert(EPT == 8, "the decoders assume 8 elements per thread");

struct StackSmem {
  alignas(128) uint8_t ring[NSLOTS][SLOT_BYTES];
  float xs[H];                      // predictor input RMSNorm_{l+1}(x_l) (rows of this CTA's W_down tiles)
  float red[2][NWARPS][2 * NB];     // per-warp partial (gate, up) dots, double buffered
  float z[128];                     // bottleneck of this layer's predictor
  float zred[CONS_THREADS];
  uint32_t own_words[MAX_WORDS];    // predicted mask words of this CTA's neuron-id range
  int32_t plan_list[COLD_LIST];     // nids, then record indices, of this CTA's active cold records
  int32_t plan_n;
  uint32_t ballot_word;
  int32_t flag;                     // consumer-wide broadcast
  int32_t abort;                    // sticky abort
  uint32_t cons_k;                  // slots consumed (for the drain)
  alignas(8) uint64_t full[NSLOTS];
  alignas(8) uint64_t empty[NSLOTS];
  alignas(8) uint64_t own_ready;    // consumers -> planner: own mask words of layer l written
  alignas(8) uint64_t plan_full;    // planner -> issuer/consumers: cold list of layer l ready
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
  float* yacc;               // [NACC][H]   partial-y accumulators
  float* zacc;               // [NACC][128] predictor bottleneck accumulators
  int32_t* status;
  uint64_t* trace;           // optional [n_layers][G][TRACE_EVENTS]
};

constexpr int TRACE_EVENTS = 24;
__device__ __forceinline__ void trace_ev(const StackParams& p, int l, int ev) {
  if (p.trace != nullptr) p.trace[((size_t)l * gridDim.x + blockIdx.x) * TRACE_EVENTS + ev] = globaltimer_ns();
}
__device__ __forceinline__ void trace_add(const StackParams& p, int l, int ev, uint64_t v) {
  if (p.trace != nullptr) p.trace[((size_t)l * gridDim.x + blockIdx.x) * TRACE_EVENTS + ev] += v;
}

constexpr size_t WS_YACC = 256;
constexpr size_t WS_ZACC = WS_YACC + sizeof(float) * NACC * H;
constexpr size_t WS_BYTES = WS_ZACC + sizeof(float) * NACC * 128;

__device__ __forceinline__ int64_t split_lo(int64_t n, int c, int G) { return n * c / G; }
// predictor tiles must fit a slot and split evenly over 8 lanes
__device__ __forceinline__ bool rank_ok(int r) { return r > 0 && r <= 96 && (r & 7) == 0; }

__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// --------------------------------------------------------------------------
// consumer helpers
// --------------------------------------------------------------------------
__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(*reinterpret_cast<const __half*>(p));
}
__device__ __forceinline__ uint32_t ld_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ int slot_of(uint32_t k) { return (int)(k % NSLOTS); }
__device__ __forceinline__ int slot_next(int s) { return s + 1 == NSLOTS ? 0 : s + 1; }

// consumer-wide broadcast of a decision taken by consumer thread 0
__device__ __forceinline__ bool cons_broadcast(StackSmem& sm, bool ok0) {
  if (threadIdx.x == 0) sm.flag = ok0 ? 1 : 0;
  named_bar(1, CONS_THREADS);
  return sm.flag != 0;
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
// wait expires flags the abort, which all threads read right after the
// group's barrier, so control flow stays uniform across named barriers.
__device__ __forceinline__ void cons_wait_group(StackSmem& sm, uint32_t k, int n, uint64_t* waited) {
  const uint64_t t0 = (waited != nullptr) ? globaltimer_ns() : 0;
  int s = slot_of(k);
  uint32_t par = (k / NSLOTS) & 1u;
  for (int i = 0; i < n; ++i) {
    if (!mbar_wait(&sm.full[s], par, WAIT_LIMIT_NS)) {
      sm.abort = 1;
      return;
    }
    s = slot_next(s);
    if (s == 0) par ^= 1u;
  }
  if (waited != nullptr) *waited += globaltimer_ns() - t0;
}
__device__ __forceinline__ void cons_release(StackSmem& sm, uint32_t k, int n) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) {
    int s = slot_of(k);
    for (int i = 0; i < n; ++i) {
      mbar_arrive(&sm.empty[s]);
      s = slot_next(s);
    }
  }
}

// block reduction over the consumer threads (result in every thread)
__device__ __forceinline__ float cons_sum(StackSmem& sm, float a) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  const int warp = threadIdx.x >> 5;
  named_bar(1, CONS_THREADS);
  if ((threadIdx.x & 31) == 0) sm.zred[warp] = a;
  named_bar(1, CONS_THREADS);
  a = 0.0f;
#pragma unroll
  for (int w = 0; w < NWARPS; ++w) a += sm.zred[w];
  return a;
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
  const uint8_t* slot[NB_HOT];
  {
    int s = slot_of(ck);
#pragma unroll
    for (int j = 0; j < NB_HOT; ++j) {
      slot[j] = sm.ring[s] + EPT * t;
      s = slot_next(s);
    }
  }
  cons_wait_group(sm, ck, nb, waited);
  float v[2 * NB_HOT];
#pragma unroll
  for (int j = 0; j < NB_HOT; ++j) {
    v[j] = 0.0f;
    v[NB_HOT + j] = 0.0f;
    if (j < nb) {
      v[j] = dot8_fp8(*reinterpret_cast<const uint2*>(slot[j]), x);
      v[NB_HOT + j] = dot8_fp8(*reinterpret_cast<const uint2*>(slot[j] + H), x);
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
      const uint2 dw = *reinterpret_cast<const uint2*>(slot[n] + 2 * H);
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
  const uint8_t* rec[NB];
  {
    int s = slot_of(ck);
#pragma unroll
    for (int j = 0; j < NB; j += 2) {
      rec[j] = sm.ring[s];
      rec[j + 1] = sm.ring[s] + REC_SLOT_OFF;
      s = slot_next(s);
    }
  }
  cons_wait_group(sm, ck, nslots, waited);
  float v[2 * NB];
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    v[j] = 0.0f;
    v[NB + j] = 0.0f;
    if (j < nb) {
      v[j] = dot8_int4(ld_int4x8(rec[j] + 4 * t), x) * ld_half(rec[j] + SCALE_OFF + gs);
      v[NB + j] = dot8_int4(ld_int4x8(rec[j] + VEC_BYTES + 4 * t), x) * ld_half(rec[j] + SCALE_OFF + 2 * NGROUPS + gs);
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
      const __half c16 = __float2half_rn(an * ld_half(rec[n] + SCALE_OFF + 4 * NGROUPS + gs));
      const __half c16s = __hmul(c16, __float2half(0.0625f));    // exact unless subnormal; csb tracks it
      csa += __half2float(c16);
      csb += __half2float(c16s);
      uint32_t h[4];
      int4_pairs(ld_int4x8(rec[n] + 2 * VEC_BYTES + 4 * t), h);
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

// grid barrier: arrive (after this CTA's atomics) ...
__device__ __forceinline__ void grid_arrive(const StackParams& p) {
  named_bar(1, CONS_THREADS);
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(p.bar_count, 1u);
  }
}
// ... and wait (thread 0 spins, bounded; result broadcast)
__device__ bool grid_wait(StackSmem& sm, const StackParams& p, uint32_t target) {
  bool ok0 = true;
  if (threadIdx.x == 0) {
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

// --------------------------------------------------------------------------
// producer helpers
// --------------------------------------------------------------------------
struct Producer {
  uint32_t k = 0;       // fills issued
  uint64_t pol = 0;
  bool ok = true;
};

// issuer lane 0: take the next slot (bounded wait for it to be empty)
__device__ __forceinline__ uint8_t* prod_slot(StackSmem& sm, Producer& pr, uint32_t bytes, uint64_t* waited) {
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

// per-layer work split of CTA c (shared by all three roles)
struct Split {
  int64_t h0, h1;       // hot neurons
  int u0, u1;           // own W_up tiles == own mask words (neuron ids [32 u0, 32 u1))
  int d0, d1;           // W_down tiles of the next layer's predictor
};
__device__ __forceinline__ Split make_split(const StackParams& p, const hc_layer_desc& d, bool pred_next, int c,
                                            int G) {
  Split s;
  s.h0 = split_lo(d.n_hot, c, G);
  s.h1 = split_lo(d.n_hot, c + 1, G);
  s.u0 = (int)split_lo(p.words, c, G);
  s.u1 = (int)split_lo(p.words, c + 1, G);
  const int nd = H / WD_ROWS;
  s.d0 = pred_next ? (int)split_lo(nd, c, G) : 0;
  s.d1 = pred_next ? (int)split_lo(nd, c + 1, G) : 0;
  return s;
}
// layer l computes its own mask words from its predictor (else they are given or all ones)
__device__ __forceinline__ bool layer_logits(const StackParams& p, const hc_layer_desc& d, int l) {
  return l > 0 && !p.masks_given && d.pred_w_up != nullptr && rank_ok(d.rank);
}
__device__ __forceinline__ bool next_pred(const StackParams& p, int l) {
  if (l + 1 >= p.n_layers || p.masks_given) return false;
  const hc_layer_desc& dn = p.layers[l + 1];
  return dn.pred_w_up != nullptr && rank_ok(dn.rank);
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
      mbar_init(&sm.empty[s], NWARPS);
    }
    mbar_init(&sm.own_ready, 1);
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
    // Per layer: wait for the CTA's own mask words, then list the active cold
    // ids of its neuron range in ascending order, resolve them to record
    // indices (batched table loads) and prefetch the records into L2.
    const int lane = tid & 31;
    bool ok = true;
    for (int l = 0; l < p.n_layers && ok; ++l) {
      const hc_layer_desc d = p.layers[l];
      const Split sp = make_split(p, d, false, c, G);
      if (l > 0) {
        if (lane == 0) ok = mbar_wait(&sm.plan_empty, (uint32_t)(l - 1) & 1u, WAIT_LIMIT_NS);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
      }
      if (lane == 0) ok = mbar_wait(&sm.own_ready, (uint32_t)l & 1u, WAIT_LIMIT_NS);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const int nw = sp.u1 - sp.u0;
      // lane-contiguous word chunks; counts, prefix
      const int wpl = (nw + 31) / 32;
      const int wb = lane * wpl, we = min(nw, wb + wpl);
      int mycnt = 0;
      for (int w = wb; w < we; ++w) {
        const uint32_t m = sm.own_words[w] & __ldg(d.fetch_bits + sp.u0 + w);
        sm.own_words[w] = m;
        mycnt += __popc(m);
      }
      int incl = mycnt;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
      }
      int cnt = __shfl_sync(0xffffffffu, incl, 31);
      if (cnt > COLD_LIST) {
        if (lane == 0) atomicOr(p.status, HC_ERR_UNSUPPORTED);
        cnt = COLD_LIST;
      }
      int rank = incl - mycnt;
      for (int w = wb; w < we && rank < cnt; ++w) {
        uint32_t m = sm.own_words[w];
        while (m && rank < cnt) {
          const int bit = __ffs(m) - 1;
          m &= m - 1;
          sm.plan_list[rank++] = (sp.u0 + w) * 32 + bit;
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
    // Lane 0 streams the CTA's units in the consumers' order: this layer's own
    // W_up tiles, hot neurons, the next predictor's W_down tiles, the
    // planner's cold records.  At each layer start it prefetches the layer's
    // static ranges into L2 so HBM keeps streaming across the grid barrier.
    const int lane = tid & 31;
    Producer pr;
    if (lane == 0) {
      pr.pol = l2_evict_first_policy();
      for (int l = 0; l < p.n_layers && pr.ok; ++l) {
        const hc_layer_desc d = p.layers[l];
        const bool pred_next = next_pred(p, l);
        const bool logits = layer_logits(p, d, l);
        const Split sp = make_split(p, d, pred_next, c, G);
        const hc_layer_desc* dn = pred_next ? &p.layers[l + 1] : nullptr;
        const int rank_n = pred_next ? dn->rank : 0;
        trace_ev(p, l, 10);
        if (sp.h1 > sp.h0) prefetch_l2_range(d.hot + sp.h0 * HOT_BYTES, (size_t)(sp.h1 - sp.h0) * HOT_BYTES);
        if (sp.d1 > sp.d0)
          prefetch_l2_range(dn->pred_w_down_t + (size_t)sp.d0 * WD_ROWS * rank_n,
                            (size_t)(sp.d1 - sp.d0) * WD_ROWS * rank_n * 4);
        if (pred_next && sp.u1 > sp.u0) {
          const int rows = min(sp.u1 * WU_ROWS, p.inter) - sp.u0 * WU_ROWS;
          prefetch_l2_range(dn->pred_w_up + (size_t)sp.u0 * WU_ROWS * rank_n, (size_t)rows * rank_n * 4);
        }
        uint64_t iw_hot = 0, iw_cold = 0;
        // own W_up tiles of this layer's predictor (consumed first)
        if (logits) {
          for (int u = sp.u0; u < sp.u1 && pr.ok; ++u) {
            const int rows = min(WU_ROWS, p.inter - u * WU_ROWS);
            const uint32_t wbytes = rows * d.rank * 4, bbytes = rows * 4;
            uint8_t* dst = prod_slot(sm, pr, wbytes + bbytes, nullptr);
            if (!dst) break;
            uint64_t* bar = &sm.full[pr.k % NSLOTS];
            bulk_g2s(dst, d.pred_w_up + (size_t)u * WU_ROWS * d.rank, wbytes, bar, pr.pol);
            bulk_g2s(dst + WU_ROWS * d.rank * 4, d.pred_b_up + (size_t)u * WU_ROWS, bbytes, bar, pr.pol);
            ++pr.k;
          }
        }
        // hot neurons
        for (int64_t i = sp.h0; i < sp.h1 && pr.ok; ++i) {
          uint8_t* dst = prod_slot(sm, pr, HOT_BYTES, p.trace ? &iw_hot : nullptr);
          if (!dst) break;
          bulk_g2s(dst, d.hot + i * HOT_BYTES, HOT_BYTES, &sm.full[pr.k % NSLOTS], pr.pol);
          ++pr.k;
        }
        trace_ev(p, l, 11);
        // W_down tiles of the next layer's predictor
        for (int u = sp.d0; u < sp.d1 && pr.ok; ++u) {
          const uint32_t bytes = WD_ROWS * rank_n * 4;
          uint8_t* dst = prod_slot(sm, pr, bytes, nullptr);
          if (!dst) break;
          bulk_g2s(dst, dn->pred_w_down_t + (size_t)u * WD_ROWS * rank_n, bytes, &sm.full[pr.k % NSLOTS], pr.pol);
          ++pr.k;
        }
        if (!pr.ok) break;
        trace_ev(p, l, 12);
        // the planner's cold records, two per slot
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
    const int t = tid, lane = t & 31;
    uint32_t ck = 0;
    int gbuf = 0;
    bool ok = true;
    float x[EPT];
    {
      const float4* src = reinterpret_cast<const float4*>(p.x_in + EPT * t);
      const float4 q0 = __ldg(src), q1 = __ldg(src + 1);
      x[0] = q0.x; x[1] = q0.y; x[2] = q0.z; x[3] = q0.w; x[4] = q1.x; x[5] = q1.y; x[6] = q1.z; x[7] = q1.w;
    }
    for (int l = 0; l < p.n_layers && ok; ++l) {
      const hc_layer_desc d = p.layers[l];
      const bool pred_next = next_pred(p, l);
      const bool logits = layer_logits(p, d, l);
      if (t == 0 && c == 0 && !p.masks_given && d.pred_w_up != nullptr && !rank_ok(d.rank))
        atomicOr(p.status, HC_ERR_UNSUPPORTED);
      const Split sp = make_split(p, d, pred_next, c, G);
      const hc_layer_desc* dn = pred_next ? &p.layers[l + 1] : nullptr;
      const int rank_n = pred_next ? dn->rank : 0;
      if (t == 0) trace_ev(p, l, 0);
      uint64_t w_hot = 0, w_cold = 0;

      // ---- layer boundary: x_l = x_{l-1} + y_{l-1} once every CTA has added its part
      if (l > 0) {
        ok = grid_wait(sm, p, (uint32_t)l * G);
        if (!ok) break;
        const float4* yv = reinterpret_cast<const float4*>(p.yacc + (size_t)((l - 1) % NACC) * H + EPT * t);
        const float4 a = __ldcg(yv), b = __ldcg(yv + 1);
        x[0] += a.x; x[1] += a.y; x[2] += a.z; x[3] += a.w; x[4] += b.x; x[5] += b.y; x[6] += b.z; x[7] += b.w;
        if (p.x_hist && c == 0) {
          float4* h = reinterpret_cast<float4*>(p.x_hist + (size_t)(l - 1) * H + EPT * t);
          h[0] = make_float4(x[0], x[1], x[2], x[3]);
          h[1] = make_float4(x[4], x[5], x[6], x[7]);
        }
      }
      // clear the accumulators layer l+1 adds into (last read before the barrier just passed)
      {
        float* yz = p.yacc + (size_t)((l + 1) % NACC) * H;
        for (int i = (int)split_lo(H / 4, c, G) + t; i < (int)split_lo(H / 4, c + 1, G); i += CONS_THREADS)
          reinterpret_cast<float4*>(yz)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c == 0 && t < 128) p.zacc[(size_t)((l + 2) % NACC) * 128 + t] = 0.0f;
      }
      if (t == 0) trace_ev(p, l, 1);

      // ---- RMSNorm (engine.py:295; torch.nn.RMSNorm); x as f16 pairs in registers
      float y[EPT];
      XRegs xr;
      {
        float nw[EPT];
        if (d.norm_w) {
          const float4* wsrc = reinterpret_cast<const float4*>(d.norm_w + EPT * t);
          const float4 w0 = __ldg(wsrc), w1 = __ldg(wsrc + 1);
          nw[0] = w0.x; nw[1] = w0.y; nw[2] = w0.z; nw[3] = w0.w; nw[4] = w1.x; nw[5] = w1.y; nw[6] = w1.z; nw[7] = w1.w;
        } else {
#pragma unroll
          for (int i = 0; i < EPT; ++i) nw[i] = 1.0f;
        }
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < EPT; ++i) ss = fmaf(x[i], x[i], ss);
        ss = cons_sum(sm, ss);
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
          // only the rows of this CTA's W_down tiles are read
          const int r0 = sp.d0 * WD_ROWS, r1 = sp.d1 * WD_ROWS;
          if (EPT * t + EPT > r0 && EPT * t < r1) {
#pragma unroll
            for (int i = 0; i < EPT; ++i) {
              const float w = dn->norm_w ? __ldg(dn->norm_w + EPT * t + i) : 1.0f;
              sm.xs[EPT * t + i] = x[i] * rstd * w;
            }
          }
        }
#pragma unroll
        for (int i = 0; i < EPT; ++i) y[i] = 0.0f;
      }
      if (t == 0) trace_ev(p, l, 2);

      // ---- own mask words of layer l (predictor logits of the own id range)
      {
        const int nw = sp.u1 - sp.u0;
        uint32_t* mrow = p.masks + (size_t)l * p.words;
        if (!logits) {
          for (int w = t; w < nw; w += CONS_THREADS) {
            uint32_t m;
            if (l == 0 || p.masks_given) {
              m = __ldcg(mrow + sp.u0 + w);
            } else {
              // no predictor: fetch every cold neuron (engine.py:282-283)
              const int valid = min(32, p.inter - 32 * (sp.u0 + w));
              m = valid >= 32 ? 0xffffffffu : ((1u << valid) - 1u);
              mrow[sp.u0 + w] = m;
            }
            sm.own_words[w] = m;
          }
        } else if (nw > 0) {
          // z of this layer (complete: summed into zacc by all CTAs before the barrier)
          if (t < d.rank) sm.z[t] = __ldcg(p.zacc + (size_t)(l % NACC) * 128 + t);
          named_bar(1, CONS_THREADS);
          const int per = d.rank / 8;
          for (int u = sp.u0; u < sp.u1 && ok; ++u) {
            ok = cons_acquire(sm, ck, 1);
            if (!ok) break;
            const float* tile = reinterpret_cast<const float*>(sm.ring[slot_of(ck)]);
            const int rows = min(WU_ROWS, p.inter - u * WU_ROWS);
            const int j = (t < 256) ? (t >> 3) : WU_ROWS, part = t & 7;   // 256 threads: 32 neurons x 8
            float acc = 0.0f;
            if (j < rows)
              for (int i = 0; i < per; ++i) acc = fmaf(tile[j * d.rank + part * per + i], sm.z[part * per + i], acc);
            acc += __shfl_xor_sync(0xffffffffu, acc, 4);
            acc += __shfl_xor_sync(0xffffffffu, acc, 2);
            acc += __shfl_xor_sync(0xffffffffu, acc, 1);
            const float lg = acc + ((j < rows) ? tile[WU_ROWS * d.rank + j] : 0.0f);
            const bool on = (j < rows) && (lg >= p.thr);
            const unsigned b = __ballot_sync(0xffffffffu, on && part == 0);
            if (lane == 0 && t < 256) {
              const uint32_t nib = ((b >> 0) & 1u) | (((b >> 8) & 1u) << 1) | (((b >> 16) & 1u) << 2) |
                                   (((b >> 24) & 1u) << 3);
              atomicOr(&sm.ballot_word, nib << (4 * (t >> 5)));
            }
            named_bar(1, CONS_THREADS);
            if (t == 0) {
              sm.own_words[u - sp.u0] = sm.ballot_word;
              mrow[u] = sm.ballot_word;
              sm.ballot_word = 0;
            }
            cons_release(sm, ck, 1);
            ck += 1;
          }
        }
        named_bar(1, CONS_THREADS);
        if (t == 0) mbar_arrive(&sm.own_ready);
      }
      if (!ok) break;
      if (t == 0) trace_ev(p, l, 3);

      // ---- hot neurons, groups of NB_HOT
      for (int64_t i = sp.h0; i < sp.h1; i += NB_HOT) {
        const int nb = (int)(sp.h1 - i < NB_HOT ? sp.h1 - i : NB_HOT);
        if (hot_group(sm, p, d.hot_scale, i, nb, ck, gbuf, xr, y, (t == 0 && p.trace) ? &w_hot : nullptr)) {
          ok = false;
          break;
        }
        ck += nb;
        gbuf ^= 1;
      }
      if (!ok) break;
      if (t == 0) trace_ev(p, l, 4);

      // ---- W_down tiles of predictor l+1 -> z partials added into zacc
      for (int u = sp.d0; u < sp.d1 && ok; ++u) {
        ok = cons_acquire(sm, ck, 1);
        if (!ok) break;
        const float* tile = reinterpret_cast<const float*>(sm.ring[slot_of(ck)]);
        const int parts = CONS_THREADS / rank_n;
        float acc = 0.0f;
        const int r = t % rank_n, part = t / rank_n;
        if (part < parts)
          for (int row = part; row < WD_ROWS; row += parts)
            acc = fmaf(tile[row * rank_n + r], sm.xs[u * WD_ROWS + row], acc);
        sm.zred[t] = acc;
        named_bar(1, CONS_THREADS);
        if (t < rank_n) {
          float s = 0.0f;
          for (int q = 0; q < parts; ++q) s += sm.zred[q * rank_n + t];
          atomicAdd(p.zacc + (size_t)((l + 1) % NACC) * 128 + t, s);
        }
        named_bar(1, CONS_THREADS);
        cons_release(sm, ck, 1);
        ck += 1;
      }
      if (!ok) break;
      if (t == 0) trace_ev(p, l, 5);

      // ---- cold records: the planner's list of this CTA's active cold neurons
      {
        bool ok0 = true;
        if (t == 0) ok0 = mbar_wait(&sm.plan_full, (uint32_t)l & 1u, WAIT_LIMIT_NS);
        ok = cons_broadcast(sm, ok0);
        if (!ok) break;
        while (!mbar_try_wait(&sm.plan_full, (uint32_t)l & 1u)) {
        }
        const int cnt = sm.plan_n;
        named_bar(1, CONS_THREADS);
        if (t == 0) {
          mbar_arrive(&sm.plan_empty);
          trace_ev(p, l, 6);
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
      if (!ok) break;
      if (t == 0) {
        trace_ev(p, l, 7);
        trace_add(p, l, 15, w_hot);
        trace_add(p, l, 16, w_cold);
      }
      // ---- add this CTA's partial y, arrive at the layer's grid barrier
      {
        float* ya = p.yacc + (size_t)(l % NACC) * H + EPT * t;
        red_add_v4(ya, y[0], y[1], y[2], y[3]);
        red_add_v4(ya + 4, y[4], y[5], y[6], y[7]);
      }
      grid_arrive(p);
      if (t == 0) trace_ev(p, l, 8);
    }
    // ---- output: x_L = x_{L-1} + y_{L-1}
    if (ok) {
      const int L = p.n_layers;
      ok = grid_wait(sm, p, (uint32_t)L * G);
      if (ok && c == 0) {
        const float4* yv = reinterpret_cast<const float4*>(p.yacc + (size_t)((L - 1) % NACC) * H + EPT * t);
        const float4 a = __ldcg(yv), b = __ldcg(yv + 1);
        const float4 o0 = make_float4(x[0] + a.x, x[1] + a.y, x[2] + a.z, x[3] + a.w);
        const float4 o1 = make_float4(x[4] + b.x, x[5] + b.y, x[6] + b.z, x[7] + b.w);
        float4* out = reinterpret_cast<float4*>(p.x_out + EPT * t);
        out[0] = o0;
        out[1] = o1;
        if (p.x_hist) {
          float4* h = reinterpret_cast<float4*>(p.x_hist + (size_t)(L - 1) * H + EPT * t);
          h[0] = o0;
          h[1] = o1;
        }
      }
    }
    if (t == 0) {
      sm.cons_k = ck;
      if (!ok) atomicOr(p.status, HC_ERR_TIMEOUT);
    }
    __syncthreads();
  }

  // Once every CTA is past its last read: reset the barrier counters and clear
  // the accumulators, so the next launch starts from a clean workspace.
  __shared__ int s_last;
  if (tid == 0) {
    __threadfence();
    s_last = atomicAdd(p.exit_count, 1u) == (uint32_t)G - 1;
  }
  __syncthreads();
  if (s_last) {
    __threadfence();
    for (int i = tid; i < NACC * H / 4; i += STACK_THREADS)
      reinterpret_cast<float4*>(p.yacc)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = tid; i < NACC * 128; i += STACK_THREADS) p.zacc[i] = 0.0f;
    if (tid == 0) {
      *p.bar_count = 0;
      *p.exit_count = 0;
    }
    __threadfence();
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
  return (int64_t)WS_BYTES;
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
  const int words = (inter + 31) / 32;
  if ((int64_t)((words + G - 1) / G) * 32 > COLD_LIST) return HC_ERR_UNSUPPORTED;   // own range too wide
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
  p.words = words;
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
  p.yacc = reinterpret_cast<float*>(ws + WS_YACC);
  p.zacc = reinterpret_cast<float*>(ws + WS_ZACC);
  p.status = status;
  p.trace = trace;
  void* args[] = {&p};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(ffn_stack_kernel), dim3(G),
                                              dim3(STACK_THREADS), args, smem, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}
