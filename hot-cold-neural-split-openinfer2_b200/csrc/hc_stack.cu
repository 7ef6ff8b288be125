// Fused hot/cold sparse FFN over a stack of layers (batch-1 decode).
//
// Per layer l this computes what SparseFFNLayer.forward does
// (engine.py:292-312): x_{l+1} = x_l + sparse_ffn(RMSNorm(x_l)), where
// sparse_ffn (engine.py:173-209) is the hot FP8 neurons plus the cold INT4
// neurons selected by the predictor, summed in-kernel (exact by linearity of
// down_proj in the neuron dimension, engine.py:184-188).  Layer l+1's
// predictor runs on layer l's input, as DesdemonaEngine.forward's lookahead
// prefetch does (engine.py:421-438).  Layer 0's mask words are the caller's
// (masks_given = 0) or, with masks_given = 2, predicted by the kernel itself
// at its start from RMSNorm_0(x_0) (engine.py:422), the same way.
//
// One persistent cooperative launch, one CTA per SM, one grid barrier per
// layer.  CTA c owns a contiguous neuron-id range (its predictor logits and
// the active cold records in it) and a slice of the next predictor's W_down
// rows.  Every CTA publishes its ascending list of active cold records into a
// per-layer global pool; once the pool is complete, CTA c streams the pool
// entries [c n / G, (c+1) n / G) and then the hot neurons [c n_hot / G, (c+1)
// n_hot / G), so every SM moves the same bytes whatever the distribution of
// active ids.  Layer l+1's logits are computed at the end of layer l, once a
// global counter shows every CTA has added its W_down partials, so layer
// l+1's cold list is built, and its records are streamed in, while the grid
// waits at the layer boundary.
//
// Roles:
//  * issuer warp: streams the CTA's groups (cold records, hot neurons)
//    through a ring of shared-memory entries with 1-D bulk copies (TMA
//    engine) completing on mbarriers, and prefetches the layer's static
//    ranges into L2;
//  * planner warp: runs the next layer's predictor for the CTA's share (its
//    W_down rows, then, once every CTA's share is in, the logits of its
//    neuron-id range), and turns the mask words into the ascending list of
//    its active cold records (ColdWeightStore's id -> record lookup), which
//    it prefetches into L2;
//  * 4 consumer subgroups of 128 threads: group g of a layer belongs to
//    subgroup g % 4; thread u owns elements [32u, 32u+32) of every row and of
//    its subgroup's partial y.  FP8 rows are dotted with RMSNorm(x) in f16
//    (f16 x f16 products, fp32 sums); INT4 rows with RMSNorm(x) as 16-bit
//    fixed point (two byte digits per element, dp4a, exact integer sums); down
//    columns are added
//    into y with f16 x f16 products and fp32 sums, skipping neurons whose
//    gated activation is exactly zero.
// Layer boundary: the subgroups' partial y are summed in shared memory, added
// to a per-layer global accumulator with one 16 KB bulk reduction
// (cp.reduce.async.bulk add.f32, performed in L2), and after the grid barrier
// every CTA reads x_{l+1} = x_l + y_l.  The float reductions make the
// summation order, and so the last bits, vary between runs.
// Every wait on another agent (slot, mbarrier, grid barrier) is bounded by a
// time limit; on expiry the kernel ORs HC_ERR_TIMEOUT into the status word,
// waits (bounded) for its own copies in flight and returns.
#include <algorithm>

#include "hc_common.cuh"

namespace hc {

constexpr int CONS_THREADS = 512;
constexpr int NWARPS = CONS_THREADS / 32;
constexpr int EPT = H / CONS_THREADS;   // element layout: x[8t, 8t+8) per consumer thread
constexpr int NSG = 4;                  // consumer subgroups
constexpr int SG_THREADS = CONS_THREADS / NSG;
constexpr int SG_WARPS = SG_THREADS / 32;
constexpr int SPT = H / SG_THREADS;     // 32 elements per subgroup thread
constexpr int STACK_THREADS = CONS_THREADS + 64;   // + issuer warp + planner warp
constexpr int HALF_BYTES = 12800;       // one hot neuron (12288) or two cold records (2 x 6352)
constexpr int ENTRY_BYTES = 2 * HALF_BYTES;   // one group: two halves
constexpr int NE = 7;                   // ring entries
constexpr int REC_SLOT_OFF = 6352;      // second cold record in a half
constexpr int NB_HOT = 2;               // hot neurons per group (one per slot)
constexpr int NB_COLD = 4;              // cold records per group (two per slot)
constexpr int WD_ROWS = 32;             // W_down tile: 32 k-rows x rank
constexpr int WU_ROWS = 32;             // W_up tile: 32 neurons x rank (+ bias) == one mask word
constexpr int COLD_LIST = 1024;         // neuron ids one CTA owns (and so cold records per layer)
constexpr int OWN_WORDS = COLD_LIST / 32;
constexpr int HOT_BYTES = 3 * H;        // 12288
constexpr int NACC = 3;                 // rotating y / z / hot-claim accumulators
constexpr int YCOPIES = 1;              // CTA c adds its partial y into copy c % YCOPIES
constexpr int POOL_CAP = 32768;         // cold-pool entries per layer (>= inter)
constexpr int WD_TILES = 4096 / 32;     // W_down tiles of a predictor (H / WD_ROWS)
constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;   // 2 s: default limit of every wait on another agent
static_assert(HALF_BYTES % 128 == 0 && REC_SLOT_OFF % 16 == 0, "halves must stay 16-byte aligned");
static_assert(HOT_BYTES <= HALF_BYTES && REC_SLOT_OFF + REC_COPY <= HALF_BYTES, "half too small");
constexpr int PRED_RANK_MAX = 96;       // in-kernel predictors: rank <= 96, a multiple of 8
constexpr int PBUF_BYTES = WU_ROWS * PRED_RANK_MAX * 4 + WU_ROWS * 4;   // one W_up tile + bias (>= a W_down tile)
static_assert(WD_ROWS * PRED_RANK_MAX * 4 <= PBUF_BYTES, "predictor tiles must fit the planner buffer");
static_assert(NE > NSG, "the subgroups' entries advance by NSG per group");
static_assert(SPT == 32 && EPT == 8, "the decoders assume 32 elements per subgroup thread");

enum : uint8_t { UNIT_HOT = 1, UNIT_COLD = 2 };

// Written by the issuer before it arms an entry's mbarrier.
struct SlotInfo {
  uint32_t pos;      // ring position of this fill
  int16_t layer;
  uint8_t kind;      // UNIT_*
  uint8_t n;         // units in the group (1..NB_*)
  int32_t index;     // first hot neuron / tile of the group
  int32_t pad;
};

struct StackSmem {
  alignas(128) uint8_t pbuf[PBUF_BYTES];   // planner: one predictor tile (W_down or W_up + bias)
  __half xh[H];                     // RMSNorm_l(x) as f16 (hot neurons, xslot order); with xq, a y stage later
  uint4 xq[CONS_THREADS];           // the same as 16-bit fixed point, byte digits per 8 elements (xslot order)
  float ystage[H];                  // partial y stage of the layer-end tree (ypos4 layout); earlier in
                                    // the layer, the planner's W_down rows RMSNorm_{l+1}(x_l)
  float z[128];                     // planner: bottleneck of the next layer's predictor
  float rstd0;                      // consumers -> planner: 1 / RMS of x_0 (layer 0's own prediction)
  int2 chunk[H / SPT];              // per 32 elements: (-8 * sum of the fixed-point values, bits of 2^-s)
  float zred[NWARPS];
  float red[NSG][2][SG_WARPS][2 * NB_COLD];
  int32_t sgdec[NSG][2][2];         // per-subgroup decision of its poller: (result, claimed group)
  int32_t gnext[2];                 // next group of layer l to claim (l & 1), shared by the subgroups
  uint64_t tstat[8];                // trace counters of subgroup 0's poller
  int32_t plan_list[COLD_LIST];     // nids, then record indices, of this CTA's active cold records
  uint32_t own_words[OWN_WORDS];    // predicted mask words of this CTA's neuron-id range
  SlotInfo info[NE];
  int32_t ngroups[4];               // groups issued per layer (l & 3)
  int32_t sealed;                   // last layer whose groups are all issued
  int32_t cons_layer;               // last layer the consumers started
  int32_t abort;
  int32_t flag;
  int32_t last;
  alignas(8) uint64_t full[NE];
  alignas(8) uint64_t empty[NE];
  alignas(8) uint64_t phase0_done;  // consumers -> planner: normalised input (and W_down rows) ready
  alignas(8) uint64_t pbar;         // planner's own tile copies
  alignas(8) uint64_t wdown_done;   // planner -> consumers: done with the W_down rows in ystage
};
constexpr size_t RING_OFF = (sizeof(StackSmem) + 127) / 128 * 128;
static_assert(RING_OFF + (size_t)NE * ENTRY_BYTES <= 227 * 1024, "stack kernel shared memory exceeds 227 KB");

struct StackParams {
  const hc_layer_desc* layers;
  int n_layers;
  int n_compute;             // layers computed: n_layers, or n_layers - 1 when the last is only predicted
  int inter;
  int words;                 // ceil(inter / 32)
  int words_lo, words_n;     // mask words (neuron ids / 32) this GPU owns
  int tp_size, tp_rank;      // GPUs sharing each layer's neurons, this GPU's index
  void* const* peer_buf;     // [tp_size] every GPU's exchange buffer (device pointers)
  uint32_t seq_base;         // launches so far x n_layers, identical on every GPU
  const void* x_in;          // [H] fp32, or fp16 with io_f16
  uint32_t* masks;           // [n_layers][words]
  int masks_given;
  void* x_out;               // [H] fp32, or fp16 with io_f16
  int io_f16;
  float* x_hist;
  float eps;
  int relu;
  int both;
  float thr;
  int pred0;                 // layer 0's mask words are predicted in the kernel too (masks_given == 2)
  uint32_t* bar_count;
  uint32_t* exit_count;
  uint32_t* hot_next;        // [NACC] hot-neuron claims per layer
  uint32_t* zdone;           // [NACC] W_down tiles added into zacc per layer
  uint32_t* gfill;           // [NACC] cold-pool entries reserved per layer
  uint32_t* gclaim;          // [NACC] cold-pool entries claimed per layer
  uint32_t* gdone;           // [NACC] CTAs that published their cold list per layer
  int32_t* gpool;            // [NACC][POOL_CAP] cold record indices of the layer, all CTAs
  float* yacc;               // [NACC][YCOPIES][H] partial-y accumulators
  float* zacc;               // [NACC][128] predictor bottleneck accumulators
  float* xbuf;               // [NACC][H]   x_l, written by CTA 0
  int32_t* status;
  uint64_t* trace;           // optional [n_layers][G][TRACE_EVENTS]
  uint64_t wait_ns;          // limit of every wait on another agent (CTA, GPU, copy engine)
};

constexpr int TRACE_EVENTS = 40;
__device__ __forceinline__ void trace_ev(const StackParams& p, int l, int ev) {
  if (p.trace != nullptr) p.trace[((size_t)l * gridDim.x + blockIdx.x) * TRACE_EVENTS + ev] = globaltimer_ns();
}
__device__ __forceinline__ void trace_set(const StackParams& p, int l, int ev, uint64_t v) {
  if (p.trace != nullptr) p.trace[((size_t)l * gridDim.x + blockIdx.x) * TRACE_EVENTS + ev] = v;
}

constexpr size_t WS_EXIT = 16;
constexpr size_t WS_HOT_NEXT = 32;
constexpr size_t WS_ZDONE = 48;
constexpr size_t WS_GFILL = 64;
constexpr size_t WS_GCLAIM = 80;
constexpr size_t WS_GDONE = 96;
constexpr size_t WS_YACC = 256;
constexpr size_t WS_ZACC = WS_YACC + sizeof(float) * NACC * YCOPIES * H;
constexpr size_t WS_XBUF = WS_ZACC + sizeof(float) * NACC * 128;
constexpr size_t WS_POOL = WS_XBUF + sizeof(float) * NACC * H;
constexpr size_t WS_BYTES = WS_POOL + sizeof(int32_t) * NACC * POOL_CAP;

__device__ __forceinline__ int64_t split_lo(int64_t n, int c, int G) { return n * c / G; }
// predictor tiles must fit a slot and split evenly over 4 threads per neuron
__device__ __forceinline__ bool rank_ok(int r) { return r > 0 && r <= PRED_RANK_MAX && (r & 7) == 0; }

// Exchange buffer of one GPU (tensor-parallel mode): a 256-byte header, then
// per slot (exchange number % NACC) and sender one row of H words of 8 bytes,
// (sequence number << 32) | bits of the float.  An aligned 8-byte store is
// single-copy atomic, so a receiver that reads the exchange's sequence number
// in a word also reads that word's value: the data carries its own arrival
// flag, and no fence or counter is needed between the stores and the reads.
constexpr size_t XCHG_HDR = 256;
constexpr int TP_MAX = 8;              // GPUs per tensor-parallel group
constexpr int KP_MAX = 32;             // CTAs that push slices of a GPU's partial to its peers
__device__ __forceinline__ unsigned long long* xchg_row(void* buf, int slot, int sender, int tp) {
  return reinterpret_cast<unsigned long long*>(reinterpret_cast<char*>(buf) + XCHG_HDR) +
         ((size_t)slot * tp + sender) * H;
}
__device__ __forceinline__ void st_pair_sys(unsigned long long* dst, unsigned long long a, unsigned long long b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(dst), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ ulonglong2 ld_pair_sys(const unsigned long long* src) {
  ulonglong2 v;
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(src) : "memory");
  return v;
}

// Slot of consumer thread t's 8 normalised elements [8t, 8t+8) in the xh / xq
// arrays (16 bytes each): subgroup thread u = t / 4 owns elements
// [32u, 32u+32), its j-th 16 bytes at slot j x 128 + u, so that the 128
// threads' loads of their j-th word are contiguous (no bank conflicts).
__device__ __forceinline__ int xslot(int t) { return (t & 3) * SG_THREADS + (t >> 2); }

// Shared-memory stage of the partial y: the 4 elements [32 u + 4 j, +4) of
// subgroup thread u sit at float4 index 8 u + (j ^ (u & 7)), so that u's 8
// float4 stores and consumer thread t's reads of its elements [8t, 8t+8) (two
// float4) are free of bank conflicts.
__device__ __forceinline__ int ypos4(int u, int j) { return 8 * u + (j ^ (u & 7)); }
__device__ __forceinline__ int ypos4_of_thread(int t, int h) { return ypos4(t >> 2, 2 * (t & 3) + h); }

// This GPU's partial y of layer l (summed over its CTAs): the local accumulator.
__device__ __forceinline__ void load_y_local(const StackParams& p, int l, int t, float4& a, float4& b) {
  a = make_float4(0.f, 0.f, 0.f, 0.f);
  b = a;
#pragma unroll
  for (int k = 0; k < YCOPIES; ++k) {
    const float4* yv = reinterpret_cast<const float4*>(p.yacc + ((size_t)(l % NACC) * YCOPIES + k) * H + 8 * t);
    const float4 u = __ldcg(yv), v = __ldcg(yv + 1);
    a.x += u.x; a.y += u.y; a.z += u.z; a.w += u.w;
    b.x += v.x; b.y += v.y; b.z += v.z; b.w += v.w;
  }
}

// Peer s's partial y of the exchange `seq`, elements [8t, 8t+8): poll (bounded)
// until all 8 words carry seq.  False if the wait ran out.
__device__ bool load_y_peer(const StackParams& p, int s, uint32_t seq, int t, float4& a, float4& b) {
  const unsigned long long* src = xchg_row(p.peer_buf[p.tp_rank], (int)(seq % NACC), s, p.tp_size) + 8 * t;
  ulonglong2 w[4];
  uint64_t t0 = 0;
  for (uint32_t i = 0;; ++i) {
    bool all = true;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      w[k] = ld_pair_sys(src + 2 * k);
      all = all && (uint32_t)(w[k].x >> 32) == seq && (uint32_t)(w[k].y >> 32) == seq;
    }
    if (all) break;
    if (i == 0) t0 = globaltimer_ns();
    else if ((i & 63) == 0 && globaltimer_ns() - t0 > p.wait_ns) return false;
    __nanosleep(32);
  }
  a = make_float4(__uint_as_float((uint32_t)w[0].x), __uint_as_float((uint32_t)w[0].y),
                  __uint_as_float((uint32_t)w[1].x), __uint_as_float((uint32_t)w[1].y));
  b = make_float4(__uint_as_float((uint32_t)w[2].x), __uint_as_float((uint32_t)w[2].y),
                  __uint_as_float((uint32_t)w[3].x), __uint_as_float((uint32_t)w[3].y));
  return true;
}

// x_l[8t, 8t+8) = x_{l-1} + y_{l-1}; with several GPUs, y is the sum of every
// GPU's partial in GPU order, so all GPUs compute identical bits.  Returns
// false (in every consumer thread of the CTA) if a peer's partial did not
// arrive in time; the caller then stops.
__device__ __forceinline__ bool load_x(StackSmem& sm, const StackParams& p, int lm1, int t, float (&x)[8]) {
  const float4* xv = reinterpret_cast<const float4*>(p.xbuf + (size_t)(lm1 % NACC) * H + 8 * t);
  float4 a = __ldcg(xv), b = __ldcg(xv + 1);
  bool ok = true;
  const uint32_t seq = p.seq_base + (uint32_t)lm1 + 1u;
  for (int s = 0; s < p.tp_size; ++s) {
    float4 u, v;
    if (s == p.tp_rank) {
      load_y_local(p, lm1, t, u, v);
    } else if (!load_y_peer(p, s, seq, t, u, v)) {
      ok = false;
      break;
    }
    a.x += u.x; a.y += u.y; a.z += u.z; a.w += u.w;
    b.x += v.x; b.y += v.y; b.z += v.z; b.w += v.w;
  }
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  if (p.tp_size == 1) return true;
  if (!ok) {
    sm.abort = 1;
    atomicOr(p.status, HC_ERR_TIMEOUT);
  }
  uint32_t all;
  asm volatile(
      "{\n\t.reg .pred pi, po;\n\t"
      "setp.ne.u32 pi, %1, 0;\n\t"
      "bar.red.and.pred po, 1, %2, pi;\n\t"
      "selp.u32 %0, 1, 0, po;\n\t}"
      : "=r"(all)
      : "r"((uint32_t)ok), "r"(CONS_THREADS)
      : "memory");
  return all != 0;
}

// generic-proxy shared-memory writes -> visible to the bulk-copy (async) proxy
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// dst[i] += src[i] (fp32), bytes % 16 == 0, both 16-byte aligned, done by the L2
__device__ __forceinline__ void bulk_reduce_add_f32(float* dst, const float* src, uint32_t bytes) {
  asm volatile("cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// wait until this thread's bulk groups completed (their writes performed)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void red_add_v4(float* dst, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
__device__ __forceinline__ int ld_vol(const int32_t* p) { return *reinterpret_cast<const volatile int32_t*>(p); }
__device__ __forceinline__ uint32_t ld_vol_u(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// --------------------------------------------------------------------------
// per-layer work split of CTA c (shared by all roles)
// --------------------------------------------------------------------------
struct Split {
  int64_t h0, h1;       // static hot neurons
  int64_t n_static;     // hot neurons [n_static, n_hot) are claimed dynamically
  int u0, u1;           // own W_up tiles == own mask words (neuron ids [32 u0, 32 u1))
  int d0, d1;           // W_down tiles of the next layer's predictor
};
__device__ __forceinline__ Split make_split(const StackParams& p, const hc_layer_desc& d, bool pred_next, int c,
                                            int G) {
  Split s;
  s.n_static = 0;
  s.h0 = split_lo(s.n_static, c, G);
  s.h1 = split_lo(s.n_static, c + 1, G);
  s.u0 = p.words_lo + (int)split_lo(p.words_n, c, G);
  s.u1 = p.words_lo + (int)split_lo(p.words_n, c + 1, G);
  const int nd = H / WD_ROWS;
  s.d0 = pred_next ? (int)split_lo(nd, c, G) : 0;
  s.d1 = pred_next ? (int)split_lo(nd, c + 1, G) : 0;
  return s;
}
// layer 0 predicts its own mask words in the kernel (requested, and it has a usable predictor)
__device__ __forceinline__ bool first_pred(const StackParams& p) {
  if (!p.pred0) return false;
  const hc_layer_desc& d = p.layers[0];
  return d.pred_w_up != nullptr && d.pred_w_down_t != nullptr && rank_ok(d.rank);
}
__device__ __forceinline__ bool next_pred(const StackParams& p, int l) {
  if (l + 1 >= p.n_layers || p.masks_given) return false;
  const hc_layer_desc& dn = p.layers[l + 1];
  return dn.pred_w_up != nullptr && rank_ok(dn.rank);
}

// --------------------------------------------------------------------------
// consumer helpers
// --------------------------------------------------------------------------
__device__ __forceinline__ float ld_half(const uint8_t* p) {
  return __half2float(*reinterpret_cast<const __half*>(p));
}
__device__ __forceinline__ bool cons_broadcast(StackSmem& sm, bool ok0) {
  if (threadIdx.x == 0) sm.flag = ok0 ? 1 : 0;
  named_bar(1, CONS_THREADS);
  return sm.flag != 0;
}
// sum over the 512 consumer threads (result in every thread)
__device__ __forceinline__ float cons_sum(StackSmem& sm, float a) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
  named_bar(1, CONS_THREADS);
  if ((threadIdx.x & 31) == 0) sm.zred[threadIdx.x >> 5] = a;
  named_bar(1, CONS_THREADS);
  a = 0.0f;
#pragma unroll
  for (int w = 0; w < NWARPS; ++w) a += sm.zred[w];
  return a;
}

// One thread polls ring position q (entry e, phase parity par).  Returns 1
// when it holds a fill of layer l, 0 when layer l's stream ended before it
// (the fill belongs to the next layer, or the issuer sealed layer l with
// fewer groups), -1 when the wait limit passed.  Position q is looked at once
// the entry's info names it: the issuer writes that only after the entry's
// previous fill was consumed, so the mbarrier parity test is then exact.  The
// poller's observation of the completed phase reaches the rest of its
// subgroup through the subgroup barrier that follows.
__device__ __forceinline__ int poll_pos(StackSmem& sm, uint32_t q, int e, uint32_t par, int l, int gi,
                                        uint64_t* waited, uint64_t limit_ns) {
  if (ld_vol_u(&sm.info[e].pos) == q && mbar_test_wait(&sm.full[e], par)) return (sm.info[e].layer == l) ? 1 : 0;
  const uint64_t c0 = (waited != nullptr) ? (uint64_t)clock64() : 0;
  const uint64_t t0 = globaltimer_ns();
  int r = -1;
  for (uint32_t i = 0;; ++i) {
    // suspends until the phase completes or ~200 ns pass
    if (ld_vol_u(&sm.info[e].pos) == q && mbar_try_wait_hint(&sm.full[e], par, 200)) {
      r = (sm.info[e].layer == l) ? 1 : 0;
      break;
    }
    if (ld_vol(&sm.sealed) >= l) {
      __threadfence_block();
      if (gi >= ld_vol(&sm.ngroups[l & 3])) {
        r = 0;
        break;
      }
    }
    if ((i & 15) == 15 && globaltimer_ns() - t0 > limit_ns) break;
  }
  if (waited != nullptr) *waited += (uint64_t)clock64() - c0;
  return r;
}
// The same test without waiting: 1 / 0 as poll_pos, 2 when position q is not
// filled yet (the caller then waits with poll_pos once it holds no entry the
// fill could need).
__device__ __forceinline__ int poll_once(StackSmem& sm, uint32_t q, int e, uint32_t par, int l, int gi) {
  if (ld_vol_u(&sm.info[e].pos) == q && mbar_test_wait(&sm.full[e], par)) return (sm.info[e].layer == l) ? 1 : 0;
  if (ld_vol(&sm.sealed) >= l) {
    __threadfence_block();
    if (gi >= ld_vol(&sm.ngroups[l & 3])) return 0;
  }
  return 2;
}
__device__ __forceinline__ void sg_release(StackSmem& sm, int e) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&sm.empty[e]);
}

// Subgroup reduction of V per-thread partials: warp-level multi-value
// reduction, one subgroup barrier, then lanes j < V of every warp sum the
// SG_WARPS warp partials of value j.
// `before_bar` runs in every thread just before the barrier (the group loop
// uses it to claim and test the subgroup's next group, whose decision the same
// barrier then publishes).
template <int V, class F>
__device__ __forceinline__ float sg_reduce(StackSmem& sm, int sg, int buf, float (&v)[V], F&& before_bar) {
  const int lane = threadIdx.x & 31, w = (threadIdx.x >> 5) & (SG_WARPS - 1);
  const float r = warp_reduce_multi<V>(v);
  constexpr int SH = 5 - (V == 16 ? 4 : V == 8 ? 3 : V == 4 ? 2 : 1);
  if ((lane & ((1 << SH) - 1)) == 0) sm.red[sg][buf][w][lane >> SH] = r;
  before_bar();
  named_bar(2 + sg, SG_THREADS);
  float s = 0.0f;
  if (lane < V) {
#pragma unroll
    for (int k = 0; k < SG_WARPS; ++k) s += sm.red[sg][buf][k][lane];
  }
  return s;
}

// Subgroup-thread copy of the layer's normalised input as fixed point: for
// word j (elements 8j..8j+7 of the thread's 32) d[4j..4j+3] = high digits of
// the even / odd elements (signed bytes), low digits of the even / odd
// elements (unsigned bytes); x = (256 * high + low) * 2^-s.
struct XFix {
  uint32_t d[16];
  int corr;      // -8 * sum of the 32 fixed-point values (removes the +8 nibble bias)
  float scale;   // 2^-s
};

// The thread's 32 INT4 elements of a record field (bytes [2 + 16u, 18 + 16u)
// of the field, which starts 2 bytes past a 16-byte boundary) as 4 words.
__device__ __forceinline__ void int4_words(const uint8_t* aligned, uint32_t (&w)[4]) {
  const uint4 a = *reinterpret_cast<const uint4*>(aligned);
  uint32_t e = __shfl_down_sync(0xffffffffu, a.x, 1);      // lane i+1 holds bytes [16, 20) of lane i
  if ((threadIdx.x & 31) == 31) e = *reinterpret_cast<const uint32_t*>(aligned + 16);
  w[0] = shift2(a.x, a.y);
  w[1] = shift2(a.y, a.z);
  w[2] = shift2(a.z, a.w);
  w[3] = shift2(a.w, e);
}

// INT4 field (32 elements) dotted with x: exact integer sum, one float scale
__device__ __forceinline__ float dot32_int4(const uint8_t* aligned, const XFix& xf) {
  uint32_t w[4];
  int4_words(aligned, w);
  int acc_h = 0;
  uint32_t acc_l = (uint32_t)xf.corr;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t lo = (w[j] & 0x0F0F0F0Fu) ^ 0x08080808u;          // elements 0,2,4,6 as q + 8
    const uint32_t hi = ((w[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;   // elements 1,3,5,7 as q + 8
    acc_h = dp4a_us(lo, xf.d[4 * j + 0], acc_h);
    acc_h = dp4a_us(hi, xf.d[4 * j + 1], acc_h);
    acc_l = dp4a_uu(lo, xf.d[4 * j + 2], acc_l);
    acc_l = dp4a_uu(hi, xf.d[4 * j + 3], acc_l);
  }
  return (float)(int)((uint32_t)acc_h * 256u + acc_l) * xf.scale;
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

// y += c * q over the thread's 32 elements of an INT4 down row (biased: the
// caller removes 1032 * c from even and 1152 * c/16 from odd elements)
__device__ __forceinline__ void axpy32_int4(const uint8_t* aligned, unsigned short cb, unsigned short cs,
                                            float (&y)[SPT]) {
  uint32_t w[4];
  int4_words(aligned, w);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint32_t h[4];
    int4_pairs(w[j], h);
    fma2_f16_f32(y[8 * j + 0], y[8 * j + 4], h[0], cb);
    fma2_f16_f32(y[8 * j + 1], y[8 * j + 5], h[1], cs);
    fma2_f16_f32(y[8 * j + 2], y[8 * j + 6], h[2], cb);
    fma2_f16_f32(y[8 * j + 3], y[8 * j + 7], h[3], cs);
  }
}

// 32 FP8 weights dotted with 32 f16 x (pairs in xp): two fp32 chains
__device__ __forceinline__ float dot32_fp8(const uint8_t* row, const uint32_t (&xp)[16]) {
  const uint4 a = *reinterpret_cast<const uint4*>(row);
  const uint4 b = *reinterpret_cast<const uint4*>(row + 16);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
  float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    fma2_f16f16_f32(s0, s1, e4m3x2_to_f16x2(w[i]), xp[2 * i]);
    fma2_f16f16_f32(s0, s1, e4m3x2_to_f16x2(w[i] >> 16), xp[2 * i + 1]);
  }
  return s0 + s1;
}
__device__ __forceinline__ void axpy32_fp8(const uint8_t* row, unsigned short a16, float (&y)[SPT]) {
  const uint4 a = *reinterpret_cast<const uint4*>(row);
  const uint4 b = *reinterpret_cast<const uint4*>(row + 16);
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    fma2_f16_f32(y[4 * i + 0], y[4 * i + 1], e4m3x2_to_f16x2(w[i]), a16);
    fma2_f16_f32(y[4 * i + 2], y[4 * i + 3], e4m3x2_to_f16x2(w[i] >> 16), a16);
  }
}

// Hot group: n (<= NB_HOT) FP8 neurons, one per slot.
template <class F>
__device__ __forceinline__ void sg_hot(StackSmem& sm, const StackParams& p, const float* hot_scale,
                                       const uint8_t* slot0, const uint8_t* slot1, int n, int64_t i0, int sg, int buf,
                                       float (&y)[SPT], F&& before_bar) {
  const int u = threadIdx.x & (SG_THREADS - 1), lane = threadIdx.x & 31;
  uint32_t xp[16];
  {
    const uint4* src = reinterpret_cast<const uint4*>(sm.xh) + u;        // word i at [i][u] (xslot)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = src[i * SG_THREADS];
      xp[4 * i] = v.x; xp[4 * i + 1] = v.y; xp[4 * i + 2] = v.z; xp[4 * i + 3] = v.w;
    }
  }
  float v[2 * NB_HOT];
  v[0] = dot32_fp8(slot0 + SPT * u, xp);
  v[NB_HOT] = dot32_fp8(slot0 + H + SPT * u, xp);
  v[1] = 0.0f;
  v[NB_HOT + 1] = 0.0f;
  if (n > 1) {
    v[1] = dot32_fp8(slot1 + SPT * u, xp);
    v[NB_HOT + 1] = dot32_fp8(slot1 + H + SPT * u, xp);
  }
  const float s = sg_reduce<2 * NB_HOT>(sm, sg, buf, v, before_bar);
  const float uu = __shfl_down_sync(0xffffffffu, s, NB_HOT);   // lane j < n: gate j, lane NB_HOT + j: up j
  float a = 0.0f;
  if (lane < n) {
    float sgs = 1.0f, sus = 1.0f, sds = 1.0f;
    if (hot_scale != nullptr) {
      const float* s3 = hot_scale + (i0 + lane) * 3;
      sgs = __ldg(s3);
      sus = __ldg(s3 + 1);
      sds = __ldg(s3 + 2);
    }
    a = gated(s * sgs, uu * sus, p.relu, p.both) * sds;
  }
  // a neuron whose gated activation is exactly zero (dReLU: either branch <= 0)
  // adds nothing: its down column is skipped (every warp holds the same a's)
  const float a0 = __shfl_sync(0xffffffffu, a, 0), a1 = __shfl_sync(0xffffffffu, a, 1);
  if (a0 != 0.0f) axpy32_fp8(slot0 + 2 * H + SPT * u, __half_as_ushort(__float2half_rn(a0)), y);
  if (n > 1 && a1 != 0.0f) axpy32_fp8(slot1 + 2 * H + SPT * u, __half_as_ushort(__float2half_rn(a1)), y);
}

// Cold group: n (<= NB_COLD) INT4 records, two per slot.
// The decoded down rows carry a bias (1032 / 1152 per element, int4_pairs):
// the f16 coefficients are summed into csa / csb and the bias is removed once
// per layer (cold_bias_out), which keeps it small against fp32's precision.
template <class F>
__device__ __forceinline__ void sg_cold(StackSmem& sm, const StackParams& p, const uint8_t* slot0,
                                        const uint8_t* slot1, int n, int sg, int buf, float (&y)[SPT], float& csa,
                                        float& csb, F&& before_bar) {
  const int u = threadIdx.x & (SG_THREADS - 1), lane = threadIdx.x & 31;
  XFix xf;
  {
    const uint4* src = sm.xq + u;                                          // word j at [j][u] (xslot)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = src[j * SG_THREADS];
      xf.d[4 * j] = v.x; xf.d[4 * j + 1] = v.y; xf.d[4 * j + 2] = v.z; xf.d[4 * j + 3] = v.w;
    }
    const int2 ch = sm.chunk[u];
    xf.corr = ch.x;
    xf.scale = __int_as_float(ch.y);
  }
  const int gs = 2 * (u >> 2);                 // byte offset of this thread's INT4 group scale
  const uint8_t* rec[NB_COLD] = {slot0, slot0 + REC_SLOT_OFF, slot1, slot1 + REC_SLOT_OFF};
  float v[2 * NB_COLD];
#pragma unroll
  for (int j = 0; j < NB_COLD; ++j) {
    v[j] = 0.0f;
    v[NB_COLD + j] = 0.0f;
    if (j < n) {
      v[j] = dot32_int4(rec[j] + 16 * u, xf) * ld_half(rec[j] + SCALE_OFF + gs);
      v[NB_COLD + j] = dot32_int4(rec[j] + VEC_BYTES + 16 * u, xf) * ld_half(rec[j] + SCALE_OFF + 2 * NGROUPS + gs);
    }
  }
  const float s = sg_reduce<2 * NB_COLD>(sm, sg, buf, v, before_bar);
  const float uu = __shfl_down_sync(0xffffffffu, s, NB_COLD);
  float a = 0.0f;
  if (lane < n) a = gated(s, uu, p.relu, p.both);
#pragma unroll
  for (int j = 0; j < NB_COLD; ++j) {
    const float aj = __shfl_sync(0xffffffffu, a, j);
    // a zero activation (dReLU) adds nothing: skip the record's down column
    if (j < n && aj != 0.0f) {
      const __half c16 = __float2half_rn(aj * ld_half(rec[j] + SCALE_OFF + 4 * NGROUPS + gs));
      const __half c16s = __hmul(c16, __float2half(0.0625f));    // exact unless subnormal; csb tracks it
      csa += __half2float(c16);
      csb += __half2float(c16s);
      axpy32_int4(rec[j] + 2 * VEC_BYTES + 16 * u, __half_as_ushort(c16), __half_as_ushort(c16s), y);
    }
  }
}
__device__ __forceinline__ void cold_bias_out(float (&y)[SPT], float csa, float csb) {
#pragma unroll
  for (int k = 0; k < SPT; ++k) y[k] = (k & 1) ? fmaf(-1152.0f, csb, y[k]) : fmaf(-1032.0f, csa, y[k]);
}

// grid barrier: arrive (after this CTA's atomics) ...
__device__ __forceinline__ void grid_arrive(const StackParams& p) {
  named_bar(1, CONS_THREADS);
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar_count) : "memory");
}
// ... and wait (thread 0 spins, bounded; result broadcast)
// (thread 0's part: spin on the counter; false on timeout or abort)
__device__ bool grid_spin(StackSmem& sm, const StackParams& p, uint32_t target) {
  bool ok0 = true;
  {
    if (ld_acquire_u32(p.bar_count) < target) {
      const uint64_t t0 = globaltimer_ns();
      uint32_t spins = 0;
      while (ld_acquire_u32(p.bar_count) < target) {
        if ((++spins & 255) == 0 && globaltimer_ns() - t0 > p.wait_ns) {
          ok0 = false;
          break;
        }
        __nanosleep(32);
      }
    }
    // (the acquire loads order what follows; the consumers' barrier carries it to the CTA)
    if (!ok0 || ld_vol(&sm.abort) != 0) {
      ok0 = false;
      sm.abort = 1;
      atomicOr(p.status, HC_ERR_TIMEOUT);
    }
  }
  return ok0;
}
__device__ bool grid_wait(StackSmem& sm, const StackParams& p, uint32_t target, int lm1) {
  bool ok0 = true;
  if (threadIdx.x == 0) {
    ok0 = grid_spin(sm, p, target);
    trace_ev(p, lm1, 32);
  }
  return cons_broadcast(sm, ok0);
}

// Wait until y of layer lm1 is complete: every CTA of this GPU added its
// partial.  With several GPUs, the first kp = min(grid, 32) CTAs then each
// store one slice (1/kp) of this GPU's partial, as (sequence number, value)
// words, into every peer's exchange buffer with plain NVLink stores; load_x
// reads the peers' partials as their words arrive.
__device__ bool layer_wait(StackSmem& sm, const StackParams& p, int lm1) {
  const uint32_t target = (uint32_t)(lm1 + 1) * gridDim.x;
  const bool ok = grid_wait(sm, p, target, lm1);     // thread 0 saw every local partial; so does every thread
  if (p.tp_size == 1 || !ok) return ok;              // on a local timeout the peers time out too
  const int t = threadIdx.x, c = blockIdx.x;
  const int kp = min((int)gridDim.x, KP_MAX);
  if (c < kp) {
    const uint32_t seq = p.seq_base + (uint32_t)lm1 + 1u;
    const int slot = (int)(seq % NACC);
    const unsigned long long tag = (unsigned long long)seq << 32;
    const int lo = c * (H / 2) / kp, hi = (c + 1) * (H / 2) / kp;      // this CTA's float2 slice
    for (int i = lo + t; i < hi; i += CONS_THREADS) {
      float2 a = make_float2(0.f, 0.f);
#pragma unroll
      for (int k = 0; k < YCOPIES; ++k) {       // the order of load_y_local: identical sums on every GPU
        const float2 v = __ldcg(reinterpret_cast<const float2*>(p.yacc + ((size_t)(lm1 % NACC) * YCOPIES + k) * H) + i);
        a.x += v.x;
        a.y += v.y;
      }
      const unsigned long long w0 = tag | __float_as_uint(a.x), w1 = tag | __float_as_uint(a.y);
      for (int s = 0; s < p.tp_size; ++s) {
        if (s == p.tp_rank) continue;
        st_pair_sys(xchg_row(p.peer_buf[s], slot, p.tp_rank, p.tp_size) + 2 * i, w0, w1);
      }
    }
    if (t == 0) trace_ev(p, lm1, 36);
  }
  return true;
}

// --------------------------------------------------------------------------
// issuer helpers
// --------------------------------------------------------------------------
struct Producer {
  uint32_t k = 0;       // ring positions issued
  uint64_t pol = 0;
  bool ok = true;
};

// Take the next ring position (bounded wait for its entry to be empty), write
// its info, arm its mbarrier with the group's bytes and start the copies.
struct Copy {
  const void* src;
  uint32_t bytes;
  uint32_t off;      // destination offset in the entry
};
template <int NCP>
__device__ __forceinline__ void issue_entry(StackSmem& sm, uint8_t* ring, Producer& pr, int l, uint8_t kind, int n,
                                            int64_t index, const Copy (&cp)[NCP], uint64_t* waited,
                                            uint64_t limit_ns) {
  const uint32_t q = pr.k;
  const int e = (int)(q % (uint32_t)NE);
  const uint32_t round = q / (uint32_t)NE;
  if (round > 0) {
    const uint64_t t0 = (waited != nullptr) ? globaltimer_ns() : 0;
    if (!mbar_wait(&sm.empty[e], (round - 1) & 1u, limit_ns)) {
      pr.ok = false;
      return;
    }
    if (waited != nullptr) *waited += globaltimer_ns() - t0;
  }
  SlotInfo& inf = sm.info[e];
  inf.layer = (int16_t)l;
  inf.kind = kind;
  inf.n = (uint8_t)n;
  inf.index = (int32_t)index;
  *reinterpret_cast<volatile uint32_t*>(&inf.pos) = q;
  uint8_t* dst = ring + (size_t)e * ENTRY_BYTES;
  uint32_t total = 0;
#pragma unroll
  for (int i = 0; i < NCP; ++i) total += cp[i].bytes;
  mbar_arrive_expect_tx(&sm.full[e], total);
#pragma unroll
  for (int i = 0; i < NCP; ++i)
    if (cp[i].bytes) bulk_g2s(dst + cp[i].off, cp[i].src, cp[i].bytes, &sm.full[e], pr.pol);
  ++pr.k;
}

// --------------------------------------------------------------------------
// the kernel
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(STACK_THREADS, 1) ffn_stack_kernel(StackParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  StackSmem& sm = *reinterpret_cast<StackSmem*>(smem_raw);
  uint8_t* ring = smem_raw + RING_OFF;
  float* xs = sm.ystage;
  const int tid = threadIdx.x;
  const int G = gridDim.x;
  const int c = blockIdx.x;

  if (tid == 0) {
    trace_ev(p, 0, 33);        // the CTA started (layer 0's slot)
    for (int e = 0; e < NE; ++e) {
      mbar_init(&sm.full[e], 1);
      mbar_init(&sm.empty[e], SG_WARPS);
      sm.info[e].pos = 0xFFFFFFFFu;
    }
    mbar_init(&sm.phase0_done, 1);
    mbar_init(&sm.pbar, 1);
    mbar_init(&sm.wdown_done, 1);
    sm.abort = 0;
    sm.flag = 1;
    sm.sealed = -1;
    sm.cons_layer = -1;
    sm.gnext[0] = 0;
    sm.gnext[1] = 0;
    mbar_fence_init();
  }
  __syncthreads();

  if (tid >= CONS_THREADS + 32) {
    // ============================ planner warp =============================
    // List of layer 0 from `masks`; then per layer l: the CTA's W_down rows of
    // layer l+1's predictor (once the consumers normalised x_l), and, once
    // every CTA's rows are in, the logits of its neuron-id range -> its mask
    // words of layer l+1 (or `masks` when given, or all ones without a
    // predictor) -> the ascending list of its active cold records.
    const int lane = tid & 31;
    bool ok = true;
    const int u0 = p.words_lo + (int)split_lo(p.words_n, c, G);
    const int nw = p.words_lo + (int)split_lo(p.words_n, c + 1, G) - u0;
    uint32_t pphase = 0, p0phase = 0;
    // one tile into pbuf with the planner's own bulk copy (bounded wait)
    auto load_tile = [&](const void* a, uint32_t abytes, const void* b, uint32_t bbytes, uint32_t boff) -> bool {
      if (lane == 0) {
        mbar_arrive_expect_tx(&sm.pbar, abytes + bbytes);
        bulk_g2s(sm.pbuf, a, abytes, &sm.pbar, 0ull);
        if (bbytes) bulk_g2s(sm.pbuf + boff, b, bbytes, &sm.pbar, 0ull);
      }
      bool done = mbar_wait(&sm.pbar, pphase & 1u, p.wait_ns);
      // a copy that outlived a short limit still lands: never leave it in flight
      if (!done) mbar_wait(&sm.pbar, pphase & 1u, WAIT_LIMIT_NS);
      ++pphase;
      return __all_sync(0xffffffffu, done);
    };
    // The static part of a layer's lookup (fetch_bits word and table entries
    // of the own id range) is loaded early, so only shared-memory work
    // remains once the own mask words are known.
    uint32_t fetch = 0;
    auto preload = [&](int l) {
      const hc_layer_desc& d = p.layers[l];
      fetch = (lane < nw) ? __ldg(d.fetch_bits + u0 + lane) : 0u;
      const int id0 = u0 * 32, nid = min((u0 + nw) * 32, p.inter) - id0;
      for (int i = lane; i < nid; i += 32) sm.plan_list[i] = __ldg(d.table + id0 + i);
      __syncwarp();
    };
    // own words (one per lane) & fetch bits -> ascending record list of layer l
    auto build = [&](int l, uint32_t own) {
      const hc_layer_desc& dl = p.layers[l];
      const int n_records = dl.n_records;
      // in-place compaction word by word: word w's entries are read (one per
      // lane) before its writes, which land below 32 (w + 1)
      const uint32_t mw = own & fetch;
      int cnt = 0;
      for (int w = 0; w < nw; ++w) {
        const uint32_t m = __shfl_sync(0xffffffffu, mw, w);
        if (m == 0) continue;
        const bool on = (m >> lane) & 1u;
        int r = on ? sm.plan_list[w * 32 + lane] : 0;
        __syncwarp();
        if (on) {
          if (r < 0 || r >= n_records) {
            atomicOr(p.status, HC_ERR_RANGE);
            r = 0;
          }
          sm.plan_list[cnt + __popc(m & ((1u << lane) - 1u))] = r;
        }
        cnt += __popc(m);
        __syncwarp();
      }
      // Publish into the layer's pool, which every CTA's issuer takes from.  The
      // pool's counters were cleared in layer l-2, before this CTA's consumers
      // started layer l-1.
      if (lane == 0 && l > 0) {
        const uint64_t t0 = globaltimer_ns();
        uint32_t i = 0;
        while (ld_vol(&sm.cons_layer) < l - 1) {
          if ((++i & 63) == 0 && globaltimer_ns() - t0 > p.wait_ns) {
            ok = false;
            break;
          }
        }
        __threadfence();
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      uint32_t base = 0;
      if (lane == 0 && ok) base = atomicAdd(p.gfill + l % NACC, (uint32_t)cnt);
      base = __shfl_sync(0xffffffffu, base, 0);
      int32_t* pool = p.gpool + (size_t)(l % NACC) * POOL_CAP;
      if (ok)
        for (int i = lane; i < cnt; i += 32) pool[base + i] = sm.plan_list[i];
      __syncwarp();
      if (lane == 0 && ok) {
        __threadfence();
        atomicAdd(p.gdone + l % NACC, 1u);
        trace_ev(p, l, 20);
        trace_set(p, l, 17, (uint64_t)cnt);
      }
      // the records come from L2 for whichever CTA takes them
      if (ok)
        for (int i = lane; i < cnt; i += 32)
          prefetch_l2(dl.cold_records + (size_t)sm.plan_list[i] * REC_BYTES, REC_COPY);
    };
    // mask words of layer l without its predictor: given, or all ones
    auto words_without_predictor = [&](int l) -> uint32_t {
      uint32_t* mrow = p.masks + (size_t)l * p.words;
      if (lane >= nw) return 0u;
      if ((l == 0 && !p.pred0) || p.masks_given) return __ldcg(mrow + u0 + lane);
      // no predictor: fetch every cold neuron (engine.py:282-283)
      const int valid = min(32, p.inter - 32 * (u0 + lane));
      const uint32_t m = valid >= 32 ? 0xffffffffu : ((1u << valid) - 1u);
      mrow[u0 + lane] = m;
      return m;
    };
    // W_down tiles [d0, d1) of layer lp's predictor on the normalised rows
    // xrow(r) -> z of layer lp (slot lp % NACC), then the tile count
    auto wdown = [&](const hc_layer_desc& dp, int lp, int d0, int d1, auto xrow) -> bool {
      const int rank = dp.rank;
      for (int tile = d0; tile < d1; ++tile) {
        if (!load_tile(dp.pred_w_down_t + (size_t)tile * WD_ROWS * rank, WD_ROWS * rank * 4, nullptr, 0, 0))
          return false;
        const float* t = reinterpret_cast<const float*>(sm.pbuf);
        for (int r = lane; r < rank; r += 32) {
          float acc = 0.0f;
#pragma unroll 8
          for (int row = 0; row < WD_ROWS; ++row) acc = fmaf(t[row * rank + r], xrow(tile * WD_ROWS + row), acc);
          atomicAdd(p.zacc + (size_t)(lp % NACC) * 128 + r, acc);
        }
        __syncwarp();      // pbuf is reused by the next copy
      }
      return true;
    };
    auto wdown_count = [&](int lp, int d0, int d1) {
      if (lane == 0 && d1 > d0) {
        __threadfence();
        atomicAdd(p.zdone + lp % NACC, (uint32_t)(d1 - d0));
      }
    };
    // once every CTA's W_down tiles of layer lp are in: the logits of the own
    // neuron-id range -> own mask words (lane w holds word w), also stored in
    // masks row lp
    auto own_logits = [&](const hc_layer_desc& dp, int lp, uint32_t& own) -> bool {
      const int rank = dp.rank;
      bool good = true;
      if (lane == 0) {
        const uint32_t* cnt = p.zdone + lp % NACC;
        const uint64_t t0 = globaltimer_ns();
        uint32_t i = 0;
        while (ld_acquire_u32(cnt) < (uint32_t)WD_TILES) {
          if ((++i & 63) == 0 && globaltimer_ns() - t0 > p.wait_ns) {
            good = false;
            break;
          }
          __nanosleep(100);
        }
      }
      if (!__shfl_sync(0xffffffffu, good, 0)) return false;
      __syncwarp();      // lane 0's acquire orders every lane's reads of z below
      for (int i = lane; i < rank; i += 32) sm.z[i] = __ldcg(p.zacc + (size_t)(lp % NACC) * 128 + i);
      __syncwarp();
      // one W_up tile (32 neurons == one mask word) at a time
      for (int w = 0; w < nw; ++w) {
        const int tile = u0 + w;
        const int rows = min(WU_ROWS, p.inter - tile * WU_ROWS);
        if (!load_tile(dp.pred_w_up + (size_t)tile * WU_ROWS * rank, rows * rank * 4,
                       dp.pred_b_up + (size_t)tile * WU_ROWS, rows * 4, WU_ROWS * rank * 4))
          return false;
        const float* t = reinterpret_cast<const float*>(sm.pbuf);
        float acc = 0.0f;
        if (lane < rows) {
          // lane = neuron; the rotated start keeps the 32 rows on distinct banks
          const float* row = t + lane * rank;
          int k = lane % rank;
          for (int i = 0; i < rank; ++i) {
            acc = fmaf(row[k], sm.z[k], acc);
            k = (k + 1 == rank) ? 0 : k + 1;
          }
          acc += t[WU_ROWS * rank + lane];
        }
        const uint32_t word = __ballot_sync(0xffffffffu, lane < rows && acc >= p.thr);
        if (lane == w) own = word;
        __syncwarp();
      }
      if (lane < nw) p.masks[(size_t)lp * p.words + u0 + lane] = own;
      if (lane == 0) trace_ev(p, lp, 21);
      return true;
    };
    const int nd = H / WD_ROWS;
    const int d0 = (int)split_lo(nd, c, G), d1 = (int)split_lo(nd, c + 1, G);
    if (first_pred(p)) {
      // ---- layer 0's own prediction on RMSNorm_0(x_0) (engine.py:422), as for
      // the later layers, once the consumers have x_0's RMS
      const hc_layer_desc& d0l = p.layers[0];
      if (lane == 0) ok = mbar_wait(&sm.phase0_done, p0phase & 1u, p.wait_ns);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // the layer-0 arrival is also the one the loop below waits for at l = 0
      if (!next_pred(p, 0)) ++p0phase;
      const float rstd0 = sm.rstd0;
      uint32_t own = 0;
      if (ok)
        ok = wdown(d0l, 0, d0, d1, [&](int r) {
          const float xr = p.io_f16 ? __half2float(__ldg(static_cast<const __half*>(p.x_in) + r))
                                    : __ldg(static_cast<const float*>(p.x_in) + r);
          return xr * rstd0 * (d0l.norm_w ? __ldg(d0l.norm_w + r) : 1.0f);
        });
      if (ok) wdown_count(0, d0, d1);
      preload(0);
      if (ok && nw > 0) ok = own_logits(d0l, 0, own);
      if (ok) build(0, own);
    } else {
      preload(0);
      build(0, words_without_predictor(0));
    }
    for (int l = 0; l + 1 < p.n_layers && ok; ++l) {
      const bool pred_next = next_pred(p, l);
      const hc_layer_desc& dn = p.layers[l + 1];
      uint32_t own = 0;
      if (pred_next) {
        // ---- W_down rows [d0, d1) of layer l+1's predictor on RMSNorm_{l+1}(x_l)
        // (one phase per layer with a next predictor, like wdown_done)
        if (lane == 0) ok = mbar_wait(&sm.phase0_done, p0phase & 1u, p.wait_ns);
        ++p0phase;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        ok = wdown(dn, l + 1, d0, d1, [&](int r) { return xs[r - d0 * WD_ROWS]; });
        if (!ok) break;
        if (lane == 0) mbar_arrive(&sm.wdown_done);       // ystage is the consumers' again
        wdown_count(l + 1, d0, d1);
        preload(l + 1);
        if (nw > 0) {
          ok = own_logits(dn, l + 1, own);
          if (!ok) break;
        }
      } else {
        preload(l + 1);
        own = words_without_predictor(l + 1);
      }
      build(l + 1, own);
      if (!ok) break;
    }
    if (lane == 0 && !ok) {
      sm.abort = 1;
      atomicOr(p.status, HC_ERR_TIMEOUT);
    }
    __syncwarp();
    __syncthreads();
  } else if (tid >= CONS_THREADS) {
    // ============================ issuer warp ==============================
    // Lane 0 streams the CTA's groups of layer l in order: cold records taken
    // from the layer's pool (all CTAs' lists) until it is empty, then hot
    // neurons claimed from the layer's counter until none are left; then it
    // seals the layer.
    const int lane = tid & 31;
    Producer pr;
    if (lane == 0) {
      pr.pol = l2_evict_first_policy();
      for (int l = 0; l < p.n_compute && pr.ok; ++l) {
        // stay at most two layers ahead of the consumers (ngroups is indexed l & 3)
        {
          const uint64_t t0 = globaltimer_ns();
          uint32_t i = 0;
          while (ld_vol(&sm.cons_layer) < l - 2) {
            if ((++i & 63) == 0 && globaltimer_ns() - t0 > p.wait_ns) {
              pr.ok = false;
              break;
            }
          }
          if (!pr.ok) break;
        }
        const hc_layer_desc d = p.layers[l];
        const bool pred_next = next_pred(p, l);
        const Split sp = make_split(p, d, pred_next, c, G);
        const hc_layer_desc* dn = pred_next ? &p.layers[l + 1] : nullptr;
        const int rank_n = pred_next ? dn->rank : 0;
        uint64_t iw = 0;
        uint64_t* iwp = p.trace ? &iw : nullptr;
        int ng = 0;
        trace_ev(p, l, 10);
        // L2 prefetch: static hot slice, a 1/G share of the dynamic hot range, next predictor tiles
        if (sp.h1 > sp.h0) prefetch_l2_range(d.hot + sp.h0 * HOT_BYTES, (size_t)(sp.h1 - sp.h0) * HOT_BYTES);
        {
          const int64_t nd = d.n_hot - sp.n_static;
          const int64_t a = sp.n_static + split_lo(nd, c, G), b = sp.n_static + split_lo(nd, c + 1, G);
          if (b > a) prefetch_l2_range(d.hot + a * HOT_BYTES, (size_t)(b - a) * HOT_BYTES);
        }
        if (sp.d1 > sp.d0)
          prefetch_l2_range(dn->pred_w_down_t + (size_t)sp.d0 * WD_ROWS * rank_n,
                            (size_t)(sp.d1 - sp.d0) * WD_ROWS * rank_n * 4);
        if (pred_next && sp.u1 > sp.u0) {
          const int rows = min(sp.u1 * WU_ROWS, p.inter) - sp.u0 * WU_ROWS;
          prefetch_l2_range(dn->pred_w_up + (size_t)sp.u0 * WU_ROWS * rank_n, (size_t)rows * rank_n * 4);
        }
        // The layer's counters (cold pool, hot neurons) were cleared in layer
        // l-2, which this CTA's consumers passed once they started layer l-1.
        {
          const uint64_t t0 = globaltimer_ns();
          uint32_t i = 0;
          while (ld_vol(&sm.cons_layer) < l - 1) {
            if ((++i & 63) == 0 && globaltimer_ns() - t0 > p.wait_ns) {
              pr.ok = false;
              break;
            }
          }
          if (!pr.ok) break;
          __threadfence();
        }
        // This CTA streams its static share of the layer: pool entries
        // [c n / G, (c+1) n / G) of the layer's cold-record pool (once every CTA
        // has published its list) and hot neurons [c n_hot / G, (c+1) n_hot / G),
        // two per group.  Equal shares of both kinds give every SM the same
        // bytes, so the layer's CTAs finish together (no claims, no counter
        // round trips).  Cold first (the costlier groups early, so the subgroups'
        // claims even out the end of the layer), except at a launch's first
        // layer, whose pool the planners are still building: its hot groups,
        // which need nothing, stream meanwhile.
        uint64_t claimed = 0, cold_taken = 0;
        auto issue_hot = [&]() {
          trace_ev(p, l, 13);
          const int64_t hA = split_lo(d.n_hot, c, G), hB = split_lo(d.n_hot, c + 1, G);
          const int64_t hsz = (hB - hA >= 8) ? NB_HOT : 1;     // single neurons when the CTA has few
          for (int64_t i = hA; pr.ok && i < hB; i += hsz) {
            const int n = (int)min(hsz, hB - i);
            Copy cp[2];
#pragma unroll
            for (int k = 0; k < 2; ++k)
              cp[k] = {k < n ? d.hot + (i + k) * HOT_BYTES : nullptr, k < n ? (uint32_t)HOT_BYTES : 0u,
                       (uint32_t)(k * HALF_BYTES)};
            issue_entry(sm, ring, pr, l, UNIT_HOT, n, i, cp, iwp, p.wait_ns);
            ++ng;
            claimed += n;
          }
          trace_ev(p, l, 37);
        };
        auto issue_cold = [&]() {
          {
            const uint64_t t0 = globaltimer_ns();
            uint32_t i = 0;
            while (ld_acquire_u32(p.gdone + l % NACC) < (uint32_t)G) {
              if ((++i & 63) == 0 && globaltimer_ns() - t0 > p.wait_ns) {
                pr.ok = false;
                break;
              }
              __nanosleep(64);
            }
            if (!pr.ok) return;
          }
          trace_ev(p, l, 11);
          const uint32_t total = __ldcg(p.gfill + l % NACC);
          const int32_t* pool = p.gpool + (size_t)(l % NACC) * POOL_CAP;
          const uint32_t i0 = (uint32_t)split_lo(total, c, G), i1 = (uint32_t)split_lo(total, c + 1, G);
          // groups of up to NB_COLD records, smaller when the CTA has few (at least
          // 4 cold groups for the 4 subgroups when it has 4 records or more)
          const uint32_t gsz = max(1u, min((uint32_t)NB_COLD, (i1 - i0) / 4u));
          for (uint32_t i = i0; pr.ok && i < i1; i += gsz) {
            const int m = (int)min(gsz, i1 - i);
            int rec[NB_COLD];
#pragma unroll
            for (int k = 0; k < NB_COLD; ++k) rec[k] = (k < m) ? __ldcg(pool + i + k) : 0;
            Copy cp[NB_COLD];
#pragma unroll
            for (int k = 0; k < NB_COLD; ++k)
              cp[k] = {k < m ? d.cold_records + (size_t)rec[k] * REC_BYTES : nullptr,
                       k < m ? (uint32_t)REC_COPY : 0u,
                       (uint32_t)((k >> 1) * HALF_BYTES + (k & 1) * REC_SLOT_OFF)};
            issue_entry(sm, ring, pr, l, UNIT_COLD, m, (int64_t)i, cp, iwp, p.wait_ns);
            ++ng;
            cold_taken += m;
          }
          trace_ev(p, l, 12);
        };
        if (l == 0) {
          issue_hot();
          if (pr.ok) issue_cold();
        } else {
          issue_cold();
          if (pr.ok) issue_hot();
        }
        if (!pr.ok) break;
        sm.ngroups[l & 3] = ng;
        __threadfence_block();
        *reinterpret_cast<volatile int32_t*>(&sm.sealed) = l;
        trace_ev(p, l, 14);
        trace_set(p, l, 15, claimed);
        trace_set(p, l, 30, cold_taken);
        trace_set(p, l, 18, iw);
        trace_set(p, l, 19, (uint64_t)ng);
      }
      if (!pr.ok) {
        sm.abort = 1;
        atomicOr(p.status, HC_ERR_TIMEOUT);
      }
    }
    __syncwarp();
    __syncthreads();
    // drain: every issued copy must have landed before the CTA exits (the
    // last fill of each slot; earlier ones completed before it was issued)
    if (lane == 0) {
      const uint32_t first = pr.k > (uint32_t)NE ? pr.k - (uint32_t)NE : 0u;
      for (uint32_t q = first; q < pr.k; ++q)
        if (!mbar_wait(&sm.full[q % (uint32_t)NE], (q / (uint32_t)NE) & 1u, WAIT_LIMIT_NS)) {   // copies land by themselves
          atomicOr(p.status, HC_ERR_TIMEOUT);
          break;
        }
    }
  } else {
    // ============================ consumer threads =========================
    const int t = tid;
    const int sg = t / SG_THREADS, u = t & (SG_THREADS - 1);
    uint32_t base = 0;       // ring position of the layer's first group
    uint32_t wd_phase = 0;   // layers with a next predictor so far (wdown_done phases)
    int rbuf = 0, dbuf = 0;
    bool ok = true;
    for (int l = 0; l < p.n_compute && ok; ++l) {
      const hc_layer_desc d = p.layers[l];
      const bool pred_next = next_pred(p, l);
      if (t == 0 && c == 0 && !p.masks_given && d.pred_w_up != nullptr && !rank_ok(d.rank))
        atomicOr(p.status, HC_ERR_UNSUPPORTED);
      const Split sp = make_split(p, d, pred_next, c, G);
      const hc_layer_desc* dn = pred_next ? &p.layers[l + 1] : nullptr;

      // this layer's RMSNorm weights, loaded before the barrier wait below so
      // that their latency hides behind it
      float nw[EPT];
      if (d.norm_w) {
        const float4* wsrc = reinterpret_cast<const float4*>(d.norm_w + EPT * t);
        const float4 w0 = __ldg(wsrc), w1 = __ldg(wsrc + 1);
        nw[0] = w0.x; nw[1] = w0.y; nw[2] = w0.z; nw[3] = w0.w; nw[4] = w1.x; nw[5] = w1.y; nw[6] = w1.z; nw[7] = w1.w;
      } else {
#pragma unroll
        for (int i = 0; i < EPT; ++i) nw[i] = 1.0f;
      }

      // ---- layer boundary: x_l = x_{l-1} + y_{l-1} once every CTA has added its part
      float x[EPT];
      if (l == 0) {
        if (p.io_f16) {
          const uint4 q = __ldg(reinterpret_cast<const uint4*>(static_cast<const __half*>(p.x_in) + EPT * t));
          const uint32_t qw[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&qw[i]));
            x[2 * i] = f.x;
            x[2 * i + 1] = f.y;
          }
        } else {
          const float4* src = reinterpret_cast<const float4*>(static_cast<const float*>(p.x_in) + EPT * t);
          const float4 q0 = __ldg(src), q1 = __ldg(src + 1);
          x[0] = q0.x; x[1] = q0.y; x[2] = q0.z; x[3] = q0.w; x[4] = q1.x; x[5] = q1.y; x[6] = q1.z; x[7] = q1.w;
        }
      } else {
        ok = layer_wait(sm, p, l - 1);
        if (!ok) break;
        ok = load_x(sm, p, l - 1, t, x);
        if (!ok) break;
        if (t == 0) trace_ev(p, l - 1, 35);
        if (p.x_hist && c == 0) {
          float4* h = reinterpret_cast<float4*>(p.x_hist + (size_t)(l - 1) * H + EPT * t);
          h[0] = make_float4(x[0], x[1], x[2], x[3]);
          h[1] = make_float4(x[4], x[5], x[6], x[7]);
        }
      }
      if (c == 0) {
        // x_l for every CTA at layer l+1 (x_{l-3}'s readers all passed the barrier above)
        float4* xo = reinterpret_cast<float4*>(p.xbuf + (size_t)(l % NACC) * H + EPT * t);
        xo[0] = make_float4(x[0], x[1], x[2], x[3]);
        xo[1] = make_float4(x[4], x[5], x[6], x[7]);
      }
      if (t == 0) trace_ev(p, l, 0);
      // Clear accumulators ahead of use (their previous users finished before the
      // barrier above): y of layer l+1 is added after barrier l+1; z of layer
      // l+2 and its tile count during layer l+1; the cold pool of layer l+2 is
      // filled, and its hot and cold counters claimed, only once the CTA doing
      // it has started layer l+1.
      {
        float* yz = p.yacc + (size_t)((l + 1) % NACC) * YCOPIES * H;
        constexpr int NV = YCOPIES * H / 4;
        for (int i = (int)split_lo(NV, c, G) + t; i < (int)split_lo(NV, c + 1, G); i += CONS_THREADS)
          reinterpret_cast<float4*>(yz)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c == 0 && t < 128) p.zacc[(size_t)((l + 2) % NACC) * 128 + t] = 0.0f;
        if (c == 0 && t == 0) p.hot_next[(l + 2) % NACC] = 0u;
        if (c == 0 && t == 1) p.zdone[(l + 2) % NACC] = 0u;
        if (c == 0 && t == 2) p.gfill[(l + 2) % NACC] = 0u;
        if (c == 0 && t == 3) p.gclaim[(l + 2) % NACC] = 0u;
        if (c == 0 && t == 4) p.gdone[(l + 2) % NACC] = 0u;
      }

      // ---- RMSNorm (engine.py:295; torch.nn.RMSNorm) -> f16 and fixed-point copies
      {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < EPT; ++i) ss = fmaf(x[i], x[i], ss);
        ss = cons_sum(sm, ss);
        const float rstd = rsqrtf(ss / (float)H + p.eps);
        float xn[EPT];
        float am = 0.0f;
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
          xn[i] = x[i] * rstd * nw[i];
          am = fmaxf(am, fabsf(xn[i]));
        }
        {
          __half2 h2[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) h2[i] = __floats2half2_rn(xn[2 * i], xn[2 * i + 1]);
          reinterpret_cast<uint4*>(sm.xh)[xslot(t)] = *reinterpret_cast<const uint4*>(h2);
        }
        // 16-bit fixed point per 32 elements (4 threads): |x| * 2^s < 2^15
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        int sh = 14 - (((__float_as_int(am) >> 23) & 255) - 127);
        sh = max(-126, min(126, sh));
        const float sc = __int_as_float((127 + sh) << 23), isc = __int_as_float((127 - sh) << 23);
        int xi[EPT];
        int sum = 0;
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
          xi[i] = max(-32768, min(32767, __float2int_rn(xn[i] * sc)));
          sum += xi[i];
        }
        auto hb = [](int v) { return (uint32_t)((v >> 8) & 0xFF); };
        auto lb = [](int v) { return (uint32_t)(v & 0xFF); };
        uint4 dq;
        dq.x = hb(xi[0]) | (hb(xi[2]) << 8) | (hb(xi[4]) << 16) | (hb(xi[6]) << 24);
        dq.y = hb(xi[1]) | (hb(xi[3]) << 8) | (hb(xi[5]) << 16) | (hb(xi[7]) << 24);
        dq.z = lb(xi[0]) | (lb(xi[2]) << 8) | (lb(xi[4]) << 16) | (lb(xi[6]) << 24);
        dq.w = lb(xi[1]) | (lb(xi[3]) << 8) | (lb(xi[5]) << 16) | (lb(xi[7]) << 24);
        sm.xq[xslot(t)] = dq;
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((t & 3) == 0) sm.chunk[t >> 2] = make_int2(-8 * sum, __float_as_int(isc));
        if (l == 0 && t == 0) sm.rstd0 = rstd;       // layer 0's own prediction (first_pred)
        if (pred_next) {
          // the rows of this CTA's W_down tiles of the next predictor: RMSNorm_{l+1}(x_l)
          const int r0 = sp.d0 * WD_ROWS, r1 = sp.d1 * WD_ROWS;
          if (EPT * t >= r0 && EPT * t < r1) {
#pragma unroll
            for (int i = 0; i < EPT; ++i) {
              const float w = dn->norm_w ? __ldg(dn->norm_w + EPT * t + i) : 1.0f;
              xs[EPT * t + i - r0] = x[i] * rstd * w;
            }
          }
        }
      }
      if (t == 0) *reinterpret_cast<volatile int32_t*>(&sm.cons_layer) = l;
      // layer l+1's claim counter: its last users (layer l-1) are done
      if (t == 1) sm.gnext[(l + 1) & 1] = 0;
      named_bar(1, CONS_THREADS);
      if (t == 0) {
        // the planner's W_down rows (xs), and at layer 0 the RMS of x_0, are written
        if (pred_next || (l == 0 && first_pred(p))) mbar_arrive(&sm.phase0_done);
        trace_ev(p, l, 1);
      }

      // ---- subgroup phase: groups g = sg, sg + 4, ... of the layer's stream
      float y[SPT];
#pragma unroll
      for (int k = 0; k < SPT; ++k) y[k] = 0.0f;
      float csa = 0.0f, csb = 0.0f;      // f16 coefficient sums of the cold rows (bias removed at the end)
      // trace counters (subgroup 0's poller, SM cycles): 0 fill waits, 1 cold,
      // 2 hot, 4 group barrier, 5 group setup, 6 release, 7 start
      const bool tr = p.trace != nullptr && t == 0;
      if (tr) {
        for (int k = 0; k < 7; ++k) sm.tstat[k] = 0;
        sm.tstat[7] = (uint64_t)clock64();
      }
      // The subgroups claim the layer's groups in stream order from a shared
      // counter (ring position base + group), so a subgroup that drew cheap
      // groups takes more of them and the four finish together.  A subgroup's
      // poller claims and tests its next group just before the reduction
      // barrier of the current one, which publishes the decision: one
      // subgroup barrier per group.  Decisions alternate between two slots
      // (a slot is rewritten only after the barrier that follows its reads).
      int r, gi;
      {
        uint64_t tb = 0;
        if (u == 0) {
          gi = atomicAdd(&sm.gnext[l & 1], 1);
          const uint32_t qc = base + (uint32_t)gi;
          r = poll_pos(sm, qc, (int)(qc % (uint32_t)NE), (qc / (uint32_t)NE) & 1u, l, gi,
                       tr ? &sm.tstat[0] : nullptr, p.wait_ns);
          if (ld_vol(&sm.abort) != 0) r = -1;
          if (r < 0) sm.abort = 1;
          sm.sgdec[sg][dbuf][0] = r;
          sm.sgdec[sg][dbuf][1] = gi;
          if (tr) tb = (uint64_t)clock64();
        }
        named_bar(2 + sg, SG_THREADS);
        if (tr) sm.tstat[4] += (uint64_t)clock64() - tb;
        r = sm.sgdec[sg][dbuf][0];
        gi = sm.sgdec[sg][dbuf][1];
        dbuf ^= 1;
      }
      while (r > 0) {
        const int e = (int)((base + (uint32_t)gi) % (uint32_t)NE);
        const SlotInfo inf = sm.info[e];
        const uint8_t* s0 = ring + (size_t)e * ENTRY_BYTES;
        const uint8_t* s1 = s0 + HALF_BYTES;
        const int db = dbuf;
        // claim the next group and test it once (published by the reduction barrier)
        auto claim_next = [&]() {
          if (u == 0) {
            const int g2 = atomicAdd(&sm.gnext[l & 1], 1);
            const uint32_t q2 = base + (uint32_t)g2;
            int r2 = poll_once(sm, q2, (int)(q2 % (uint32_t)NE), (q2 / (uint32_t)NE) & 1u, l, g2);
            if (ld_vol(&sm.abort) != 0) r2 = -1;
            sm.sgdec[sg][db][0] = r2;
            sm.sgdec[sg][db][1] = g2;
          }
        };
        const uint64_t tg0 = tr ? (uint64_t)clock64() : 0;
        if (inf.kind == UNIT_COLD) {
          sg_cold(sm, p, s0, s1, inf.n, sg, rbuf, y, csa, csb, claim_next);
        } else {
          sg_hot(sm, p, d.hot_scale, s0, s1, inf.n, inf.index, sg, rbuf, y, claim_next);
        }
        rbuf ^= 1;
        uint64_t tg1 = 0;
        if (tr) {
          tg1 = (uint64_t)clock64();
          sm.tstat[inf.kind == UNIT_COLD ? 1 : 2] += tg1 - tg0;
        }
        sg_release(sm, e);
        if (tr) sm.tstat[6] += (uint64_t)clock64() - tg1;
        r = sm.sgdec[sg][db][0];
        gi = sm.sgdec[sg][db][1];
        dbuf ^= 1;
        if (r == 2) {
          // not filled at the test: wait for it now (this subgroup holds no entry)
          uint64_t tb = 0;
          if (u == 0) {
            const uint32_t qc = base + (uint32_t)gi;
            int r3 = poll_pos(sm, qc, (int)(qc % (uint32_t)NE), (qc / (uint32_t)NE) & 1u, l, gi,
                              tr ? &sm.tstat[0] : nullptr, p.wait_ns);
            if (ld_vol(&sm.abort) != 0) r3 = -1;
            sm.sgdec[sg][dbuf][0] = r3;
            if (tr) tb = (uint64_t)clock64();
          }
          named_bar(2 + sg, SG_THREADS);
          if (tr) sm.tstat[4] += (uint64_t)clock64() - tb;
          r = sm.sgdec[sg][dbuf][0];
          dbuf ^= 1;
        }
        if (r < 0 && u == 0) sm.abort = 1;
      }
      if (p.trace != nullptr && u == 0) trace_ev(p, l, 4 + sg);
      if (tr) {
        trace_set(p, l, 16, sm.tstat[0]);
        trace_set(p, l, 2, sm.tstat[1]);
        trace_set(p, l, 3, sm.tstat[2]);
        trace_set(p, l, 23, sm.tstat[3]);
        trace_set(p, l, 24, sm.tstat[4]);
        trace_set(p, l, 25, sm.tstat[5]);
        trace_set(p, l, 26, sm.tstat[6]);
        trace_set(p, l, 27, (uint64_t)clock64() - sm.tstat[7]);
      }
      // ---- all subgroups done: remove the cold rows' bias, one abort decision for
      // everyone, then sum the partial y (fixed tree in shared memory) and add it to
      // the layer's accumulator
      cold_bias_out(y, csa, csb);
      if (t == 0) {
        bool okw = true;
        if (pred_next) okw = mbar_wait(&sm.wdown_done, wd_phase & 1u, p.wait_ns);
        if (!okw) {
          sm.abort = 1;
          atomicOr(p.status, HC_ERR_TIMEOUT);
        }
        sm.flag = ld_vol(&sm.abort) ? 0 : 1;
      }
      if (pred_next) ++wd_phase;
      named_bar(1, CONS_THREADS);
      if (t == 0) trace_ev(p, l, 38);
      if (sm.flag == 0) {
        ok = false;
        break;
      }
      base += (uint32_t)ld_vol(&sm.ngroups[l & 3]);
      {
        // Fixed tree over the four subgroups' partial y in shared memory (ypos4
        // layout, conflict-free): subgroups 2 and 3 stage theirs, subgroups 0 and 1
        // add them in place, then thread t adds the two stages' elements
        // [8t, 8t+8) and stores them in element order for one bulk reduction.
        // bufA = ystage (the planner released it: wdown_done above), bufB = xh + xq
        // (dead until the next layer's input is normalised).
        float4* bufA = reinterpret_cast<float4*>(sm.ystage);
        float4* bufB = reinterpret_cast<float4*>(sm.xh);
        float4* mine = (sg & 1) ? bufB : bufA;
        if (sg >= 2) {
#pragma unroll
          for (int j = 0; j < SPT / 4; ++j)
            mine[ypos4(u, j)] = make_float4(y[4 * j], y[4 * j + 1], y[4 * j + 2], y[4 * j + 3]);
        }
        named_bar(1, CONS_THREADS);
        if (sg < 2) {
#pragma unroll
          for (int j = 0; j < SPT / 4; ++j) {
            const float4 o = mine[ypos4(u, j)];
            mine[ypos4(u, j)] = make_float4(y[4 * j] + o.x, y[4 * j + 1] + o.y, y[4 * j + 2] + o.z,
                                            y[4 * j + 3] + o.w);
          }
        }
        named_bar(1, CONS_THREADS);
        if (t == 0) trace_ev(p, l, 39);
        float4 e0 = bufA[ypos4_of_thread(t, 0)], e1 = bufA[ypos4_of_thread(t, 1)];
        {
          const float4 f0 = bufB[ypos4_of_thread(t, 0)], f1 = bufB[ypos4_of_thread(t, 1)];
          e0.x += f0.x; e0.y += f0.y; e0.z += f0.z; e0.w += f0.w;
          e1.x += f1.x; e1.y += f1.y; e1.z += f1.z; e1.w += f1.w;
        }
        named_bar(1, CONS_THREADS);       // every stage read before bufA is overwritten
        {
          // element order; lanes 4-7 of each quarter warp store their second half
          // first, so both stores are conflict-free
          const int f = (t >> 2) & 1;
          bufA[2 * t + f] = f ? e1 : e0;
          bufA[2 * t + 1 - f] = f ? e0 : e1;
        }
        fence_proxy_async_smem();
        named_bar(1, CONS_THREADS);
        if (t == 0) {
          trace_ev(p, l, 9);
          // y_l += this CTA's partial: the L2 adds 16 KB in one bulk operation
          bulk_reduce_add_f32(p.yacc + ((size_t)(l % NACC) * YCOPIES + c % YCOPIES) * H,
                              reinterpret_cast<const float*>(bufA), H * sizeof(float));
          bulk_wait_all();
          trace_ev(p, l, 28);
          // then the grid-barrier arrival, ordered after the reduction's writes
          asm volatile("fence.proxy.async.global;" ::: "memory");
          trace_ev(p, l, 29);
          asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(p.bar_count) : "memory");
          trace_ev(p, l, 8);
        }
      }
    }
    // ---- output: x_L = x_{L-1} + y_{L-1}
    if (ok) {
      const int L = p.n_compute;
      ok = layer_wait(sm, p, L - 1);
      float xo[EPT];
      if (ok && c == 0) ok = load_x(sm, p, L - 1, t, xo);
      if (ok && c == 0) {
        const float4 o0 = make_float4(xo[0], xo[1], xo[2], xo[3]);
        const float4 o1 = make_float4(xo[4], xo[5], xo[6], xo[7]);
        if (p.io_f16) {
          const __half2 h0 = __floats2half2_rn(xo[0], xo[1]), h1 = __floats2half2_rn(xo[2], xo[3]);
          const __half2 h2 = __floats2half2_rn(xo[4], xo[5]), h3 = __floats2half2_rn(xo[6], xo[7]);
          uint4 q;
          q.x = *reinterpret_cast<const uint32_t*>(&h0);
          q.y = *reinterpret_cast<const uint32_t*>(&h1);
          q.z = *reinterpret_cast<const uint32_t*>(&h2);
          q.w = *reinterpret_cast<const uint32_t*>(&h3);
          *reinterpret_cast<uint4*>(static_cast<__half*>(p.x_out) + EPT * t) = q;
        } else {
          float4* out = reinterpret_cast<float4*>(static_cast<float*>(p.x_out) + EPT * t);
          out[0] = o0;
          out[1] = o1;
        }
        if (p.x_hist) {
          float4* h = reinterpret_cast<float4*>(p.x_hist + (size_t)(L - 1) * H + EPT * t);
          h[0] = o0;
          h[1] = o1;
        }
      }
    }
    if (t == 0 && !ok) atomicOr(p.status, HC_ERR_TIMEOUT);
    __syncthreads();
  }

  // Once every CTA is past its last read: reset the barrier counters and clear
  // the accumulators, so the next launch starts from a clean workspace.
  if (tid == 0) {
    trace_ev(p, 0, 34);        // the CTA is done (layer 0's slot)
    __threadfence();
    sm.last = atomicAdd(p.exit_count, 1u) == (uint32_t)G - 1;
  }
  __syncthreads();
  if (sm.last) {
    __threadfence();
    for (int i = tid; i < NACC * YCOPIES * H / 4; i += STACK_THREADS)
      reinterpret_cast<float4*>(p.yacc)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = tid; i < NACC * 128; i += STACK_THREADS) p.zacc[i] = 0.0f;
    if (tid < NACC) p.hot_next[tid] = 0u;
    if (tid < NACC) p.zdone[tid] = 0u;
    if (tid < NACC) p.gfill[tid] = 0u;
    if (tid < NACC) p.gclaim[tid] = 0u;
    if (tid < NACC) p.gdone[tid] = 0u;
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

extern "C" int64_t hc_tp_buffer_bytes(int32_t tp_size) {
  if (tp_size < 1 || tp_size > TP_MAX) return -1;
  return (int64_t)(XCHG_HDR + sizeof(unsigned long long) * (size_t)NACC * tp_size * H);
}

extern "C" int hc_ffn_stack_tp(const hc_layer_desc* layers, int32_t n_layers, int32_t inter, const void* x_in,
                               uint32_t* masks, int32_t masks_given, void* x_out, float* x_hist, float eps,
                               int32_t act, int32_t act_on_both, float logit_threshold, int32_t grid,
                               void* workspace, int32_t* status, uint64_t* trace, const hc_tp_desc* tp,
                               hc_stream_t stream) {
  if (!layers || n_layers <= 0 || n_layers > 32767 || !x_in || !masks || !x_out || !workspace || !status)
    return HC_ERR_ARG;
  if (masks_given < 0 || masks_given > 2) return HC_ERR_ARG;
  // predicting the last layer only needs a layer before it and the kernel's own prediction
  if (tp && tp->predict_last && (n_layers < 2 || masks_given == 1)) return HC_ERR_ARG;
  if (inter <= 0 || inter > 32768 || (inter & 3) != 0 || (act != HC_ACT_SILU && act != HC_ACT_RELU))
    return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x_in) & 15) || (reinterpret_cast<uintptr_t>(x_out) & 15) ||
      (reinterpret_cast<uintptr_t>(workspace) & 15) || (x_hist && (reinterpret_cast<uintptr_t>(x_hist) & 15)))
    return HC_ERR_ARG;
  int G = grid > 0 ? grid : hc_ffn_stack_grid();
  if (G <= 0) return HC_ERR_CUDA;
  const int words = (inter + 31) / 32;
  int words_lo = 0, words_n = words, tp_size = 1, tp_rank = 0;
  if (tp) {
    if (tp->size < 1 || hc_tp_buffer_bytes(tp->size) < 0 || tp->rank < 0 || tp->rank >= tp->size ||
        tp->words_lo < 0 || tp->words_n < 0 || tp->words_lo + tp->words_n > words || (tp->size > 1 && !tp->peer_buf))
      return HC_ERR_ARG;
    words_lo = tp->words_lo;
    words_n = tp->words_n;
    tp_size = tp->size;
    tp_rank = tp->rank;
  }
  if ((words_n + G - 1) / G > OWN_WORDS) return HC_ERR_UNSUPPORTED;   // own neuron-id range too wide
  int dev = 0, smem_max = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
    return HC_ERR_CUDA;
  const size_t smem_need = RING_OFF + (size_t)NE * ENTRY_BYTES;
  if ((long)smem_need > (long)smem_max) return HC_ERR_UNSUPPORTED;
  const int smem = (int)smem_need;
  if (cudaFuncSetAttribute(ffn_stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return HC_ERR_CUDA;
  StackParams p;
  p.layers = layers;
  p.n_layers = n_layers;
  p.n_compute = n_layers - ((tp && tp->predict_last) ? 1 : 0);
  p.inter = inter;
  p.words = words;
  p.words_lo = words_lo;
  p.words_n = words_n;
  p.tp_size = tp_size;
  p.tp_rank = tp_rank;
  p.peer_buf = tp ? tp->peer_buf : nullptr;
  p.seq_base = tp ? tp->seq_base : 0u;
  p.x_in = x_in;
  p.masks = masks;
  p.masks_given = masks_given == 1;
  p.pred0 = masks_given == 2;
  p.x_out = x_out;
  p.io_f16 = (tp && tp->io_f16) ? 1 : 0;
  p.x_hist = x_hist;
  p.eps = eps;
  p.relu = act == HC_ACT_RELU;
  p.both = act_on_both != 0;
  p.thr = logit_threshold;
  char* ws = static_cast<char*>(workspace);
  p.bar_count = reinterpret_cast<uint32_t*>(ws);
  p.hot_next = reinterpret_cast<uint32_t*>(ws + WS_HOT_NEXT);
  p.zdone = reinterpret_cast<uint32_t*>(ws + WS_ZDONE);
  p.gfill = reinterpret_cast<uint32_t*>(ws + WS_GFILL);
  p.gclaim = reinterpret_cast<uint32_t*>(ws + WS_GCLAIM);
  p.gdone = reinterpret_cast<uint32_t*>(ws + WS_GDONE);
  p.gpool = reinterpret_cast<int32_t*>(ws + WS_POOL);
  p.exit_count = reinterpret_cast<uint32_t*>(ws + WS_EXIT);
  p.yacc = reinterpret_cast<float*>(ws + WS_YACC);
  p.zacc = reinterpret_cast<float*>(ws + WS_ZACC);
  p.xbuf = reinterpret_cast<float*>(ws + WS_XBUF);
  p.status = status;
  p.trace = trace;
  p.wait_ns = (tp && tp->wait_ns > 0) ? tp->wait_ns : WAIT_LIMIT_NS;
  void* args[] = {&p};
  cudaError_t e = cudaLaunchCooperativeKernel(reinterpret_cast<const void*>(ffn_stack_kernel), dim3(G),
                                              dim3(STACK_THREADS), args, smem, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_ffn_stack(const hc_layer_desc* layers, int32_t n_layers, int32_t inter, const float* x_in,
                            uint32_t* masks, int32_t masks_given, float* x_out, float* x_hist, float eps,
                            int32_t act, int32_t act_on_both, float logit_threshold, int32_t grid, void* workspace,
                            int32_t* status, uint64_t* trace, hc_stream_t stream) {
  return hc_ffn_stack_tp(layers, n_layers, inter, x_in, masks, masks_given, x_out, x_hist, eps, act, act_on_both,
                         logit_threshold, grid, workspace, status, trace, nullptr, stream);
}
