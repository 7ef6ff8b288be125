// Batched decode of one hot/cold sparse-FFN layer (B tokens, one fetch set)
// on the 5th-generation tensor cores (tcgen05.mma, accumulators in TMEM).
//
// The reference's sparse_ffn takes x [B, 4096] (engine.py:173-209); the
// batched configuration of this path runs every token through the union of
// the tokens' fetch sets.  Per layer and pass of up to 64 tokens (N = the
// token count rounded up to 16):
//
//   k_norm     RMSNorm_l(x_b) -> f16 operand tiles, twice: natural element
//              order for the FP8 hot rows, and the nibble order of the INT4
//              decoder (each 8-element run stored as 0,4,1,5,2,6,3,7) for the
//              cold rows -- a dot product may permute K as long as both
//              operands do
//   k_gu       gate and up GEMMs, D[128 neurons][N tokens], persistent over
//              64-wide K steps of every tile: 512 decoder threads turn FP8
//              rows (exact in f16) or INT4 rows (q * group scale, rounded
//              once to f16) into the A operand in TMEM (tcgen05.st); one
//              thread issues tcgen05.mma with A from TMEM and the token tile
//              from shared memory; 4 warps move finished accumulators out of
//              TMEM as fp32 partial sums of the CTA's K range
//   k_act      sum of the K partials, per-neuron FP8 scales, gated
//              activation -> act [slot][N] f16
//   k_down     D[128 output rows][N tokens] per CTA over a neuron range:
//              A = down columns (FP8 exact, INT4 q exact; MN-major tiles),
//              B = act (times the INT4 group scale of the CTA's 128 rows);
//              the epilogue adds the tile straight into the residual rows
//              x_b with float reductions (a warp covers 32 consecutive
//              elements of one token)
//
// Two ways to reach the cold records:
//   gathered   (k_gu, k_act, k_down) the union's ascending record list is
//              walked; each record's fields are fetched where they lie in the
//              store (cp.async windows around the 2-byte field offset)
//   packed     (k_gu_p, k_act_p, k_down_p) for large batches, where the union
//              covers most records: a load-time unit-major copy of the layer
//              (hc_batch_pack) is streamed whole with one bulk copy per block,
//              and records outside the union get a zero activation
//
// Shared-memory operand layout (SWIZZLE_NONE canonical form): 8x16-byte core
// matrices; SBO = the byte stride between core matrices along M/N, LBO =
// along K.  Every weight byte is read once per pass.
#include <cuda.h>
#include <string.h>
#include <utility>
#include <cudaTypedefs.h>

#include "hc_common.cuh"

namespace hcb {
using namespace hc;

constexpr int NMAX = 64;             // tokens per pass
constexpr int TILE = 128;            // MMA M: neurons per gate/up tile, output rows per down tile
constexpr int KC = 64;               // K per pipeline stage
constexpr int HOT_ROW = 3 * H;       // packed hot neuron: gate row | up row | down column (e4m3)
constexpr int A_TILE_BYTES = TILE * KC * 2;    // 16 KB of f16
constexpr uint64_t WAIT_NS = 1000000000ull;
constexpr uint64_t DRAIN_NS = 2000000000ull;       // copies and MMAs in flight complete by themselves

// ---------------------------------------------------------------------------
// tcgen05 helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t sdesc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  // start >> 4 [0,14), LBO >> 4 [16,30), SBO >> 4 [32,46), descriptor version 1 at [46,48),
  // base offset 0, SWIZZLE_NONE
  return (uint64_t)((addr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// kind::f16 instruction descriptor: f16 A and B, f32 accumulate, M = 128
__host__ __device__ constexpr uint32_t idesc_f16(int n, int a_mn, int b_mn) {
  return (1u << 4) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(TILE >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// A from TMEM (128 lanes x 8 columns of f16 pairs = 16 K), B from shared memory
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// 16 consecutive 32-bit columns of this thread's TMEM lane, then wait for the store
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
// the same store without the wait (several stores, then one tmem_wait_st)
__device__ __forceinline__ void tmem_st16_nowait(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Programmatic dependent launch (the packed-mode kernels are launched with
// programmatic stream serialisation): a kernel lets the next one be scheduled
// as soon as every one of its CTAs has started, and the next one does its
// independent set-up (barriers, TMEM, weight copies) before waiting, in
// pdl_wait, for its predecessor to complete with all its memory visible.
// Without the launch attribute both are no-ops.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// global -> shared bulk copy (16-byte aligned, size % 16 == 0) completing on `bar`
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// 2-D tiled tensor copy, coordinates {x (bytes), y (rows)}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// four rows y0..y3 of a one-row-high box at byte offset x, stored one after another
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int x, int y0, int y1, int y2, int y3,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y0), "r"(y1), "r"(y2), "r"(y3),
      "r"(smem_u32(bar))
      : "memory");
}

// 8 consecutive fp32 columns of this thread's TMEM lane
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// ---------------------------------------------------------------------------
// element decoders into 16-byte operand pieces (8 f16)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cvt_e4m3x2(uint32_t two_bytes) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(static_cast<unsigned short>(two_bytes & 0xFFFFu)));
  return r;
}
// 8 e4m3 (lo, hi words) -> 8 f16 in natural order
__device__ __forceinline__ uint4 fp8_piece_nat(uint32_t lo, uint32_t hi) {
  return make_uint4(cvt_e4m3x2(lo), cvt_e4m3x2(lo >> 16), cvt_e4m3x2(hi), cvt_e4m3x2(hi >> 16));
}
// 8 e4m3 -> 8 f16 in the order 0,4,1,5,2,6,3,7
__device__ __forceinline__ uint4 fp8_piece_perm(uint32_t lo, uint32_t hi) {
  const uint32_t a = __byte_perm(lo, hi, 0x5140), b = __byte_perm(lo, hi, 0x7362);
  return make_uint4(cvt_e4m3x2(a), cvt_e4m3x2(a >> 16), cvt_e4m3x2(b), cvt_e4m3x2(b >> 16));
}
// 8 signed INT4 (element e in bits 4e..4e+3) -> 8 f16 q values in the order 0,4,1,5,2,6,3,7:
// (q + 8) | 0x6400 is the f16 1024 + q + 8 exactly; subtracting 1032 leaves q.
__device__ __forceinline__ uint4 int4_piece_perm(uint32_t w) {
  const uint32_t u = w ^ 0x88888888u;
  const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));
  uint32_t o[4];
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t h = ((u >> (4 * s)) & 0x000F000Fu) | 0x64006400u;
    const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&h), bias);
    o[s] = *reinterpret_cast<const uint32_t*>(&q);
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}
__device__ __forceinline__ uint4 scale_piece(uint4 p, __half s) {
  const __half2 s2 = __halves2half2(s, s);
  uint32_t* w = reinterpret_cast<uint32_t*>(&p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 v = __hmul2(*reinterpret_cast<const __half2*>(&w[i]), s2);
    w[i] = *reinterpret_cast<const uint32_t*>(&v);
  }
  return p;
}
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ldg128(const void* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint32_t ldg32(const void* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }

// position p of a 16-byte piece in the INT4 order holds element perm8(p)
__device__ __forceinline__ int perm8(int p) { return (p >> 1) + ((p & 1) << 2); }

struct LayerArgs {
  const uint8_t* hot;
  const float* hot_scale;
  int n_hot;
  const uint8_t* cold;
  int n_records;
  const int32_t* rec;
  const int32_t* count;
  int max_cold;
  int relu, both;
  int32_t* status;
  const uint8_t* flags;   // dense cold mode: [n_records] 1 = in the batch's fetch set; NULL = gathered list
};

// cold rows of the gathered work list
__device__ __forceinline__ int cold_count(const LayerArgs& a) { return min(*a.count, a.max_cold); }
__device__ __forceinline__ int checked_rec(const LayerArgs& a, int i) {
  const int r = __ldg(a.rec + i);
  if (r < 0 || r >= a.n_records) {
    atomicOr(a.status, HC_ERR_RANGE);
    return -1;
  }
  return r;
}

// ---------------------------------------------------------------------------
// k_norm: token b of the pass -> operand tiles.  Byte offset of (token, k) in
// a tile set of N tokens: chunk (k / 64) * N * 128 + ((k % 64) / 8) * 16 N +
// (b / 8) * 128 + (b % 8) * 16 + position * 2.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_norm(const float* __restrict__ x, int nb, int N, const float* __restrict__ w,
                                              float eps, uint8_t* __restrict__ xs_nat, uint8_t* __restrict__ xs_perm) {
  __shared__ float red[8];
  const int b = blockIdx.x, t = threadIdx.x;
  constexpr int NP = H / 8 / 256;               // 8-element pieces per thread: t, t + 256
  pdl_launch_dependents();
  // the RMSNorm weights do not depend on the previous layer: read them before waiting
  float wv[NP][8];
  const bool w16 = (reinterpret_cast<uintptr_t>(w) & 15) == 0;    // vector loads only when aligned
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    if (w && !w16) {
#pragma unroll
      for (int e = 0; e < 8; ++e) wv[j][e] = __ldg(w + (t + 256 * j) * 8 + e);
    } else if (w) {
      const float4 a0 = __ldg(reinterpret_cast<const float4*>(w + (t + 256 * j) * 8));
      const float4 a1 = __ldg(reinterpret_cast<const float4*>(w + (t + 256 * j) * 8) + 1);
      wv[j][0] = a0.x; wv[j][1] = a0.y; wv[j][2] = a0.z; wv[j][3] = a0.w;
      wv[j][4] = a1.x; wv[j][5] = a1.y; wv[j][6] = a1.z; wv[j][7] = a1.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) wv[j][e] = 1.0f;
    }
  }
  pdl_wait();                                   // x is the previous layer's output
  // each thread reads its pieces of x once: the sum of squares and the scaled values
  float v[NP][8];
  if (b < nb) {
    float ss = 0.0f;
#pragma unroll
    for (int j = 0; j < NP; ++j) {
      const float4* src = reinterpret_cast<const float4*>(x + (size_t)b * H + (t + 256 * j) * 8);
      const float4 a0 = src[0], a1 = src[1];
      v[j][0] = a0.x; v[j][1] = a0.y; v[j][2] = a0.z; v[j][3] = a0.w;
      v[j][4] = a1.x; v[j][5] = a1.y; v[j][6] = a1.z; v[j][7] = a1.w;
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += v[j][e] * v[j][e];
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((t & 31) == 0) red[t >> 5] = ss;
    __syncthreads();
    ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += red[k];
    const float rstd = rsqrtf(ss / (float)H + eps);
#pragma unroll
    for (int j = 0; j < NP; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] *= rstd * wv[j][e];
  } else {
#pragma unroll
    for (int j = 0; j < NP; ++j)
#pragma unroll
      for (int e = 0; e < 8; ++e) v[j][e] = 0.0f;
  }
#pragma unroll
  for (int j = 0; j < NP; ++j) {
    const int k0 = (t + 256 * j) * 8;
    __half hn[8], hp[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      hn[p] = __float2half_rn(v[j][p]);
      hp[p] = __float2half_rn(v[j][perm8(p)]);
    }
    const size_t off = (size_t)(k0 / KC) * N * 128 + (size_t)((k0 % KC) / 8) * 16 * N + (b / 8) * 128 + (b % 8) * 16;
    *reinterpret_cast<uint4*>(xs_nat + off) = *reinterpret_cast<const uint4*>(hn);
    *reinterpret_cast<uint4*>(xs_perm + off) = *reinterpret_cast<const uint4*>(hp);
  }
}

// ---------------------------------------------------------------------------
// Persistent schedule of k_gu / k_down: U work units are split into G
// contiguous ranges, one per CTA (G = grid size); unit x belongs to CTA
// ((x + 1) G - 1) / U.  A unit is one 64-wide K step of one output tile.
// ---------------------------------------------------------------------------
constexpr int GU_PROD = 512;                       // k_gu decoder threads: (row, matrix, K half)
constexpr int GU_THREADS = GU_PROD + 64 + 128;     // + MMA warp + token-tile warp + 4 epilogue warps
// Raw weights of one unit: two 8 KB matrix regions (gate, up).  Hot: 128 rows
// x 64 bytes (one 2-D tensor copy per matrix).  Cold: row r's 48-byte window
// of the unit's 32 field bytes (the field starts 2 bytes into it) at 48 r, and
// the 16-byte window holding the row's fp16 group scale at 6144 + 16 r.
constexpr int GU_REGION = 8192;
constexpr int GU_RAW_SLOT = 2 * GU_REGION;
constexpr int GU_COLD_WIN = 48;
constexpr int GU_SCALE_OFF = TILE * GU_COLD_WIN;
constexpr int GU_STAGES = 4;                       // k_gu: TMEM A stages = token-tile stages
constexpr int GUP_GROUP = 4;                       // k_gu_p: units per bulk-copied group (up to 64 KB)
constexpr int GUP_GSLOTS = 3;                      // k_gu_p: group slots (two groups in flight)
constexpr int GU_A_COL = 256;                      // TMEM columns [256, 512): A stages of 64 columns
constexpr int GU_SMEM_FLOOR = 120 * 1024;          // at least this much keeps k_gu at one CTA (all 512 TMEM columns) per SM
constexpr int DN_PROD = 256;                       // k_down producer threads: (neuron, 32-row quarter)
constexpr int DN_THREADS = DN_PROD + 32 + 128;
// The packed kernels' weight-copy issuer runs in a warp of its own: two lanes of
// one warp that block in different mbarrier waits serialise each other.
constexpr int GUP_THREADS = GU_THREADS + 64;       // k_gu_p: + issuer warp (warp 22) + up-MMA warp (warp 23)
constexpr int DNP_PROD = 2 * DN_PROD;              // k_down_p: two producer groups of 8 warps
constexpr int DNP_THREADS = DNP_PROD + 64 + 128 + 32;   // + 2 MMA warps + 4 epilogue warps + issuer warp (warp 22)
constexpr int GUP_DEC_WARPS = GU_PROD / 64;        // k_gu_p: warps of one decoder group (two groups)
constexpr int RAW_DEPTH = 4;                       // k_down: units of copies in flight per thread
constexpr int GU_DEPTH = 8;                        // k_gu: raw weight slots
constexpr int GU_AHEAD = GU_DEPTH - 2;             // k_gu: copies issued this many units ahead, so a refilled
                                                   // slot was last read two units back (no lockstep wait)
constexpr int DN_PIECES = 5;                       // 2 weight, 2 act, 1 scale
constexpr int DN_PSTRIDE = DN_PROD * 16;
constexpr int REC_AHEAD = RAW_DEPTH;               // k_down: record indices copied this many units early
constexpr int REC_RING = 2 * RAW_DEPTH;
constexpr int MAX_CTAS = 256;

__device__ __forceinline__ int range_lo(int c, int U, int G) { return (int)(((int64_t)c * U) / G); }
__device__ __forceinline__ int unit_owner(int x, int U, int G) { return (int)((((int64_t)x + 1) * G - 1) / U); }

__device__ __forceinline__ void cp16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
// arrive on `bar` once this thread's earlier cp.async copies have landed (the arrival is one of the expected count)
__device__ __forceinline__ void cp_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int K>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(K) : "memory"); }
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
// the fp16 at a 2-byte aligned address, from the aligned 4-byte word holding it
__device__ __forceinline__ __half half_of(uint32_t word, uint32_t upper) {
  return __ushort_as_half(static_cast<unsigned short>(upper ? (word >> 16) : (word & 0xFFFFu)));
}
__device__ __forceinline__ const void* align16(const void* p) {
  return reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(15));
}
__device__ __forceinline__ const void* align4(const void* p) {
  return reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(3));
}
__device__ __forceinline__ uint32_t upper_half(const void* p) {
  return static_cast<uint32_t>((reinterpret_cast<uintptr_t>(p) >> 1) & 1);
}
// Bounded wait: the thread parks in try_wait (woken when the phase completes),
// so waiting warps take few issue slots from the decoders.
__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = WAIT_NS) {
  if (mbar_test_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 7) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}
__device__ __forceinline__ void fail(const LayerArgs& a, volatile int* abort_flag) {
  atomicOr(a.status, HC_ERR_TIMEOUT);
  *abort_flag = 1;
}

// barriers and TMEM slot after the operand stages and the raw ring
struct Bars {
  uint64_t* full;    // [8] producers -> MMA: stage filled
  uint64_t* empty;   // [8] MMA commit -> producers: stage free
  uint64_t* accf;    // [2] MMA commit -> epilogue: accumulator buffer complete
  uint64_t* tfree;   // [2] epilogue -> MMA: accumulator buffer drained
  uint64_t* xfull;   // [8] bulk copy -> MMA: token tile landed
  uint64_t* xempty;  // [8] MMA commit -> token-tile warp: tile read
  uint64_t* rawfull;   // [16] copies -> decoders: raw weights landed
  uint64_t* rawempty;  // [16] decoders -> issuer: raw slot read
  uint64_t* tmaf;      // [8] k_gu: tensor copy of a hot unit landed (count 1, armed by its issuer)
  uint64_t* mdrain;    // [2] MMA issuer i: every tcgen05 operation it issued has completed
  uint32_t* tslot;
  volatile int* abort_flag;
};
__device__ __forceinline__ Bars carve_bars(uint8_t* p) {
  Bars b;
  uint64_t* u = reinterpret_cast<uint64_t*>(p);
  b.full = u;
  b.empty = u + 8;
  b.accf = u + 16;
  b.tfree = u + 18;
  b.xfull = u + 20;
  b.rawfull = u + 28;
  b.rawempty = u + 44;
  b.xempty = u + 60;
  b.tslot = reinterpret_cast<uint32_t*>(u + 68);
  b.abort_flag = reinterpret_cast<volatile int*>(u + 68) + 1;
  b.tmaf = u + 69;
  b.mdrain = u + 77;
  return b;
}
__device__ __forceinline__ void init_bars(const Bars& b, int stages, int producers, int rawfull_count = -1,
                                          int xempty_count = 1, int rawempty_count = -1, int mma_issuers = 1) {
  for (int s = 0; s < stages; ++s) {
    mbar_init(&b.full[s], producers);
    mbar_init(&b.empty[s], mma_issuers);
  }
  for (int k = 0; k < 2; ++k) {
    mbar_init(&b.accf[k], mma_issuers);
    mbar_init(&b.tfree[k], 128);
  }
  for (int k = 0; k < 8; ++k) {
    mbar_init(&b.xfull[k], 1);
    mbar_init(&b.xempty[k], xempty_count);
  }
  for (int k = 0; k < 16; ++k) {
    mbar_init(&b.rawfull[k], rawfull_count < 0 ? producers : rawfull_count);
    mbar_init(&b.rawempty[k], rawempty_count < 0 ? producers : rawempty_count);
  }
  for (int k = 0; k < 8; ++k) mbar_init(&b.tmaf[k], 1);
  for (int k = 0; k < 2; ++k) mbar_init(&b.mdrain[k], 1);
  *b.abort_flag = 0;
  mbar_fence_init();
}
constexpr int BAR_BYTES = 640;

// Exit drain (every path, including an expired wait): a thread that armed
// count-1 barriers with copies waits, bounded, for the last armed phase of
// each slot; armed[s] = times slot s was armed.
template <int NS>
__device__ __forceinline__ void drain_slots(uint64_t* bars, const int (&armed)[NS], const LayerArgs& a) {
#pragma unroll 1
  for (int s = 0; s < NS; ++s)
    if (armed[s] > 0 && !bwait(&bars[s], (armed[s] - 1) & 1, DRAIN_NS)) atomicOr(a.status, HC_ERR_TIMEOUT);
}
// ... and an MMA issuer waits until every tcgen05 operation it issued has
// completed before the CTA frees its TMEM and exits.
__device__ __forceinline__ void drain_mma(uint64_t* bar, const LayerArgs& a) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
  if (!bwait(bar, 0, DRAIN_NS)) atomicOr(a.status, HC_ERR_TIMEOUT);
}

// Optional timeline of k_gu / k_down launches (profiling hook, off unless
// hc_batch_set_trace gave a buffer): per CTA 64 %globaltimer stamps.
constexpr int TRACE_SLOTS = 64;
__device__ __forceinline__ void stamp(uint64_t* tr, int c, int e) {
  if (tr) tr[(size_t)c * TRACE_SLOTS + e] = globaltimer_ns();
}

// ---------------------------------------------------------------------------
// k_gu: gate and up GEMMs, D[128 neurons][N tokens], persistent.
//   Tiles: hot tiles first (ceil(n_hot / 128)), then tiles of the union's cold
//   list; unit x = (tile x / 64, K step x % 64).  A CTA's range covers pieces
//   ("segments") of one or more tiles; each segment's fp32 partial goes to
//   block (tile + CTA) of part [blocks][128][2N] (gate N, then up N), unique
//   because ranges are contiguous.
// Weights reach shared memory GU_AHEAD units ahead of their decode, in
//   GU_DEPTH raw slots: a hot unit is one 2-D tensor copy per matrix (128
//   rows x 64 bytes of the packed hot rows, issued by thread 0); a cold unit
//   is copied with cp.async by the decoders themselves, thread t taking piece
//   t % 4 of row t / 4 of both matrices (three 16-byte pieces of the 48-byte
//   window holding the unit's 32 field bytes, which start 2 bytes into it,
//   and the 16-byte window holding the group's fp16 scale).  Rows past the
//   union's end decode as zeros.
// TMEM (512 columns): accumulator buffers tb = 0, 1 at columns [2N tb, 2N tb
//   + 2N) (gate, up); A stages s = 0..3 at [256 + 64 s, +64) (gate 32
//   columns, up 32 columns; column c of a row holds K elements 2c, 2c + 1).
// Threads: 512 decoders -- warp w decodes rows 32 (w & 3) + lane (its TMEM
//   lane quarter) of matrix (w >> 2) & 1, K half w >> 3 of each unit to f16
//   pairs and stores them with tcgen05.st; warp 16 issues tcgen05.mma (A from
//   TMEM, B = the token tile in shared memory, K-major: k-group stride 16 N,
//   token-group stride 128); warp 17 bulk-copies each unit's token tile;
//   warps 18-21 drain finished accumulator buffers.
// ---------------------------------------------------------------------------
struct GuParams {
  LayerArgs a;
  const uint8_t* xs_nat;
  const uint8_t* xs_perm;
  float* part;
  int N, hot_tiles;
  uint64_t* trace;
  CUtensorMap tm_hot;      // packed hot rows: {12288 bytes, n_hot rows}, box {64, 128}
};

__global__ void __launch_bounds__(GU_THREADS, 1) k_gu(const __grid_constant__ GuParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const LayerArgs& a = p.a;
  const int N = p.N, G = gridDim.x, c = blockIdx.x;
  const int cnt = cold_count(a);
  const int tiles = p.hot_tiles + (cnt + TILE - 1) / TILE;
  const int U = tiles * (H / KC);
  const int lo = range_lo(c, U, G), hi = range_lo(c + 1, U, G);
  if (lo >= hi) return;                                     // uniform: before any barrier
  const int nunits = hi - lo;
  uint64_t* tr = p.trace;
  if (t == 0) stamp(tr, c, 0);

  const int x_bytes = N * KC * 2;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t rbase = sbase;                             // [GU_DEPTH][GU_RAW_SLOT] raw weights (1 KB aligned)
  const uint32_t xbase = rbase + GU_DEPTH * GU_RAW_SLOT;    // [GU_STAGES][x_bytes] token tiles
  const Bars bar = carve_bars(smem + GU_DEPTH * GU_RAW_SLOT + GU_STAGES * x_bytes);

  if (t == 0) init_bars(bar, GU_STAGES, GU_PROD / 32, GU_PROD);   // decoders signal per warp; copies per thread
  if (warp == 0) tmem_alloc(bar.tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tslot;
  if (t == 0) stamp(tr, c, 1);

  if (t < GU_PROD) {
    // ---- decoders, which also issue the weight copies GU_AHEAD units ahead.
    // Cold unit: thread t copies piece t % 4 of row t / 4 for both matrices --
    // pieces 0-2 the row's 48-byte field window, piece 3 the 16-byte window
    // holding the group's fp16 scale -- so a warp's copy covers 8 whole rows.
    // Hot unit: thread 0 issues one 2-D tensor copy per matrix.
    const int q = warp & 3, m = (warp >> 2) & 1, h = warp >> 3;
    const int r = q * 32 + lane;                            // decoded row
    const int crow = t >> 2, cpiece = t & 3;                // copied row and piece
    const uint32_t a_lane = tmem + ((uint32_t)(q * 32) << 16) + GU_A_COL + 32 * m + 16 * h;
    // record index of `row` in cold tile T: -1 past the union's end, -2 out of range
    auto rec_of = [&](int T, int row) -> int {
      if (T < p.hot_tiles || T >= tiles) return -1;
      const int j = (T - p.hot_tiles) * TILE + row;
      return j < cnt ? __ldg(a.rec + j) : -1;
    };
    auto checked = [&](int R) -> int {
      if (R < -1 || R >= a.n_records) {
        atomicOr(a.status, HC_ERR_RANGE);
        return -2;
      }
      return R;
    };
    // issue side: tile being copied, its record for crow; next tile's, loaded a tile early
    int cT = -1, cR = -1, cnT = lo >> 6, cnR = rec_of(cnT, crow);
    int tma_armed[GU_DEPTH];                                // thread 0: hot-unit tensor copies per raw slot
#pragma unroll
    for (int k = 0; k < GU_DEPTH; ++k) tma_armed[k] = 0;
    auto issue = [&](int i) {
      if (i < nunits && !*bar.abort_flag) {
        const int x = lo + i, T = x >> 6, k = x & (H / KC - 1);
        const int slot = i % GU_DEPTH, use = i / GU_DEPTH;
        if (T != cT) {
          cR = checked(T == cnT ? cnR : rec_of(T, crow));
          cT = T;
          cnT = T + 1;
          cnR = rec_of(cnT, crow);
        }
        // the slot's previous unit has been decoded by every thread; if that wait
        // expires, nothing more is copied into the slot (it may still be read)
        if (use > 0 && !bwait(&bar.rawempty[slot], (use - 1) & 1)) {
          fail(a, bar.abort_flag);
          return;
        }
        const uint32_t dst = rbase + slot * GU_RAW_SLOT;
        if (T < p.hot_tiles) {
          // the tensor copies complete on tmaf[slot] (count 1), so their landing can be
          // awaited on every path; rawfull counts every thread's arrival as for cold units
          if (t == 0) {
            mbar_arrive_expect_tx(&bar.tmaf[slot], 2 * KC * TILE);
            tma_load_2d(dst, &p.tm_hot, k * KC, T * TILE, &bar.tmaf[slot]);
            tma_load_2d(dst + GU_REGION, &p.tm_hot, H + k * KC, T * TILE, &bar.tmaf[slot]);
            ++tma_armed[slot];
          }
          mbar_arrive(&bar.rawfull[slot]);
        } else {
          if (cR >= 0) {
            const uint8_t* rb = a.cold + (size_t)cR * REC_BYTES;
#pragma unroll
            for (int mm = 0; mm < 2; ++mm) {
              if (cpiece < 3)
                cp16(dst + mm * GU_REGION + crow * GU_COLD_WIN + 16 * cpiece,
                     rb + mm * VEC_BYTES + k * (KC / 2) + 16 * cpiece);
              else
                cp16(dst + mm * GU_REGION + GU_SCALE_OFF + crow * 16,
                     align16(rb + SCALE_OFF + mm * 2 * NGROUPS + 2 * (k >> 1)));
            }
          }
          cp_arrive(&bar.rawfull[slot]);
        }
      }
    };
#pragma unroll 1
    for (int i = 0; i < GU_AHEAD; ++i) issue(i);
    int dT = -1, dR = -1, dnT = lo >> 6, dnR = rec_of(dnT, r);    // decode side: this row's record
    for (int i = 0; i < nunits; ++i) {
      const int x = lo + i, T = x >> 6, k = x & (H / KC - 1);
      if (T != dT) {
        dR = T == dnT ? dnR : rec_of(T, r);
        dT = T;
        dnT = T + 1;
        dnR = rec_of(dnT, r);
      }
      issue(i + GU_AHEAD);
      const int slot = i % GU_DEPTH, s = i % GU_STAGES, round = i / GU_STAGES;
      bool ok = bwait(&bar.rawfull[slot], (i / GU_DEPTH) & 1);
      // hot units come first in a CTA's range, so every earlier use of this slot was hot too
      ok = ok && (T >= p.hot_tiles || bwait(&bar.tmaf[slot], (i / GU_DEPTH) & 1));
      ok = ok && (round == 0 || bwait(&bar.empty[s], (round - 1) & 1));
      if (!ok) fail(a, bar.abort_flag);
      // tcgen05.st is warp-collective: leave the loop as a whole warp
      if (!__all_sync(0xffffffffu, ok) || __any_sync(0xffffffffu, *bar.abort_flag != 0)) break;
      tc_fence_after();                                     // the MMAs that read stage s are done
      const uint32_t reg = rbase + slot * GU_RAW_SLOT + m * GU_REGION;
      uint32_t v[16];
      if (T < p.hot_tiles) {
        const uint4 w0 = lds128(reg + r * KC + 32 * h), w1 = lds128(reg + r * KC + 32 * h + 16);
        const uint4 p0 = fp8_piece_nat(w0.x, w0.y), p1 = fp8_piece_nat(w0.z, w0.w);
        const uint4 p2 = fp8_piece_nat(w1.x, w1.y), p3 = fp8_piece_nat(w1.z, w1.w);
        v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w; v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
        v[8] = p2.x; v[9] = p2.y; v[10] = p2.z; v[11] = p2.w; v[12] = p3.x; v[13] = p3.y; v[14] = p3.z; v[15] = p3.w;
      } else if (dR >= 0 && dR < a.n_records) {
        const uint32_t wa = reg + r * GU_COLD_WIN + 16 * h;
        const uint4 w0 = lds128(wa);
        const uint32_t w4 = lds32(wa + 16);
        // fp16 scale of group k / 2 at record byte 6146 + 64 m + 2 (k / 2), in the copied 16-byte window
        const uint32_t so = (2 + 2 * (k >> 1)) & 15;
        const __half sc = half_of(lds32(reg + GU_SCALE_OFF + r * 16 + (so & ~3u)), (so >> 1) & 1);
        const uint4 p0 = scale_piece(int4_piece_perm(shift2(w0.x, w0.y)), sc);
        const uint4 p1 = scale_piece(int4_piece_perm(shift2(w0.y, w0.z)), sc);
        const uint4 p2 = scale_piece(int4_piece_perm(shift2(w0.z, w0.w)), sc);
        const uint4 p3 = scale_piece(int4_piece_perm(shift2(w0.w, w4)), sc);
        v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w; v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
        v[8] = p2.x; v[9] = p2.y; v[10] = p2.z; v[11] = p2.w; v[12] = p3.x; v[13] = p3.y; v[14] = p3.z; v[15] = p3.w;
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = 0u;            // past the union's end, or a bad record
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.rawempty[slot]);      // raw slot read by the warp
      tmem_st16(a_lane + 64 * s, v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.full[s]);
    }
    cp_wait<0>();
    if (t == 0) drain_slots(bar.tmaf, tma_armed, a);
  } else if (t == GU_PROD) {
    // ---- MMA issuer
    const uint32_t idesc = idesc_f16(N, 0, 0);
    int seg = 0;
    for (int i = 0; i < nunits; ++i) {
      const int k = (lo + i) & (H / KC - 1);
      const bool first = i == 0 || k == 0, last = i == nunits - 1 || k == H / KC - 1;
      const int tb = seg & 1;
      if (first && seg >= 2 && !bwait(&bar.tfree[tb], ((seg >> 1) - 1) & 1)) fail(a, bar.abort_flag);
      const int s = i % GU_STAGES, round = i / GU_STAGES;
      if (!bwait(&bar.full[s], round & 1) || !bwait(&bar.xfull[s], round & 1)) fail(a, bar.abort_flag);
      if (*bar.abort_flag) break;
      tc_fence_after();
      const uint32_t X = xbase + s * x_bytes;
      const uint32_t dt = tmem + tb * 2 * N;
      const uint32_t at = tmem + GU_A_COL + 64 * s;
#pragma unroll
      for (int j = 0; j < KC / 16; ++j) {
        const uint64_t bd = sdesc(X + j * 2 * 16 * N, 16 * N, 128);
        const uint32_t acc = !(first && j == 0);
        umma_f16_ts(dt, at + 8 * j, bd, idesc, acc);
        umma_f16_ts(dt + N, at + 32 + 8 * j, bd, idesc, acc);
      }
      umma_commit(&bar.empty[s]);
      if (last) {
        umma_commit(&bar.accf[tb]);
        ++seg;
      }
    }
    drain_mma(&bar.mdrain[0], a);
  } else if (t == GU_PROD + 32) {
    // ---- token tiles: unit i's K step of the hot or cold operand tile set
    int x_armed[GU_STAGES] = {};
    for (int i = 0; i < nunits; ++i) {
      const int x = lo + i, T = x >> 6, k = x & (H / KC - 1);
      const int s = i % GU_STAGES, round = i / GU_STAGES;
      if (round > 0 && !bwait(&bar.empty[s], (round - 1) & 1)) fail(a, bar.abort_flag);
      if (*bar.abort_flag) break;
      mbar_arrive_expect_tx(&bar.xfull[s], x_bytes);
      bulk_copy(xbase + s * x_bytes, (T < p.hot_tiles ? p.xs_nat : p.xs_perm) + (size_t)k * x_bytes, x_bytes,
                &bar.xfull[s]);
      ++x_armed[s];
    }
    drain_slots(bar.xfull, x_armed, a);
  } else if (t >= GU_PROD + 64) {
    // ---- epilogue: warp (18..21) & 3 reads TMEM lanes [32 q, 32 q + 32)
    const int q = warp & 3, r = q * 32 + lane;
    int seg = 0;
    for (int x0 = lo; x0 < hi; ++seg) {
      const int T = x0 >> 6;
      const int x1 = min(hi, (T + 1) * (H / KC));
      const int tb = seg & 1;
      const bool done = bwait(&bar.accf[tb], (seg >> 1) & 1);
      if (!done) fail(a, bar.abort_flag);
      const bool go = __all_sync(0xffffffffu, done) && !__any_sync(0xffffffffu, *bar.abort_flag != 0);
      if (!go) break;
      tc_fence_after();
      const bool hotT = T < p.hot_tiles;
      const int row = (hotT ? T : T - p.hot_tiles) * TILE + r;
      const bool valid = row < (hotT ? a.n_hot : cnt);
      float* dst = p.part + ((size_t)(T + c) * TILE + r) * (2 * N);
      for (int col = 0; col < 2 * N; col += 8) {
        float v[8];
        tmem_ld8(tmem + ((uint32_t)(q * 32) << 16) + tb * 2 * N + col, v);
        if (valid) {
          reinterpret_cast<float4*>(dst + col)[0] = make_float4(v[0], v[1], v[2], v[3]);
          reinterpret_cast<float4*>(dst + col)[1] = make_float4(v[4], v[5], v[6], v[7]);
        }
      }
      tc_fence_before();
      mbar_arrive(&bar.tfree[tb]);
      x0 = x1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (t == 0) {
    stamp(tr, c, 56);
    if (tr) tr[(size_t)c * TRACE_SLOTS + 57] = (uint64_t)nunits;
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// k_act: act[slot][b] = gated(g * sg, u * su) * sd (f16), g and u summed over
// the segments of the slot's tile in ascending CTA order.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_act(LayerArgs a, const float* __restrict__ part, int hot_tiles, int G,
                                             int N, __half* __restrict__ act) {
  const int cnt = cold_count(a);
  const int total = a.n_hot + cnt;
  const int U = (hot_tiles + (cnt + TILE - 1) / TILE) * (H / KC);
  const int groups = N / 8;
  const int i = blockIdx.x * 256 + threadIdx.x;
  const int slot = i / groups, g = i % groups;
  if (slot >= total) return;
  const int T = slot < a.n_hot ? slot / TILE : hot_tiles + (slot - a.n_hot) / TILE;
  const int r = slot < a.n_hot ? slot % TILE : (slot - a.n_hot) % TILE;
  const int c0 = unit_owner(T * (H / KC), U, G), c1 = unit_owner(T * (H / KC) + H / KC - 1, U, G);
  float gs[8], us[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) gs[e] = us[e] = 0.0f;
  for (int cc = c0; cc <= c1; ++cc) {
    const float* row = part + ((size_t)(T + cc) * TILE + r) * (2 * N) + g * 8;
    const float4 g0 = reinterpret_cast<const float4*>(row)[0], g1 = reinterpret_cast<const float4*>(row)[1];
    const float4 u0 = reinterpret_cast<const float4*>(row + N)[0], u1 = reinterpret_cast<const float4*>(row + N)[1];
    gs[0] += g0.x; gs[1] += g0.y; gs[2] += g0.z; gs[3] += g0.w; gs[4] += g1.x; gs[5] += g1.y; gs[6] += g1.z; gs[7] += g1.w;
    us[0] += u0.x; us[1] += u0.y; us[2] += u0.z; us[3] += u0.w; us[4] += u1.x; us[5] += u1.y; us[6] += u1.z; us[7] += u1.w;
  }
  float sg = 1.0f, su = 1.0f, sd = 1.0f;
  if (slot < a.n_hot && a.hot_scale) {
    sg = __ldg(a.hot_scale + (size_t)slot * 3);
    su = __ldg(a.hot_scale + (size_t)slot * 3 + 1);
    sd = __ldg(a.hot_scale + (size_t)slot * 3 + 2);
  }
  __half o[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(gated(gs[e] * sg, us[e] * su, a.relu, a.both) * sd);
  *reinterpret_cast<uint4*>(act + (size_t)slot * N + g * 8) = *reinterpret_cast<const uint4*>(o);
}

// ---------------------------------------------------------------------------
// k_down: x_b[e] += sum_n down[n][e] * act[n][b], persistent.
//   Unit x = (output tile x / nsub, neuron step x % nsub), nsub = ceil(slots
//   / 64).  Producer thread (q, j): neuron q of the step, rows [32 j, 32 j +
//   32) of the tile.  Stage: A 128 rows x 64 neurons f16 MN-major (row-group
//   stride 128 B = SBO, neuron-group stride 2048 B = LBO; rows of a 16-byte
//   piece in the order 0,4,1,5,2,6,3,7); B 64 neurons x N tokens MN-major
//   (token-group stride 128 B, neuron-group stride 16 N).  Each segment's
//   tile is added into the residual rows x_b with float reductions.
// ---------------------------------------------------------------------------
// xe[b * H] += v[b - col] for tokens b in [col, col + 8) below nb (xe = row e of token 0)
__device__ __forceinline__ void add_to_rows(float* xe, int col, int nb, const float (&v)[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k)
    if (col + k < nb) asm volatile("red.global.add.f32 [%0], %1;" ::"l"(xe + (size_t)(col + k) * H), "f"(v[k]) : "memory");
}

struct DownParams {
  LayerArgs a;
  const __half* act;
  float* x;                 // the pass's token rows [nb][4096], updated in place
  int N, nb, stages;
  uint32_t tmem_cols;
  uint64_t* trace;
};

__global__ void __launch_bounds__(DN_THREADS, 1) k_down(DownParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const LayerArgs& a = p.a;
  const int N = p.N, G = gridDim.x, c = blockIdx.x;
  const int total = a.n_hot + cold_count(a);
  const int nsub = (total + KC - 1) / KC;
  const int U = (H / TILE) * nsub;
  const int lo = range_lo(c, U, G), hi = range_lo(c + 1, U, G);
  if (lo >= hi) return;
  const int nunits = hi - lo;

  const int b_bytes = KC * N * 2;
  const int stage_bytes = A_TILE_BYTES + b_bytes;
  const int raw_slot = DN_PIECES * DN_PSTRIDE;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t rbase = sbase + p.stages * stage_bytes;
  const uint32_t recbase = rbase + RAW_DEPTH * raw_slot;    // [REC_RING][DN_PROD] record indices
  const Bars bar = carve_bars(smem + p.stages * stage_bytes + RAW_DEPTH * raw_slot + REC_RING * DN_PROD * 4);

  if (t == 0) init_bars(bar, p.stages, DN_PROD / 32);
  if (warp == 0) tmem_alloc(bar.tslot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tslot;

  if (t < DN_PROD) {
    // neuron q, output rows [32 j, 32 j + 32): a quarter-warp holds 8 neurons of one j,
    // so its 16-byte stage stores land on distinct banks
    const int q = (warp << 3) | (lane & 7), j = lane >> 3;
    const int groups = N / 8;
    uint32_t meta = 0;                        // 3 bits per raw slot: kind (2), scale half (1)
    // record index of the neuron of unit u, copied REC_AHEAD units before the
    // unit's own copies are issued (range-checked where used)
    auto rec_copy = [&](int u) {
      if (u >= nunits) return;
      const int slot = ((lo + u) % nsub) * KC + q;
      if (slot >= a.n_hot && slot < total)
        cp4(recbase + ((u % REC_RING) * DN_PROD + t) * 4, a.rec + (slot - a.n_hot));
    };
    auto issue = [&](int i) {
      rec_copy(i + REC_AHEAD);
      if (i < nunits) {
        const int x = lo + i, et = x / nsub, slot = (x % nsub) * KC + q;
        int R = -1;
        if (slot >= a.n_hot && slot < total) {
          R = (int)lds32(recbase + ((i % REC_RING) * DN_PROD + t) * 4);
          if (R < 0 || R >= a.n_records) {
            atomicOr(a.status, HC_ERR_RANGE);
            R = -1;
          }
        }
        const int rs = i % RAW_DEPTH;
        const uint32_t d = rbase + rs * raw_slot + t * 16;
        uint32_t md = 0;
        if (slot < a.n_hot) {
          const uint8_t* dd = a.hot + (size_t)slot * HOT_ROW + 2 * H + et * TILE + 32 * j;
          cp16(d, dd);
          cp16(d + DN_PSTRIDE, dd + 16);
          md = 1;
        } else if (slot < total && R >= 0) {
          const uint8_t* rb = a.cold + (size_t)R * REC_BYTES;
          const uint8_t* dd = rb + 2 * VEC_BYTES + et * (TILE / 2) + 16 * j;     // aligned; field at +2
          cp16(d, dd);
          cp16(d + DN_PSTRIDE, dd + 16);
          const uint8_t* sp = rb + SCALE_OFF + 4 * NGROUPS + 2 * et;
          cp4(d + 4 * DN_PSTRIDE, align4(sp));
          md = 2 | (upper_half(sp) << 2);
        }
        if (md) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int g = j + 4 * h;
            if (g < groups) cp16(d + (2 + h) * DN_PSTRIDE, p.act + (size_t)slot * N + g * 8);
          }
        }
        meta = (meta & ~(7u << (3 * rs))) | (md << (3 * rs));
      }
      cp_commit();
    };
    for (int u = 0; u < REC_AHEAD; ++u) rec_copy(u);
    cp_commit();
    cp_wait<0>();
#pragma unroll
    for (int i = 0; i < RAW_DEPTH - 1; ++i) issue(i);
    for (int i = 0; i < nunits; ++i) {
      issue(i + RAW_DEPTH - 1);
      cp_wait<RAW_DEPTH - 1>();
      const int s = i % p.stages, round = i / p.stages;
      if (round > 0 && !bwait(&bar.empty[s], (round - 1) & 1)) fail(a, bar.abort_flag);
      if (__any_sync(0xffffffffu, *bar.abort_flag != 0)) break;     // warp-uniform: the warp signals as one
      const int rs = i % RAW_DEPTH;
      const uint32_t d = rbase + rs * raw_slot + t * 16;
      const uint32_t md = (meta >> (3 * rs)) & 7u;
      const uint32_t A = sbase + s * stage_bytes + (q >> 3) * 2048 + (4 * j) * 128 + (q & 7) * 16;
      __half ds = __float2half(1.0f);
      if ((md & 3) == 1) {
        const uint4 w0 = lds128(d), w1 = lds128(d + DN_PSTRIDE);
        sts128(A + 0 * 128, fp8_piece_perm(w0.x, w0.y));
        sts128(A + 1 * 128, fp8_piece_perm(w0.z, w0.w));
        sts128(A + 2 * 128, fp8_piece_perm(w1.x, w1.y));
        sts128(A + 3 * 128, fp8_piece_perm(w1.z, w1.w));
      } else if ((md & 3) == 2) {
        const uint4 w0 = lds128(d);
        const uint32_t w4 = lds32(d + DN_PSTRIDE);
        ds = half_of(lds32(d + 4 * DN_PSTRIDE), md >> 2);
        sts128(A + 0 * 128, int4_piece_perm(shift2(w0.x, w0.y)));
        sts128(A + 1 * 128, int4_piece_perm(shift2(w0.y, w0.z)));
        sts128(A + 2 * 128, int4_piece_perm(shift2(w0.z, w0.w)));
        sts128(A + 3 * 128, int4_piece_perm(shift2(w0.w, w4)));
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) sts128(A + k * 128, make_uint4(0, 0, 0, 0));
      }
      const uint32_t B = sbase + s * stage_bytes + A_TILE_BYTES + (q >> 3) * 16 * N + (q & 7) * 16;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int g = j + 4 * h;
        if (g < groups) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (md & 3) v = lds128(d + (2 + h) * DN_PSTRIDE);
          if ((md & 3) == 2) v = scale_piece(v, ds);
          sts128(B + g * 128, v);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.full[s]);
    }
    cp_wait<0>();
  } else if (t == DN_PROD) {
    const uint32_t idesc = idesc_f16(N, 1, 1);
    int seg = 0;
    for (int i = 0; i < nunits; ++i) {
      const int sub = (lo + i) % nsub;
      const bool first = i == 0 || sub == 0, last = i == nunits - 1 || sub == nsub - 1;
      const int tb = seg & 1;
      if (first && seg >= 2 && !bwait(&bar.tfree[tb], ((seg >> 1) - 1) & 1)) fail(a, bar.abort_flag);
      const int s = i % p.stages, round = i / p.stages;
      if (!bwait(&bar.full[s], round & 1)) fail(a, bar.abort_flag);
      if (*bar.abort_flag) break;
      tc_fence_after();
      const uint32_t st = sbase + s * stage_bytes;
      const uint32_t dt = tmem + tb * N;
#pragma unroll
      for (int k = 0; k < KC / 16; ++k)
        umma_f16(dt, sdesc(st + k * 2 * 2048, 2048, 128), sdesc(st + A_TILE_BYTES + k * 2 * 16 * N, 16 * N, 128),
                 idesc, !(first && k == 0));
      umma_commit(&bar.empty[s]);
      if (last) {
        umma_commit(&bar.accf[tb]);
        ++seg;
      }
    }
    drain_mma(&bar.mdrain[0], a);
  } else if (t >= DN_PROD + 32) {
    const int qd = warp & 3, m = qd * 32 + lane;
    int seg = 0;
    for (int x0 = lo; x0 < hi; ++seg) {
      const int et = x0 / nsub;
      const int x1 = min(hi, (et + 1) * nsub);
      const int tb = seg & 1;
      const bool done = bwait(&bar.accf[tb], (seg >> 1) & 1);
      if (!done) fail(a, bar.abort_flag);
      const bool go = __all_sync(0xffffffffu, done) && !__any_sync(0xffffffffu, *bar.abort_flag != 0);
      if (!go) break;
      tc_fence_after();
      const int e = et * TILE + (m & ~7) + perm8(m & 7);
      for (int col = 0; col < N; col += 8) {
        float v[8];
        tmem_ld8(tmem + ((uint32_t)(qd * 32) << 16) + tb * N + col, v);
        add_to_rows(p.x + e, col, p.nb, v);
      }
      tc_fence_before();
      mbar_arrive(&bar.tfree[tb]);
      x0 = x1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_free(tmem, p.tmem_cols);
  }
}

constexpr int DD_DEPTH = 8;                         // k_down_p: weight block slots (8 KB each)
constexpr int DD_ACTS = 4;                          // k_down_p: activation block slots
constexpr int DD_STAGES = 4;                        // k_down_p: f16 operand stages

// ===========================================================================
// Packed dense mode.  Once per layer (hc_batch_pack), the weights are copied
// into unit-major blocks so that every 64-wide K step of a 128-row gate/up
// tile, and every 64-neuron step of a 128-row down tile, is ONE contiguous
// block read by ONE bulk copy.  Neuron slots: hot neurons [0, 128 ht) (ht =
// ceil(n_hot / 128), padded with zero rows), then every record of the section
// in storage order [128 ht, 128 ht + n_records).  Block layouts (16-byte
// chunks are XOR-swizzled so the decoders' 16-byte shared-memory reads of 8
// neighbouring rows fall on distinct banks):
//   gate/up hot   [m 2][row 128][64 B]  e4m3, chunk c of row r at c ^ ((r >> 1) & 3)      16384 B
//   gate/up cold  [m 2][row 128][32 B]  INT4 field bytes, chunk c at c ^ ((r >> 2) & 1)
//                 + [m][row] fp16 group scale                                              8704 B
//   down hot      [row 64][128 B]       e4m3 of output rows 128 et .., chunk c at c ^ (row & 7)  8192 B
//   down cold     [row 64][64 B]        INT4 field bytes, chunk c at c ^ ((row >> 1) & 3),
//                 + [row] fp16 group scale                                                4224 B
// ===========================================================================
constexpr int PG_HOT = 16384, PG_COLD = 8704, PD_HOT = 8192, PD_COLD = 4224;

struct PackLayout {
  int hot_tiles, cold_tiles, hot_blocks, cold_blocks;
  size_t gu_hot, gu_cold, dn_hot, dn_cold, total;
};
__host__ __device__ inline PackLayout pack_layout(int n_hot, int n_records) {
  PackLayout L;
  L.hot_tiles = (n_hot + TILE - 1) / TILE;
  L.cold_tiles = (n_records + TILE - 1) / TILE;
  L.hot_blocks = 2 * L.hot_tiles;
  L.cold_blocks = (n_records + KC - 1) / KC;
  size_t o = 0;
  L.gu_hot = o;  o += (size_t)L.hot_tiles * (H / KC) * PG_HOT;
  L.gu_cold = o; o += (size_t)L.cold_tiles * (H / KC) * PG_COLD;
  L.dn_hot = o;  o += (size_t)(H / TILE) * L.hot_blocks * PD_HOT;
  L.dn_cold = o; o += (size_t)(H / TILE) * L.cold_blocks * PD_COLD;
  L.total = (o + 1023) / 1024 * 1024;
  return L;
}

// one thread per 16-byte output chunk (scales: one thread per fp16)
__global__ void k_pack(const uint8_t* __restrict__ hot, int n_hot, const uint8_t* __restrict__ cold, int n_records,
                       uint8_t* __restrict__ out) {
  const PackLayout L = pack_layout(n_hot, n_records);
  const int64_t n_gu_hot = (int64_t)L.hot_tiles * (H / KC) * PG_HOT / 16;
  const int64_t n_gu_cold = (int64_t)L.cold_tiles * (H / KC) * (2 * TILE * 2);       // 16-byte chunks
  const int64_t n_gu_sc = (int64_t)L.cold_tiles * (H / KC) * (2 * TILE);             // fp16 scales
  const int64_t n_dn_hot = (int64_t)(H / TILE) * L.hot_blocks * PD_HOT / 16;
  const int64_t n_dn_cold = (int64_t)(H / TILE) * L.cold_blocks * (KC * 4);
  const int64_t n_dn_sc = (int64_t)(H / TILE) * L.cold_blocks * KC;
  const int64_t total = n_gu_hot + n_gu_cold + n_gu_sc + n_dn_hot + n_dn_cold + n_dn_sc;
  auto field16 = [&](const uint8_t* p) {          // 16 unaligned bytes
    uint8_t b[16];
    for (int i = 0; i < 16; ++i) b[i] = p[i];
    return *reinterpret_cast<const uint4*>(b);
  };
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t k = i;
    if (k < n_gu_hot) {                           // (unit, m, row, c)
      const int c = k & 3, r = (k >> 2) & 127, m = (k >> 9) & 1;
      const int64_t unit = k >> 10;
      const int T = (int)(unit / (H / KC)), kb = (int)(unit % (H / KC));
      const int row = T * TILE + r;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (row < n_hot) v = *reinterpret_cast<const uint4*>(hot + (size_t)row * HOT_ROW + m * H + kb * KC + 16 * c);
      *reinterpret_cast<uint4*>(out + L.gu_hot + unit * PG_HOT + m * (TILE * KC) + r * KC +
                                16 * (c ^ ((r >> 1) & 3))) = v;
      continue;
    }
    k -= n_gu_hot;
    if (k < n_gu_cold) {                          // (unit, m, row, c)
      const int c = k & 1, r = (k >> 1) & 127, m = (k >> 8) & 1;
      const int64_t unit = k >> 9;
      const int T = (int)(unit / (H / KC)), kb = (int)(unit % (H / KC));
      const int R = T * TILE + r;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (R < n_records) v = field16(cold + (size_t)R * REC_BYTES + 2 + m * VEC_BYTES + kb * (KC / 2) + 16 * c);
      *reinterpret_cast<uint4*>(out + L.gu_cold + unit * PG_COLD + m * (TILE * 32) + r * 32 +
                                16 * (c ^ ((r >> 2) & 1))) = v;
      continue;
    }
    k -= n_gu_cold;
    if (k < n_gu_sc) {                            // (unit, m, row)
      const int r = k & 127, m = (k >> 7) & 1;
      const int64_t unit = k >> 8;
      const int T = (int)(unit / (H / KC)), kb = (int)(unit % (H / KC));
      const int R = T * TILE + r;
      uint16_t v = 0;
      if (R < n_records) {
        const uint8_t* sp = cold + (size_t)R * REC_BYTES + SCALE_OFF + m * 2 * NGROUPS + 2 * (kb >> 1);
        v = (uint16_t)(sp[0] | (sp[1] << 8));
      }
      *reinterpret_cast<uint16_t*>(out + L.gu_cold + unit * PG_COLD + 2 * TILE * 32 + (m * TILE + r) * 2) = v;
      continue;
    }
    k -= n_gu_sc;
    if (k < n_dn_hot) {                           // (et, block, q, c)
      const int c = k & 7, q = (k >> 3) & 63;
      const int64_t ub = k >> 9;                  // et * hot_blocks + block
      const int et = (int)(ub / L.hot_blocks), nb = (int)(ub % L.hot_blocks);
      const int n = nb * KC + q;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (n < n_hot) v = *reinterpret_cast<const uint4*>(hot + (size_t)n * HOT_ROW + 2 * H + et * TILE + 16 * c);
      *reinterpret_cast<uint4*>(out + L.dn_hot + ub * PD_HOT + q * TILE + 16 * (c ^ (q & 7))) = v;
      continue;
    }
    k -= n_dn_hot;
    if (k < n_dn_cold) {                          // (et, block, q, c)
      const int c = k & 3, q = (k >> 2) & 63;
      const int64_t ub = k >> 8;
      const int et = (int)(ub / L.cold_blocks), nb = (int)(ub % L.cold_blocks);
      const int R = nb * KC + q;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (R < n_records) v = field16(cold + (size_t)R * REC_BYTES + 2 + 2 * VEC_BYTES + et * (TILE / 2) + 16 * c);
      *reinterpret_cast<uint4*>(out + L.dn_cold + ub * PD_COLD + q * 64 + 16 * (c ^ ((q >> 1) & 3))) = v;
      continue;
    }
    k -= n_dn_cold;
    {                                             // (et, block, q)
      const int q = k & 63;
      const int64_t ub = k >> 6;
      const int et = (int)(ub / L.cold_blocks), nb = (int)(ub % L.cold_blocks);
      const int R = nb * KC + q;
      uint16_t v = 0;
      if (R < n_records) {
        const uint8_t* sp = cold + (size_t)R * REC_BYTES + SCALE_OFF + 4 * NGROUPS + 2 * et;
        v = (uint16_t)(sp[0] | (sp[1] << 8));
      }
      *reinterpret_cast<uint16_t*>(out + L.dn_cold + ub * PD_COLD + KC * 64 + q * 2) = v;
    }
  }
}

// 16-byte chunk index swizzle of activation rows (2N bytes) written by k_act_p,
// read by k_down_p: keeps the reads of 8 neighbouring rows on distinct banks
__host__ __device__ inline int act_swz(int slot, int N) {
  return N == 64 ? (slot & 7) : N == 32 ? ((slot >> 1) & 3) : N == 16 ? ((slot >> 2) & 1) : 0;
}

struct PackedParams {
  LayerArgs a;
  const uint8_t* packed;
  const uint8_t* xs_nat;
  const uint8_t* xs_perm;
  float* part;
  int N;
  uint64_t* trace;
};

// ---------------------------------------------------------------------------
// k_gu_p: k_gu over the packed blocks.  Units x = (tile x / 64, K step x % 64)
// over hot tiles then cold tiles (every record of the section).  Lane 0 of
// warp 22 bulk-copies groups of GUP_GROUP units (one copy per run of
// contiguous blocks, up to 64 KB) into GUP_GSLOTS group slots; lane 0 of warp
// 17 copies the token tiles (one per A stage, freed with it); two decoder
// groups of 8 warps take alternate units (each warp a whole K step of its
// rows); warps 16 and 23 issue the gate and the up MMAs; epilogue as in k_gu.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(GUP_THREADS, 1) k_gu_p(const __grid_constant__ PackedParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const LayerArgs& a = p.a;
  const PackLayout L = pack_layout(a.n_hot, a.n_records);
  const int N = p.N, G = gridDim.x, c = blockIdx.x;
  const int tiles = L.hot_tiles + L.cold_tiles;
  const int U = tiles * (H / KC);
  const int lo = range_lo(c, U, G), hi = range_lo(c + 1, U, G);
  if (lo >= hi) return;
  pdl_launch_dependents();
  const int nunits = hi - lo;
  uint64_t* tr = p.trace;
  if (t == 0) stamp(tr, c, 0);

  const int x_bytes = N * KC * 2;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t rbase = sbase;                             // [GUP_GSLOTS][GUP_GROUP * PG_HOT] raw unit groups
  const uint32_t xbase = rbase + GUP_GSLOTS * GUP_GROUP * PG_HOT;   // [GU_STAGES][x_bytes] token tiles
  const Bars bar = carve_bars(smem + GUP_GSLOTS * GUP_GROUP * PG_HOT + GU_STAGES * x_bytes);
  // packed source and size of local unit i; a group's units sit back to back in its slot
  auto usrc = [&](int i) -> const uint8_t* {
    const int x = lo + i;
    return p.packed + (x < L.hot_tiles * (H / KC) ? L.gu_hot + (size_t)x * PG_HOT
                                                   : L.gu_cold + (size_t)(x - L.hot_tiles * (H / KC)) * PG_COLD);
  };
  auto usize = [&](int i) -> uint32_t { return lo + i < L.hot_tiles * (H / KC) ? PG_HOT : PG_COLD; };

  // group g = local units [4 g, 4 g + 4): one bulk copy per run of contiguous blocks (the hot
  // blocks, then the cold ones), issued by the issuer warp two groups ahead
  const int ngroups = (nunits + GUP_GROUP - 1) / GUP_GROUP;
  int g_armed[GUP_GSLOTS] = {};                             // issuer: group copies per slot
  auto issue = [&](int g) {
    if (g >= ngroups) return;
    const int slot = g % GUP_GSLOTS, use = g / GUP_GSLOTS;
    // if the slot is not released in time, nothing more is copied into it (it may still be read)
    if (use > 0 && !bwait(&bar.rawempty[slot], (use - 1) & 1)) {
      fail(a, bar.abort_flag);
      return;
    }
    ++g_armed[slot];
    const int i0 = g * GUP_GROUP, i1 = min(nunits, i0 + GUP_GROUP);
    uint32_t total = 0;
    for (int i = i0; i < i1; ++i) total += usize(i);
    mbar_arrive_expect_tx(&bar.rawfull[slot], total);
    uint32_t off = 0;
    for (int i = i0; i < i1;) {
      int j = i + 1;
      uint32_t run = usize(i);
      while (j < i1 && usrc(j) == usrc(j - 1) + usize(j - 1)) run += usize(j++);
      bulk_copy(rbase + slot * (GUP_GROUP * PG_HOT) + off, usrc(i), run, &bar.rawfull[slot]);
      off += run;
      i = j;
    }
  };

  // full: the 8 warps of the unit's decoder group; rawempty: those 8 warps for each of a group's units
  // empty / accf: one commit from each of the two MMA issuers (a tcgen05.commit costs about as much as an MMA)
  if (t == 0) init_bars(bar, GU_STAGES, GUP_DEC_WARPS, 1, 1, GUP_DEC_WARPS * GUP_GROUP, 2);
  if (warp == 0) tmem_alloc(bar.tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tslot;

  if (t < GU_PROD) {
    // Two decoder groups of 8 warps take alternate units, so that one unit's
    // latency chain (waits, shared loads, decode, TMEM store, signal) overlaps
    // the other's.  Warp (q, m) of a group decodes rows 32 q .. 32 q + 31 (its
    // TMEM lane quarter) of matrix m over the unit's whole 64-wide K step.
    const int q = warp & 3, m = (warp >> 2) & 1, gd = warp >> 3;
    const int r = q * 32 + lane;
    const uint32_t a_lane = tmem + ((uint32_t)(q * 32) << 16) + GU_A_COL + 32 * m;
    for (int i = gd; i < nunits; i += 2) {
      const int g = i / GUP_GROUP;
      const int x = lo + i, T = x >> 6;
      const int slot = g % GUP_GSLOTS, s = i % GU_STAGES, round = i / GU_STAGES;
      bool ok = bwait(&bar.rawfull[slot], (g / GUP_GSLOTS) & 1);
      ok = ok && (round == 0 || bwait(&bar.empty[s], (round - 1) & 1));
      if (!ok) fail(a, bar.abort_flag);
      if (!__all_sync(0xffffffffu, ok) || __any_sync(0xffffffffu, *bar.abort_flag != 0)) break;
      tc_fence_after();
      uint32_t uoff = 0;
      for (int i2 = g * GUP_GROUP; i2 < i; ++i2) uoff += usize(i2);
      const uint32_t blk = rbase + slot * (GUP_GROUP * PG_HOT) + uoff;
      uint32_t v0[16], v1[16];
      if (T < L.hot_tiles) {
        const uint32_t row = blk + m * (TILE * KC) + r * KC;
        const int sw = (r >> 1) & 3;
        const uint4 w0 = lds128(row + ((0 ^ sw) << 4)), w1 = lds128(row + ((1 ^ sw) << 4));
        const uint4 w2 = lds128(row + ((2 ^ sw) << 4)), w3 = lds128(row + ((3 ^ sw) << 4));
        const uint4 p0 = fp8_piece_nat(w0.x, w0.y), p1 = fp8_piece_nat(w0.z, w0.w);
        const uint4 p2 = fp8_piece_nat(w1.x, w1.y), p3 = fp8_piece_nat(w1.z, w1.w);
        v0[0] = p0.x; v0[1] = p0.y; v0[2] = p0.z; v0[3] = p0.w; v0[4] = p1.x; v0[5] = p1.y; v0[6] = p1.z; v0[7] = p1.w;
        v0[8] = p2.x; v0[9] = p2.y; v0[10] = p2.z; v0[11] = p2.w; v0[12] = p3.x; v0[13] = p3.y; v0[14] = p3.z; v0[15] = p3.w;
        const uint4 p4 = fp8_piece_nat(w2.x, w2.y), p5 = fp8_piece_nat(w2.z, w2.w);
        const uint4 p6 = fp8_piece_nat(w3.x, w3.y), p7 = fp8_piece_nat(w3.z, w3.w);
        v1[0] = p4.x; v1[1] = p4.y; v1[2] = p4.z; v1[3] = p4.w; v1[4] = p5.x; v1[5] = p5.y; v1[6] = p5.z; v1[7] = p5.w;
        v1[8] = p6.x; v1[9] = p6.y; v1[10] = p6.z; v1[11] = p6.w; v1[12] = p7.x; v1[13] = p7.y; v1[14] = p7.z; v1[15] = p7.w;
      } else {
        const uint32_t rowc = blk + m * (TILE * 32) + r * 32;
        const int sw = (r >> 2) & 1;
        const uint4 w0 = lds128(rowc + ((0 ^ sw) << 4)), w1 = lds128(rowc + ((1 ^ sw) << 4));
        const uint32_t scw = lds32(blk + 2 * TILE * 32 + ((m * TILE + r) * 2 & ~3));
        const __half sc = half_of(scw, r & 1);
        const uint4 p0 = scale_piece(int4_piece_perm(w0.x), sc), p1 = scale_piece(int4_piece_perm(w0.y), sc);
        const uint4 p2 = scale_piece(int4_piece_perm(w0.z), sc), p3 = scale_piece(int4_piece_perm(w0.w), sc);
        v0[0] = p0.x; v0[1] = p0.y; v0[2] = p0.z; v0[3] = p0.w; v0[4] = p1.x; v0[5] = p1.y; v0[6] = p1.z; v0[7] = p1.w;
        v0[8] = p2.x; v0[9] = p2.y; v0[10] = p2.z; v0[11] = p2.w; v0[12] = p3.x; v0[13] = p3.y; v0[14] = p3.z; v0[15] = p3.w;
        const uint4 p4 = scale_piece(int4_piece_perm(w1.x), sc), p5 = scale_piece(int4_piece_perm(w1.y), sc);
        const uint4 p6 = scale_piece(int4_piece_perm(w1.z), sc), p7 = scale_piece(int4_piece_perm(w1.w), sc);
        v1[0] = p4.x; v1[1] = p4.y; v1[2] = p4.z; v1[3] = p4.w; v1[4] = p5.x; v1[5] = p5.y; v1[6] = p5.z; v1[7] = p5.w;
        v1[8] = p6.x; v1[9] = p6.y; v1[10] = p6.z; v1[11] = p6.w; v1[12] = p7.x; v1[13] = p7.y; v1[14] = p7.z; v1[15] = p7.w;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.rawempty[slot]);      // this warp's reads of the unit are done
      tmem_st16_nowait(a_lane + 64 * s, v0);                 // K [0, 32) of the step
      tmem_st16_nowait(a_lane + 64 * s + 16, v1);            // K [32, 64)
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.full[s]);
    }
  } else if (t == GU_PROD || t == GU_PROD + 224) {
    // MMA issuers: warp 16 the gate accumulator, warp 23 the up accumulator (one
    // tcgen05.mma takes ~135 cycles to issue, so two threads double the rate)
    const int mu = t == GU_PROD ? 0 : 1;
    const uint32_t idesc = idesc_f16(N, 0, 0);
    int seg = 0;
    for (int i = 0; i < nunits; ++i) {
      const int kb = (lo + i) & (H / KC - 1);
      const bool first = i == 0 || kb == 0, last = i == nunits - 1 || kb == H / KC - 1;
      const int tb = seg & 1;
      if (first && seg >= 2 && !bwait(&bar.tfree[tb], ((seg >> 1) - 1) & 1)) fail(a, bar.abort_flag);
      const int s = i % GU_STAGES, round = i / GU_STAGES;
      if (!bwait(&bar.full[s], round & 1)) fail(a, bar.abort_flag);
      if (!bwait(&bar.xfull[s], round & 1)) fail(a, bar.abort_flag);
      if (*bar.abort_flag) break;
      tc_fence_after();
      const uint32_t X = xbase + s * x_bytes;
      const uint32_t dt = tmem + tb * 2 * N + mu * N;
      const uint32_t at = tmem + GU_A_COL + 64 * s + 32 * mu;
#pragma unroll
      for (int j = 0; j < KC / 16; ++j)
        umma_f16_ts(dt, at + 8 * j, sdesc(X + j * 2 * 16 * N, 16 * N, 128), idesc, !(first && j == 0));
      umma_commit(&bar.empty[s]);                          // frees A stage s and token tile s
      if (last) {
        umma_commit(&bar.accf[tb]);
        ++seg;
      }
    }
    drain_mma(&bar.mdrain[mu], a);
  } else if (t == GU_PROD + 192) {
    for (int g = 0; g < ngroups && !*bar.abort_flag; ++g) issue(g);
    drain_slots(bar.rawfull, g_armed, a);
  } else if (t == GU_PROD + 32) {
    // token tiles: tile s belongs to A stage s and is freed by the same commits
    pdl_wait();                                 // the tiles are k_norm's output
    int x_armed[GU_STAGES] = {};
    for (int i = 0; i < nunits; ++i) {
      const int x = lo + i, T = x >> 6, kb = x & (H / KC - 1);
      const int s = i % GU_STAGES, round = i / GU_STAGES;
      if (round > 0 && !bwait(&bar.empty[s], (round - 1) & 1)) fail(a, bar.abort_flag);
      if (*bar.abort_flag) break;
      mbar_arrive_expect_tx(&bar.xfull[s], x_bytes);
      bulk_copy(xbase + s * x_bytes, (T < L.hot_tiles ? p.xs_nat : p.xs_perm) + (size_t)kb * x_bytes, x_bytes,
                &bar.xfull[s]);
      ++x_armed[s];
    }
    drain_slots(bar.xfull, x_armed, a);
  } else if (t >= GU_PROD + 64 && t < GU_PROD + 192) {                 // epilogue warps 18-21
    const int q = warp & 3, r = q * 32 + lane;
    int seg = 0;
    for (int x0 = lo; x0 < hi; ++seg) {
      const int T = x0 >> 6;
      const int x1 = min(hi, (T + 1) * (H / KC));
      const int tb = seg & 1;
      const bool done = bwait(&bar.accf[tb], (seg >> 1) & 1);
      if (!done) fail(a, bar.abort_flag);
      const bool go = __all_sync(0xffffffffu, done) && !__any_sync(0xffffffffu, *bar.abort_flag != 0);
      if (!go) break;
      tc_fence_after();
      float* dst = p.part + ((size_t)(T + c) * TILE + r) * (2 * N);
      for (int col = 0; col < 2 * N; col += 8) {
        float v[8];
        tmem_ld8(tmem + ((uint32_t)(q * 32) << 16) + tb * 2 * N + col, v);
        reinterpret_cast<float4*>(dst + col)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(dst + col)[1] = make_float4(v[4], v[5], v[6], v[7]);
      }
      tc_fence_before();
      mbar_arrive(&bar.tfree[tb]);
      x0 = x1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (t == 0) stamp(tr, c, 56);
  if (warp == 0) {
    tc_fence_after();
    tmem_free(tmem, 512);
  }
}

// act[slot][b] (swizzled 16-byte chunks) for every packed slot; records outside the fetch set -> 0
__global__ void __launch_bounds__(256) k_act_p(LayerArgs a, const float* __restrict__ part, int G, int N,
                                               __half* __restrict__ act) {
  pdl_launch_dependents();
  pdl_wait();                                   // part is k_gu_p's output
  const PackLayout L = pack_layout(a.n_hot, a.n_records);
  const int U = (L.hot_tiles + L.cold_tiles) * (H / KC);
  const int slots = (L.hot_blocks + L.cold_blocks) * KC;
  const int groups = N / 8;
  const int i = blockIdx.x * 256 + threadIdx.x;
  const int slot = i / groups, g = i % groups;
  if (slot >= slots) return;
  const int hot_slots = L.hot_tiles * TILE;
  bool live;
  float sg = 1.0f, su = 1.0f, sd = 1.0f;
  if (slot < hot_slots) {
    live = slot < a.n_hot;
    if (live && a.hot_scale) {
      sg = __ldg(a.hot_scale + (size_t)slot * 3);
      su = __ldg(a.hot_scale + (size_t)slot * 3 + 1);
      sd = __ldg(a.hot_scale + (size_t)slot * 3 + 2);
    }
  } else {
    const int j = slot - hot_slots;
    live = j < a.n_records && __ldg(a.flags + j);
  }
  __half o[8];
  if (live) {
    const int T = slot / TILE, r = slot % TILE;
    const int c0 = unit_owner(T * (H / KC), U, G), c1 = unit_owner(T * (H / KC) + H / KC - 1, U, G);
    float gs[8], us[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) gs[e] = us[e] = 0.0f;
    for (int cc = c0; cc <= c1; ++cc) {
      const float* row = part + ((size_t)(T + cc) * TILE + r) * (2 * N) + g * 8;
      const float4 g0 = reinterpret_cast<const float4*>(row)[0], g1 = reinterpret_cast<const float4*>(row)[1];
      const float4 u0 = reinterpret_cast<const float4*>(row + N)[0], u1 = reinterpret_cast<const float4*>(row + N)[1];
      gs[0] += g0.x; gs[1] += g0.y; gs[2] += g0.z; gs[3] += g0.w; gs[4] += g1.x; gs[5] += g1.y; gs[6] += g1.z; gs[7] += g1.w;
      us[0] += u0.x; us[1] += u0.y; us[2] += u0.z; us[3] += u0.w; us[4] += u1.x; us[5] += u1.y; us[6] += u1.z; us[7] += u1.w;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(gated(gs[e] * sg, us[e] * su, a.relu, a.both) * sd);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __float2half_rn(0.0f);
  }
  *reinterpret_cast<uint4*>(act + (size_t)slot * N + ((g ^ act_swz(slot, N)) * 8)) = *reinterpret_cast<const uint4*>(o);
}

// ---------------------------------------------------------------------------
// k_down_p: k_down over the packed blocks.  Unit x = (output tile x / nblk,
// 64-slot block x % nblk).  Lane 0 of warp 22 bulk-copies each unit's
// weight block into a DD_DEPTH ring and its 64 activation rows into a DD_ACTS
// ring, the weights DD_DEPTH - DD_ACTS units further ahead; two producer
// groups of 8 warps build the f16 A / B stages (DD_STAGES) of alternate units;
// two threads issue the MMAs (even / odd 16-neuron steps into two accumulator
// chains), and 4 epilogue warps add each finished tile into the residual
// rows x_b with float reductions.
// ---------------------------------------------------------------------------

__global__ void __launch_bounds__(DNP_THREADS, 1) k_down_p(const __grid_constant__ PackedParams p, const __half* act,
                                                          float* x, int nb, uint32_t tmem_cols) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const LayerArgs& a = p.a;
  const PackLayout L = pack_layout(a.n_hot, a.n_records);
  const int N = p.N, G = gridDim.x, c = blockIdx.x;
  const int nblk = L.hot_blocks + L.cold_blocks;
  const int U = (H / TILE) * nblk;
  const int lo = range_lo(c, U, G), hi = range_lo(c + 1, U, G);
  if (lo >= hi) return;
  pdl_launch_dependents();
  const int nunits = hi - lo;

  const int b_bytes = KC * N * 2;
  const int stage_bytes = A_TILE_BYTES + b_bytes;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t wbase = sbase;                             // [DD_DEPTH][PD_HOT] weight blocks
  const uint32_t abase = wbase + DD_DEPTH * PD_HOT;         // [DD_ACTS][KC * 2 NMAX] activation blocks
  const uint32_t stbase = abase + DD_ACTS * KC * NMAX * 2;  // [DD_STAGES][stage_bytes]
  const Bars bar = carve_bars(smem + DD_DEPTH * PD_HOT + DD_ACTS * KC * NMAX * 2 + DD_STAGES * stage_bytes);

  // full / rawempty / xempty: the 8 warps of the unit's producer group; empty / accf: both MMA issuers
  if (t == 0) init_bars(bar, DD_STAGES, DN_PROD / 32, 1, DN_PROD / 32, DN_PROD / 32, 2);
  if (warp == 0) tmem_alloc(bar.tslot, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tslot;

  // issuer (warp 22): weight blocks (from DRAM) and activation blocks (from L2)
  int w_armed[DD_DEPTH] = {}, a_armed[DD_ACTS] = {};       // issuer: copies per weight / activation slot
  auto issue_w = [&](int i) {
    if (i >= nunits || *bar.abort_flag) return;
    const int x = lo + i, et = x / nblk, nb = x % nblk;
    const int slot = i % DD_DEPTH, use = i / DD_DEPTH;
    // if the slot is not released in time, nothing more is copied into it (it may still be read)
    if (use > 0 && !bwait(&bar.rawempty[slot], (use - 1) & 1)) {
      fail(a, bar.abort_flag);
      return;
    }
    ++w_armed[slot];
    const bool hotB = nb < L.hot_blocks;
    const uint8_t* src = p.packed + (hotB ? L.dn_hot + ((size_t)et * L.hot_blocks + nb) * PD_HOT
                                          : L.dn_cold + ((size_t)et * L.cold_blocks + (nb - L.hot_blocks)) * PD_COLD);
    const uint32_t wbytes = hotB ? PD_HOT : PD_COLD;
    mbar_arrive_expect_tx(&bar.rawfull[slot], wbytes);
    bulk_copy(wbase + slot * PD_HOT, src, wbytes, &bar.rawfull[slot]);
  };
  auto issue_a = [&](int i) {
    if (i >= nunits || *bar.abort_flag) return;
    if (i == 0) pdl_wait();                     // the activation rows are k_act_p's output
    const int nb = (lo + i) % nblk;
    const int slot = i % DD_ACTS, use = i / DD_ACTS;
    if (use > 0 && !bwait(&bar.xempty[slot], (use - 1) & 1)) {
      fail(a, bar.abort_flag);
      return;
    }
    ++a_armed[slot];
    mbar_arrive_expect_tx(&bar.xfull[slot], b_bytes);
    bulk_copy(abase + slot * (KC * NMAX * 2), act + (size_t)nb * KC * N, b_bytes, &bar.xfull[slot]);
  };
  if (t < DNP_PROD) {
    // two producer groups of 8 warps take alternate units; in a group, thread
    // (q, j) builds neuron q, output rows [32 j, 32 j + 32) (a quarter-warp
    // holds 8 neurons of one j: conflict-free stage stores)
    const int gd = warp >> 3;
    const int q = ((warp & 7) << 3) | (lane & 7), j = lane >> 3;
    const int groups = N / 8;
    for (int i = gd; i < nunits; i += 2) {
      const int x = lo + i, et = x / nblk, nb = x % nblk;
      const int rs = i % DD_DEPTH, as = i % DD_ACTS, s = i % DD_STAGES, round = i / DD_STAGES;
      bool ok = bwait(&bar.rawfull[rs], (i / DD_DEPTH) & 1) && bwait(&bar.xfull[as], (i / DD_ACTS) & 1);
      ok = ok && (round == 0 || bwait(&bar.empty[s], (round - 1) & 1));
      if (!ok) fail(a, bar.abort_flag);
      if (!__all_sync(0xffffffffu, ok) || __any_sync(0xffffffffu, *bar.abort_flag != 0)) break;
      const uint32_t raw = wbase + rs * PD_HOT;
      const uint32_t actb = abase + as * (KC * NMAX * 2);
      const uint32_t A = stbase + s * stage_bytes + (q >> 3) * 2048 + (4 * j) * 128 + (q & 7) * 16;
      const uint32_t B = stbase + s * stage_bytes + A_TILE_BYTES + (q >> 3) * 16 * N + (q & 7) * 16;
      const int slot_q = nb * KC + q;
      const int asw = act_swz(slot_q, N);
      if (nb < L.hot_blocks) {
        const uint32_t row = raw + q * TILE;
        const uint4 w0 = lds128(row + (((2 * j) ^ (q & 7)) << 4));
        const uint4 w1 = lds128(row + (((2 * j + 1) ^ (q & 7)) << 4));
        sts128(A + 0 * 128, fp8_piece_perm(w0.x, w0.y));
        sts128(A + 1 * 128, fp8_piece_perm(w0.z, w0.w));
        sts128(A + 2 * 128, fp8_piece_perm(w1.x, w1.y));
        sts128(A + 3 * 128, fp8_piece_perm(w1.z, w1.w));
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int g = j + 4 * hh;
          if (g < groups) sts128(B + g * 128, lds128(actb + q * N * 2 + ((g ^ asw) << 4)));
        }
      } else {
        const uint4 w = lds128(raw + q * 64 + 16 * (j ^ ((q >> 1) & 3)));
        const __half ds = half_of(lds32(raw + KC * 64 + ((q * 2) & ~3)), q & 1);
        sts128(A + 0 * 128, int4_piece_perm(w.x));
        sts128(A + 1 * 128, int4_piece_perm(w.y));
        sts128(A + 2 * 128, int4_piece_perm(w.z));
        sts128(A + 3 * 128, int4_piece_perm(w.w));
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int g = j + 4 * hh;
          if (g < groups) sts128(B + g * 128, scale_piece(lds128(actb + q * N * 2 + ((g ^ asw) << 4)), ds));
        }
      }
      (void)et;
      fence_async_smem();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&bar.rawempty[rs]);
        mbar_arrive(&bar.xempty[as]);
        mbar_arrive(&bar.full[s]);
      }
    }
  } else if (t == DNP_PROD + 192) {
    // weights run DD_DEPTH - DD_ACTS units further ahead than the activation blocks
    for (int i = 0; i < nunits && !*bar.abort_flag; ++i) {
      issue_w(i);
      if (i >= DD_DEPTH - DD_ACTS) issue_a(i - (DD_DEPTH - DD_ACTS));
    }
    for (int i = max(0, nunits - (DD_DEPTH - DD_ACTS)); i < nunits && !*bar.abort_flag; ++i) issue_a(i);
    drain_slots(bar.rawfull, w_armed, a);
    drain_slots(bar.xfull, a_armed, a);
  } else if (t == DNP_PROD || t == DNP_PROD + 32) {
    // two MMA issuers (warps 16, 17): chain ch accumulates the unit's 16-neuron
    // steps ch and ch + 2 into its own TMEM columns; the epilogue adds the chains
    const int ch = t == DNP_PROD ? 0 : 1;
    const uint32_t idesc = idesc_f16(N, 1, 1);
    int seg = 0;
    for (int i = 0; i < nunits; ++i) {
      const int nb = (lo + i) % nblk;
      const bool first = i == 0 || nb == 0, last = i == nunits - 1 || nb == nblk - 1;
      const int tb = seg & 1;
      if (first && seg >= 2 && !bwait(&bar.tfree[tb], ((seg >> 1) - 1) & 1)) fail(a, bar.abort_flag);
      const int s = i % DD_STAGES, round = i / DD_STAGES;
      if (!bwait(&bar.full[s], round & 1)) fail(a, bar.abort_flag);
      if (*bar.abort_flag) break;
      tc_fence_after();
      const uint32_t st = stbase + s * stage_bytes;
      const uint32_t dt = tmem + (2 * tb + ch) * N;
#pragma unroll
      for (int kk = 0; kk < 2; ++kk) {
        const int k = ch + 2 * kk;
        umma_f16(dt, sdesc(st + k * 2 * 2048, 2048, 128), sdesc(st + A_TILE_BYTES + k * 2 * 16 * N, 16 * N, 128),
                 idesc, !(first && kk == 0));
      }
      umma_commit(&bar.empty[s]);
      if (last) {
        umma_commit(&bar.accf[tb]);
        ++seg;
      }
    }
    drain_mma(&bar.mdrain[ch], a);
  } else if (t >= DNP_PROD + 64 && t < DNP_PROD + 192) {              // epilogue warps 18-21
    const int qd = warp & 3, m = qd * 32 + lane;
    int seg = 0;
    for (int x0 = lo; x0 < hi; ++seg) {
      const int et = x0 / nblk;
      const int x1 = min(hi, (et + 1) * nblk);
      const int tb = seg & 1;
      const bool done = bwait(&bar.accf[tb], (seg >> 1) & 1);
      if (!done) fail(a, bar.abort_flag);
      const bool go = __all_sync(0xffffffffu, done) && !__any_sync(0xffffffffu, *bar.abort_flag != 0);
      if (!go) break;
      tc_fence_after();
      const int e = et * TILE + (m & ~7) + perm8(m & 7);
      for (int col = 0; col < N; col += 8) {
        float v[8], v1[8];
        tmem_ld8(tmem + ((uint32_t)(qd * 32) << 16) + 2 * tb * N + col, v);
        tmem_ld8(tmem + ((uint32_t)(qd * 32) << 16) + (2 * tb + 1) * N + col, v1);
#pragma unroll
        for (int u = 0; u < 8; ++u) v[u] += v1[u];
        add_to_rows(x + e, col, nb, v);
      }
      tc_fence_before();
      mbar_arrive(&bar.tfree[tb]);
      x0 = x1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_free(tmem, tmem_cols);
  }
}

// ---------------------------------------------------------------------------
// Union of B tokens' mask words & fetch bits -> ascending record list.
// ---------------------------------------------------------------------------
// blockIdx.x = layer: masks + layer * layer_stride, fetch + layer * words,
// table + layer * 65536, rec_out + layer * rec_stride, count + layer.
__global__ void __launch_bounds__(1024) k_union(const uint32_t* __restrict__ masks, int64_t layer_stride, int batch,
                                                int64_t token_stride, int words, const uint32_t* __restrict__ fetch,
                                                const int32_t* __restrict__ table, int32_t* __restrict__ rec_out,
                                                int64_t rec_stride, int32_t* __restrict__ count,
                                                uint8_t* __restrict__ flags, int64_t flag_stride) {
  __shared__ int warp_tot[32];
  __shared__ int base_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int layer = blockIdx.x;
  masks += (size_t)layer * layer_stride;
  fetch += (size_t)layer * words;
  table += (size_t)layer * TABLE_SIZE;
  rec_out += (size_t)layer * rec_stride;
  if (flags) {
    flags += (size_t)layer * flag_stride;
    for (int64_t i = tid; i < flag_stride; i += 1024) flags[i] = 0;
  }
  if (tid == 0) base_s = 0;
  __syncthreads();
  for (int w0 = 0; w0 < words; w0 += 1024) {
    const int w = w0 + tid;
    uint32_t m = 0;
    if (w < words) {
      // 16 independent loads in flight per round
      int b = 0;
      for (; b + 16 <= batch; b += 16) {
        uint32_t v[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = __ldg(masks + (size_t)(b + k) * token_stride + w);
#pragma unroll
        for (int k = 0; k < 16; ++k) m |= v[k];
      }
      for (; b < batch; ++b) m |= __ldg(masks + (size_t)b * token_stride + w);
      m &= __ldg(fetch + w);
    }
    const int mine = __popc(m);
    int incl = mine;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int v = warp_tot[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      warp_tot[lane] = v;
    }
    __syncthreads();
    int pos = base_s + (warp ? warp_tot[warp - 1] : 0) + incl - mine;
    while (m) {
      const int bit = __ffs(m) - 1;
      m &= m - 1;
      const int r = __ldg(table + w * 32 + bit);
      rec_out[pos++] = r;
      if (flags && r >= 0 && r < flag_stride) flags[r] = 1;
    }
    __syncthreads();
    if (tid == 0) base_s += warp_tot[31];
    __syncthreads();
  }
  if (tid == 0) count[layer] = base_s;
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct WsLayout {
  size_t xs_nat, xs_perm, act, part, total;
};
static size_t align_up(size_t v, size_t al) { return (v + al - 1) / al * al; }
static WsLayout ws_layout(int64_t max_neurons) {
  WsLayout w;
  size_t o = 0;
  const size_t xs = (size_t)NMAX * H * 2;
  const size_t blocks = (size_t)(max_neurons + TILE - 1) / TILE + 1 + MAX_CTAS;
  w.xs_nat = o; o = align_up(o + xs, 1024);
  w.xs_perm = o; o = align_up(o + xs, 1024);
  w.act = o; o = align_up(o + (size_t)max_neurons * NMAX * 2, 1024);
  w.part = o; o = align_up(o + blocks * TILE * 2 * NMAX * 4, 1024);
  w.total = o;
  return w;
}
static uint32_t tmem_cols_for(int n) {
  uint32_t c = 32;
  while (c < (uint32_t)n) c <<= 1;
  return c;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}
// rows of `row_bytes` bytes, one after another from `base` (16-byte aligned), read in boxes of box_x bytes x box_y rows
static bool encode_rows(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows, uint32_t box_x,
                        uint32_t box_y, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_NONE) {
  PFN_cuTensorMapEncodeTiled_v12000 fn = tmap_encoder();
  if (!fn || rows == 0) return false;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_x, box_y};
  cuuint32_t es[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static uint64_t* g_trace_gu = nullptr;
static uint64_t* g_trace_down = nullptr;

}  // namespace hcb

using namespace hcb;

// launch with programmatic stream serialisation (see pdl_wait)
template <typename... P, typename... A>
static cudaError_t launch_pdl(void (*kernel)(P...), int grid, int block, size_t smem, cudaStream_t s, A&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<A>(args)...);
}

extern "C" int hc_batch_set_trace(uint64_t* gu, uint64_t* down) {
  g_trace_gu = gu;
  g_trace_down = down;
  return HC_OK;
}

extern "C" int64_t hc_ffn_batch_workspace_bytes(int32_t max_neurons) {
  if (max_neurons <= 0) return -1;
  return (int64_t)ws_layout((int64_t)max_neurons + 2 * TILE).total;   // + the packed mode's slot padding
}

extern "C" int64_t hc_batch_pack_bytes(int32_t n_hot, int32_t n_records) {
  if (n_hot < 0 || n_records < 0) return -1;
  return (int64_t)pack_layout(n_hot, n_records).total;
}

extern "C" int hc_batch_pack(const hc_layer_desc* layer, void* packed, hc_stream_t stream) {
  if (!layer || !packed || !layer->hot || (layer->n_records > 0 && !layer->cold_records) || layer->n_hot < 0 ||
      (reinterpret_cast<uintptr_t>(packed) & 15) || (reinterpret_cast<uintptr_t>(layer->hot) & 15))
    return HC_ERR_ARG;
  k_pack<<<1184, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      layer->hot, layer->n_hot, layer->cold_records, layer->n_records, static_cast<uint8_t*>(packed));
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_union_cold(const uint32_t* masks, int32_t batch, int64_t token_stride, int32_t inter,
                             const uint32_t* fetch_bits, const int32_t* table, int32_t* rec_out, int32_t* count,
                             hc_stream_t stream) {
  return hc_union_cold_layers(masks, 1, 0, batch, token_stride, inter, fetch_bits, table, rec_out, 0, count, nullptr,
                              0, stream);
}

extern "C" int hc_union_cold_layers(const uint32_t* masks, int32_t n_layers, int64_t layer_stride, int32_t batch,
                                    int64_t token_stride, int32_t inter, const uint32_t* fetch_bits,
                                    const int32_t* table, int32_t* rec_out, int64_t rec_stride, int32_t* count,
                                    uint8_t* flags_out, int64_t flag_stride, hc_stream_t stream) {
  if (!masks || !fetch_bits || !table || !rec_out || !count || n_layers <= 0 || batch <= 0 || inter <= 0 ||
      inter > 65536 || (n_layers > 1 && rec_stride <= 0) || (flags_out && flag_stride <= 0))
    return HC_ERR_ARG;
  k_union<<<n_layers, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      masks, layer_stride, batch, token_stride, (inter + 31) / 32, fetch_bits, table, rec_out, rec_stride, count,
      flags_out, flag_stride);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

// y_out == nullptr: x_b += FFN(x_b); else y_out_b += FFN(x_b) and x is only read
static int batch_layer(const hc_layer_desc* layer, const void* packed, float* x, int32_t batch, const int32_t* rec,
                       const int32_t* count, int32_t max_cold, const uint8_t* rec_flags, float eps, int32_t act,
                       int32_t act_on_both, void* workspace, float* y_out, int32_t* status, hc_stream_t stream) {
  if (!layer || !x || batch <= 0 || !rec || !count || max_cold < 0 || !workspace || !status ||
      (act != HC_ACT_SILU && act != HC_ACT_RELU) || (rec_flags && !packed) ||
      (packed && (reinterpret_cast<uintptr_t>(packed) & 15)))
    return HC_ERR_ARG;
  if (rec_flags) max_cold = layer->n_records;        // packed: every record of the section
  if (!layer->hot || !layer->cold_records || layer->n_hot < 0 || max_cold > layer->n_records)
    return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15) ||
      (reinterpret_cast<uintptr_t>(y_out) & 15) ||
      (reinterpret_cast<uintptr_t>(layer->hot) & 15) || (reinterpret_cast<uintptr_t>(layer->cold_records) & 15))
    return HC_ERR_ARG;
  constexpr int GU_RAW = GU_DEPTH * GU_RAW_SLOT;
  constexpr int GU_SMEM = GU_STAGES * NMAX * KC * 2 + GU_RAW + BAR_BYTES;
  constexpr int GU_SMEM_LAUNCH = GU_SMEM > GU_SMEM_FLOOR ? GU_SMEM : GU_SMEM_FLOOR;
  static_assert(GU_SMEM_LAUNCH <= 227 * 1024, "k_gu shared memory");
  constexpr int DN_RAW = RAW_DEPTH * DN_PIECES * DN_PSTRIDE + REC_RING * DN_PROD * 4;
  constexpr int GU_SMEM_MAX = GU_SMEM_LAUNCH;
  constexpr int GUP_SMEM_NEED = GUP_GSLOTS * GUP_GROUP * PG_HOT + GU_STAGES * NMAX * KC * 2 + BAR_BYTES;
  constexpr int GUP_SMEM = GUP_SMEM_NEED > GU_SMEM_FLOOR ? GUP_SMEM_NEED : GU_SMEM_FLOOR;
  constexpr int DDP_SMEM =
      DD_DEPTH * PD_HOT + DD_ACTS * KC * NMAX * 2 + DD_STAGES * (A_TILE_BYTES + KC * NMAX * 2) + BAR_BYTES;
  static_assert(GUP_SMEM <= 227 * 1024 && DDP_SMEM <= 227 * 1024, "packed kernels' shared memory");
  constexpr int DN_SMEM_MAX = 3 * (A_TILE_BYTES + KC * NMAX * 2) + DN_RAW + BAR_BYTES;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(k_gu, cudaFuncAttributeMaxDynamicSharedMemorySize, GU_SMEM_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, DN_SMEM_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_gu_p, cudaFuncAttributeMaxDynamicSharedMemorySize, GUP_SMEM) != cudaSuccess ||
        cudaFuncSetAttribute(k_down_p, cudaFuncAttributeMaxDynamicSharedMemorySize, DDP_SMEM) != cudaSuccess)
      return HC_ERR_CUDA;
    attr = true;
  }
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return HC_ERR_CUDA;
  const int ctas = sms < MAX_CTAS ? sms : MAX_CTAS;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int max_total = layer->n_hot + max_cold;
  const WsLayout wl = ws_layout((int64_t)max_total + 2 * TILE);
  uint8_t* ws = static_cast<uint8_t*>(workspace);

  LayerArgs la;
  la.hot = layer->hot;
  la.hot_scale = layer->hot_scale;
  la.n_hot = layer->n_hot;
  la.cold = layer->cold_records;
  la.n_records = layer->n_records;
  la.rec = rec;
  la.count = count;
  la.max_cold = max_cold;
  la.relu = act == HC_ACT_RELU;
  la.both = act_on_both != 0;
  la.status = status;
  la.flags = rec_flags;

  const int hot_tiles = (layer->n_hot + TILE - 1) / TILE;
  const int tiles_max = hot_tiles + (max_cold + TILE - 1) / TILE;
  for (int b0 = 0; b0 < batch; b0 += NMAX) {
    const int nb = batch - b0 < NMAX ? batch - b0 : NMAX;
    const int N = (nb + 15) / 16 * 16;
    float* xb = x + (size_t)b0 * H;
    float* ob = (y_out ? y_out : x) + (size_t)b0 * H;      // where the down tiles are added
    if (rec_flags && max_total > 0) {
      // packed mode: the four kernels overlap each one's set-up with its predecessor's tail
      if (launch_pdl(k_norm, N, 256, 0, s, (const float*)xb, nb, N, layer->norm_w, eps, ws + wl.xs_nat,
                     ws + wl.xs_perm) != cudaSuccess)
        return HC_ERR_CUDA;
      const PackLayout L = pack_layout(layer->n_hot, layer->n_records);
      PackedParams pp;
      memset(&pp, 0, sizeof(pp));
      pp.a = la;
      pp.packed = static_cast<const uint8_t*>(packed);
      pp.xs_nat = ws + wl.xs_nat;
      pp.xs_perm = ws + wl.xs_perm;
      pp.part = reinterpret_cast<float*>(ws + wl.part);
      pp.N = N;
      pp.trace = g_trace_gu;
      const int gu_units = (L.hot_tiles + L.cold_tiles) * (H / KC);
      const int gu_grid = gu_units < ctas ? gu_units : ctas;
      if (launch_pdl(k_gu_p, gu_grid, GUP_THREADS, GUP_SMEM, s, pp) != cudaSuccess) return HC_ERR_CUDA;
      const int slots = (L.hot_blocks + L.cold_blocks) * KC;
      __half* actb = reinterpret_cast<__half*>(ws + wl.act);
      if (launch_pdl(k_act_p, (slots * (N / 8) + 255) / 256, 256, 0, s, la, (const float*)pp.part, gu_grid, N,
                     actb) != cudaSuccess)
        return HC_ERR_CUDA;
      const int dn_units = (H / TILE) * (L.hot_blocks + L.cold_blocks);
      const int dn_grid = dn_units < ctas ? dn_units : ctas;
      if (launch_pdl(k_down_p, dn_grid, DNP_THREADS, DDP_SMEM, s, pp, (const __half*)actb, ob, nb,
                     tmem_cols_for(4 * N)) != cudaSuccess)
        return HC_ERR_CUDA;
    } else if (max_total > 0) {
      k_norm<<<N, 256, 0, s>>>(xb, nb, N, layer->norm_w, eps, ws + wl.xs_nat, ws + wl.xs_perm);
      GuParams g;
      memset(&g, 0, sizeof(g));
      g.a = la;
      g.xs_nat = ws + wl.xs_nat;
      g.xs_perm = ws + wl.xs_perm;
      g.part = reinterpret_cast<float*>(ws + wl.part);
      g.N = N;
      g.hot_tiles = hot_tiles;
      g.trace = g_trace_gu;
      if (layer->n_hot > 0 && !encode_rows(&g.tm_hot, layer->hot, HOT_ROW, layer->n_hot, KC, TILE))
        return HC_ERR_CUDA;
      const int gu_grid = tiles_max * (H / KC) < ctas ? tiles_max * (H / KC) : ctas;
      k_gu<<<gu_grid, GU_THREADS, GU_SMEM_LAUNCH, s>>>(g);

      const int act_threads = max_total * (N / 8);
      k_act<<<(act_threads + 255) / 256, 256, 0, s>>>(la, g.part, hot_tiles, gu_grid, N,
                                                       reinterpret_cast<__half*>(ws + wl.act));

      DownParams d;
      d.a = la;
      d.act = reinterpret_cast<const __half*>(ws + wl.act);
      d.x = ob;
      d.nb = nb;
      d.N = N;
      d.stages = 3;
      d.tmem_cols = tmem_cols_for(2 * N);
      d.trace = g_trace_down;
      const int dn_units = (H / TILE) * ((max_total + KC - 1) / KC);
      const int dn_grid = dn_units < ctas ? dn_units : ctas;
      const int dn_smem = d.stages * (A_TILE_BYTES + KC * N * 2) + DN_RAW + BAR_BYTES;
      k_down<<<dn_grid, DN_THREADS, dn_smem, s>>>(d);

    }
  }
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_ffn_batch_layer(const hc_layer_desc* layer, const void* packed, float* x, int32_t batch,
                                  const int32_t* rec, const int32_t* count, int32_t max_cold,
                                  const uint8_t* rec_flags, float eps, int32_t act, int32_t act_on_both,
                                  void* workspace, int32_t* status, hc_stream_t stream) {
  return batch_layer(layer, packed, x, batch, rec, count, max_cold, rec_flags, eps, act, act_on_both, workspace,
                     nullptr, status, stream);
}

extern "C" int hc_ffn_batch_layer_partial(const hc_layer_desc* layer, const void* packed, const float* x,
                                          int32_t batch, const int32_t* rec, const int32_t* count, int32_t max_cold,
                                          const uint8_t* rec_flags, float eps, int32_t act, int32_t act_on_both,
                                          void* workspace, float* y_out, int32_t* status, hc_stream_t stream) {
  if (!y_out) return HC_ERR_ARG;
  return batch_layer(layer, packed, const_cast<float*>(x), batch, rec, count, max_cold, rec_flags, eps, act,
                     act_on_both, workspace, y_out, status, stream);
}
