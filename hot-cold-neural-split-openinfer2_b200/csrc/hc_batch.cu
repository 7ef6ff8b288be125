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
//   k_gu       gate and up GEMMs, D[128 neurons][N tokens] per CTA over a
//              K range: 256 producer threads decode FP8 rows (exact in f16)
//              or INT4 rows (q * group scale, rounded once to f16) into
//              K-major shared-memory tiles; one thread issues tcgen05.mma
//              per 16-K step; 8 warps move the accumulators out of TMEM as
//              fp32 partial sums (K split over up to 4 CTAs to fill the GPU)
//   k_act      sum of the K partials, per-neuron FP8 scales, gated
//              activation -> act [slot][N] f16
//   k_down     D[128 output rows][N tokens] per CTA over a neuron range:
//              A = down columns (FP8 exact, INT4 q exact; MN-major tiles),
//              B = act (times the INT4 group scale of the CTA's 128 rows);
//              the tile is added to y [4096][N] with vector float atomics
//   k_resid    x_b += y[:, b]; y = 0
//
// Shared-memory operand layout (SWIZZLE_NONE canonical form): 8x16-byte core
// matrices; SBO = the byte stride between core matrices along M/N, LBO =
// along K.  Every weight byte is read once per pass.
#include "hc_common.cuh"

namespace hcb {
using namespace hc;

constexpr int NMAX = 64;             // tokens per pass
constexpr int TILE = 128;            // MMA M: neurons per gate/up tile, output rows per down tile
constexpr int KC = 64;               // K per pipeline stage
constexpr int HOT_ROW = 3 * H;       // packed hot neuron: gate row | up row | down column (e4m3)
constexpr int A_TILE_BYTES = TILE * KC * 2;    // 16 KB of f16
constexpr uint64_t WAIT_NS = 1000000000ull;

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
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
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
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}"
      ::"r"(d_tmem), "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
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
// global -> shared bulk copy (16-byte aligned, size % 16 == 0) completing on `bar`
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
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
};

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
  float rstd = 0.0f;
  if (b < nb) {
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)b * H);
    float ss = 0.0f;
    for (int i = t; i < H / 4; i += 256) {
      const float4 v = src[i];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((t & 31) == 0) red[t >> 5] = ss;
    __syncthreads();
    ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += red[k];
    rstd = rsqrtf(ss / (float)H + eps);
  }
  for (int piece = t; piece < H / 8; piece += 256) {
    const int k0 = piece * 8;
    float v[8];
    if (b < nb) {
      const float4 a0 = reinterpret_cast<const float4*>(x + (size_t)b * H + k0)[0];
      const float4 a1 = reinterpret_cast<const float4*>(x + (size_t)b * H + k0)[1];
      v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] *= rstd * (w ? __ldg(w + k0 + e) : 1.0f);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.0f;
    }
    __half hn[8], hp[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      hn[p] = __float2half_rn(v[p]);
      hp[p] = __float2half_rn(v[perm8(p)]);
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
constexpr int GU_PROD = 512;                       // k_gu producer threads: (row, matrix, K half)
constexpr int GU_THREADS = GU_PROD + 64 + 128;     // + MMA warp + token-tile warp + 4 epilogue warps
constexpr int GU_STAGES = 4;                       // k_gu: TMEM A stages = token-tile stages
constexpr int GU_A_COL = 256;                      // TMEM columns [256, 512): A stages of 64 columns
constexpr int GU_SMEM_FLOOR = 120 * 1024;          // keeps k_gu at one CTA (all 512 TMEM columns) per SM
constexpr int DN_PROD = 256;                       // k_down producer threads: (neuron, 32-row quarter)
constexpr int DN_THREADS = DN_PROD + 32 + 128;
constexpr int RAW_DEPTH = 4;                       // units of copies in flight per thread
constexpr int GU_PIECES = 2;                       // per thread and unit: 2 weight pieces
constexpr int DN_PIECES = 5;                       // 2 weight, 2 act, 1 scale
constexpr int GU_PSTRIDE = GU_PROD * 16;           // bytes between piece j and j + 1 of one raw slot
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
__device__ __forceinline__ const void* align4(const void* p) {
  return reinterpret_cast<const void*>(reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(3));
}
__device__ __forceinline__ uint32_t upper_half(const void* p) {
  return static_cast<uint32_t>((reinterpret_cast<uintptr_t>(p) >> 1) & 1);
}
__device__ __forceinline__ void fail(const LayerArgs& a, volatile int* abort_flag) {
  atomicOr(a.status, HC_ERR_TIMEOUT);
  *abort_flag = 1;
}

// barriers and TMEM slot after the operand stages and the raw ring
struct Bars {
  uint64_t* full;    // [4] producers -> MMA: stage filled
  uint64_t* empty;   // [4] MMA commit -> producers: stage free
  uint64_t* accf;    // [2] MMA commit -> epilogue: accumulator buffer complete
  uint64_t* tfree;   // [2] epilogue -> MMA: accumulator buffer drained
  uint64_t* xfull;   // [4] bulk copy -> MMA: token tile landed
  uint32_t* tslot;
  volatile int* abort_flag;
};
__device__ __forceinline__ Bars carve_bars(uint8_t* p) {
  Bars b;
  uint64_t* u = reinterpret_cast<uint64_t*>(p);
  b.full = u;
  b.empty = u + 4;
  b.accf = u + 8;
  b.tfree = u + 10;
  b.xfull = u + 12;
  b.tslot = reinterpret_cast<uint32_t*>(u + 16);
  b.abort_flag = reinterpret_cast<volatile int*>(u + 16) + 1;
  return b;
}
__device__ __forceinline__ void init_bars(const Bars& b, int stages, int producers) {
  for (int s = 0; s < stages; ++s) {
    mbar_init(&b.full[s], producers);
    mbar_init(&b.empty[s], 1);
  }
  for (int k = 0; k < 2; ++k) {
    mbar_init(&b.accf[k], 1);
    mbar_init(&b.tfree[k], 128);
  }
  for (int k = 0; k < 4; ++k) mbar_init(&b.xfull[k], 1);
  *b.abort_flag = 0;
  mbar_fence_init();
}
constexpr int BAR_BYTES = 160;

// ---------------------------------------------------------------------------
// k_gu: gate and up GEMMs, D[128 neurons][N tokens], persistent.
//   Tiles: hot tiles first (ceil(n_hot / 128)), then tiles of the union's cold
//   list; unit x = (tile x / 64, K step x % 64).  A CTA's range covers pieces
//   ("segments") of one or more tiles; each segment's fp32 partial goes to
//   block (tile + CTA) of part [blocks][128][2N] (gate N, then up N), unique
//   because ranges are contiguous.
// TMEM (512 columns): accumulator buffers tb = 0, 1 at columns [2N tb, 2N tb
//   + 2N) (gate, up); A stages s = 0..3 at [256 + 64 s, +64) (gate 32
//   columns, up 32 columns; column c of a row holds K elements 2c, 2c + 1).
// Threads: 512 producers -- warp w decodes rows 32 (w & 3) + lane (its TMEM
//   lane quarter) of matrix (w >> 2) & 1, K half w >> 3 of each unit, from a
//   private cp.async ring RAW_DEPTH units deep, and stores the f16 pairs with
//   tcgen05.st; warp 16 issues tcgen05.mma (A from TMEM, B = the token tile
//   from shared memory, K-major: k-group stride 16 N, token-group stride
//   128); warp 17 bulk-copies each unit's token tile; warps 18-21 drain
//   finished accumulator buffers.
// ---------------------------------------------------------------------------
struct GuParams {
  LayerArgs a;
  const uint8_t* xs_nat;
  const uint8_t* xs_perm;
  float* part;
  int N, hot_tiles;
};

__global__ void __launch_bounds__(GU_THREADS, 1) k_gu(GuParams p) {
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

  const int x_bytes = N * KC * 2;
  const int raw_slot = GU_PIECES * GU_PSTRIDE;
  const uint32_t sbase = smem_u32(smem);
  const uint32_t xbase = sbase;                             // [GU_STAGES][x_bytes] token tiles
  const uint32_t rbase = xbase + GU_STAGES * x_bytes;       // [RAW_DEPTH][GU_PIECES][GU_PROD][16]
  const uint32_t scbase = rbase + RAW_DEPTH * raw_slot;     // [RAW_DEPTH][GU_PROD] 4-byte scale words
  const Bars bar = carve_bars(smem + GU_STAGES * x_bytes + RAW_DEPTH * (raw_slot + GU_PROD * 4));

  if (t == 0) init_bars(bar, GU_STAGES, GU_PROD);
  if (warp == 0) tmem_alloc(bar.tslot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tslot;

  if (t < GU_PROD) {
    const int q = warp & 3, m = (warp >> 2) & 1, h = warp >> 3;
    const int r = q * 32 + lane;
    int curT = -1, kindT = 0;
    const uint8_t* src = nullptr;
    const uint8_t* scl = nullptr;
    uint32_t meta = 0;                                      // 3 bits per raw slot: kind (2), scale half (1)
    // record index of this thread's row in cold tile T (raw; checked where used)
    auto raw_rec = [&](int T) -> int {
      if (T < p.hot_tiles || T >= tiles) return -1;
      const int row = (T - p.hot_tiles) * TILE + r;
      return row < cnt ? __ldg(a.rec + row) : -1;
    };
    int nextT = lo >> 6, nextR = raw_rec(nextT);            // the next tile's record, loaded a tile early
    auto issue = [&](int i) {
      if (i < nunits) {
        const int x = lo + i, T = x >> 6, k = x & (H / KC - 1);
        if (T != curT) {
          curT = T;
          const int R = T == nextT ? nextR : raw_rec(T);
          nextT = T + 1;
          nextR = raw_rec(nextT);
          const bool hotT = T < p.hot_tiles;
          const int row = (hotT ? T : T - p.hot_tiles) * TILE + r;
          kindT = 0;
          if (hotT) {
            if (row < a.n_hot) {
              src = a.hot + (size_t)row * HOT_ROW + (size_t)m * H;
              kindT = 1;
            }
          } else if (row < cnt) {
            if (R < 0 || R >= a.n_records) {
              atomicOr(a.status, HC_ERR_RANGE);
            } else {
              const uint8_t* rb = a.cold + (size_t)R * REC_BYTES;
              src = rb + (size_t)m * VEC_BYTES;             // aligned; the field starts at +2
              scl = rb + SCALE_OFF + m * 2 * NGROUPS;
              kindT = 2;
            }
          }
        }
        const int slot = i % RAW_DEPTH;
        const uint32_t d = rbase + slot * raw_slot + t * 16;
        uint32_t md = kindT;
        if (kindT == 1) {
          const uint8_t* w = src + k * KC + 32 * h;
          cp16(d, w);
          cp16(d + GU_PSTRIDE, w + 16);
        } else if (kindT == 2) {
          const uint8_t* w = src + k * (KC / 2) + 16 * h;   // field bytes [32k + 16h, +16) at +2
          cp16(d, w);
          cp4(d + GU_PSTRIDE, w + 16);
          const uint8_t* sp = scl + 2 * (k >> 1);           // group of 128 = two K steps
          cp4(scbase + (slot * GU_PROD + t) * 4, align4(sp));
          md |= upper_half(sp) << 2;
        }
        meta = (meta & ~(7u << (3 * slot))) | (md << (3 * slot));
      }
      cp_commit();
    };
#pragma unroll
    for (int i = 0; i < RAW_DEPTH - 1; ++i) issue(i);
    const uint32_t a_lane = tmem + ((uint32_t)(q * 32) << 16) + GU_A_COL + 32 * m + 16 * h;
    for (int i = 0; i < nunits; ++i) {
      issue(i + RAW_DEPTH - 1);
      cp_wait<RAW_DEPTH - 1>();                             // this thread's copies of unit i landed
      const int s = i % GU_STAGES, round = i / GU_STAGES;
      bool ok = round == 0 || mbar_wait(&bar.empty[s], (round - 1) & 1, WAIT_NS);
      if (!ok) fail(a, bar.abort_flag);
      // tcgen05.st is warp-collective: leave the loop as a whole warp
      if (!__all_sync(0xffffffffu, ok) || __any_sync(0xffffffffu, *bar.abort_flag != 0)) break;
      tc_fence_after();                                     // the MMAs that read stage s are done
      const int slot = i % RAW_DEPTH;
      const uint32_t d = rbase + slot * raw_slot + t * 16;
      const uint32_t md = (meta >> (3 * slot)) & 7u;
      uint32_t v[16];
      if ((md & 3) == 1) {
        const uint4 w0 = lds128(d), w1 = lds128(d + GU_PSTRIDE);
        const uint4 p0 = fp8_piece_nat(w0.x, w0.y), p1 = fp8_piece_nat(w0.z, w0.w);
        const uint4 p2 = fp8_piece_nat(w1.x, w1.y), p3 = fp8_piece_nat(w1.z, w1.w);
        v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w; v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
        v[8] = p2.x; v[9] = p2.y; v[10] = p2.z; v[11] = p2.w; v[12] = p3.x; v[13] = p3.y; v[14] = p3.z; v[15] = p3.w;
      } else if ((md & 3) == 2) {
        const uint4 w0 = lds128(d);
        const uint32_t w4 = lds32(d + GU_PSTRIDE);
        const __half sc = half_of(lds32(scbase + (slot * GU_PROD + t) * 4), md >> 2);
        const uint4 p0 = scale_piece(int4_piece_perm(shift2(w0.x, w0.y)), sc);
        const uint4 p1 = scale_piece(int4_piece_perm(shift2(w0.y, w0.z)), sc);
        const uint4 p2 = scale_piece(int4_piece_perm(shift2(w0.z, w0.w)), sc);
        const uint4 p3 = scale_piece(int4_piece_perm(shift2(w0.w, w4)), sc);
        v[0] = p0.x; v[1] = p0.y; v[2] = p0.z; v[3] = p0.w; v[4] = p1.x; v[5] = p1.y; v[6] = p1.z; v[7] = p1.w;
        v[8] = p2.x; v[9] = p2.y; v[10] = p2.z; v[11] = p2.w; v[12] = p3.x; v[13] = p3.y; v[14] = p3.z; v[15] = p3.w;
      } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) v[k] = 0u;
      }
      tmem_st16(a_lane + 64 * s, v);
      tc_fence_before();
      mbar_arrive(&bar.full[s]);
    }
    cp_wait<0>();
  } else if (t == GU_PROD) {
    // ---- MMA issuer
    const uint32_t idesc = idesc_f16(N, 0, 0);
    int seg = 0;
    for (int i = 0; i < nunits; ++i) {
      const int k = (lo + i) & (H / KC - 1);
      const bool first = i == 0 || k == 0, last = i == nunits - 1 || k == H / KC - 1;
      const int tb = seg & 1;
      if (first && seg >= 2 && !mbar_wait(&bar.tfree[tb], ((seg >> 1) - 1) & 1, WAIT_NS)) fail(a, bar.abort_flag);
      const int s = i % GU_STAGES, round = i / GU_STAGES;
      if (!mbar_wait(&bar.full[s], round & 1, WAIT_NS) || !mbar_wait(&bar.xfull[s], round & 1, WAIT_NS))
        fail(a, bar.abort_flag);
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
  } else if (t == GU_PROD + 32) {
    // ---- token tiles: unit i's K step of the hot or cold operand tile set
    for (int i = 0; i < nunits; ++i) {
      const int x = lo + i, T = x >> 6, k = x & (H / KC - 1);
      const int s = i % GU_STAGES, round = i / GU_STAGES;
      if (round > 0 && !mbar_wait(&bar.empty[s], (round - 1) & 1, WAIT_NS)) fail(a, bar.abort_flag);
      if (*bar.abort_flag) break;
      mbar_arrive_expect_tx(&bar.xfull[s], x_bytes);
      bulk_copy(xbase + s * x_bytes, (T < p.hot_tiles ? p.xs_nat : p.xs_perm) + (size_t)k * x_bytes, x_bytes,
                &bar.xfull[s]);
    }
  } else if (t >= GU_PROD + 64) {
    // ---- epilogue: warp (18..21) & 3 reads TMEM lanes [32 q, 32 q + 32)
    const int q = warp & 3, r = q * 32 + lane;
    int seg = 0;
    for (int x0 = lo; x0 < hi; ++seg) {
      const int T = x0 >> 6;
      const int x1 = min(hi, (T + 1) * (H / KC));
      const int tb = seg & 1;
      const bool done = mbar_wait(&bar.accf[tb], (seg >> 1) & 1, WAIT_NS);
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
// k_down: y[e][b] += sum_n down[n][e] * act[n][b], persistent.
//   Unit x = (output tile x / nsub, neuron step x % nsub), nsub = ceil(slots
//   / 64).  Producer thread (q, j): neuron q of the step, rows [32 j, 32 j +
//   32) of the tile.  Stage: A 128 rows x 64 neurons f16 MN-major (row-group
//   stride 128 B = SBO, neuron-group stride 2048 B = LBO; rows of a 16-byte
//   piece in the order 0,4,1,5,2,6,3,7); B 64 neurons x N tokens MN-major
//   (token-group stride 128 B, neuron-group stride 16 N).  Each segment's
//   tile is added to y [4096][N] with vector float atomics.
// ---------------------------------------------------------------------------
struct DownParams {
  LayerArgs a;
  const __half* act;
  float* y;
  int N, stages;
  uint32_t tmem_cols;
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

  if (t == 0) init_bars(bar, p.stages, DN_PROD);
  if (warp == 0) tmem_alloc(bar.tslot, p.tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *bar.tslot;

  if (t < DN_PROD) {
    const int q = t >> 2, j = t & 3;
    const int groups = N / 8;
    uint32_t meta = 0;                        // 3 bits per raw slot: kind (2), scale half (1)
    // record index of the neuron of unit u, copied REC_AHEAD units before the
    // unit's own copies are issued (range-checked where used)
    auto rec_copy = [&](int u) {
      if (u >= nunits) return;
      const int slot = ((lo + u) % nsub) * KC + q;
      if (slot >= a.n_hot && slot < total) cp4(recbase + ((u % REC_RING) * DN_PROD + t) * 4, a.rec + (slot - a.n_hot));
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
      if (round > 0 && !mbar_wait(&bar.empty[s], (round - 1) & 1, WAIT_NS)) fail(a, bar.abort_flag);
      if (*bar.abort_flag) break;
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
      mbar_arrive(&bar.full[s]);
    }
    cp_wait<0>();
  } else if (t == DN_PROD) {
    const uint32_t idesc = idesc_f16(N, 1, 1);
    int seg = 0;
    for (int i = 0; i < nunits; ++i) {
      const int sub = (lo + i) % nsub;
      const bool first = i == 0 || sub == 0, last = i == nunits - 1 || sub == nsub - 1;
      const int tb = seg & 1;
      if (first && seg >= 2 && !mbar_wait(&bar.tfree[tb], ((seg >> 1) - 1) & 1, WAIT_NS)) fail(a, bar.abort_flag);
      const int s = i % p.stages, round = i / p.stages;
      if (!mbar_wait(&bar.full[s], round & 1, WAIT_NS)) fail(a, bar.abort_flag);
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
  } else if (t >= DN_PROD + 32) {
    const int qd = warp & 3, m = qd * 32 + lane;
    int seg = 0;
    for (int x0 = lo; x0 < hi; ++seg) {
      const int et = x0 / nsub;
      const int x1 = min(hi, (et + 1) * nsub);
      const int tb = seg & 1;
      const bool done = mbar_wait(&bar.accf[tb], (seg >> 1) & 1, WAIT_NS);
      if (!done) fail(a, bar.abort_flag);
      const bool go = __all_sync(0xffffffffu, done) && !__any_sync(0xffffffffu, *bar.abort_flag != 0);
      if (!go) break;
      tc_fence_after();
      const int e = et * TILE + (m & ~7) + perm8(m & 7);
      float* yr = p.y + (size_t)e * N;
      for (int col = 0; col < N; col += 8) {
        float v[8];
        tmem_ld8(tmem + ((uint32_t)(qd * 32) << 16) + tb * N + col, v);
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(yr + col), "f"(v[0]), "f"(v[1]),
                     "f"(v[2]), "f"(v[3])
                     : "memory");
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(yr + col + 4), "f"(v[4]), "f"(v[5]),
                     "f"(v[6]), "f"(v[7])
                     : "memory");
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

// x_b[e] += y[e][b] for b < nb; y is cleared for the next pass
__global__ void __launch_bounds__(256) k_resid(float* __restrict__ x, int nb, int N, float* __restrict__ y) {
  const int e = blockIdx.x * 256 + threadIdx.x, g = blockIdx.y;
  float4* yr = reinterpret_cast<float4*>(y + (size_t)e * N) + g;
  const float4 v = *yr;
  const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (4 * g + k < nb) x[(size_t)(4 * g + k) * H + e] += vv[k];
  *yr = make_float4(0.f, 0.f, 0.f, 0.f);
}

// ---------------------------------------------------------------------------
// Union of B tokens' mask words & fetch bits -> ascending record list.
// ---------------------------------------------------------------------------
// blockIdx.x = layer: masks + layer * layer_stride, fetch + layer * words,
// table + layer * 65536, rec_out + layer * rec_stride, count + layer.
__global__ void __launch_bounds__(1024) k_union(const uint32_t* __restrict__ masks, int64_t layer_stride, int batch,
                                                int64_t token_stride, int words, const uint32_t* __restrict__ fetch,
                                                const int32_t* __restrict__ table, int32_t* __restrict__ rec_out,
                                                int64_t rec_stride, int32_t* __restrict__ count) {
  __shared__ int warp_tot[32];
  __shared__ int base_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int layer = blockIdx.x;
  masks += (size_t)layer * layer_stride;
  fetch += (size_t)layer * words;
  table += (size_t)layer * TABLE_SIZE;
  rec_out += (size_t)layer * rec_stride;
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
      rec_out[pos++] = __ldg(table + w * 32 + bit);
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
  size_t xs_nat, xs_perm, act, part, y, total;
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
  w.y = o; o = align_up(o + (size_t)H * NMAX * 4, 1024);
  w.total = o;
  return w;
}
static uint32_t tmem_cols_for(int n) {
  uint32_t c = 32;
  while (c < (uint32_t)n) c <<= 1;
  return c;
}

}  // namespace hcb

using namespace hcb;

extern "C" int64_t hc_ffn_batch_workspace_bytes(int32_t max_neurons) {
  if (max_neurons <= 0) return -1;
  return (int64_t)ws_layout(max_neurons).total;
}

extern "C" int hc_union_cold(const uint32_t* masks, int32_t batch, int64_t token_stride, int32_t inter,
                             const uint32_t* fetch_bits, const int32_t* table, int32_t* rec_out, int32_t* count,
                             hc_stream_t stream) {
  return hc_union_cold_layers(masks, 1, 0, batch, token_stride, inter, fetch_bits, table, rec_out, 0, count, stream);
}

extern "C" int hc_union_cold_layers(const uint32_t* masks, int32_t n_layers, int64_t layer_stride, int32_t batch,
                                    int64_t token_stride, int32_t inter, const uint32_t* fetch_bits,
                                    const int32_t* table, int32_t* rec_out, int64_t rec_stride, int32_t* count,
                                    hc_stream_t stream) {
  if (!masks || !fetch_bits || !table || !rec_out || !count || n_layers <= 0 || batch <= 0 || inter <= 0 ||
      inter > 65536 || (n_layers > 1 && rec_stride <= 0))
    return HC_ERR_ARG;
  k_union<<<n_layers, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      masks, layer_stride, batch, token_stride, (inter + 31) / 32, fetch_bits, table, rec_out, rec_stride, count);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_ffn_batch_layer(const hc_layer_desc* layer, float* x, int32_t batch, const int32_t* rec,
                                  const int32_t* count, int32_t max_cold, float eps, int32_t act,
                                  int32_t act_on_both, void* workspace, int32_t* status, hc_stream_t stream) {
  if (!layer || !x || batch <= 0 || !rec || !count || max_cold < 0 || !workspace || !status ||
      (act != HC_ACT_SILU && act != HC_ACT_RELU))
    return HC_ERR_ARG;
  if (!layer->hot || !layer->cold_records || layer->n_hot < 0 || max_cold > layer->n_records)
    return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(workspace) & 15) ||
      (reinterpret_cast<uintptr_t>(layer->hot) & 15) || (reinterpret_cast<uintptr_t>(layer->cold_records) & 15))
    return HC_ERR_ARG;
  constexpr int GU_RAW = RAW_DEPTH * (GU_PIECES * GU_PSTRIDE + GU_PROD * 4);
  constexpr int GU_SMEM = GU_STAGES * NMAX * KC * 2 + GU_RAW + BAR_BYTES;
  static_assert(GU_SMEM <= GU_SMEM_FLOOR, "k_gu shared memory");
  constexpr int DN_RAW = RAW_DEPTH * DN_PIECES * DN_PSTRIDE + REC_RING * DN_PROD * 4;
  constexpr int GU_SMEM_MAX = GU_SMEM_FLOOR;
  constexpr int DN_SMEM_MAX = 3 * (A_TILE_BYTES + KC * NMAX * 2) + DN_RAW + BAR_BYTES;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(k_gu, cudaFuncAttributeMaxDynamicSharedMemorySize, GU_SMEM_MAX) != cudaSuccess ||
        cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, DN_SMEM_MAX) != cudaSuccess)
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
  const WsLayout wl = ws_layout(max_total > 0 ? max_total : 1);
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

  const int hot_tiles = (layer->n_hot + TILE - 1) / TILE;
  const int tiles_max = hot_tiles + (max_cold + TILE - 1) / TILE;
  for (int b0 = 0; b0 < batch; b0 += NMAX) {
    const int nb = batch - b0 < NMAX ? batch - b0 : NMAX;
    const int N = (nb + 15) / 16 * 16;
    float* xb = x + (size_t)b0 * H;
    k_norm<<<N, 256, 0, s>>>(xb, nb, N, layer->norm_w, eps, ws + wl.xs_nat, ws + wl.xs_perm);
    if (max_total > 0) {
      GuParams g;
      g.a = la;
      g.xs_nat = ws + wl.xs_nat;
      g.xs_perm = ws + wl.xs_perm;
      g.part = reinterpret_cast<float*>(ws + wl.part);
      g.N = N;
      g.hot_tiles = hot_tiles;
      const int gu_grid = tiles_max * (H / KC) < ctas ? tiles_max * (H / KC) : ctas;
      k_gu<<<gu_grid, GU_THREADS, GU_SMEM_FLOOR, s>>>(g);

      const int act_threads = max_total * (N / 8);
      k_act<<<(act_threads + 255) / 256, 256, 0, s>>>(la, g.part, hot_tiles, gu_grid, N,
                                                       reinterpret_cast<__half*>(ws + wl.act));

      DownParams d;
      d.a = la;
      d.act = reinterpret_cast<const __half*>(ws + wl.act);
      d.y = reinterpret_cast<float*>(ws + wl.y);
      d.N = N;
      d.stages = 3;
      d.tmem_cols = tmem_cols_for(2 * N);
      const int dn_units = (H / TILE) * ((max_total + KC - 1) / KC);
      const int dn_grid = dn_units < ctas ? dn_units : ctas;
      const int dn_smem = d.stages * (A_TILE_BYTES + KC * N * 2) + DN_RAW + BAR_BYTES;
      k_down<<<dn_grid, DN_THREADS, dn_smem, s>>>(d);
    }
    k_resid<<<dim3(H / 256, N / 4), 256, 0, s>>>(xb, nb, N, reinterpret_cast<float*>(ws + wl.y));
  }
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}
