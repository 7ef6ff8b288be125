// Cold store kernels: the nid -> record table, request-id mapping, and the
// batched INT4 gather + dequantise that replaces ColdWeightStore.read_neurons
// (splitter.py:354-403) and dequantize_int4 (splitter.py:111-124).
//
// Records are read straight from the uploaded image of cold_weights.bin.
// A record starts 16 B after a page-aligned section header plus r * 6400, so
// its start is 16-byte aligned, but every field begins 2 bytes later (after
// the u16 id).  Threads load aligned words and funnel-shift by 16 bits.
#include <algorithm>

#include "hc_common.cuh"

namespace hc {

// --------------------------------------------------------------------------
// nid -> record index (ColdWeightStore._section_offsets, splitter.py:332-352)
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(256) build_table_kernel(const uint8_t* __restrict__ base,
                                                          int64_t image_bytes,
                                                          const int64_t* __restrict__ sec_off,
                                                          const int32_t* __restrict__ n_rec,
                                                          int32_t* __restrict__ table,
                                                          int32_t* __restrict__ status) {
  const int layer = blockIdx.y;
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t off = sec_off[layer];
  if (off < 0 || (off & 15) != 0) {
    if (r == 0 && status) atomicOr(status, HC_ERR_ARG);
    return;
  }
  if (r >= n_rec[layer]) return;
  if (off + SECTION_HEADER + (int64_t)r * REC_BYTES + REC_COPY > image_bytes) {
    if (status) atomicOr(status, HC_ERR_RANGE);   // cold_index points past the image
    return;
  }
  const uint16_t nid = *reinterpret_cast<const uint16_t*>(base + off + SECTION_HEADER + (int64_t)r * REC_BYTES);
  // the reference keeps the last duplicate (dict overwrite order == record order)
  atomicMax(&table[(int64_t)layer * TABLE_SIZE + nid], r);
}

// --------------------------------------------------------------------------
// request ids -> record indices in request order, absent ids dropped
// (splitter.py:370-372).  One CTA of 1024 threads, chunked block scan.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) map_ids_kernel(const int64_t* __restrict__ ids, int n,
                                                       const int32_t* __restrict__ table,
                                                       int32_t* __restrict__ rec_out,
                                                       int32_t* __restrict__ nid_out,
                                                       int32_t* __restrict__ count) {
  __shared__ int warp_tot[32];
  __shared__ int base_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) base_s = 0;
  __syncthreads();
  for (int start = 0; start < n; start += 1024) {
    const int i = start + tid;
    int rec = -1;
    int64_t id = -1;
    if (i < n) {
      id = ids[i];
      if (id >= 0 && id < TABLE_SIZE) rec = table[id];
    }
    const bool keep = rec >= 0;
    const unsigned bal = __ballot_sync(0xffffffffu, keep);
    const int before = __popc(bal & ((1u << lane) - 1u));
    if (lane == 31) warp_tot[warp] = before + (keep ? 1 : 0);
    __syncthreads();
    if (warp == 0) {
      int v = warp_tot[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += u;
      }
      warp_tot[lane] = v;  // inclusive
    }
    __syncthreads();
    const int wbase = (warp ? warp_tot[warp - 1] : 0) + base_s;
    if (keep) {
      rec_out[wbase + before] = rec;
      if (nid_out) nid_out[wbase + before] = static_cast<int32_t>(id);
    }
    __syncthreads();
    if (tid == 0) base_s += warp_tot[31];
    __syncthreads();
  }
  if (tid == 0) *count = base_s;
}

// --------------------------------------------------------------------------
// gather + dequantise.  128 threads per record, 2 records per CTA.  A vector's
// 4096 elements are 512 chunks of 8 (4 bytes of INT4 each); thread t owns
// chunks t, t + 128, t + 256 and t + 384, so each warp-wide load reads 128
// contiguous bytes of the field and each warp-wide store writes 512 (bf16) or
// 2 x 512 (fp32) contiguous bytes of the output row -- whole lines, where a
// thread owning 32 consecutive elements would leave every store instruction
// covering a quarter of 16 lines.  A field starts 2 bytes past a 16-byte
// boundary: chunk m's nibbles are aligned words m and m + 1 of the field's
// aligned span, funnel-shifted by 16 bits (word m + 1 comes from the next lane).
// --------------------------------------------------------------------------
template <typename OutT>
__device__ __forceinline__ void store8(OutT* dst, const float (&f)[8]);

template <>
__device__ __forceinline__ void store8<float>(float* dst, const float (&f)[8]) {
  float4* d = reinterpret_cast<float4*>(dst);
  d[0] = make_float4(f[0], f[1], f[2], f[3]);
  d[1] = make_float4(f[4], f[5], f[6], f[7]);
}

template <>
__device__ __forceinline__ void store8<__nv_bfloat16>(__nv_bfloat16* dst, const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __nv_bfloat162 b = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
    w[j] = *reinterpret_cast<const uint32_t*>(&b);
  }
  *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
}

constexpr int GD_CHUNKS = H / 8 / 128;     // 4 chunks of 8 elements per thread and vector

template <typename OutT>
__global__ void __launch_bounds__(256) gather_dequant_kernel(
    const uint8_t* __restrict__ base, int64_t image_bytes, const int64_t* __restrict__ sec_off,
    const int32_t* __restrict__ n_rec, const int32_t* __restrict__ rec_idx, int K, const int32_t* __restrict__ count,
    OutT* __restrict__ gate_out, OutT* __restrict__ up_out, OutT* __restrict__ down_out,
    int32_t* __restrict__ status) {
  const int layer = blockIdx.y;
  const int k = blockIdx.x * 2 + (threadIdx.x >> 7);      // uniform over each 128-thread half (4 whole warps)
  const int t = threadIdx.x & 127, lane = threadIdx.x & 31;
  if (k >= K) return;
  if (count != nullptr && k >= count[layer]) return;
  const int64_t row = ((int64_t)layer * K + k) * H;
  OutT* outs[3] = {gate_out + row, up_out + row, down_out + row};
  const int32_t r = rec_idx[(int64_t)layer * K + k];
  const int64_t off = sec_off[layer];
  const bool bad_off = off < 0 || (off & 15) != 0;
  if (bad_off || r < 0 || r >= n_rec[layer] ||
      off + SECTION_HEADER + (int64_t)r * REC_BYTES + REC_COPY > image_bytes) {
    float z[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) z[i] = 0.0f;
    for (int v = 0; v < 3; ++v)
#pragma unroll
      for (int j = 0; j < GD_CHUNKS; ++j) store8<OutT>(outs[v] + 8 * (t + 128 * j), z);
    if (t == 0) atomicOr(status, bad_off ? HC_ERR_ARG : HC_ERR_RANGE);
    return;
  }
  const uint8_t* rec = base + off + SECTION_HEADER + (int64_t)r * REC_BYTES;
  const uint32_t* rw = reinterpret_cast<const uint32_t*>(rec);   // 16-byte aligned
  // issue all loads first: the chunks' words, the last lane's next words, one
  // group scale per lane (lane g holds group g's)
  uint32_t w[3][GD_CHUNKS], nx[3][GD_CHUNKS];
  uint16_t s16[3];
#pragma unroll
  for (int v = 0; v < 3; ++v) {
#pragma unroll
    for (int j = 0; j < GD_CHUNKS; ++j) w[v][j] = __ldg(rw + (VEC_BYTES / 4) * v + t + 128 * j);
    s16[v] = __ldg(reinterpret_cast<const unsigned short*>(rec + SCALE_OFF + v * 2 * NGROUPS + 2 * lane));
  }
  if (lane == 31) {
#pragma unroll
    for (int v = 0; v < 3; ++v)
#pragma unroll
      for (int j = 0; j < GD_CHUNKS; ++j) nx[v][j] = __ldg(rw + (VEC_BYTES / 4) * v + t + 128 * j + 1);
  }
#pragma unroll
  for (int v = 0; v < 3; ++v) {
#pragma unroll
    for (int j = 0; j < GD_CHUNKS; ++j) {
      const uint32_t up1 = __shfl_down_sync(0xffffffffu, w[v][j], 1);
      const uint32_t hi = lane == 31 ? nx[v][j] : up1;
      const int m = t + 128 * j;                                   // chunk: elements [8m, 8m + 8)
      const float sc = __half2float(__ushort_as_half(
          (unsigned short)__shfl_sync(0xffffffffu, (uint32_t)s16[v], m >> 4)));   // group m / 16 (< 32)
      float q[8];
      int4x8_to_f32(shift2(w[v][j], hi), q);
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] *= sc;                      // exact in fp32 (splitter.py:124)
      store8<OutT>(outs[v] + 8 * m, q);
    }
  }
}

// --------------------------------------------------------------------------
// record staging: the cold tier kept outside HBM.  The reference keeps the
// store on disk / in host memory and reads only the fetched neurons
// (splitter.py:307-330, :354-403); here a layer's fetched records are copied,
// raw, from the store's section (pinned host memory read over the bus, or any
// device-readable memory) to the same record offsets of a device buffer that
// the fused kernels then read as the layer's section.  One warp per record:
// every lane issues its 13 16-byte loads before its stores, so a warp keeps a
// whole record in flight.
// --------------------------------------------------------------------------
constexpr int REC_WORDS = REC_COPY / 16;                 // 397 words read per record
constexpr int STAGE_PER_LANE = (REC_WORDS + 31) / 32;    // 13
constexpr int STAGE_THREADS = 256;
constexpr int STAGE_MAX_CTAS = 148 * 8;

__global__ void __launch_bounds__(STAGE_THREADS) stage_records_kernel(
    const uint8_t* __restrict__ src, int64_t src_bytes, const int32_t* __restrict__ rec_idx,
    const int32_t* __restrict__ count, int max_count, int n_records, uint8_t* __restrict__ dst, int64_t dst_bytes,
    int32_t* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  const int warp = (blockIdx.x * STAGE_THREADS + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * STAGE_THREADS) >> 5;
  int n = max_count;
  if (count != nullptr) {
    const int c = __ldg(count);
    if (c > max_count && warp == 0 && lane == 0) atomicOr(status, HC_ERR_RANGE);   // list longer than its buffer
    n = min(max(c, 0), max_count);
  }
  for (int k = warp; k < n; k += nwarps) {
    const int32_t r = __ldg(rec_idx + k);
    const int64_t off = (int64_t)r * REC_BYTES;
    if (r < 0 || r >= n_records || off + REC_COPY > src_bytes || off + REC_COPY > dst_bytes) {
      if (lane == 0) atomicOr(status, HC_ERR_RANGE);
      continue;
    }
    const uint4* s = reinterpret_cast<const uint4*>(src + off);
    uint4* d = reinterpret_cast<uint4*>(dst + off);
    uint4 v[STAGE_PER_LANE];
#pragma unroll
    for (int i = 0; i < STAGE_PER_LANE; ++i)
      if (lane + 32 * i < REC_WORDS) v[i] = __ldg(s + lane + 32 * i);
#pragma unroll
    for (int i = 0; i < STAGE_PER_LANE; ++i)
      if (lane + 32 * i < REC_WORDS) d[lane + 32 * i] = v[i];
  }
}

}  // namespace hc

using namespace hc;

extern "C" int hc_cold_stage(const void* src_records, int64_t src_bytes, const int32_t* rec_idx,
                             const int32_t* count, int32_t max_count, int32_t n_records, void* dst_records,
                             int64_t dst_bytes, int32_t* status, hc_stream_t stream) {
  if (!src_records || !dst_records || !status || max_count < 0 || n_records < 0 || src_bytes < 0 ||
      dst_bytes < 0 || (max_count > 0 && !rec_idx))
    return HC_ERR_ARG;
  if ((reinterpret_cast<uintptr_t>(src_records) & 15) || (reinterpret_cast<uintptr_t>(dst_records) & 15))
    return HC_ERR_ARG;
  if (max_count == 0) return HC_OK;
  const int warps = max_count;
  const int ctas = std::min((warps + STAGE_THREADS / 32 - 1) / (STAGE_THREADS / 32), STAGE_MAX_CTAS);
  stage_records_kernel<<<ctas, STAGE_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src_records), src_bytes, rec_idx, count, max_count, n_records,
      static_cast<uint8_t*>(dst_records), dst_bytes, status);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_build_record_table(const void* cold_base, int64_t image_bytes, const int64_t* section_offsets,
                                     const int32_t* n_records, int32_t n_layers, int32_t max_records,
                                     int32_t* table, int32_t* status, hc_stream_t stream) {
  if (!cold_base || !section_offsets || !n_records || !table || n_layers <= 0 || max_records < 0 ||
      n_layers > 65535)
    return HC_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(table, 0xFF, sizeof(int32_t) * (size_t)TABLE_SIZE * n_layers, s) != cudaSuccess)
    return HC_ERR_CUDA;
  if (max_records == 0) return HC_OK;
  dim3 grid((max_records + 255) / 256, n_layers);
  build_table_kernel<<<grid, 256, 0, s>>>(static_cast<const uint8_t*>(cold_base), image_bytes, section_offsets, n_records,
                                          table, status);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_map_ids(const int64_t* ids, int32_t n, const int32_t* table, int32_t* rec_out,
                          int32_t* nid_out, int32_t* count, hc_stream_t stream) {
  if (n < 0 || n > (1 << 20) || !table || !rec_out || !count || (n > 0 && !ids)) return HC_ERR_ARG;
  map_ids_kernel<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(ids, n, table, rec_out, nid_out, count);
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}

extern "C" int hc_cold_gather_dequant(const void* cold_base, int64_t image_bytes, const int64_t* section_offsets,
                                      const int32_t* n_records, int32_t n_layers, const int32_t* rec_idx,
                                      int32_t K, const int32_t* count, int32_t out_dtype, void* gate_out,
                                      void* up_out, void* down_out, int32_t* status, hc_stream_t stream) {
  if (!cold_base || !section_offsets || !n_records || !rec_idx || !gate_out || !up_out || !down_out || !status ||
      n_layers <= 0 || n_layers > 65535 || K < 0)
    return HC_ERR_ARG;
  if (K == 0) return HC_OK;
  if ((reinterpret_cast<uintptr_t>(cold_base) & 15) || (reinterpret_cast<uintptr_t>(gate_out) & 15) ||
      (reinterpret_cast<uintptr_t>(up_out) & 15) || (reinterpret_cast<uintptr_t>(down_out) & 15))
    return HC_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  dim3 grid((K + 1) / 2, n_layers);
  const uint8_t* b = static_cast<const uint8_t*>(cold_base);
  if (out_dtype == HC_F32) {
    gather_dequant_kernel<float><<<grid, 256, 0, s>>>(b, image_bytes, section_offsets, n_records, rec_idx, K, count,
                                                      static_cast<float*>(gate_out), static_cast<float*>(up_out),
                                                      static_cast<float*>(down_out), status);
  } else if (out_dtype == HC_BF16) {
    gather_dequant_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(
        b, image_bytes, section_offsets, n_records, rec_idx, K, count, static_cast<__nv_bfloat16*>(gate_out),
        static_cast<__nv_bfloat16*>(up_out), static_cast<__nv_bfloat16*>(down_out), status);
  } else {
    return HC_ERR_UNSUPPORTED;
  }
  return cudaGetLastError() == cudaSuccess ? HC_OK : HC_ERR_CUDA;
}
