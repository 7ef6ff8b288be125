/*
 * hotcold.h -- C ABI of the B200 (sm_100a) hot/cold sparse-FFN library
 * (libhotcold.so).
 *
 * The reference (Hot-Cold-Neural-Split-OpenInfer2) is pure Python; these entry
 * points replace the Python/torch functions on its per-token FFN path.  Each
 * declaration names the reference function it stands in for (file:line).
 *
 * Conventions
 *  - Every pointer argument is a DEVICE pointer unless its comment says host.
 *  - Functions are asynchronous on `stream` and return an HC_* status for
 *    argument / launch errors.  Errors found by a kernel (an index out of
 *    range, a bounded wait that expired) are OR-ed into the caller's device
 *    word `status` (HC_ERR_* bits); read it after synchronising.
 *  - Nothing allocates: scratch space is a caller-owned workspace whose size
 *    comes from the matching *_workspace_bytes query and which must be zeroed
 *    once after allocation (kernels leave it re-usable).
 *  - Thread safety: calls are independent as long as they do not share a
 *    workspace or a status word while in flight.
 *  - Cold records are read in the reference's on-disk layout
 *    (splitter.py:23-37): the image of cold_weights.bin is uploaded unchanged.
 */
#ifndef HOTCOLD_H
#define HOTCOLD_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* hc_stream_t; /* == cudaStream_t */

#if defined(__GNUC__)
#define HC_API __attribute__((visibility("default")))
#else
#define HC_API
#endif

/* ---- status codes (return values and device status bits) ---------------- */
#define HC_OK 0
#define HC_ERR_ARG 1         /* bad argument, detected on the host            */
#define HC_ERR_CUDA 2        /* a CUDA runtime call failed                    */
#define HC_ERR_RANGE 4       /* device: an index pointed outside its table    */
#define HC_ERR_TIMEOUT 8     /* device: a bounded wait expired                */
#define HC_ERR_UNSUPPORTED 16 /* shape or mode this build does not handle    */

/* ---- dtypes ------------------------------------------------------------- */
#define HC_F32 0
#define HC_BF16 1
#define HC_F16 2

/* ---- activations (engine.py:163-170) ------------------------------------ */
#define HC_ACT_SILU 0
#define HC_ACT_RELU 1

/* Library identity / device checks.  hc_version returns HC_ABI_VERSION. */
#define HC_ABI_VERSION 3
HC_API int hc_version(void);
HC_API const char* hc_status_string(int status);
/* Number of SMs of the current device, or -1 when no CUDA device is usable. */
HC_API int hc_device_sm_count(void);

/* ======================================================================= */
/* Cold store                                                              */
/* ======================================================================= */

/*
 * hc_build_record_table -- replaces ColdWeightStore._section_offsets
 * (splitter.py:332-352): scans each layer's section once and records, for
 * every u16 neuron id, its record index (-1 when absent; a later duplicate
 * wins, like the reference's dict).
 *   cold_base        image of cold_weights.bin (device or mapped pinned host)
 *   image_bytes      host: size of that image; records reaching past it are
 *                    left out of the table and flag HC_ERR_RANGE
 *   section_offsets  [n_layers] byte offset of each section header (device);
 *                    must be a multiple of 16 (the reference page-aligns them)
 *   n_records        [n_layers] n_cold of each section (device)
 *   max_records      host: upper bound of n_records (grid size)
 *   table            [n_layers][65536] int32 output (device)
 *   status           device status word (may be NULL)
 */
HC_API int hc_build_record_table(const void* cold_base, int64_t image_bytes, const int64_t* section_offsets,
                          const int32_t* n_records, int32_t n_layers, int32_t max_records,
                          int32_t* table, int32_t* status, hc_stream_t stream);

/*
 * hc_map_ids -- the id handling of ColdWeightStore.read_neurons
 * (splitter.py:365-372): maps requested neuron ids to record indices in
 * request order, dropping ids that have no record.
 *   ids [n] int64 requested ids; table [65536] of the layer;
 *   rec_out [n] int32 record indices (first *count entries valid);
 *   nid_out [n] int32 kept ids (may be NULL); count [1] int32 output.
 * Single CTA; n <= 1<<20.
 */
HC_API int hc_map_ids(const int64_t* ids, int32_t n, const int32_t* table, int32_t* rec_out,
               int32_t* nid_out, int32_t* count, hc_stream_t stream);

/*
 * hc_cold_gather_dequant -- replaces the per-neuron loop of
 * ColdWeightStore.read_neurons + dequantize_int4 (splitter.py:354-403,
 * :111-124).  For each layer j and each of K record indices, decodes the
 * record's gate / up / down INT4 vectors with their fp16 group scales into
 * neuron-major rows: out[j][k][0:4096] = q * s (exact in fp32; bf16 is the
 * round-to-nearest-even of that fp32 value).
 *   cold_base, image_bytes, section_offsets[n_layers], n_records[n_layers]:
 *              as above (records reaching past image_bytes flag HC_ERR_RANGE)
 *   rec_idx    [n_layers][K] int32; an index outside [0, n_records) sets
 *              HC_ERR_RANGE and writes zeros for that row
 *   count      optional [n_layers] int32 (NULL = K): rows k >= count[j] are
 *              left untouched (lets the caller pass a device-side count)
 *   out_dtype  HC_F32 or HC_BF16; gate/up/down_out [n_layers][K][4096]
 */
HC_API int hc_cold_gather_dequant(const void* cold_base, int64_t image_bytes, const int64_t* section_offsets,
                           const int32_t* n_records, int32_t n_layers, const int32_t* rec_idx,
                           int32_t K, const int32_t* count, int32_t out_dtype, void* gate_out,
                           void* up_out, void* down_out, int32_t* status, hc_stream_t stream);

/*
 * hc_cold_stage -- the per-layer fetch of a cold tier kept outside HBM.  The
 * reference keeps cold_weights.bin on disk / in host memory and reads only
 * the neurons it fetches (ColdWeightStore, splitter.py:307-330, :354-403);
 * here the fetched records of one layer are copied raw (their first 6352
 * bytes: id, INT4 fields, scales) from the store's section to the same
 * offsets of a device buffer, which the fused kernels (hc_ffn_stack,
 * hc_ffn_batch_layer) are then given as that layer's cold_records.
 *   src_records  the section's first record (section offset + 16) in device
 *                memory or mapped pinned host memory (read over the bus);
 *                16-byte aligned
 *   src_bytes    host: bytes readable from src_records
 *   rec_idx      [max_count] int32 record indices (hc_union_cold's list)
 *   count        optional [1] int32 (device): entries of rec_idx in use;
 *                NULL = max_count; a count above max_count sets HC_ERR_RANGE
 *   n_records    host: records in the section; an index outside [0,
 *                n_records) or past src_bytes / dst_bytes sets HC_ERR_RANGE
 *                and is skipped
 *   dst_records  device buffer laid out like the section (record r at
 *                r * 6400); 16-byte aligned; dst_bytes its size
 * Records not listed are left untouched.
 */
HC_API int hc_cold_stage(const void* src_records, int64_t src_bytes, const int32_t* rec_idx, const int32_t* count,
                         int32_t max_count, int32_t n_records, void* dst_records, int64_t dst_bytes,
                         int32_t* status, hc_stream_t stream);

/* ======================================================================= */
/* Predictor                                                               */
/* ======================================================================= */

/*
 * hc_predictor_workspace_bytes -- scratch for hc_predictor_forward.
 */
HC_API int64_t hc_predictor_workspace_bytes(int32_t batch, int32_t rank, int32_t inter);

/*
 * hc_predictor_forward -- replaces NeuronPredictor.forward / predict_mask
 * (predictor.py:70-79), PredictorRegistry.predict (predictor.py:435-456) and
 * the id selection of SparseFFNLayer._cold_ids_for (engine.py:274-283).
 *   x        [batch][4096] fp32 predictor input
 *   norm_w   optional [4096] fp32: when given, each row is first RMS-normalised
 *            (x * rsqrt(mean(x^2) + eps) * norm_w), as SparseFFNLayer does
 *            before querying the predictor (engine.py:289); NULL = x as is
 *   w_down   [rank][4096] fp32   (nn.Linear weight of `down`)
 *   w_up     [inter][rank] fp32  (nn.Linear weight of `up`), b_up [inter]
 *   logit_threshold  mask bit = (logit >= logit_threshold); the host picks the
 *            smallest fp32 logit whose torch.sigmoid reaches the probability
 *            threshold, so the decision equals `sigmoid(logit) >= threshold`
 *   mask_out [batch][ceil(inter/32)] uint32 bit masks (required)
 *   probs_out / logits_out  optional [batch][inter] fp32 (NULL to skip)
 *   fetch_bits optional [ceil(inter/32)] uint32: ids eligible for the cold
 *            fetch (a record exists and the id is not hot); when given, row 0's
 *            mask & fetch_bits is compacted in ascending id order into
 *            ids_out [inter] int32 (+ rec_out via `table`, may be NULL) with
 *            the number in count_out[0]
 *   workspace  hc_predictor_workspace_bytes(batch, rank, inter) bytes, zeroed once
 * Limits: rank <= 128, inter <= 65536, batch <= 64.
 */
HC_API int hc_predictor_forward(const float* x, int32_t batch, const float* norm_w, float eps,
                                const float* w_down, const float* w_up,
                         const float* b_up, int32_t rank, int32_t inter, float logit_threshold,
                         uint32_t* mask_out, float* probs_out, float* logits_out,
                         const uint32_t* fetch_bits, const int32_t* table, int32_t* ids_out,
                         int32_t* rec_out, int32_t* count_out, void* workspace, int32_t* status,
                         hc_stream_t stream);

/*
 * hc_predictor_forward_static -- no counterpart in the reference.  The same
 * computation and arguments as hc_predictor_forward, minus the workspace,
 * for callers that cannot allocate device memory (a serving process whose
 * allocator is frozen after start-up, an embedded runtime or a plugin host
 * that owns every allocation).  The scratch is a file-scope device array of
 * about 66 KB inside the library (held by every GPU that loads it until the
 * process exits), so it supports batch * rank <= 512 and returns
 * HC_ERR_UNSUPPORTED beyond that without launching anything.  Bad arguments
 * return HC_ERR_ARG, as for hc_predictor_forward, before anything is
 * enqueued.  The first call on a device looks up that array's address
 * (cudaGetSymbolAddress) for the current device and context, and again after
 * the device's context was replaced (cudaDeviceReset); make that first call
 * before any stream capture.  Each call clears the array's counters on
 * `stream` first; calls that overlap on the GPU share the array and race, so
 * serialise them (one stream, or events).  Nothing here calls cudaMalloc or
 * cudaFree.
 */
HC_API int hc_predictor_forward_static(const float* x, int32_t batch, const float* norm_w, float eps,
                                       const float* w_down, const float* w_up, const float* b_up,
                                       int32_t rank, int32_t inter, float logit_threshold,
                                       uint32_t* mask_out, float* probs_out, float* logits_out,
                                       const uint32_t* fetch_bits, const int32_t* table, int32_t* ids_out,
                                       int32_t* rec_out, int32_t* count_out, int32_t* status,
                                       hc_stream_t stream);

/* ======================================================================= */
/* Fused sparse FFN (hot FP8 + cold INT4), one layer or a stack of layers  */
/* ======================================================================= */

/*
 * Per-layer description consumed by hc_ffn_stack.  All pointers are device
 * pointers.  Layout notes:
 *  - hot: n_hot neurons, each 3 x 4096 e4m3 bytes in the order gate row, up
 *    row, down column (the reference stores down as [4096][n_hot],
 *    splitter.py:225; the host re-lays it out once at load time);
 *    hot_scale [n_hot][3] fp32 or NULL (the reference's direct cast = 1.0)
 *  - cold_records: first record of the layer's section inside the uploaded
 *    cold_weights.bin image (16-byte aligned)
 *  - fetch_bits [ceil(inter/32)]: 1 = cold id with a record and not hot
 *  - pred_w_down_t [4096][rank] (transposed), pred_w_up [inter][rank],
 *    pred_b_up [inter]: this layer's predictor, or all NULL
 */
typedef struct hc_layer_desc {
  const uint8_t* hot;
  const float* hot_scale;
  const float* norm_w;
  const uint8_t* cold_records;
  const int32_t* table;
  const uint32_t* fetch_bits;
  const float* pred_w_down_t;
  const float* pred_w_up;
  const float* pred_b_up;
  int32_t n_hot;
  int32_t n_records;
  int32_t inter;
  int32_t rank;
} hc_layer_desc;

/* Grid size the stack kernel uses on the current device (1 CTA per SM). */
HC_API int hc_ffn_stack_grid(void);
HC_API int64_t hc_ffn_stack_workspace_bytes(int32_t grid, int32_t inter);

/*
 * hc_ffn_stack -- replaces, per layer, SparseFFNLayer.forward
 * (engine.py:292-312: RMSNorm -> sparse_ffn -> residual) with sparse_ffn
 * (engine.py:173-209: hot FP8 half + cold INT4 half, summed in-kernel), and
 * the cross-layer predictor prefetch of DesdemonaEngine.forward
 * (engine.py:421-438: layer l+1's fetch set comes from layer l's input).
 *   layers     [n_layers] hc_layer_desc (device array); every layer has
 *              `inter` neurons (inter % 4 == 0, inter <= 32768); a predictor
 *              rank must be a multiple of 8 and <= 96 (else HC_ERR_UNSUPPORTED,
 *              no predictor); CTA c owns the neuron ids of mask words
 *              [c*W/grid, (c+1)*W/grid), W = ceil(inter/32), and at most 1024
 *              of them, i.e. ceil(W/grid)*32 <= 1024 (else HC_ERR_UNSUPPORTED)
 *   x_in       [4096] fp32 input hidden state (batch 1)
 *   masks      [n_layers][ceil(inter/32)] uint32 predicted-active bits.
 *              masks_given = 0: row 0 is filled by the caller (e.g. by
 *              hc_predictor_forward on x_in); row l+1 is written by the kernel
 *              from layer l+1's predictor on RMSNorm_{l+1}(x_l) (all ones when
 *              that layer has no predictor -- the reference's fetch-everything
 *              fallback, engine.py:282-283).  masks_given = 2: the same, and
 *              row 0 too is written by the kernel, from layer 0's predictor on
 *              RMSNorm_0(x_in) (engine.py:422; all ones without a predictor),
 *              saving the caller's predictor launches.  masks_given = 1: every
 *              row is an input.  The cold neurons a layer computes are
 *              masks[l] & fetch_bits.
 *   x_out      [4096] fp32 output; x_hist optional [n_layers][4096] fp32
 *   eps        RMSNorm epsilon; act = HC_ACT_*; act_on_both = dReLU form
 *   logit_threshold  as in hc_predictor_forward
 *   grid       0 = hc_ffn_stack_grid(); tests may pass fewer CTAs
 *   workspace  hc_ffn_stack_workspace_bytes(grid, inter), zeroed once; the
 *              kernel leaves it zeroed again when it completes
 *   trace      optional [n_layers][grid][40] uint64, zeroed by the caller:
 *              %globaltimer stamps (ns) per CTA and layer -- 0: layer start
 *              (grid barrier passed), 1: normalised input ready, 4-7:
 *              consumer subgroup 0-3 done, 9: partial y added, 8: grid
 *              barrier arrival; issuer 10: layer start, 11: the layer's
 *              cold pool complete, 12: cold records issued, 13 / 37: hot
 *              groups start / issued (layer 0 of a launch: hot groups before
 *              the cold pool), 14: layer sealed; CTA thread 0 at the layer
 *              end: 38 all subgroups done, 39 tree staged; layer 0's slot
 *              also holds 33: the CTA started, 34: the CTA done; 21: own mask words ready (stamped at the end of the
 *              previous layer), 22: planner took them, 20: own cold list
 *              published -- plus 15: hot neurons claimed, 30: cold records
 *              taken from the pool, 17: active cold records of the own id
 *              range, 18: ns the issuer waited for empty slots, 19: groups
 *              issued; SM cycles of
 *              subgroup 0's poller: 16 waiting for fills, 2/3/23 on cold /
 *              hot / predictor groups, 24/25/26 in its group barrier / seeing
 *              the fills / releasing, 27 in total;
 *              32: local partials complete (every CTA); under tensor
 *              parallelism 35: all peers' partials seen (layers before the
 *              last), 36: this CTA's slice pushed (pushing CTAs only);
 *              NULL = off
 * The layer outputs are sums of per-CTA float partials added with atomics, so
 * their last bits can differ between launches.
 */
HC_API int hc_ffn_stack(const hc_layer_desc* layers, int32_t n_layers, int32_t inter, const float* x_in,
                 uint32_t* masks, int32_t masks_given, float* x_out, float* x_hist, float eps,
                 int32_t act, int32_t act_on_both, float logit_threshold, int32_t grid,
                 void* workspace, int32_t* status, uint64_t* trace, hc_stream_t stream);

/*
 * Tensor-parallel decode stack: the neuron dimension of every layer is split
 * over `size` GPUs, one process per GPU (the reference's down_proj is linear
 * in the neuron dimension, engine.py:184-188, so y = sum over GPUs of each
 * GPU's partial).  GPU `rank` holds its slice of the hot neurons (its own
 * hc_layer_desc.hot / n_hot), computes the predictor logits and cold records
 * of mask words [words_lo, words_lo + words_n), and runs the full W_down of
 * every predictor.  Per layer, each GPU sums its CTAs' partial y; its first
 * kp = min(grid, 32) CTAs each store one slice of that sum into every peer's
 * exchange buffer over NVLink (plain peer stores, no multicast) as 8-byte
 * words (exchange number << 32 | float bits), exchange number q = seq_base +
 * layer + 1, in slot q % 3.  An aligned 8-byte store is single-copy atomic,
 * so every word carries its own arrival flag: each CTA polls (bounded) its
 * elements' words until they show q, then adds the partials in GPU order, so
 * all GPUs hold bit-identical hidden states.  No fence or counter is used.
 *   peer_buf   device array [size] of every GPU's exchange buffer
 *              (hc_tp_buffer_bytes(size) bytes from hc_tp_alloc, zeroed once,
 *              opened in the other processes with hc_ipc_open); size <= 8
 *   seq_base   layers exchanged through these buffers by earlier launches;
 *              every GPU passes the same value and runs the same grid
 * All `size` kernels must be running at the same time (one per GPU, issued
 * by each rank in the same order); a GPU that does not reach a layer within
 * `wait_ns` (default 2 s) makes the others return HC_ERR_TIMEOUT: the kernel
 * ORs it into `status`, waits for its own copies in flight and returns,
 * leaving the workspace clean and the context usable.  masks[] rows are
 * written only for the mask words this GPU owns.  A tp with size 1 only
 * sets the wait limit.
 */
typedef struct hc_tp_desc {
  int32_t size, rank;
  int32_t words_lo, words_n;
  void* const* peer_buf;
  uint32_t seq_base;
  uint64_t wait_ns;   /* limit of every bounded wait of the launch; 0 = 2 s */
  /* 1: the last layer of `layers` is not computed, only its mask row is
   * predicted, on RMSNorm_last(input of the layer before it) -- the engine's
   * lookahead across an attention block (engine.py:430-438): a launch over
   * [layer l, layer l+1] computes layer l and predicts layer l+1's set.
   * Needs n_layers >= 2 and masks_given 0 or 2. */
  int32_t predict_last;
  /* 1: x_in and x_out are fp16 [4096] (16-byte aligned) instead of fp32 -- the
   * engine's fp16 hidden state handed over without conversions; the layers
   * still compute in fp32 and x_hist stays fp32. */
  int32_t io_f16;
} hc_tp_desc;

HC_API int64_t hc_tp_buffer_bytes(int32_t tp_size);
/* tp == NULL is hc_ffn_stack. */
HC_API int hc_ffn_stack_tp(const hc_layer_desc* layers, int32_t n_layers, int32_t inter, const void* x_in,
                    uint32_t* masks, int32_t masks_given, void* x_out, float* x_hist, float eps,
                    int32_t act, int32_t act_on_both, float logit_threshold, int32_t grid,
                    void* workspace, int32_t* status, uint64_t* trace, const hc_tp_desc* tp,
                    hc_stream_t stream);

/* Exchange-buffer plumbing for the tensor-parallel stack (host side). */
HC_API int hc_tp_alloc(int64_t bytes, void** ptr);     /* cudaMalloc + zero on the current device */
HC_API int hc_tp_free(void* ptr);
HC_API int hc_ipc_get_handle(void* ptr, uint8_t* handle);          /* 64-byte cudaIpcMemHandle_t */
HC_API int hc_ipc_open(const uint8_t* handle, void** ptr);         /* peer access enabled lazily */
HC_API int hc_ipc_close(void* ptr);

/* ======================================================================= */
/* Batched decode (B tokens through one layer, one fetch set per batch)    */
/* ======================================================================= */

/*
 * hc_union_cold -- the batched form of the id selection of
 * SparseFFNLayer._cold_ids_for (engine.py:274-283): the cold records a batch
 * fetches are the union of its tokens' active masks, restricted to fetch_bits,
 * in ascending neuron-id order.
 *   masks      [batch][token_stride] uint32 active bits, ceil(inter/32) words
 *              per token; fetch_bits, table as in hc_layer_desc
 *   rec_out    [n_records] int32 record indices; count [1] int32 output
 * Single CTA; inter <= 65536.
 */
HC_API int hc_union_cold(const uint32_t* masks, int32_t batch, int64_t token_stride, int32_t inter,
                         const uint32_t* fetch_bits, const int32_t* table, int32_t* rec_out,
                         int32_t* count, hc_stream_t stream);
/*
 * The same for n_layers layers at once (one CTA per layer), when every
 * layer's masks are known up front: layer l reads masks + l * layer_stride,
 * fetch_bits + l * ceil(inter/32), table + l * 65536 and writes
 * rec_out + l * rec_stride, count[l].  flags_out (optional, [n_layers][flag_stride]
 * bytes, flag_stride >= every layer's record count) receives 1 for each record
 * in the union and 0 elsewhere -- the input of the dense cold mode below.
 */
HC_API int hc_union_cold_layers(const uint32_t* masks, int32_t n_layers, int64_t layer_stride, int32_t batch,
                                int64_t token_stride, int32_t inter, const uint32_t* fetch_bits,
                                const int32_t* table, int32_t* rec_out, int64_t rec_stride, int32_t* count,
                                uint8_t* flags_out, int64_t flag_stride, hc_stream_t stream);

/*
 * hc_ffn_batch_layer -- SparseFFNLayer.forward (engine.py:292-312) for a
 * batch of B tokens sharing one fetch set: x_b += sparse_ffn(RMSNorm(x_b))
 * over the layer's hot neurons and the cold records rec[0..*count).
 *   layer      host pointer to the layer's hc_layer_desc (its device pointers
 *              are used; the predictor fields are ignored)
 *   x          [batch][4096] fp32 hidden states, updated in place
 *   rec/count  device cold record list (hc_union_cold), at most max_cold
 *              entries (more sets HC_ERR_RANGE and drops the excess)
 *   packed     the layer's packed copy (hc_batch_pack) or NULL; required
 *              when rec_flags is given
 *   rec_flags  NULL: compute the listed records.  Otherwise dense mode:
 *              every record of the section is streamed from `packed` (one
 *              bulk copy per tile step instead of per-record pieces) and
 *              rec_flags[n_records] (1 = in the fetch set) zeroes the rest --
 *              the same result, cheaper once the union covers a large part of
 *              the section; max_cold is then the section's record count
 *   workspace  hc_ffn_batch_workspace_bytes(n_hot + max_cold) bytes (scratch;
 *              no initial contents needed)
 * Tokens are processed 64 at a time on the tcgen05 tensor cores: every weight
 * byte is read once per 64 tokens.  Operands are f16 (FP8 weights and INT4 q
 * exact; RMSNorm(x), q * group scale and the activations rounded once each),
 * accumulation fp32.  Each down tile is added into x with float reductions,
 * so the last bits can differ between launches.
 */
HC_API int64_t hc_ffn_batch_workspace_bytes(int32_t max_neurons);
/*
 * Profiling hook: later hc_ffn_batch_layer launches write %globaltimer
 * stamps of their gate/up and down kernels into gu / down ([grid][64] uint64,
 * device; NULL = off).  Not for concurrent use.
 */
HC_API int hc_batch_set_trace(uint64_t* gu, uint64_t* down);
HC_API int hc_ffn_batch_layer(const hc_layer_desc* layer, const void* packed, float* x, int32_t batch,
                              const int32_t* rec, const int32_t* count, int32_t max_cold,
                              const uint8_t* rec_flags, float eps, int32_t act, int32_t act_on_both,
                              void* workspace, int32_t* status, hc_stream_t stream);
/*
 * hc_ffn_batch_layer_partial -- the same layer, with its output added into
 * y_out ([batch][4096] fp32, device; the caller zeroes it) instead of x, which
 * is only read.  This is the per-GPU step of the neuron-sharded batched decode
 * (engine.py:184-188: down_proj is linear in the neuron dimension): each GPU
 * passes the descriptor of its share of the layer's hot neurons and cold
 * records, and the partial outputs are summed across GPUs (one all-reduce of
 * [batch][4096] per layer) before x += y.
 */
HC_API int hc_ffn_batch_layer_partial(const hc_layer_desc* layer, const void* packed, const float* x, int32_t batch,
                                      const int32_t* rec, const int32_t* count, int32_t max_cold,
                                      const uint8_t* rec_flags, float eps, int32_t act, int32_t act_on_both,
                                      void* workspace, float* y_out, int32_t* status, hc_stream_t stream);
/*
 * Packed copy of a layer for the dense mode of hc_ffn_batch_layer: the hot
 * rows and every cold record re-laid out once, unit-major, so that each
 * 64-wide K step of a 128-row gate/up tile and each 64-neuron step of a
 * 128-row down tile is one contiguous block (INT4 bytes without the record's
 * 2-byte offset, fp16 scales beside them).  Values are copied bit for bit.
 * hc_batch_pack_bytes: size of the copy; hc_batch_pack: fills it (layer is a
 * host pointer; its hot / cold_records device pointers are read).
 */
HC_API int64_t hc_batch_pack_bytes(int32_t n_hot, int32_t n_records);
HC_API int hc_batch_pack(const hc_layer_desc* layer, void* packed, hc_stream_t stream);

/*
 * hc_xchg_sum -- the one exchange per layer of the neuron-sharded batched
 * decode (the reference's down_proj is linear in the neuron dimension,
 * engine.py:184-188): out += sum over the `size` GPUs of their `part`, in GPU
 * order, so every GPU gets bit-identical sums.  Each GPU stores its partial
 * into every peer's exchange buffer with plain NVLink stores (CUDA IPC
 * mappings from hc_tp_alloc / hc_ipc_open), releases once per CTA and adds to
 * the peers' arrival counters; it then waits (bounded by tp->wait_ns, default
 * 2 s; HC_ERR_TIMEOUT in `status` and `out` untouched on expiry) for all
 * peers.  An ordinary kernel: a CUDA graph can hold it.
 *   part, out   [n] fp32 (16-byte aligned), n % 4 == 0, n <= max_floats
 *   tp          size (2..8), rank, peer_buf (device array of every GPU's
 *               buffer of hc_xchg_buffer_bytes(size, max_floats) bytes, zeroed
 *               once), wait_ns; seq_base is not used: the buffers count the
 *               exchanges themselves, so a CUDA graph can replay the call
 * Every GPU of the group must make the same sequence of calls on its buffers.
 */
HC_API int64_t hc_xchg_buffer_bytes(int32_t size, int64_t max_floats);
HC_API int hc_xchg_sum(const float* part, int64_t n, float* out, int64_t max_floats, const hc_tp_desc* tp,
                       int32_t* status, hc_stream_t stream);

/* ======================================================================= */
/* Decode-step attention projections                                       */
/* ======================================================================= */

/*
 * hc_fp8_gemv -- the batch-1 form of the attention projections F.linear(x, W)
 * in GroupedQueryAttention.forward (engine.py:100-102, :123), whose weights
 * the reference stores as FP8 e4m3 at rest and casts to fp16 for every call
 * (engine.py:77-82): y = W x, reading the e4m3 bytes directly.
 *   w          [rows][cols] e4m3 (row-major, 16-byte aligned); cols == 4096
 *   row_scale  optional [rows] fp32 per-row scale (NULL = 1, the reference's
 *              direct cast)
 *   x          [cols] fp16 (16-byte aligned); y [rows] fp16
 * fp32 accumulation of exact f16 x f16 products; one launch, no workspace.
 */
HC_API int hc_fp8_gemv(const uint8_t* w, const float* row_scale, int64_t rows, int32_t cols, const void* x,
                       void* y, hc_stream_t stream);

/*
 * hc_fp8_gemv_ex -- hc_fp8_gemv with the decoder layer's neighbours fused:
 *   norm_w     optional [cols] fp16 (16-byte aligned): x is first RMS-normalised
 *              (the layer's input_layernorm, engine.py:98-100): the products
 *              use fp16(x * norm_w) and the fp32 sums are scaled by
 *              1 / sqrt(mean(x^2) + eps); NULL = x as given
 *   residual   optional [rows] fp16: y = residual + W x with one rounding (the
 *              decoder layer's x + attention(x), engine.py:421-429); may be y
 *              itself, must not otherwise overlap y
 */
HC_API int hc_fp8_gemv_ex(const uint8_t* w, const float* row_scale, int64_t rows, int32_t cols, const void* x,
                          const void* norm_w, float eps, const void* residual, void* y, hc_stream_t stream);

/*
 * hc_attn_decode -- one token's grouped-query attention of one layer
 * (LlamaAttention.forward for T = 1, engine.py:100-125, rotary embedding
 * engine.py:130-158): RoPE on q and k at position *pos, k / v written into the
 * cache at *pos, causal softmax attention of every query head over cache
 * positions 0..*pos of its key-value head (query head h reads key-value head
 * h / (n_q_heads / n_kv_heads)), out = softmax(q k^T / sqrt(d)) v.
 *   qkv        [(n_q_heads + 2 n_kv_heads) head_dim] fp16: q, k, v before RoPE
 *   cos_t/sin_t [capacity][head_dim / 2] fp32 rotary tables (angle pos x
 *              theta^(-i / (head_dim / 2)))
 *   pos        device int64 scalar (read by the kernel, so a captured graph
 *              replays the step); *pos outside [0, capacity) -> HC_ERR_RANGE
 *              in *status and nothing is written
 *   k_cache / v_cache  this layer's [n_kv_heads][capacity][head_dim] fp16
 *   out        [n_q_heads head_dim] fp16
 * head_dim must be 128 and n_q_heads / n_kv_heads <= 8.  One cluster of 8
 * CTAs per key-value head splits the sequence; the CTAs' partial softmaxes
 * (fp32) are combined through distributed shared memory after a cluster
 * barrier.  No workspace; launches on one cache must not overlap.
 */
HC_API int hc_attn_decode(const void* qkv, const float* cos_t, const float* sin_t, const int64_t* pos,
                          void* k_cache, void* v_cache, int32_t capacity, int32_t n_q_heads, int32_t n_kv_heads,
                          int32_t head_dim, void* out, int32_t* status, hc_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* HOTCOLD_H */
