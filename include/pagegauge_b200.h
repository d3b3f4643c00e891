/*
 * PageGauge-B200: C ABI of the INT8 page-affine paged decode path.
 *
 * Every entry point takes raw device pointers, element strides and sizes, and
 * a cudaStream_t (passed as void*); it validates what it can, launches on the
 * given stream, never allocates device memory, and returns PG_OK or an error
 * code.  pg_last_error() returns the message of the last failure on the
 * calling thread; the messages of the checks that mirror the reference's
 * host validation are kept verbatim so callers can match on them.
 *
 * Fixed geometry: head_dim 128, 16-token pages, NHD page layout
 * [pages, 16, Hkv, 128]; GQA group Hq/Hkv in 1..8.
 *
 * Reference interfaces replaced (paths inside ahmed123hds/PageGauge):
 *   pg_rope_append_fp16          <- rope_append_fp16[_dynamic]
 *                                   tests/page_gauge_append_extension.cu:644-745
 *   pg_rope_append_page_gauge    <- rope_append_page_gauge[_dynamic]
 *                                   tests/page_gauge_append_extension.cu:747-948
 *   pg_exact_tail_merge_center   <- exact_tail_merge_center
 *                                   tests/page_gauge_append_extension.cu:950-1028
 *   pg_decode_plan               <- BatchDecodeWithPagedKVCacheWrapper.plan as
 *                                   called by plan()
 *                                   scripts/benchmark_flashinfer_page_affine_int8.py:363-389
 *   pg_decode_run                <- wrapper.run(q, (k_codes, v_codes), k_scale,
 *                                   v_scale, sm_scale, out=, lse=)
 *                                   scripts/benchmark_flashinfer_page_affine_int8.py:581-590
 *                                   (INT8 segment), the FP16 tail run :591-597,
 *                                   and the single-launch run_decode ABI
 *                                   scripts/page_gauge_heterogeneous_fa2.py:330-379
 *   pg_merge_state_in_place      <- flashinfer.merge_state_in_place
 *                                   scripts/benchmark_page_gauge_transformer.py:2300-2305
 *   pg_quantize_affine_group16   <- quantize_pages (affine_group16)
 *                                   scripts/benchmark_flashinfer_page_affine_int8.py:234-253
 *   pg_quantize_pages            <- quantize_completed_kv_pages
 *                                   scripts/benchmark_page_gauge_overheads.py:208-239
 *                                   and the codes/scales of quantize_page_gauge
 *                                   scripts/benchmark_flashinfer_page_affine_int8.py:256-278
 */
#ifndef PAGEGAUGE_B200_H_
#define PAGEGAUGE_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  PG_OK = 0,
  PG_ERR_INVALID = 1,   /* argument validation failed (message set) */
  PG_ERR_CUDA = 2,      /* a CUDA runtime/driver call failed */
  PG_ERR_CAPACITY = 3   /* a caller-provided buffer is too small */
};

/* Device-side guard codes reported by pg_read_device_error. */
enum {
  PG_DEV_OK = 0,
  PG_DEV_WAIT_TIMEOUT = 1, /* a bounded mbarrier wait gave up */
  PG_DEV_BAD_POSITION = 2, /* device position outside cache / RoPE table */
  PG_DEV_BAD_PAGE_ID = 3   /* page table entry outside the cache */
};

/* Message of the last error on this thread ("" if none). */
const char* pg_last_error(void);

/* ABI version (major*100 + minor). */
int32_t pg_abi_version(void);

/* sizeof of pg_decode_args, pg_gemm_args, pg_segment, pg_plan_info and
 * pg_decode_item as compiled into the library (a binding checks its own
 * structure layouts against these before the first call).                */
int32_t pg_struct_sizes(int64_t* out, int32_t n);

/* Read and clear the device guard word of the current device. */
int32_t pg_read_device_error(int32_t* code_out);

/* Exchange buffer of the tensor-parallel GEMM reduction, for up to
 * tiles_cap output tiles of 64 rows: created zeroed on the current device
 * with a CUDA IPC handle (64 bytes) the other ranks open.                 */
int64_t pg_tp_exchange_bytes(int32_t tiles_cap);
int32_t pg_tp_exchange_create(int32_t tiles_cap, void** buffer_out, void* ipc_handle_out);
int32_t pg_tp_exchange_open(const void* ipc_handle, void** buffer_out);
int32_t pg_tp_exchange_close(void* peer_buffer);
int32_t pg_tp_exchange_destroy(void* buffer);

/* Publish this rank's partial product computed by another GEMM (FP16
 * src [batch, tiles * 64], e.g. cuBLAS's row-parallel o_proj / down_proj
 * output) to every rank's exchange buffer (peers[r] = rank r's buffer as
 * mapped here), so that pg_tp_reduce with PG_TP_PAYLOAD_F16 replaces the
 * all-reduce (and the residual add + RMSNorm after it).  The values travel
 * as FP16 pairs, half the bytes of the FP32 tiles a tensor-parallel
 * pg_skinny_gemm publishes.  Every rank must launch the same sequence.    */
enum {
  PG_TP_PAYLOAD_F32 = 0, /* tiles published by a tensor-parallel pg_skinny_gemm */
  PG_TP_PAYLOAD_F16 = 1  /* tiles published by pg_tp_publish */
};
int32_t pg_tp_publish(void* const* peers, int32_t world, int32_t rank, int32_t tiles_cap,
                      int32_t tiles, int32_t batch, const void* src, int64_t src_stride,
                      void* stream);

/* Consume a tensor-parallel GEMM's published tiles on this rank: wait
 * (about a second at most, then PG_DEV_WAIT_TIMEOUT, and a row whose tiles
 * did not all arrive stores nothing, so residual and out keep their
 * contents and the step can be repeated) until all `world`
 * ranks' tiles of the `tiles` output tiles have arrived in this rank's
 * `exchange` buffer, sum them in rank order (FP32; identical on every
 * rank) and, per batch row (batch = the GEMM's rows):
 *   residual != NULL: residual = f16(residual + f16(sum)), then out =
 *                     RMSNorm(residual) with norm_weight (MistralRMSNorm),
 *                     or out = residual without it
 *   residual == NULL: out = f16(sum)
 * payload names the publisher of the tiles: PG_TP_PAYLOAD_F32 after a
 * tensor-parallel pg_skinny_gemm, PG_TP_PAYLOAD_F16 after pg_tp_publish
 * (every rank of one exchange uses the same publisher).                   */
int32_t pg_tp_reduce(const void* exchange, int32_t world, int32_t tiles_cap, int32_t tiles,
                     int32_t batch, void* residual, int64_t residual_stride,
                     const void* norm_weight, float eps, void* out, int64_t out_stride,
                     int32_t payload, void* stream);

/* Device address of a page-locked, mapped host buffer (cudaHostAlloc /
 * pinned memory): kernels may take it wherever an input or output pointer
 * is expected and then read or write the host buffer directly over the
 * host link (zero copy).  Fails for memory that is not mapped.            */
int32_t pg_host_device_pointer(const void* host, void** device_out);

/* ---------------------------------------------------------------------- */
/* Fused RoPE + FP16 append (the comparator path).                         */
/* query [B,Hq,128], key/value [B,Hkv,128] fp16 with contiguous heads;      */
/* cosine/sine: one [128] row (device_position == NULL, position used) or   */
/* a [rope_rows,128] table indexed by *device_position.                     */
/* key_pages/value_pages fp16 [num_pages,16,Hkv,128], request-major.        */
int32_t pg_rope_append_fp16(const void* query, const void* key,
                            const void* value, const void* cosine,
                            const void* sine, void* rotated_query,
                            void* key_pages, void* value_pages,
                            int64_t query_batch_stride,
                            int64_t key_batch_stride,
                            int64_t value_batch_stride, int32_t batch,
                            int32_t query_heads, int32_t kv_heads,
                            int64_t num_pages, int64_t position,
                            const int32_t* device_position,
                            int64_t rope_row_stride, int64_t rope_rows,
                            void* stream);

/* Fused RoPE + centred append into the exact FP16 ring + INT8 finalisation
 * of the page closed by this token (codes [code_pages,16,Hkv,128] int8,
 * scales [code_pages,Hkv] fp16).  centers: [B,Hkv,128] (center_batch_stride
 * = Hkv*128) or one [Hkv,128] shared centre for batch one (stride 0).     */
int32_t pg_rope_append_page_gauge(
    const void* query, const void* key, const void* value,
    const void* cosine, const void* sine, const void* key_center,
    const void* value_center, void* rotated_query, void* exact_key_pages,
    void* exact_value_pages, void* key_codes, void* value_codes,
    void* key_scales, void* value_scales, int64_t query_batch_stride,
    int64_t key_batch_stride, int64_t value_batch_stride,
    int64_t center_batch_stride, int32_t batch, int32_t query_heads,
    int32_t kv_heads, int64_t exact_pages, int64_t code_pages,
    int64_t exact_sink_pages, int64_t position,
    const int32_t* device_position, int64_t rope_row_stride,
    int64_t rope_rows, void* stream);

/* Per-request-position forms of the two appends above: positions is a
 * device int32 [B] tensor (request r appends at positions[r]) and
 * cosine/sine are [rope_rows,128] tables.  A ragged serving batch has one
 * position per request; the reference's extension takes one position for
 * the whole batch, and its per-request append is the Triton
 * append_finalize_page_gauge (scripts/benchmark_page_gauge_overheads.py:113-205,
 * page ids and in-page offsets per request, no RoPE).  An out-of-range
 * position skips that request and sets the device guard word.              */
int32_t pg_rope_append_fp16_batched(const void* query, const void* key,
                                    const void* value, const void* cosine,
                                    const void* sine, void* rotated_query,
                                    void* key_pages, void* value_pages,
                                    int64_t query_batch_stride,
                                    int64_t key_batch_stride,
                                    int64_t value_batch_stride, int32_t batch,
                                    int32_t query_heads, int32_t kv_heads,
                                    int64_t num_pages, const int32_t* positions,
                                    int64_t rope_row_stride, int64_t rope_rows,
                                    void* stream);

/* inputs_ready != 0 declares that no kernel earlier in the stream writes
 * query / key / value (e.g. rows the host wrote into page-locked memory
 * before the call): the kernel then requests them before waiting for the
 * previous kernel, so a trip over the host link overlaps that kernel's
 * tail.  0 (the reference's behaviour): everything after the wait.        */
int32_t pg_rope_append_page_gauge_batched(
    const void* query, const void* key, const void* value,
    const void* cosine, const void* sine, const void* key_center,
    const void* value_center, void* rotated_query, void* exact_key_pages,
    void* exact_value_pages, void* key_codes, void* value_codes,
    void* key_scales, void* value_scales, int64_t query_batch_stride,
    int64_t key_batch_stride, int64_t value_batch_stride,
    int64_t center_batch_stride, int32_t batch, int32_t query_heads,
    int32_t kv_heads, int64_t exact_pages, int64_t code_pages,
    int64_t exact_sink_pages, const int32_t* positions,
    int64_t rope_row_stride, int64_t rope_rows, int32_t inputs_ready, void* stream);

/* The fused append on the served pool layout (the device side of the
 * serving decode metadata, experiments/mlsys2027/serving_v1/pagegauge_vllm/
 * decode_metadata.py:28-35, whose columns are "for a future device ABI"):
 * per batch row r, positions[r], token_slots[r] = physical code page * 16 +
 * token (pool planes [num_code_pages, 16, Hkv, 128]), exact_slots[r] = exact
 * sidecar page * 16 + token ([num_exact_pages, 16, Hkv, 128], centred FP16)
 * and center_rows[r] = the request's lease slot in the centre sidecars
 * [num_centers, Hkv, 128].  A closing page's codes go to its physical code
 * page; the row's value centre is copied to value_center_out [B, Hkv, 128]
 * for the decode.  Rows whose slots disagree with their position or fall
 * outside the pool are skipped and reported (PG_DEV_BAD_PAGE_ID).          */
int32_t pg_rope_append_page_gauge_served(
    const void* query, const void* key, const void* value, const void* cosine,
    const void* sine, const void* key_center, const void* value_center,
    void* rotated_query, void* exact_key_pages, void* exact_value_pages, void* key_codes,
    void* value_codes, void* key_scales, void* value_scales, void* value_center_out,
    int64_t query_batch_stride, int64_t key_batch_stride, int64_t value_batch_stride,
    int32_t batch, int32_t query_heads, int32_t kv_heads, int64_t num_code_pages,
    int64_t num_exact_pages, int64_t num_centers, const int32_t* positions,
    const int32_t* token_slots, const int32_t* exact_slots, const int32_t* center_rows,
    int64_t rope_row_stride, int64_t rope_rows, void* stream);

/* Zero the four planes of `count` pool pages (page_ids device int32), the
 * served pool's zero_physical_pages
 * (experiments/mlsys2027/serving_v1/pagegauge_vllm/cache_views.py:42-62). */
int32_t pg_zero_pool_pages(void* key_codes, void* value_codes, void* key_scales,
                           void* value_scales, int64_t num_pages, int32_t kv_heads,
                           const int32_t* page_ids, int32_t count, void* stream);

/* Exact FP16 tail attention merged into (old_output, old_lse) in place,
 * plus the value centre.  exact_page_indices [B*n] int32,
 * exact_last_page_len [B] int32 (device), old_lse base 2 [B,Hq].          */
int32_t pg_exact_tail_merge_center(
    const void* query, const void* exact_key_pages,
    const void* exact_value_pages, int64_t exact_pages_total,
    const int32_t* exact_page_indices, int64_t num_indices,
    const int32_t* exact_last_page_len, void* old_output, float* old_lse,
    const void* value_center, int64_t center_batch_stride, int32_t batch,
    int32_t query_heads, int32_t kv_heads, double sm_scale, void* stream);

/* ---------------------------------------------------------------------- */
/* Split-KV paged decode.  Segment 0: INT8 codes + per-(page, head) FP16     */
/* scales.  Segment 1: FP16 pages (exact tail ring or a plain FP16 cache).  */
typedef struct pg_decode_item {
  int32_t request;
  int32_t head_seg;  /* kv_head | (segment << 16) */
  int32_t idx_begin; /* absolute offset of the first page id */
  int32_t count;     /* pages; bit 31: holds the request's last page */
} pg_decode_item;

typedef struct pg_segment {
  const void* k_cache; /* NULL: segment absent */
  const void* v_cache;
  int64_t num_pages;             /* pages allocated in k_cache/v_cache */
  const int32_t* indices;        /* device page ids */
  const int32_t* last_page_len;  /* device [B] */
  const void* k_scale;           /* fp16 [num_pages, Hkv], segment 0 */
  const void* v_scale;
} pg_segment;

typedef struct pg_plan_info {
  int64_t num_items;
  int32_t max_items_per_head;
  int32_t single_item_per_head; /* 1: run may use the final epilogue */
  int32_t split_pages[2];       /* pages per work item chosen per segment */
  int32_t warps_per_cta;
} pg_plan_info;

/* Host-only planner.  indptr_s (host, [B+1]) gives each request's page-id
 * range in segment s (NULL: absent).  split_pages_s = pages per work item
 * (0: automatic, sized for one wave on num_sms SMs).  Writes at most
 * items_capacity items and item_off[B*Hkv+1]; returns PG_CAPACITY if the
 * list does not fit.                                                       */
int32_t pg_decode_plan(int32_t batch, int32_t kv_heads,
                       const int32_t* indptr0, const int32_t* indptr1,
                       int32_t split_pages0, int32_t split_pages1,
                       int32_t num_sms, int32_t warps_per_cta,
                       pg_decode_item* items, int64_t items_capacity,
                       int32_t* item_off, pg_plan_info* info);

typedef struct pg_decode_args {
  const void* q; /* fp16 [B, Hq, 128], last dim contiguous */
  int64_t q_stride_b, q_stride_h;
  int32_t batch, kv_heads, group;
  float sm_scale;
  pg_segment seg[2];
  const pg_decode_item* items; /* device, from pg_decode_plan */
  const int32_t* item_off;     /* device [B*Hkv+1] */
  int32_t num_items;
  int32_t warps_per_cta;
  float* part_o;   /* device workspace [num_items*group*128] */
  float* part_lse; /* device workspace [num_items*group] */
  int32_t final_mode; /* 1: one item per (request, head): no merge launch */
  void* out;          /* fp16 [B, Hq, 128] */
  int64_t out_stride_b, out_stride_h;
  float* lse_out; /* base-2 [B, Hq] or NULL */
  const void* extra_o; /* optional state merged in (may alias out) */
  int64_t extra_stride_b, extra_stride_h;
  const float* extra_lse;
  const void* value_center; /* fp16 [B,Hkv,128] or NULL */
  int64_t vc_stride_b;
  int32_t stage_mask; /* 0 or 3: split + merge; 1: split kernel only;
                         2: merge kernel only (stages on separate calls) */
  int32_t* merge_sem; /* device [B*Hkv] int32, zero when idle (the planner's
                         workspace provides it); non-NULL: the split kernel
                         merges each head in its last CTA (one launch, no
                         merge kernel).  Launches sharing it must not run
                         concurrently. */
  int32_t cluster;    /* with merge_sem: 2..8 groups the CTAs in thread-block
                         clusters of this many consecutive work items that
                         merge through distributed shared memory (the single
                         launch of the heterogeneous run_decode ABI,
                         scripts/page_gauge_heterogeneous_fa2.py:286-379);
                         0 or 1: last-CTA merge */
  int32_t representation; /* 0: PageGauge (seg[0] scales fp16 [pages, Hkv]);
                             1: affine_group16 (seg[0].k_scale / v_scale are
                             fp16 [pages, Hkv, 8] group scales, k_bias /
                             v_bias the group biases; 16-byte aligned) -- the
                             make_affine_wrapper run(q, (k_codes, v_codes),
                             k_bias, k_scale, v_bias, v_scale, sm_scale) of
                             scripts/benchmark_flashinfer_page_affine_int8.py:166-189, :567-578 */
  const void* k_bias;
  const void* v_bias;
  int32_t int8_after_wait; /* 0: the INT8 tiles are requested before the
                              kernel waits for the previous kernel in the
                              stream (programmatic dependent launch), which
                              overlaps them with its drain; correct only if
                              none of the kernels that may still run wrote
                              those pages.  1: request them after that wait.
                              Set it when a page closed by an append is read
                              as INT8 by the next step's decode (a one-page
                              exact ring), where the append of the previous
                              step may still be running. */
} pg_decode_args;

int32_t pg_decode_run(const pg_decode_args* args, void* stream);

/* Clusters of `cluster` decode CTAs (of `warps` warps) the current GPU can
 * hold at once: the single-launch plan fits one wave when its padded item
 * count is at most cluster * *out.                                        */
int32_t pg_decode_max_clusters(int32_t warps, int32_t cluster, int32_t* out);

/* Allocation-free variant of pg_decode_plan + pg_decode_run (no counterpart
 * in the reference).  For callers that cannot allocate device memory - a
 * plugin inside a host process whose allocator owns the GPU, or a path that
 * must not allocate while it runs - the work list, the per-head item ranges
 * and the split partial states live in one file-scope device array of
 * 8 MiB inside the library instead of a caller workspace.  The caller passes
 * inputs and outputs in `args` (items, item_off, num_items, part_o,
 * part_lse, final_mode and merge_sem are ignored) plus the host indptr
 * arrays pg_decode_plan takes.  Limits: at most 4096 work items and 8192
 * (request, kv head) pairs, and the partial states must fit the array
 * (about 2 KiB per item at GQA group 4); larger plans fail with
 * PG_ERR_CAPACITY and a message.  No cudaMalloc/cudaFree is called.  The
 * first call on each device looks up the array's device address.  Each
 * call copies its plan from host memory, so a call on a stream that is
 * being captured is refused (PG_ERR_INVALID) before anything is enqueued.
 * Calls on one device share that device's
 * array and it keeps the last call's contents (nothing in it has to start
 * at zero: every call rewrites what it reads); two calls that run at the
 * same time on one GPU, e.g. on two streams, race on it. */
int32_t pg_decode_static(const pg_decode_args* args, const int32_t* indptr0,
                         const int32_t* indptr1, int32_t split_pages0,
                         int32_t split_pages1, int32_t num_sms, void* stream);

/* (v_a, s_a) <- merge((v_a, s_a), (v_b, s_b)); rows of 128 fp16, lse base 2. */
int32_t pg_merge_state_in_place(void* v_a, float* s_a, const void* v_b,
                                const float* s_b, int64_t rows,
                                int64_t va_row_stride, int64_t vb_row_stride,
                                void* stream);

/* Bulk completed-page quantisation: fp32 centring (no FP16 rounding),
 * scale = f16(max(absmax/127, 2^-20)), rounding 0 = half away from zero
 * (prefill quantiser), 1 = half to even (torch.round).  value,
 * value_center, value_codes and value_scales may all be NULL: key only. */
int32_t pg_quantize_pages(const void* key, const void* value,
                          const void* key_center, const void* value_center,
                          int64_t pages_per_center, void* key_codes,
                          void* value_codes, void* key_scales,
                          void* value_scales, int64_t num_pages,
                          int32_t kv_heads, int32_t rounding, void* stream);

/* affine_group16 bulk quantiser (quantize_pages,
 * scripts/benchmark_flashinfer_page_affine_int8.py:234-253), bit-exact:
 * values fp16 [pages, 16, Hkv, 128] -> codes int8 (same shape), bias and
 * scale fp16 [pages, Hkv, 8] (one pair per 16-dim group), reconstructed fp16
 * (same shape as values; NULL to skip).                                   */
int32_t pg_quantize_affine_group16(const void* values, int64_t num_pages, int32_t kv_heads,
                                   void* codes, void* bias, void* scale, void* reconstructed,
                                   void* stream);

/* ---------------------------------------------------------------------- */
/* Decoder-layer element-wise steps around the attention path (the Mistral   */
/* layer body of scripts/benchmark_page_gauge_transformer.py:2754-2804).    */

/* Weight-streaming skinny GEMM of the decoder projections,
 * Y[b, n] = sum_k X[b, k] W[n, k] for batch <= 32 rows (FP16 in, FP32
 * accumulation), split over the GPU "stream-K" (equal k-block ranges per
 * CTA, the last CTA of a split tile finishes it in a fixed order, so
 * results are deterministic), with the layer's element-wise step fused:
 *   mode 0  y = f16(acc)
 *   mode 1  residual = f16(residual + f16(acc))         (o_proj, down_proj)
 *   mode 2  y[b, j] = f16(f16(silu(f16(acc[b, j]))) * f16(acc[b, n/2 + j]))
 *           for the packed gate|up projection (rows [0, n/2) gate, rest up).
 * w is the weight in the packed layout pg_pack_weight writes (one 8 KB
 * block per 64 rows x 64 k, 128-byte swizzled; ldw is ignored), so each
 * pipeline stage's weights are one contiguous bulk copy.
 * The reference runs these through cuBLAS (F.linear in
 * scripts/benchmark_page_gauge_transformer.py:2754-2804).  partials and
 * counters are caller-owned scratch sized by pg_skinny_gemm_workspace;
 * counters must be zero before the first call and are left zero.  pdl = 1
 * launches as a programmatic dependent: weights are requested before the
 * previous kernel in the stream has finished, activations after.         */
typedef struct pg_gemm_args {
  const void* w;       /* [n, k] fp16 */
  int64_t ldw;
  const void* x;       /* [batch, k] fp16 */
  int64_t ldx;
  void* y;             /* mode 0: [batch, n]; mode 2: [batch, n/2] */
  int64_t ldy;
  void* residual;      /* mode 1: [batch, n], updated in place */
  int64_t ldr;
  int32_t n, k, batch, mode;
  int32_t grid;        /* CTAs; 0: all resident slots */
  int32_t pdl;
  float* partials;
  int64_t partial_floats;
  int32_t* counters;
  int32_t num_counters;
  const void* norm_weight; /* fp16 [k] or NULL: the input rows are first
                              RMS-normalised, f16(w * f16(x * rsqrt(mean(x^2)
                              + eps))) (MistralRMSNorm), inside the GEMM */
  float norm_eps;
  /* Tensor parallelism (tp_world 2..8, mode 0): the GEMM computes this
   * rank's partial product and publishes every finished FP32 tile into
   * every rank's exchange buffer (NVLink peer stores; tp_peers[r] = rank
   * r's buffer as mapped here, from pg_tp_exchange_create / _open) with an
   * arrival flag; it writes no y.  pg_tp_reduce, launched next on each
   * rank, sums the ranks' tiles and applies the epilogue: the row-parallel
   * projection and its all-reduce without a collective library
   * (o_proj / down_proj, scripts/benchmark_page_gauge_transformer.py:
   * 2754-2804 under TP).  Every rank must launch the same sequence.       */
  int32_t tp_world, tp_rank, tp_tiles_cap;
  void* tp_peers[8];
} pg_gemm_args;

/* Pack W [n, k] (row stride ld, FP16) for pg_skinny_gemm with the same
 * mode (silu_mul pairs gate row j with up row n/2 + j in one tile); out
 * holds n * k halves.                                                     */
int32_t pg_pack_weight(const void* w, int64_t ld, int32_t n, int32_t k, int32_t mode, void* out,
                       void* stream);

int32_t pg_skinny_gemm_workspace(int32_t n, int32_t k, int32_t batch, int32_t mode,
                                 int32_t grid, int32_t num_sms, int64_t* partial_floats,
                                 int32_t* counters);
int32_t pg_skinny_gemm(const pg_gemm_args* args, void* stream);

/* residual = f16(residual + delta) in place (delta may be NULL), then
 * out = f16(weight * f16(residual * rsqrt(mean(residual^2) + eps))), FP32
 * reduction; rows x hidden FP16, hidden a multiple of 8 up to 16384.       */
int32_t pg_add_rmsnorm(void* residual, const void* delta, const void* weight, void* out,
                       int32_t rows, int32_t hidden, int64_t residual_stride,
                       int64_t delta_stride, int64_t out_stride, float eps, void* stream);

/* out[r, i] = f16(f16(silu(gate[r, i])) * up[r, i]) for gate_up rows laid
 * out as gate | up (the packed gate_up projection).                        */
int32_t pg_silu_mul(const void* gate_up, void* out, int32_t rows, int32_t features,
                    int64_t in_stride, int64_t out_stride, void* stream);

/* Greedy token of each row of FP16 logits [rows, cols] (row stride ld):
 * out_idx[r] = index_offset + argmax (ties to the lowest index), out_val
 * (optional) the maximum as FP32.  index_offset places a vocabulary slice
 * of a tensor-parallel LM head in the full vocabulary.                    */
int32_t pg_argmax_rows(const void* logits, int64_t ld, int32_t rows, int32_t cols,
                       int64_t index_offset, float* out_val, int64_t* out_idx, void* stream);

/* positions[r] += advance; last_page_len[r] = positions[r] % 16 + 1 (NULL
 * last_page_len: positions only).  Keeps a captured decode step's device
 * position and exact-tail length current without host copies.             */
int32_t pg_step_positions(int32_t* positions, int32_t* last_page_len, int32_t batch,
                          int32_t advance, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* PAGEGAUGE_B200_H_ */
