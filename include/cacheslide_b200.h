/*
 * cacheslide_b200.h -- C ABI of libcacheslide_sm100.so, the B200 (sm_100a)
 * implementation of CacheSlide's reuse-time attention hot path.
 *
 * Every entry point takes plain device pointers, element strides, sizes and a
 * cudaStream_t (passed as void*), enqueues its kernels on that stream and
 * returns immediately with a cs_status code for host-side argument errors.
 * Data-dependent failures (a slot outside the arena, a non-finite WCA value,
 * an invalid contextual path, ...) are reported through an optional device
 * status word: kernels OR the CS_ST_* bits below into *status and skip the
 * offending access, they never trap.  The caller reads the word after the
 * stream has drained and maps it to the reference's exception types.
 *
 * Tensor layouts follow the reference package `cacheslide_vllm`:
 *   query [token, q_head, dim], key/value [token, kv_head, dim],
 *   positions [head, query, key], learned table E [dim, npos],
 *   native paged KV cache [block, kv_head, block_offset, 2*dim] (K | V).
 * The innermost dimension of q/k/v/out must be contiguous unless a stride for
 * it is taken explicitly.
 */
#ifndef CACHESLIDE_B200_H
#define CACHESLIDE_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define CS_API __attribute__((visibility("default")))
#else
#define CS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ codes */
typedef enum {
  CS_OK = 0,
  CS_ERR_INVALID = 1,     /* bad argument; nothing was enqueued            */
  CS_ERR_CUDA = 2,        /* a CUDA runtime call or launch failed          */
  CS_ERR_UNSUPPORTED = 3, /* shape/dtype combination this build lacks      */
  CS_ERR_TOO_LARGE = 4    /* needs more than a fixed internal capacity     */
} cs_status;

typedef enum { CS_F32 = 0, CS_F16 = 1, CS_BF16 = 2, CS_F64 = 3 } cs_dtype;

/* bits OR-ed into the optional device status word */
#define CS_ST_SLOT_RANGE (1 << 0)     /* slot outside native + sidecar range   */
#define CS_ST_NONFINITE (1 << 1)      /* non-finite WCA arithmetic / K,V       */
#define CS_ST_LOGIT_NONFINITE (1 << 2)/* attention logits not finite           */
#define CS_ST_POS_RANGE (1 << 3)      /* substituted position not in [0,npos-1]*/
#define CS_ST_PATH_NEG (1 << 4)       /* strict path: negative count           */
#define CS_ST_PATH_AVAIL (1 << 5)     /* strict path: count > available gates  */
#define CS_ST_PATH_INCR (1 << 6)      /* strict path: increasing along keys    */
#define CS_ST_PATH_GAP (1 << 7)       /* strict path: drop > coordinate gap    */
#define CS_ST_TIMEOUT (1 << 8)        /* a bounded device wait expired         */
#define CS_ST_INPUT_NONFINITE (1 << 9)/* non-finite query/key/value element    */

/* ------------------------------------------------------- paged KV arena */
/*
 * One request/layer view of the native paged cache plus its sidecar.
 * Replaces the tensor state of `NativePagedKV` (paged.py:57-128): slot s <
 * num_blocks*block_size addresses cache[s / bs, :, s % bs, :] with K in the
 * first head_dim elements and V in the next; s >= that addresses sidecar row
 * s - num_blocks*block_size (paged.py:205-240).  All strides are in elements
 * and may describe a non-contiguous view; the innermost stride may be != 1.
 */
typedef struct {
  void* cache;
  int64_t num_blocks, kv_heads, block_size, head_dim;
  int64_t stride_block, stride_head, stride_offset, stride_elem;
  void* side_k; /* [side_capacity, kv_heads, head_dim] or NULL */
  void* side_v;
  int64_t side_capacity;
  int64_t side_stride_row, side_stride_head, side_stride_elem;
  int32_t dtype; /* cs_dtype of cache and sidecar */
} cs_paged_kv;

/*
 * SLIDE gather: out_k/out_v[r] = record of slots[r] (caller order).
 * Replaces NativePagedKV.gather (paged.py:433-472).  out rows are
 * [n, kv_heads, head_dim] with the given row/head strides (elem stride 1).
 */
CS_API int cs_slide_gather(const cs_paged_kv* kv, const int64_t* slots, int64_t n,
                    void* out_k, void* out_v, int64_t out_stride_row,
                    int64_t out_stride_head, int32_t* status, void* stream);

/*
 * SLIDE scatter: record of slots[r] = (k, v)[rows ? rows[r] : r].
 * Replaces NativePagedKV._write_slots (paged.py:205-240) including the
 * `key[selected]` row selection of promote/update (paged.py:300-312, 421-426).
 */
CS_API int cs_slide_scatter(const cs_paged_kv* kv, const int64_t* slots,
                     const int64_t* rows, int64_t n, const void* k,
                     const void* v, int64_t in_stride_row,
                     int64_t in_stride_head, int32_t* status, void* stream);

/*
 * SLIDE relocate: record of dst_slots[r] = record of src_slots[r], copied
 * paged-to-paged without a dense staging buffer (promotion into the sidecar,
 * canonical mirror writes; paged.py:279-328, 474-524).  Source and
 * destination sets must not overlap.
 */
CS_API int cs_slide_relocate(const cs_paged_kv* kv, const int64_t* src_slots,
                      const int64_t* dst_slots, int64_t n, int32_t* status,
                      void* stream);

/*
 * One request of a batched SLIDE scatter: the arguments of cs_slide_scatter
 * that differ between requests (strides in elements).
 */
typedef struct {
  const int64_t* slots;
  const int64_t* rows; /* or NULL */
  int64_t n;
  const void* k;
  const void* v;
  int64_t in_stride_row, in_stride_head;
  int32_t* status;
} cs_slide_scatter_item;

/*
 * cs_slide_scatter for `count` requests into one shared paged pool, in one
 * launch per 64 requests: the baseline-snapshot writes of every
 * request of a step (NativePagedKV.load_baseline -> _write_slots,
 * paged.py:205-240, once per request in the reference).  The requests'
 * slot sets must be disjoint.
 */
CS_API int cs_slide_scatter_batch(const cs_paged_kv* kv, const cs_slide_scatter_item* items,
                                  int32_t count, void* stream);

/*
 * Page images for the dirty-page writeback that NativePagedKV.spill_order
 * only advises (paged.py:530-559, slide.py:119-156): page q of `pages` is the
 * block_size consecutive slots pages[q] * block_size .. + block_size - 1 (a
 * native block, or sidecar rows past the native pool), and its image is one
 * native block [kv_head][block_size][2*head_dim] (K then V per record) at
 * `image` + q * kv_heads * block_size * 2*head_dim elements.  Pack copies
 * the pages' records into the images (for a host copy), unpack writes
 * images back into the same slots (a reload).  Any view strides; slots
 * past the end of a partial sidecar page read as zeros; a page outside the
 * arena sets CS_ST_SLOT_RANGE and is skipped.
 */
CS_API int cs_slide_pack_pages(const cs_paged_kv* kv, const int64_t* pages, int64_t count,
                               void* image, int32_t* status, void* stream);
CS_API int cs_slide_unpack_pages(const cs_paged_kv* kv, const int64_t* pages, int64_t count,
                                 const void* image, int32_t* status, void* stream);

/* ------------------------------------------------------------------ WCA */
/*
 * Per-token squared deviation and adaptation weight in float64
 * (wca.py:55-93): dev[r] = sum_{h,d} (fresh[r] - cached[c])^2,
 * alpha[r] = dev[r] / (sum cached[c]^2 + epsilon), clamped to [0,1] when
 * `clamp`; c = cached_rows ? cached_rows[r] : r.  Either output may be NULL.
 * Non-finite inputs or results set CS_ST_NONFINITE.
 */
CS_API int cs_wca_deviation(const void* cached, int64_t c_stride_row,
                     int64_t c_stride_head, const int64_t* cached_rows,
                     const void* fresh, int64_t f_stride_row,
                     int64_t f_stride_head, int64_t n, int64_t heads,
                     int64_t dim, int32_t dtype, double epsilon, int32_t clamp,
                     double* dev_out, double* alpha_out, int32_t* status,
                     void* stream);

/*
 * Mean-head cosine (wca.py:96-112): per head, amax-scaled unit vectors,
 * dot clamped to [-1,1], mean over heads; b row = b_rows ? b_rows[r] : r.
 */
CS_API int cs_wca_cosine(const void* a, int64_t a_stride_row, int64_t a_stride_head,
                  const void* b, int64_t b_stride_row, int64_t b_stride_head,
                  const int64_t* b_rows, int64_t n, int64_t heads, int64_t dim,
                  int32_t dtype, double epsilon, double* cos_out,
                  int32_t* status, void* stream);

/*
 * Row sums of one KV-head shard, for KV-head tensor parallelism (the C5
 * layout: each rank holds `heads` of `heads_total` heads).  Replaces the
 * head reductions inside squared_deviation / adaptation_weight /
 * mean_head_cosine (wca.py:55-112) with per-shard partial sums that the
 * caller all-reduces across ranks:
 *   dev[r] = sum over the shard's heads and dims of (fresh[r] - cached[c])^2,
 *   nrm[r] = sum of cached[c]^2,
 *   cos[r] = sum over the shard's heads of the head cosine / heads_total,
 * with c = cached_rows ? cached_rows[r] : r.  Any output may be NULL.
 */
CS_API int cs_wca_row_sums(const void* cached, int64_t c_stride_row,
                    int64_t c_stride_head, const int64_t* cached_rows,
                    const void* fresh, int64_t f_stride_row,
                    int64_t f_stride_head, int64_t n, int64_t heads,
                    int64_t dim, int32_t dtype, int64_t heads_total,
                    double* dev_out, double* nrm_out, double* cos_out,
                    int32_t* status, void* stream);

/*
 * Adaptation weights from complete (all-reduced) row sums (wca.py:65-93,
 * 152-191): alpha[r] = dev[r] / (nrm[r] + epsilon), clamped to [0,1] when
 * `clamp`; with `candidate` (then `reused` and `counts_out` are required):
 * candidate = reused & dev > 0, counts_out[0] = |reused|,
 * counts_out[1] = |candidate|.  alpha_out may be NULL.
 */
CS_API int cs_wca_weights(const double* dev, const double* nrm, int64_t n,
                   double epsilon, int32_t clamp, const uint8_t* reused,
                   double* alpha_out, uint8_t* candidate, int64_t* counts_out,
                   int32_t* status, void* stream);

/*
 * Block radix top-k (wca.py:202-215): among tokens with available[i] != 0,
 * pick the `slots` largest keys[i] (float64, >= 0), descending with ties to the
 * lower index, exactly like a stable descending argsort.  Sets selected[i]=1
 * for each pick, writes the picks in that order to chosen_out (may be NULL)
 * and their number to *count_out (device int64, may be NULL).
 */
CS_API int cs_wca_select_topk(const double* keys, const uint8_t* available, int64_t n,
                       int64_t slots, uint8_t* selected, int64_t* chosen_out,
                       int64_t* count_out, int32_t* status, void* stream);

/*
 * WCA initialize reductions (wca.py:152-191): deviation, alpha, candidate =
 * reused & dev > 0, counts_out[0] = |reused|, counts_out[1] = |candidate|;
 * selected/removed (may be NULL) are cleared, as a fresh state starts.
 * cached/fresh are full [n, heads, dim] layers.
 */
CS_API int cs_wca_initialize(const void* cached, int64_t c_stride_row,
                      int64_t c_stride_head, const void* fresh,
                      int64_t f_stride_row, int64_t f_stride_head, int64_t n,
                      int64_t heads, int64_t dim, int32_t dtype,
                      const uint8_t* reused, double epsilon, int32_t clamp,
                      double* dev_out, double* alpha_out, uint8_t* candidate,
                      uint8_t* selected, uint8_t* removed,
                      int64_t* counts_out, int32_t* status, void* stream);

/*
 * Fused WCA update for the active rows (wca.py:217-304), one pass:
 *   old = cached[indices[r]], next_alpha[r] = adaptation weight(old, fresh[r]),
 *   used = mandatory[indices[r]] ? 1 : (same_layer ? next_alpha[r]
 *                                                   : alpha[indices[r]]),
 *   fused = used*fresh + (1-used)*old  (float64, cast to dtype),
 *   cosine[r] = mean-head cosine(fresh_k[r], old_k) when cos_out != NULL.
 * fused rows go to fused_k/fused_v (dense [a, heads, dim], may be NULL) and,
 * when `kv` is non-NULL, straight into the paged slots `slots[r]` (blend +
 * scatter; replaces WCAState.update + NativePagedKV.update_selected's
 * writes).  Non-finite fused values set CS_ST_NONFINITE.
 */
CS_API int cs_wca_update(const void* cached_k, const void* cached_v,
                  int64_t c_stride_row, int64_t c_stride_head,
                  const void* fresh_k, const void* fresh_v,
                  int64_t f_stride_row, int64_t f_stride_head,
                  const int64_t* indices, int64_t a, int64_t heads, int64_t dim,
                  int32_t dtype, const double* alpha, const uint8_t* mandatory,
                  int32_t same_layer, double epsilon, int32_t clamp,
                  void* fused_k, void* fused_v, double* next_alpha_out,
                  double* used_alpha_out, double* cos_out,
                  const cs_paged_kv* kv, const int64_t* slots, int32_t* status,
                  void* stream);

/*
 * WCA commit (wca.py:274-287 and 345-366): alpha[indices[r]] = next_alpha[r];
 * rows with selected[idx] and metric < threshold (metric = cos, or 1-cos when
 * distance_mode) are removed (selected=0, candidate=0, removed=1; listed in
 * removed_out in index order, count in counts_out[0]); then the free budget
 * slots are promoted by cs_wca_select_topk semantics over
 * candidate & !selected & !removed (listed in promoted_out, count in
 * counts_out[1]).  cos may be NULL (no gate at this layer).
 */
CS_API int cs_wca_commit(const int64_t* indices, int64_t a, const double* next_alpha,
                  const double* cos, double threshold, int32_t distance_mode,
                  int64_t n, int64_t budget, const double* initial_dev,
                  double* alpha, uint8_t* candidate, uint8_t* selected,
                  uint8_t* removed, int64_t* removed_out,
                  int64_t* promoted_out, int64_t* counts_out, int32_t* status,
                  void* stream);

/*
 * Batched WCA: the per-request calls of one step (one WCAState per request
 * in the reference, wca.py:152-366) as one launch per 64 requests.  Each
 * item holds the arguments of the single call
 * that differ between requests; the shared ones are function arguments.
 * Results are identical to `count` single calls.
 */
typedef struct {
  const void* cached;
  int64_t c_stride_row, c_stride_head;
  const void* fresh;
  int64_t f_stride_row, f_stride_head;
  int64_t n;
  const uint8_t* reused;
  double* dev_out;
  double* alpha_out;
  uint8_t* candidate;
  uint8_t* selected; /* or NULL */
  uint8_t* removed;  /* or NULL */
  int64_t* counts_out;
  int32_t* status;
} cs_wca_initialize_item;

CS_API int cs_wca_initialize_batch(const cs_wca_initialize_item* items, int32_t count,
                                   int64_t heads, int64_t dim, int32_t dtype, double epsilon,
                                   int32_t clamp, void* stream);

typedef struct {
  const void* cached_k;
  const void* cached_v;
  int64_t c_stride_row, c_stride_head;
  const void* fresh_k;
  const void* fresh_v;
  int64_t f_stride_row, f_stride_head;
  const int64_t* indices;
  int64_t a;
  const double* alpha;
  const uint8_t* mandatory;
  void* fused_k; /* or NULL (then fused_v NULL too) */
  void* fused_v;
  double* next_alpha_out;
  double* used_alpha_out;
  double* cos_out; /* or NULL */
  const int64_t* slots; /* paged destination rows when kv != NULL */
  int32_t* status;
  /* or NULL: the number of rows is *a_dev, read on the device and clamped to
     [0, a] (a is then the capacity); rows past it are skipped.  With the
     count of cs_wca_active_rows a layer runs on the rows the previous
     layer's commit chose without a host read. */
  const int64_t* a_dev;
} cs_wca_update_item;

/* all items share heads, dim, dtype, the update options and the paged pool */
CS_API int cs_wca_update_batch(const cs_wca_update_item* items, int32_t count, int64_t heads,
                               int64_t dim, int32_t dtype, int32_t same_layer, double epsilon,
                               int32_t clamp, const cs_paged_kv* kv, void* stream);

typedef struct {
  const int64_t* indices; /* or NULL when a == 0 */
  int64_t a;
  const double* next_alpha;
  const double* cos; /* or NULL */
  int64_t n, budget;
  const double* initial_dev;
  double* alpha;
  uint8_t* candidate;
  uint8_t* selected;
  uint8_t* removed;
  int64_t* removed_out;  /* or NULL */
  int64_t* promoted_out; /* or NULL */
  int64_t* counts_out;
  int32_t* status;
  const int64_t* a_dev; /* or NULL: as cs_wca_update_item.a_dev, for indices */
} cs_wca_commit_item;

/* one thread block per request; threshold and distance_mode are shared */
CS_API int cs_wca_commit_batch(const cs_wca_commit_item* items, int32_t count, double threshold,
                               int32_t distance_mode, void* stream);

/*
 * The layer's active rows on the device (WCAState.active_indices,
 * wca.py:194-196, and the association rows of runtime.py:448-454): rows_out
 * = the ascending indices r < n with selected[r] or mandatory[r]; sel_out[k]
 * = 1 when row rows_out[k] is selected and not mandatory; *count_out = their
 * number, all written by one kernel on `stream`.  Entries from the count up
 * to `capacity` are -1 / 0; rows beyond `capacity` are dropped and set
 * CS_ST_SLOT_RANGE.  With cs_attn_params.nq_dev = count_out the prefill of
 * the next layer runs on these rows without a host read.
 */
CS_API int cs_wca_active_rows(const uint8_t* selected, const uint8_t* mandatory, int64_t n,
                              int64_t capacity, int64_t* rows_out, uint8_t* sel_out,
                              int64_t* count_out, int32_t* status, void* stream);

/* ------------------------------------------------- selective layer loop */
/*
 * The QKV projection of a layer's active rows (runtime.py:409-460 with the
 * adapter deltas of artifacts.py:189-193), on the tensor cores:
 *   out[r] = x_r W^T + round16(x_r A^T) B^T,
 *   x_r = (row_src[r] == 0 ? src0 : src1)[row_idx[r]]
 * src0 holds the previous layer's output rows (continuing rows), src1 the
 * layer's input snapshot (rows newly selected, restored); the gather is the
 * GEMM's A-operand load.  W [n_out, hidden], A [rank, hidden], B [n_out,
 * rank], row-major 16-bit (bf16 or fp16, one dtype for all); out [a, n_out]
 * in active-row order, float32 accumulation.  hidden % 64 == 0, n_out % 256
 * == 0, rank in {0, 8, ..., 32}, 16-byte aligned rows
 * (CS_ERR_UNSUPPORTED otherwise).  A row index outside its source sets
 * CS_ST_SLOT_RANGE and computes a zero row.
 */
typedef struct {
  const void* src0;
  int64_t src0_stride, src0_rows; /* stride in elements */
  const void* src1;
  int64_t src1_stride, src1_rows;
  const int32_t* row_src; /* [a] 0 or 1 */
  const int64_t* row_idx; /* [a] */
  int64_t a, hidden, n_out;
  const void* w;
  const void* lora_a; /* or NULL when rank == 0 */
  const void* lora_b;
  int32_t rank;
  void* out;
  int64_t out_stride;
  int32_t dtype;
  int32_t* status;
  /* or NULL: the number of rows is *a_dev, read on the device and clamped to
     [0, a] (a is then the capacity the grid is sized for); rows past it are
     not computed and their output rows are not written */
  const int64_t* a_dev;
} cs_qkv_params;

CS_API int cs_qkv_gather_lora(const cs_qkv_params* p, void* stream);

/* ------------------------------------------------------------ attention */
typedef enum {
  CS_POS_CONTEXTUAL = 0, /* CoPE gates (position.py:295-307)                 */
  CS_POS_FIXED = 1,      /* caller positions [h,q,k] (position.py:495-499)   */
  CS_POS_TABLE = 2,      /* canonical table substitution (attention.py:32-57)*/
  CS_POS_CHUNK = 3       /* chunk-reset counts with carried per-chunk offsets*/
} cs_pos_mode;

/*
 * Arguments of one CoPE/CCPE attention call (cope_attention,
 * position.py:404-560).  Dense K/V are used when kv_slots == NULL, otherwise
 * key j is read from paged slot kv_slots[j] of `paged` (no gather copy).
 */
typedef struct {
  const void* q;
  int64_t q_stride_tok, q_stride_head;
  int32_t nq, hq, d;
  const int64_t* qpos; /* [nq] distinct nonnegative coordinates */

  const void* k;
  const void* v;
  int64_t k_stride_tok, k_stride_head, v_stride_tok, v_stride_head;
  cs_paged_kv paged;
  const int64_t* kv_slots; /* [nk] or NULL */
  int32_t nk, hkv, dv;
  const int64_t* kpos; /* [nk] strictly increasing or NULL (= 0..nk-1) */

  const void* E; /* [d, npos] in the accumulation dtype (f64 iff in_dtype == F64) */
  int64_t e_stride_d, e_stride_p;
  int32_t npos;
  double scale; /* 1/sqrt(d) */

  int32_t pos_mode; /* cs_pos_mode */
  /* FIXED: [h, q, k] in the accumulation dtype (f64 iff in_dtype == F64) */
  const void* fixed_pos;
  int64_t fp_stride_h, fp_stride_q, fp_stride_k;
  /* TABLE: table[h, q_row[i], k_ord[j]] for q_row >= 0 and k_ord >= 0 */
  const void* table;
  int64_t tb_stride_h, tb_stride_r, tb_stride_c;
  const int32_t* q_row;
  const int32_t* k_ord;
  /* CHUNK: key_chunk[nk] nondecreasing; chunk_off[h, i, c] (float32) >= 0
     restarts the count entering chunk c (older than the query's chunk),
     < 0 carries it */
  const int32_t* key_chunk;
  const float* chunk_off;
  int64_t co_stride_h, co_stride_q;
  int32_t nchunks;

  /* optional bool masks (uint8, key stride 1; h stride 0 = broadcast):
     gate_mask = attention_mask (gates and attention), vis_mask =
     visibility_mask (attention only) */
  const uint8_t* gate_mask;
  int64_t gm_stride_h, gm_stride_q;
  const uint8_t* vis_mask;
  int64_t vm_stride_h, vm_stride_q;
  /* SelectedAssociationPolicy (attention.py:61-72): non-NULL enables */
  const uint8_t* q_selected; /* [nq] */
  const uint8_t* k_fixed;    /* [nk] */

  int32_t strict; /* validate_contextual_path (position.py:28-114) */
  double atol;
  int32_t positions_only; /* compute out_positions only, no softmax/PV */

  void* out_positions; /* [h, q, k] accumulation dtype or NULL */
  int64_t op_stride_h, op_stride_q;

  void* out; /* [nq, hq, dv] */
  int64_t o_stride_tok, o_stride_head;
  int32_t in_dtype, out_dtype;
  int32_t* status;
  /* decode only: CS_LAUNCH_OVERLAP_PREV lets the decode start while the grid
     launched just before it on the stream still runs (a programmatic
     dependent launch).  Set it only when that grid writes none of q, qpos,
     kv_slots and E, or writes them before it signals its dependents; the
     library's cs_slide_scatter qualifies (it writes only K/V records, which
     the decode reads after waiting for it).  0 = plain stream order. */
  int32_t launch_flags;
  /* cs_cope_attn_prefill(_batch) only (the other entry points return
     CS_ERR_UNSUPPORTED when it is set): the number of live query rows is
     *nq_dev, read by the kernel from device memory and clamped to [0, nq], so
     that a count the device produced (cs_wca_active_rows) needs no host read;
     nq is then the capacity the grid is sized for.  Rows at or past the count
     are not computed and their output rows are not written. */
  const int64_t* nq_dev;
} cs_attn_params;

#define CS_LAUNCH_OVERLAP_PREV 1

/*
 * Generic CoPE/CCPE attention: every mode above, any query rows, float64 /
 * float32 / bf16 / fp16 inputs (float64 accumulates in float64, the others in
 * float32, as position.py:153-154).  One warp per (query row, KV head).
 */
CS_API int cs_cope_attn(const cs_attn_params* p, void* stream);

/*
 * Tensor-core prefill / reuse-prefill (sm_100a, tcgen05 + TMEM): bf16 or fp16
 * inputs, head_dim 64 or 128, contextual or chunk-reset positions, optional
 * association policy, paged or dense K/V.  Returns CS_ERR_UNSUPPORTED for
 * any other combination (the caller then uses cs_cope_attn).
 */
CS_API int cs_cope_attn_prefill(const cs_attn_params* p, void* stream);

/*
 * The prefill of `count` requests in one launch (the reuse-prefill layer of a
 * whole step; the reference runs cope_attention once per request,
 * runtime.py:576-609).  Every request must be supported by
 * cs_cope_attn_prefill and share hq, hkv and the input dtype; each has its
 * own queries, positions, keys / slots, tables and output.  The heaviest
 * query tiles of all requests are scheduled first, which balances the grid
 * across requests of different lengths.
 */
CS_API int cs_cope_attn_prefill_batch(const cs_attn_params* params, int32_t count,
                                      void* stream);

/*
 * Decode (one or a few query rows over a long paged context): split-key
 * kernel.  On the tensor-core path (head_dim 128, 16-bit, 16-byte aligned
 * rows) one pass over the records: each split publishes its gate totals,
 * takes the count carried from the newer splits, applies the bias, and the
 * split partials are merged; other shapes run two CUDA-core phases (logits
 * and gate totals, then the carried scan, bias and partials) and a combine.
 * `workspace` must hold cs_cope_attn_decode_workspace(p) bytes of device
 * memory (256-byte aligned); its contents need no initialisation.
 */
CS_API int64_t cs_cope_attn_decode_workspace(const cs_attn_params* p);
CS_API int cs_cope_attn_decode(const cs_attn_params* p, void* workspace,
                        void* stream);

/*
 * Decode of `count` requests in one set of launches (the per-step decode of
 * a whole batch; the reference runs runtime.py:490-508 once per request).
 * All requests must share head counts, head dims, npos, dtypes and scale;
 * each has its own queries, positions, slot table, cache view, E table and
 * output.  `workspace` holds cs_cope_attn_decode_batch_workspace(params,
 * count) bytes (256-byte aligned); requests are packed in order.
 */
CS_API int64_t cs_cope_attn_decode_batch_workspace(const cs_attn_params* params,
                                                   int32_t count);
CS_API int cs_cope_attn_decode_batch(const cs_attn_params* params, int32_t count,
                                     void* workspace, void* stream);

/*
 * Decode that allocates nothing (no counterpart in the reference; it exists
 * for callers that must not allocate device memory, e.g. a plugin inside an
 * inference engine that already gave all free HBM to its KV-cache pool, or a
 * foreign-language host without a CUDA allocator).  Same kernels and results
 * as cs_cope_attn_decode; the workspace comes from 16 MiB of static device
 * memory inside this library, held by every GPU that loads it until exit.
 * - Problems needing more than 16 MiB (cs_cope_attn_decode_workspace) return
 *   CS_ERR_TOO_LARGE without launching anything.
 * - The first call on a device resolves the array's device address with that
 *   device current; make that first call before any stream capture, and make
 *   the stream's device current for every call.  The address is kept for the
 *   life of the process: after cudaDeviceReset (or anything else that
 *   re-creates the device's primary context) it is stale, so do not call
 *   this entry point again in that process after such a reset.
 * - All calls on a device share the one array: calls that overlap on the GPU
 *   (different streams, no ordering between them) race and corrupt each
 *   other's results.  Nothing in it needs to start at zero.
 */
CS_API int cs_cope_attn_decode_noalloc(const cs_attn_params* p, void* stream);

/* ------------------------------------------- standalone CoPE operators */
/*
 * CoPE.contextual_positions (position.py:295-307): positions of [h, q, k]
 * float32/float64 logits under a uint8 allowed mask (key stride 1):
 * masked gates, reverse cumulative sum over keys, clamp to [0, npos-1].
 * Non-finite allowed logits set CS_ST_LOGIT_NONFINITE.
 */
CS_API int cs_cope_positions(const void* logits, int64_t ls_h, int64_t ls_q,
                             const uint8_t* allowed, int64_t as_h, int64_t as_q,
                             int32_t heads, int64_t nq, int64_t nk, int32_t npos,
                             int32_t dtype, void* out, int64_t os_h, int64_t os_q,
                             int32_t* status, void* stream);

/*
 * CoPE.positional_bias (position.py:309-344): per (head, query) the q.E
 * table, then floor / floor+1 interpolation at every position.  query has
 * dtype in_dtype; E, positions and out use the accumulation dtype.  Positions
 * outside [0, npos-1] or non-finite set CS_ST_POS_RANGE.
 */
CS_API int cs_cope_bias(const void* query, int64_t qs_t, int64_t qs_h,
                        const void* E, int64_t es_d, int64_t es_p, int32_t d,
                        int32_t npos, const void* positions, int64_t ps_h,
                        int64_t ps_q, int32_t heads, int64_t nq, int64_t nk,
                        int32_t in_dtype, void* out, int64_t os_h, int64_t os_q,
                        int32_t* status, void* stream);

/*
 * Compressed CCPE positions from a canonical profile: the [head, F, F]
 * tables of CCPEProfile (position.py:581-748, applied by
 * CanonicalPositionPolicy, attention.py:32-57) turned into the per-chunk
 * offsets of CS_POS_CHUNK (offsets[h, t, segment], float32).  For query row
 * r (token position qpos[r], fixed ordinal q_ord[r] or -1, segment
 * q_seg[r]) and fixed chunk f (segment seg_of_chunk[f], last token at key
 * index last_key[f] with fixed ordinal last_ord[f]) older than the query's
 * segment:
 *   offsets[h, qpos[r], seg_of_chunk[f]] = table[h, q_ord[r], last_ord[f]]
 *       - sigmoid(q[r, h] . k[last_key[f], h / (hq / hkv)] / sqrt(d)),
 * the count carried into the chunk (its last key's canonical position minus
 * that key's own gate); every other entry of the rows qpos[r] is -1 (the
 * running count is carried).  With the calibration's gates inside the fixed
 * chunks, the chunk-reset positions of fixed x fixed cells equal the table.
 * q, k in bf16 / fp16 / fp32; out-of-range ordinals set CS_ST_POS_RANGE.
 */
CS_API int cs_cope_chunk_offsets(const void* q, int64_t q_stride_tok, int64_t q_stride_head,
                                 int32_t nq, int32_t hq, int32_t d, const int64_t* qpos,
                                 const int32_t* q_ord, const int32_t* q_seg, const void* k,
                                 int64_t k_stride_tok, int64_t k_stride_head, int32_t hkv,
                                 const int64_t* last_key, const int32_t* last_ord,
                                 const int32_t* seg_of_chunk, int32_t nfixed_chunks,
                                 const float* table, int64_t tb_stride_h, int64_t tb_stride_r,
                                 int64_t tb_stride_c, int32_t tb_rows, int32_t tb_cols,
                                 int32_t dtype, float* offsets, int64_t off_stride_h,
                                 int64_t off_stride_t, int32_t nseg, int32_t* status,
                                 void* stream);

/*
 * validate_contextual_path (position.py:28-114): OR-s CS_ST_PATH_* bits for
 * failing causal cells / adjacent pairs and CS_ST_POS_RANGE for non-finite
 * positions.  mask (uint8 [h|1, q, k], may be NULL) = attention_mask.
 */
CS_API int cs_cope_validate_path(const void* positions, int64_t ps_h,
                                 int64_t ps_q, const int64_t* qpos,
                                 const int64_t* kpos, const uint8_t* mask,
                                 int64_t ms_h, int64_t ms_q, int32_t heads,
                                 int64_t nq, int64_t nk, double atol,
                                 int32_t dtype, int32_t* status, void* stream);

/* library identification: compile-time arch string and ABI version */
CS_API const char* cs_build_info(void);
CS_API int32_t cs_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* CACHESLIDE_B200_H */
