/*
 * intent_attention_b200.h -- C ABI of the B200 (sm_100a) fused selected-quant
 * paged decode attention library (libiak_b200.so).
 *
 * Plain C: device pointers, sizes, strides and POD descriptors; no torch or
 * CUDA types (a CUDA stream is passed as `void*`, NULL = legacy default
 * stream).  Every entry point returns an iak_status; on failure
 * iak_last_error() returns a thread-local message.  Entry points never
 * allocate device memory and never synchronise the stream (exceptions: the
 * iak_ipc_* helpers, which exist to allocate and map exchange areas, and
 * iak_kernel_timer_read); they are reentrant across devices (the current
 * CUDA device is used).
 *
 * Reference interfaces replaced (manishklach/intent-attention-kernel,
 * paths inside src/intent_attention/):
 *   iak_decode / iak_decode_workspace_size
 *       fused_selected_quant_decode.py:408-464  fused_selected_quant_decode()
 *       fused_selected_quant_decode.py:472-513  _launch_triton_kernel()
 *       triton_intent_quant_attention.py:342-457 intent_quant_decode_attention_triton()
 *       triton_adaptive_format_attention.py:237-329 adaptive_format_decode_attention_triton()
 *     (one decode for all three: each Python entry point fills tag_map with
 *      its own enum, so FusedKVPrecision / TritonKVPrecision /
 *      AdaptivePageFormat tags are translated at the boundary, never globally)
 *   iak_merge_partials
 *       the (m, l, acc) online-softmax recurrence of
 *       fused_selected_quant_decode.py:323-334, applied across KV splits
 *   iak_pack_metadata
 *       fused_selected_quant_decode.py:344-400  metadata_to_kernel_tensors()
 *       triton_intent_quant_attention.py:126-203 make_page_tables_from_selected_pages()
 *   iak_quantize_pages
 *       intent_quant.py:221-312 _absmax_scale() / fake_quantize_tensor()
 *       fused_selected_quant_decode.py:521-542 fake_int8_pages_from_fp16()
 *       (real packed page formats instead of fake quantisation)
 *   iak_mla_decode
 *       triton_mla_decode.py:110-152 mla_decode_triton(), mla.py:95-136
 */
#ifndef INTENT_ATTENTION_B200_H
#define INTENT_ATTENTION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define IAK_ABI_VERSION 2

typedef enum iak_status {
  IAK_OK = 0,
  IAK_ERR_INVALID_ARG = 1,   /* maps to ValueError in the Python layer   */
  IAK_ERR_UNSUPPORTED = 2,   /* shape / format combination not built      */
  IAK_ERR_CUDA = 3,          /* a CUDA runtime / driver call failed       */
  IAK_ERR_WORKSPACE = 4,     /* workspace missing or too small            */
  IAK_ERR_TIMEOUT = 5        /* a bounded device-side wait gave up        */
} iak_status;

/* element types of q / out / dense inputs */
enum { IAK_DT_F32 = 0, IAK_DT_F16 = 1, IAK_DT_BF16 = 2 };

/* page formats a tag can map to */
enum {
  IAK_FMT_SKIP = 0,    /* no load, no contribution                                */
  IAK_FMT_F16 = 1,     /* [NP, PS, D] float16                                     */
  IAK_FMT_FP8 = 2,     /* [NP, PS, D] e4m3fn codes, value = code * scale          */
  IAK_FMT_INT8 = 3,    /* [NP, PS, D] int8 codes, value = code * scale            */
  IAK_FMT_INT4 = 4,    /* [NP, PS, D/2] packed nibbles, value = code * scale      */
  IAK_FMT_INT4R = 5,   /* INT4 base plane + INT4 residual plane, two scale sets   */
  IAK_FMT_SPARSE = 6   /* adaptive SPARSE: contributes nothing (reference kernel) */
};

/* scale granularity of the quantised formats (one scale set per page) */
enum {
  IAK_SCALE_PAGE = 0,     /* 1 scale per page                    */
  IAK_SCALE_GROUP32 = 1,  /* head_dim / 32 scales per page       */
  IAK_SCALE_CHANNEL = 2   /* head_dim scales per page            */
};

/* Paged KV storage.  Pages are single-head: page p of every pool is one
 * (sequence, kv-head, logical page) slot, addressed by the page table.
 * Pools that are not used by any tag may be NULL.  Packed INT4 rows hold
 * channel d of nibble n in 32-bit word w at
 *   d = 32*(w/4) + 4*(w%4) + {0,2,16,18,1,3,17,19}[n],  stored as code + 8.
 * Base pointers must be 16-byte aligned. */
typedef struct iak_page_pools {
  void* k_f16;  void* v_f16;
  void* k_fp8;  void* v_fp8;
  void* k_i8;   void* v_i8;
  void* k_i4;   void* v_i4;
  void* k_i4r;  void* v_i4r;      /* INT4_RESIDUAL residual planes        */
  float* k_scale;     float* v_scale;      /* [NP, n_scales]              */
  float* k_res_scale; float* v_res_scale;  /* [NP, n_scales] (INT4R)      */
  int64_t num_pages;
  int32_t page_size;
  int32_t head_dim;
  int32_t scale_mode;             /* IAK_SCALE_*                           */
} iak_page_pools;

/* One decode step: B sequences, Hq query heads, Ht page-table heads
 * (G = Hq / Ht query heads share one page list: G = 1 is the reference's
 * per-head table, G > 1 is grouped-query attention). */
typedef struct iak_decode_args {
  const void* q;  int32_t q_dtype;  int64_t q_stride_b, q_stride_h;    /* elements */
  void* out;      int32_t out_dtype; int64_t out_stride_b, out_stride_h;
  int32_t batch, num_q_heads, num_table_heads;
  const int32_t* page_table;      /* [B, Ht, W]; ids < 0 are unused slots */
  int64_t pt_stride_b, pt_stride_h;
  int32_t table_width;            /* W                                     */
  const int32_t* page_counts;     /* [B, Ht] (row stride pc_stride_b) or NULL = W */
  int64_t pc_stride_b;
  const void* page_tags;          /* [NP] tag per page                      */
  int32_t tag_bytes;              /* 1 (uint8) or 4 (int32)                 */
  uint8_t tag_map[16];            /* tag -> IAK_FMT_*                       */
  uint8_t tag_default;            /* format of tags outside 0..15           */
  float sm_scale;                 /* softmax scale (1/sqrt(D) in the reference) */
  /* Optional split-KV export: when partial_l != NULL the decode writes the
   * unnormalised partial (m natural-log max, l, acc) of every query row
   * ([B*Hq], [B*Hq], [B*Hq, D] fp32) instead of `out`; iak_merge_partials
   * combines partials of several devices. */
  float* partial_m; float* partial_l; float* partial_acc;
  int32_t num_splits;             /* 0 = choose automatically               */
  int32_t kernel;                 /* IAK_KERNEL_*: 0 auto, 1 generic, 2 tensor core */
  /* Device-side waits.  The tensor-core decode is a pipeline of warps that
   * wait on one another (page copies, stage release); each wait gives up
   * after wait_budget_ns nanoseconds (0 = the default of about 2 s), after
   * which the kernel stops, lets the copies it issued land and, when status
   * is non-NULL, ORs IAK_STATUS_DECODE_TIMEOUT into *status (device memory;
   * never cleared by the library, so one word can collect many calls).  The
   * output of a call that timed out is undefined.  iak_device_status reads
   * the process-wide counters instead. */
  uint32_t* status;
  uint32_t wait_budget_ns;
} iak_decode_args;

/* bits of iak_decode_args.status */
enum { IAK_STATUS_DECODE_TIMEOUT = 1 };

/* decode kernel selection (iak_decode_args.kernel) */
enum { IAK_KERNEL_AUTO = 0, IAK_KERNEL_GENERIC = 1, IAK_KERNEL_TENSOR = 2 };

int iak_version(void);
const char* iak_last_error(void);

/* Timeout counters of the current device (no counterpart in the reference).
 * Every kernel warp whose bounded wait gave up adds one to its kernel's
 * counter: the tensor-core decode (iak_decode / iak_decode_noalloc), the
 * tcgen05 MLA decode and the tcgen05 prefill.  Copies the three counters to
 * the non-NULL outputs and, when reset != 0, sets them back to zero.  Waits
 * for the device (a synchronous copy); returns IAK_ERR_TIMEOUT when any
 * counter read was non-zero, else IAK_OK. */
int iak_device_status(uint32_t* decode_timeouts, uint32_t* mla_timeouts, uint32_t* prefill_timeouts,
                      int32_t reset);

/* Workspace (device bytes) iak_decode needs for these arguments. */
int iak_decode_workspace_size(const iak_page_pools* pools, const iak_decode_args* args,
                              size_t* bytes);

/* Fused selected-quant paged decode: gather the selected pages, dequantise
 * in registers, split-KV online softmax, LSE merge. */
int iak_decode(const iak_page_pools* pools, const iak_decode_args* args,
               void* workspace, size_t workspace_bytes, void* stream);

/* Decode without any device allocation.  No counterpart in the reference.
 *
 * For callers that cannot call cudaMalloc: serving engines that reserve all
 * device memory up front (most of it for the KV cache) and forbid allocation
 * while decoding, hosts that reach this library through an FFI holding only
 * borrowed device pointers and no allocator, and latency-critical loops that
 * cannot afford an allocation's implicit device synchronisation.
 *
 * Same arguments and results as iak_decode, but the split-KV scratch is a
 * file-scope device array of IAK_NOALLOC_SCRATCH_BYTES (8 MiB) that every GPU
 * loading the library holds until the process exits; decodes whose
 * iak_decode_workspace_size exceeds it are rejected with IAK_ERR_WORKSPACE
 * (pass fewer num_splits, or use iak_decode).  The first call on a device
 * looks up the array's device address with that device current, so make that
 * first call before any stream capture.  The address is cached per device for
 * the life of the process and belongs to the device's primary context: do not
 * use the entry point after cudaDeviceReset of that device, nor with another
 * driver context current.  All calls share the one array and it
 * keeps the last call's contents (nothing in it needs to start at zero):
 * calls that overlap on the GPU, on any streams, race.  Calls no cudaMalloc,
 * cudaFree or allocating library routine. */
#define IAK_NOALLOC_SCRATCH_BYTES (8 << 20)
int iak_decode_noalloc(const iak_page_pools* pools, const iak_decode_args* args, void* stream);

/* ------------------------------------------------------------------------
 * MLA (absorbed multi-head latent attention) decode.
 *
 * Replaces triton_mla_decode.py:110-152 mla_decode_triton() and its CPU path
 * _mla_decode_cpu() (:155-186), and the decode step of mla.py:95-136
 * mla_triton_decode().  The reference collapses heads into one absorbed
 * query row per (batch, position) and uses the whole latent vector as key
 * and value; here every query row r = (b, h) attends over its own sequence's
 * selected latent pages: score = sm_scale * q[b,h,:d_qk] . c[:d_qk],
 * context[b,h,:] = softmax-weighted sum of c[:d_v] (d_v <= d_qk; the rope
 * channels d_v..d_qk-1 are key-only).  The W_VO projection that follows in
 * the reference is a plain GEMM left to the caller.
 *
 * Latent pages are [NP, page_size, d_qk], one pool per format: dense
 * (f32 / f16 / bf16) and FP8-e4m3 codes with one fp32 scale per page
 * (value = code * scale).  page_tags + tag_map pick a page's format.
 * ------------------------------------------------------------------------ */
enum { IAK_MLA_SKIP = 0, IAK_MLA_DENSE = 1, IAK_MLA_FP8 = 2 };

typedef struct iak_mla_args {
  const void* q; int32_t q_dtype; int64_t q_stride_b, q_stride_h;     /* [B, H, d_qk], elements */
  void* out; int32_t out_dtype; int64_t out_stride_b, out_stride_h;    /* [B, H, d_v] context    */
  int32_t batch, num_heads, d_qk, d_v;
  const void* dense_pages; int32_t dense_dtype;   /* [NP, page_size, d_qk] IAK_DT_*, or NULL   */
  const uint8_t* fp8_pages; const float* fp8_scale; /* [NP, page_size, d_qk] e4m3 codes, [NP]  */
  int64_t num_pages;
  int32_t page_size;
  const int32_t* page_table;      /* [B, W]; pt_stride_b = 0 shares one list; ids < 0 unused  */
  int64_t pt_stride_b;
  int32_t table_width;
  const int32_t* page_counts;     /* [B] or NULL = W                                          */
  const void* page_tags;          /* [NP] or NULL = every page IAK_MLA_DENSE                  */
  int32_t tag_bytes;              /* 1 or 4                                                   */
  uint8_t tag_map[16];            /* tag -> IAK_MLA_*                                         */
  uint8_t tag_default;
  float sm_scale;                 /* 1/sqrt(d_qk) in the reference                            */
  /* optional export of per-row partials (rows = B*H: m [rows], l [rows],
   * acc [rows, d_v], the layout of a partial block with head_dim = d_v)
   * instead of `out` */
  float* partial_m; float* partial_l; float* partial_acc;
  int32_t num_splits;             /* 0 = choose automatically                                 */
  int32_t kernel;                 /* IAK_KERNEL_*: auto, generic (CUDA cores), tensor (tcgen05: d_qk 576,
                                     d_v 512, <= 128 heads, page_size % 64 == 0, bf16 / f16 q and
                                     dense pages, sm_scale > 0) */
} iak_mla_args;

int iak_mla_workspace_size(const iak_mla_args* args, size_t* bytes);
int iak_mla_decode(const iak_mla_args* args, void* workspace, size_t workspace_bytes, void* stream);

/* Kernel timer (measurement only; no counterpart in the reference).  While
 * enabled, each iak_decode / iak_decode_noalloc call records a CUDA event
 * pair on the caller's stream around its main decode kernel (not the query
 * preparation or merge launches), for the first max_launches calls.
 * iak_kernel_timer_read waits for the recorded events and returns the summed
 * kernel time and the number of timed launches; iak_kernel_timer_disable
 * releases the events.  Process-wide.  Launches captured into a CUDA graph
 * record graph event nodes, so each replay of the graph re-times them; enable
 * the timer before the capture and read it after the replay to be timed. */
int iak_kernel_timer_enable(int32_t max_launches);
int iak_kernel_timer_read(double* total_ms, int32_t* launches);
int iak_kernel_timer_disable(void);

/* LSE merge of S partials per row: m/l [rows, S], acc [rows, S, D] (fp32,
 * contiguous).  Writes normalised rows to out (dtype, row stride in
 * elements); rows with no contribution become 0. */
int iak_merge_partials(const float* m, const float* l, const float* acc,
                       int64_t rows, int32_t splits, int32_t head_dim,
                       void* out, int32_t out_dtype, int64_t out_row_stride, void* stream);

/* Partial blocks: merging decodes of disjoint page ranges (sequence shards
 * on several GPUs, or any split of the page lists).  No counterpart in the
 * reference, which decodes on one device.  A block holds
 * rows * (head_dim + 2) fp32 values laid out
 *     [m: rows][l: rows][acc: rows x head_dim]
 * with rows = batch * num_q_heads and row = b * num_q_heads + h.
 * iak_decode writes one when partial_m / partial_l / partial_acc point at
 * block, block + rows and block + 2 * rows.  m is the running max of the
 * scaled scores (natural-log domain), l the softmax denominator, acc the
 * unnormalised weighted sum of values; l = 0 marks a row without pages. */
#define IAK_PARTIAL_BLOCK_FLOATS(rows, head_dim) ((rows) * ((head_dim) + 2))

/* LSE merge of num_parts consecutive partial blocks (e.g. the result of an
 * all-gather over ranks) into normalised rows of out (dtype, row stride in
 * elements): m = max m_i, l = sum l_i e^(m_i - m), o = sum acc_i e^(m_i - m) / l;
 * rows without pages anywhere become 0. */
int iak_merge_partial_blocks(const float* blocks, int32_t num_parts, int64_t rows, int32_t head_dim,
                             void* out, int32_t out_dtype, int64_t out_row_stride, void* stream);

/* ------------------------------------------------------------------------
 * Peer-memory exchange of partial blocks (multi-GPU split-KV over NVLink).
 * No counterpart in the reference.  Replaces a collective all-gather of the
 * blocks with stores straight into the peers' memory.
 *
 * Every rank owns an exchange area in its own device memory
 * (iak_exchange_area_bytes): a staging block, for each of two parities a
 * receive array of `world` partial blocks and `world` uint32 arrival flags,
 * and a device-side epoch counter.  The areas are allocated with
 * iak_ipc_alloc and shared once through their 64-byte CUDA IPC handles
 * (iak_ipc_open in every other rank), so each rank can write every peer's
 * area.  Per step:
 *   1. decode with partial export into this rank's staging block
 *      (iak_exchange_staging_ptr; the block layout of IAK_PARTIAL_BLOCK_FLOATS);
 *   2. iak_exchange_push: advance the epoch e -> e+1, copy the staging block
 *      into slot `rank` of every rank's receive array of parity (e+1) & 1
 *      over NVLink, then raise those areas' flag[parity][rank] to e+1;
 *   3. iak_exchange_merge: wait until every flag of that parity in this
 *      rank's area equals e+1 (bounded by timeout_us; on expiry *status
 *      becomes 1 and the merge reads whatever arrived), then LSE-merge the
 *      world blocks into out.
 * The epoch lives in device memory, so the three steps can be captured once
 * in a CUDA graph and replayed.  Two parities let a rank run one step ahead
 * without overwriting blocks a slower peer is still merging.  All ranks must
 * run the three steps every step, in the same order.
 * ------------------------------------------------------------------------ */
#define IAK_MAX_PEERS 8
typedef struct iak_peer_exchange {
  void* areas[IAK_MAX_PEERS];     /* rank r's exchange area as mapped in this process */
  int32_t rank, world;
  int64_t rows;                   /* batch * num_q_heads                            */
  int32_t head_dim;               /* block = rows * (head_dim + 2) floats           */
} iak_peer_exchange;

int iak_exchange_area_bytes(int32_t world, int64_t rows, int32_t head_dim, size_t* bytes);

/* Decode fused with the push (no counterpart in the reference): the same decode
 * as iak_decode on the tensor-core path, but each query row's merged partial
 * (m, l, acc) is stored by the decode kernel itself into slot x->rank of every
 * rank's receive array (plain stores over NVLink), and the last work unit to
 * finish raises this rank's flag in every area and advances the epoch.  Use it
 * in place of steps 1-2 above (decode into the staging block, then
 * iak_exchange_push); step 3 (iak_exchange_merge) is unchanged.  args->out and
 * args->partial_* are not used (partial_* must be NULL); x->rows must be
 * batch * num_q_heads and x->head_dim the pools' head_dim.  Allocates nothing,
 * synchronises nothing; IAK_ERR_UNSUPPORTED outside the tensor-core shapes. */
int iak_decode_exchange(const iak_page_pools* pools, const iak_decode_args* args, const iak_peer_exchange* x,
                        void* workspace, size_t workspace_bytes, void* stream);
/* Address of the staging block inside an exchange area. */
float* iak_exchange_staging_ptr(void* area, int32_t world, int64_t rows, int32_t head_dim);
int iak_exchange_push(const iak_peer_exchange* x, void* stream);
int iak_exchange_merge(const iak_peer_exchange* x, void* out, int32_t out_dtype, int64_t out_row_stride,
                       uint32_t* status, uint32_t timeout_us, void* stream);

/* CUDA IPC helpers (device memory of the current device; handle = 64 bytes).
 * iak_ipc_alloc zero-fills the allocation. */
int iak_ipc_alloc(size_t bytes, void** ptr, void* handle);
int iak_ipc_open(const void* handle, void** ptr);
int iak_ipc_close(void* ptr);
int iak_ipc_free(void* ptr);

/* ------------------------------------------------------------------------
 * Device router: block routing + page lists for a batch of sequences.
 *
 * Replaces, per sequence, block_router.py:101-266 BlockRouter.route_layout()
 * (with intent_quant.py:77-131 IntentQuantizer.assign_block_precision() as
 * the precision policy), :283-296 selected_page_ids() and the precision map
 * of :383-421 routing_to_kernel_metadata(), followed by the page-table
 * packing of iak_pack_metadata.  Per sequence: ALWAYS / GLOBAL / RECENT
 * blocks are selected; scored ATTEND blocks are ranked by score (descending,
 * ties in layout order) and the first top_k_blocks (Python slice semantics,
 * so a negative value drops the last |k|) are selected unless the quantiser
 * assigns them SKIP; SKIP-policy blocks with a score >= score_threshold are
 * selected (with precision SKIP).  Page ids t / page_size of the selected
 * blocks are listed in routed order (pinned blocks in layout order, then the
 * top-k in score order, then the selected SKIP-policy blocks in layout
 * order), each page once, at its first covering block, which also gives its
 * precision.  Scores are doubles so that threshold tests compare exactly as
 * Python floats do; NaN stands for "no score".
 *
 * Each sequence's layout is checked on the device with the conditions of
 * block_metadata.py:41-70 BlockLayout.validate (start >= 0, end > start,
 * end <= seq_lens[b] when seq_lens is given, sorted and non-overlapping,
 * ATTEND blocks scored) plus policy < 5; a sequence that fails gets
 * num_selected[b] = -1, page_counts 0 and a padded row, where the reference
 * raises ValueError.  memory_pressure outside [0, 1] is IAK_ERR_INVALID_ARG,
 * as IntentQuantizer.__init__ (intent_quant.py:67-70) raises.
 * ------------------------------------------------------------------------ */
enum { IAK_POLICY_ALWAYS = 0, IAK_POLICY_ATTEND = 1, IAK_POLICY_SKIP = 2, IAK_POLICY_RECENT = 3,
       IAK_POLICY_GLOBAL = 4 };
enum { IAK_PREC_FP16 = 0, IAK_PREC_FP8 = 1, IAK_PREC_INT8 = 2, IAK_PREC_INT4 = 3, IAK_PREC_INT4_RESIDUAL = 4,
       IAK_PREC_SKIP = 5 };
#define IAK_ROUTE_MAX_BLOCKS 8192

typedef struct iak_route_args {
  /* layouts: block arrays [batch, layout_stride] (layout_stride 0 = one layout for the batch) */
  int32_t num_blocks;             /* blocks per layout row, <= IAK_ROUTE_MAX_BLOCKS          */
  const int32_t* block_counts;    /* [batch] blocks of sequence b (<= num_blocks) or NULL     */
  const int32_t* block_start;     /* token ranges [start, end)                                */
  const int32_t* block_end;
  const uint8_t* block_policy;    /* IAK_POLICY_*                                             */
  int64_t layout_stride;
  const double* scores;           /* [batch, score_stride] (0 = shared), NaN = no score       */
  int64_t score_stride;
  const int32_t* seq_lens;        /* [batch] total tokens for the end bound, or NULL          */
  int32_t batch, num_table_heads, page_size;
  /* RouterConfig (block_router.py:39-47) and IntentQuantizer (intent_quant.py:59-74) */
  int32_t top_k_blocks;
  int32_t preserve_recent, preserve_global;
  double score_threshold, memory_pressure;
  double high_score_threshold, medium_score_threshold;   /* 0.75 / 0.40 in the reference */
  /* outputs, as iak_pack_metadata writes them: page_table [batch, Ht, table_width]
   * holding bases[b*Ht + h] + logical page id (bases NULL = 0), pad_value
   * padded; page_counts [batch, Ht] = min(n, table_width); num_selected
   * [batch] = n before truncation or -1 (or NULL); page_prec [batch,
   * table_width] IAK_PREC_* of each listed page, IAK_PREC_SKIP padded (or
   * NULL); when page_tags is set, prec_to_tag[prec] is also stored at
   * page_tags[physical id] for every head (ids outside [0, num_tag_pages)
   * are dropped) */
  const int32_t* bases;
  int32_t table_width, pad_value;
  int32_t* page_table;
  int32_t* page_counts;
  int32_t* num_selected;
  uint8_t* page_prec;
  uint8_t* page_tags; int64_t num_tag_pages;
  uint8_t prec_to_tag[6];
  /* row_masks [batch, table_width] (or NULL; page_size <= 64): bit r of a
   * listed page = token page * page_size + r lies in a selected block (the
   * exact-token bounds iak_prefill takes); 0 padded */
  uint64_t* row_masks;
} iak_route_args;
int iak_route_pages(const iak_route_args* args, void* stream);

/* Metadata packing on the device.  Logical page ids (one list shared by
 * every (b, h), the router's selected_page_ids order) are mapped to
 * physical ids base[b*Ht + h] + logical, written -1 padded into
 * page_table [B, Ht, W] with counts min(n, W); when tags_in is non-NULL the
 * per-logical-page tags are scattered to page_tags[physical]. */
typedef struct iak_pack_args {
  const int32_t* logical_ids; int32_t num_ids;
  const uint8_t* logical_tags;    /* [num_logical_pages] or NULL            */
  int32_t num_logical_pages;
  const int32_t* bases;           /* [B*Ht] physical base per (b, h) or NULL = 0 */
  int32_t batch, num_table_heads, table_width;
  int32_t* page_table; int32_t* page_counts; uint8_t* page_tags;
  int64_t num_tag_pages;          /* length of page_tags; writes outside it are dropped */
  int32_t pad_value;              /* -1 (6-tag / adaptive) or 0 (fused API)  */
} iak_pack_args;
int iak_pack_metadata(const iak_pack_args* args, void* stream);

/* Quantise dense pages x [P, PS, D] (f32 / f16 / bf16) into the pool
 * formats, one plane (K or V) per call, with the reference's arithmetic:
 * scale = max(absmax/127, 1e-8) over the scale span, INT8/INT4 codes =
 * round_half_even(clamp(x/scale, +-127 / +-7)), FP8 = e4m3(x/scale),
 * INT4R = INT4 base + INT4 residual with its own scale, FP16 = half(x).
 * Source page i goes to pool page dst_ids[i] (NULL = i) in format
 * formats[i] (IAK_FMT_*).  given_scale / given_res_scale ([P, n_scales],
 * optional) replace the computed scales. */
typedef struct iak_quant_args {
  const void* x; int32_t x_dtype; int64_t num_src_pages;
  const int32_t* dst_ids;
  const uint8_t* formats;
  const float* given_scale; const float* given_res_scale;
  void* f16; void* fp8; void* i8; void* i4; void* i4r;   /* plane pools */
  float* scale; float* res_scale;
  int64_t num_pages;
  int32_t page_size, head_dim, scale_mode;
} iak_quant_args;
int iak_quantize_pages(const iak_quant_args* args, void* stream);

/* ------------------------------------------------------------------------
 * KV append with quantise-on-write, and page format transitions.
 *
 * iak_append_tokens replaces, on the device and for a whole batch, the
 * page writes of kv_memory_manager.py:225-256 KVMemoryManager.write_page
 * (quantise a page on write into its storage format; the device precedent is
 * triton_kernel.py:186-279 _quant_kernel) for tokens produced while decoding.
 * num_new new K/V rows of every (sequence b, table head h) go to logical
 * token positions positions[b] .. positions[b]+num_new-1, i.e. to physical
 * page bases[b*Ht+h] + pos / page_size, row pos % page_size.  Each touched
 * page is re-quantised in the format its tag names (tag_map as in
 * iak_decode_args) from the rows staged for it, with the arithmetic of
 * iak_quantize_pages, so a page always holds exactly what quantising its
 * dense rows (zeros past the last appended row) gives.  The stage keeps the
 * rows of each (b, h)'s open page between calls: a page that begins inside
 * the appended range is restaged from zero; the rows of a page opened by
 * an earlier call are taken from the stage.  Pages outside [0, num_pages)
 * are not written and are counted in *dropped (when given).
 * new_lengths[b] = positions[b] + num_new when given (may alias nothing
 * read by the call).
 * ------------------------------------------------------------------------ */
typedef struct iak_append_args {
  const void* k_new; const void* v_new;  /* [batch, Ht, num_new, head_dim] contiguous      */
  int32_t new_dtype;                     /* IAK_DT_*                                       */
  int32_t batch, num_table_heads, num_new;
  const int32_t* positions;              /* [batch] index of the first appended token      */
  int32_t* new_lengths;                  /* [batch] or NULL                                */
  const int32_t* bases;                  /* [batch*Ht] physical id of logical page 0, NULL = 0 */
  const void* page_tags; int32_t tag_bytes;              /* 1 (uint8) or 4 (int32)       */
  uint8_t tag_map[16]; uint8_t tag_default;
  float* k_stage; float* v_stage;        /* [batch*Ht, page_size, head_dim] fp32           */
  int32_t* dropped;                      /* device counter or NULL                         */
} iak_append_args;
int iak_append_tokens(const iak_page_pools* pools, const iak_append_args* args, void* stream);

/* Page format transitions (demotion / promotion): replaces
 * kv_memory_manager.py:258-274 KVMemoryManager.set_page_format as used by
 * demote_cold_pages / promote_hot_pages / _prefetch_warmup (:329-362).  Each
 * listed page is read in its current format (its tag through tag_map;
 * dequantised as the decode kernels read it: code x scale in fp32) and
 * re-quantised into new_formats[i] with the arithmetic of
 * iak_quantize_pages; then fmt_to_tag[new format] is stored as its tag.
 * A page already in its target format is left untouched (set_page_format
 * returns early); SKIP / SPARSE pages read as zeros; converting to SKIP /
 * SPARSE only retags.  page_ids must be distinct; ids outside
 * [0, num_pages) are ignored; a page whose target pool (or scales) is absent
 * is left untouched and counted in *rejected (when given).
 * page_size * head_dim <= IAK_CONVERT_MAX_ELEMS. */
#define IAK_CONVERT_MAX_ELEMS 16384
typedef struct iak_convert_args {
  const int32_t* page_ids; int32_t num_ids;
  const uint8_t* new_formats;            /* [num_ids] IAK_FMT_*                            */
  void* page_tags; int32_t tag_bytes;    /* read for the current format, then rewritten    */
  uint8_t tag_map[16]; uint8_t tag_default;
  uint8_t fmt_to_tag[8];                 /* tag written for each IAK_FMT_* target          */
  int32_t* rejected;                     /* device counter or NULL                         */
} iak_convert_args;
int iak_convert_pages(const iak_page_pools* pools, const iak_convert_args* args, void* stream);

/* ------------------------------------------------------------------------
 * Multi-query (prefill / chunked prefill) attention over selected pages.
 *
 * Replaces triton_kernel.py:74-181 _fwd_kernel and :285-410
 * _fwd_kernel_quant as driven by :668-760 semantic_block_attention_triton,
 * with the exact-token semantics of reference.py:82-130
 * semantic_block_attention (causal masks on ORIGINAL token positions,
 * reference.py:16-45) that the reference's GPU path lacks: per-page row
 * masks select the rows of partially selected pages, and a key at token
 * position (page - bases[b*Ht+h]) * page_size + row (or page_positions[b, h,
 * slot] + row) is visible to query m iff it is <= q_positions[b, m] (causal).
 * Query rows that see no key are written as 0 (the reference's softmax gives
 * NaN there).
 * q [B, Hq, M, D], out [B, Hq, M, D]; G = Hq / Ht query heads share a
 * page-table row.  page_size <= 64 when row_masks is given.
 * ------------------------------------------------------------------------ */
typedef struct iak_prefill_args {
  const void* q; int32_t q_dtype; int64_t q_stride_b, q_stride_h, q_stride_m;
  void* out; int32_t out_dtype; int64_t out_stride_b, out_stride_h, out_stride_m;
  int32_t batch, num_q_heads, num_table_heads, num_queries;
  const int32_t* q_positions;   /* [B, M] (row stride qp_stride_b) or NULL = m */
  int64_t qp_stride_b;
  int32_t causal;
  const int32_t* page_table; int64_t pt_stride_b, pt_stride_h; int32_t table_width;
  const int32_t* page_counts; int64_t pc_stride_b;    /* [B, Ht] or NULL = W     */
  const int32_t* bases;         /* [B*Ht] or NULL = 0                             */
  const int32_t* page_positions;/* [B, Ht, W] token position of row 0 of each slot's page (overrides
                                   (page - base) * page_size), or NULL                            */
  int64_t pp_stride_b, pp_stride_h;
  const uint64_t* row_masks;    /* [B, W] (row stride rm_stride_b): bit r = row r selected; NULL = all */
  int64_t rm_stride_b;
  const void* page_tags; int32_t tag_bytes; uint8_t tag_map[16]; uint8_t tag_default;
  float sm_scale;
  int32_t kernel;               /* IAK_KERNEL_AUTO / GENERIC / TENSOR: the tensor-core kernel takes
                                   head_dim 128, page_size 8..64, table_width <= 1024, 16-byte aligned
                                   pools and sm_scale > 0; TENSOR on other calls -> IAK_ERR_UNSUPPORTED */
} iak_prefill_args;
int iak_prefill(const iak_page_pools* pools, const iak_prefill_args* args, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* INTENT_ATTENTION_B200_H */
