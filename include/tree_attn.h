/*
 * tree_attn.h -- C ABI of the B200 (sm_100a) tree-shared decode-attention kernels.
 *
 * The reference (Gxj230958/tree-attention-scheduling) drives its two Triton
 * kernels from Python (src/tree_attention/kernels.py).  These entry points are
 * the boundary those launches map to; every argument is a plain pointer or
 * integer, no framework types.  Device pointers are CUDA global-memory
 * addresses on the current device; `stream` is a cudaStream_t (NULL = legacy
 * default stream).  No entry point synchronises the stream or allocates
 * memory, so all of them can be recorded into a CUDA graph.
 *
 * Layouts (all row-major, contiguous):
 *   q      [num_requests, num_q_heads, head_dim]            bf16 or f16
 *   kpool  [num_kv_heads, pool_tokens, head_dim]             same dtype as q
 *   vpool  [num_kv_heads, pool_tokens, head_dim]             same dtype as q
 *   part   [num_kv_heads, num_partials * G, head_dim]        f32 scratch
 *   lse    [num_kv_heads, num_partials * G]                  f32 scratch
 *   out    [num_requests, num_q_heads, head_dim]             dtype of q
 * with G = num_q_heads / num_kv_heads.  The reference keeps K as [H, D, T]
 * (kernels.py:144-145); here K and V share the token-major [H, T, D] layout,
 * which makes every key row one 2*head_dim-byte line for TMA and bulk copies.
 *
 * Plan metadata is one int32 device buffer holding the arrays described by
 * ta_plan_layout (offsets in int32 elements from `meta`).  The first six are
 * the reference's own arrays from prepare() (kernels.py:103-141), bit-exact:
 *   qids   [num_jobs, max_requests]   request ids of each job, zero padded
 *   kstart [num_jobs, kstart_stride]  first physical position of each job
 *   qlen   [num_jobs]                 requests per job
 *   klen   [num_jobs]                 positions per job (mutable, see below)
 *   slots  [num_requests, max_slots]  reference slot code job*max_requests+j
 *   counts [num_requests]             reference partials per request
 * followed by this implementation's own arrays.  A job is executed as one or
 * more pieces, contiguous key ranges with their own partial slots:
 *   pieces      [num_pieces, 4]             job, key offset, keys, first partial slot;
 *                                           a piece covers keys [offset, offset +
 *                                           min(keys, klen[job] - offset)) of its job
 *   pcounts     [num_requests]              partials per request (over pieces)
 *   cslots      [num_requests, max_pslots]  partial slots of each request
 *   small_tasks [num_small_tasks, 2]        (piece, 16-row tile), SIMT kernel
 *   tc_tasks    [num_tc_tasks, 4]           (piece, 256-row pair, first request of the job if its
 *                                           requests are contiguous else -1, 0), query-tile kernel
 *   kn_offsets  [kn_ctas + 1]               task range of each persistent CTA of the
 *                                           keys-in-lanes tcgen05 kernel
 *   kn_tasks    [num_kn_tasks, 4]           its task headers: first segment, segments, 0, 0
 *   kn_segs     [num_kn_segs, 12]           segments: KV head, first query row in the
 *                                           task, query rows, first partial row, first
 *                                           pool position, first key of its slot in the
 *                                           tile, keys, job | growing << 30 (growing: keys
 *                                           = min(keys, klen[job]), a decode tail), first
 *                                           request if the segment's requests are contiguous
 *                                           (else -1), index of the segment's first request
 *                                           within its job (a job's rows may be cut into
 *                                           several segments), 0, 0; a task of several
 *                                           segments is one 128-key tile
 * Every array starts at a multiple of 4 int32 (16 bytes).  Partial slot s of a
 * piece holds query rows s*G .. s*G+G-1 (one request).
 *
 * Return value: 0 on success, otherwise a TA_ERR_* code describing a rejected
 * argument or a launch failure.  Errors found on the device (a metadata index
 * out of range, a bounded wait that gave up) are OR-ed into *status (a device
 * int32 the caller owns and zeroes; may be NULL) and never trap.
 */
#ifndef TREE_ATTN_H
#define TREE_ATTN_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TA_ABI_VERSION 5

#define TA_DTYPE_BF16 1
#define TA_DTYPE_F16 2

#define TA_OK 0
#define TA_ERR_ARG 1          /* host: invalid argument, nothing launched */
#define TA_ERR_LAUNCH 2       /* host: a kernel launch failed */
#define TA_ERR_BOUNDS 4       /* device: plan index out of range, access skipped */
#define TA_ERR_TIMEOUT 8      /* device: a bounded wait gave up */
#define TA_ERR_UNSUPPORTED 16 /* host: shape or dtype without a kernel */
#define TA_ERR_TOO_LARGE 32   /* host: the problem exceeds ta_attention_noalloc's fixed scratch,
                                 or ta_plan_build's meta_capacity */

/* Size of the device scratch array behind ta_attention_noalloc, per GPU. */
#define TA_NOALLOC_SCRATCH_BYTES (32u << 20)

typedef struct ta_plan_layout {
  int32_t num_jobs;
  int32_t max_requests;
  int32_t max_slots;
  int32_t num_requests;
  int32_t num_pieces;
  int32_t num_partials;  /* partial slots: sum over pieces of their job's requests */
  int32_t max_pslots;
  int32_t num_small_tasks;
  int32_t num_tc_tasks;
  int32_t num_kn_tasks;
  int32_t num_kn_segs;
  int32_t kn_ctas;       /* persistent CTAs of the keys-in-lanes launches, all classes */
  /* keys-in-lanes tasks are grouped by query rows into classes of at most 4,
     8, 16, 32 and 64 rows, one launch per non-empty class; class c has
     kn_class_ctas[c] persistent CTAs, whose kn_offsets entries follow those
     of the classes before it (the sum is kn_ctas).  This build has kernels
     for the 4- and 8-row classes; a plan with CTAs in the others is rejected
     with TA_ERR_UNSUPPORTED. */
  int32_t kn_class_ctas[5];
  /* small tasks are sorted by padded row count: [0, e0) need 4 rows,
     [e0, e1) 8 rows, [e1, e2) 16 rows; e2 == num_small_tasks */
  int32_t small_class_end[3];
  /* longest piece among small tasks when the plan was built (a hint: the
     SIMT kernel single-buffers when every task fits one 64-key chunk) */
  int32_t small_max_keys;
  int32_t kstart_stride;
  int32_t off_qids;
  int32_t off_kstart;
  int32_t off_qlen;
  int32_t off_klen;
  int32_t off_slots;
  int32_t off_counts;
  int32_t off_pieces;
  int32_t off_pcounts;
  int32_t off_cslots;
  int32_t off_small_tasks;
  int32_t off_tc_tasks;
  int32_t off_kn_offsets;
  int32_t off_kn_tasks;
  int32_t off_kn_segs;
} ta_plan_layout;

/* ABI version of the loaded library (TA_ABI_VERSION). */
int ta_abi_version(void);

/* Human-readable name of a TA_ERR_* code or status bit set. */
const char* ta_error_string(int code);

/*
 * Partial attention of every (piece, KV head) of the plan: for each query row
 * (request of the piece's job x GQA row) the softmax-normalised output over the
 * piece's positions and its natural-log LSE, written to part/lse at the row's
 * partial slot.  A piece with zero positions writes O = 0 and LSE = -inf.
 * Replaces the reference's _segment kernel (kernels.py:8-55) and its two launch
 * phases in attention_matrix (kernels.py:158-165).
 */
int ta_segment(const ta_plan_layout* plan, const int32_t* meta, const void* q, const void* kpool,
               const void* vpool, int64_t pool_tokens, int32_t num_q_heads, int32_t num_kv_heads,
               int32_t head_dim, int32_t dtype, float* part, float* lse, int32_t* status, void* stream);

/*
 * Global log-sum-exp merge of each request's partials into out (dtype of q);
 * out_lse [num_requests, num_q_heads] f32 receives the merged LSE when not
 * NULL.  Partials with LSE = -inf contribute nothing; a request whose partials
 * are all empty gets O = 0.  Replaces the reference's _merge kernel
 * (kernels.py:58-83) launched at kernels.py:166-167.
 */
int ta_merge(const ta_plan_layout* plan, const int32_t* meta, const float* part, const float* lse,
             void* out, float* out_lse, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
             int32_t dtype, int32_t* status, void* stream);

/*
 * ta_segment followed by ta_merge on the same stream: the whole decode-step
 * attention of attention_matrix (kernels.py:152-168).
 */
int ta_attention(const ta_plan_layout* plan, const int32_t* meta, const void* q, const void* kpool,
                 const void* vpool, int64_t pool_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                 int32_t head_dim, int32_t dtype, float* part, float* lse, void* out, float* out_lse,
                 int32_t* status, void* stream);

/*
 * ta_attention for callers that cannot allocate device memory: no counterpart
 * in the reference, which always allocates its scratch in prepare().  A
 * process whose device memory is owned by another allocator, a binding without
 * access to a CUDA allocator, or a serving loop that must not allocate on its
 * decode path passes only its inputs and outputs; the
 * partial outputs and LSEs live in one file-scope device array of
 * TA_NOALLOC_SCRATCH_BYTES per GPU (held by every GPU that loads the library,
 * until exit).  Problems needing more than that -- num_kv_heads * num_partials
 * * G * (head_dim + 1) floats plus 256 bytes -- return TA_ERR_TOO_LARGE without
 * launching.  The first call on a device looks the array's address up (make it
 * before any stream capture).  All calls share the array: calls whose kernels
 * overlap on the GPU race on it and must be serialised by the caller; nothing
 * in it needs to start at zero.  Allocates nothing.
 */
int ta_attention_noalloc(const ta_plan_layout* plan, const int32_t* meta, const void* q, const void* kpool,
                         const void* vpool, int64_t pool_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                         int32_t head_dim, int32_t dtype, void* out, float* out_lse, int32_t* status, void* stream);

/*
 * klen[tail_jobs[i]] = value for i < num_tails, on the device: the per-step
 * update of a reused decode plan, CachedDecodePlan.update (kernels.py:184-186).
 * A growing tail job must be a single piece (offset 0, keys >= every value).
 */
int ta_update_tail_klen(int32_t* klen, const int32_t* tail_jobs, int32_t num_tails, int32_t value,
                        int32_t num_jobs, int32_t* status, void* stream);

/*
 * One decode step's KV append for one layer, fused into one launch: for every
 * request r < num_requests and KV head h < num_kv_heads, the new rows
 * k_new[r * new_stride_request + h * new_stride_head + (0 .. head_dim)] (and
 * likewise v_new; strides in elements, rows contiguous) are written to
 * kpool / vpool [num_kv_heads, pool_tokens, head_dim] at position targets[r]
 * (device int64).  Replaces the two index_copy_ calls of the reference's
 * decode step (qwen.py:89-90).  When klen is not NULL the same launch also sets
 * klen[tail_jobs[i]] = *count + offset for i < num_tails, with count a device
 * int64: CachedDecodePlan.update (kernels.py:184-186) without a host value, so
 * a captured step advances on the device.  A target outside [0, pool_tokens),
 * a tail index outside [0, num_jobs) or a length outside int32 is skipped and
 * TA_ERR_BOUNDS is OR-ed into *status.  Pointers must be 4-byte aligned and
 * head_dim and the strides even (rows move as bf16/f16 pairs).
 */
int ta_decode_append(void* kpool, void* vpool, const void* k_new, const void* v_new, int64_t new_stride_request,
                     int64_t new_stride_head, const int64_t* targets, int32_t num_requests, int32_t num_kv_heads,
                     int64_t pool_tokens, int32_t head_dim, int32_t dtype, int32_t* klen, const int32_t* tail_jobs,
                     int32_t num_tails, const int64_t* count, int32_t offset, int32_t num_jobs, int32_t* status,
                     void* stream);

/*
 * Host-side plan builder: the metadata buffer and layout of a physical job list
 * that ta_segment / ta_merge / ta_attention consume.  Replaces the array loops
 * of the reference's prepare (kernels.py:103-141): qids, kids, qlen, klen,
 * slots and counts are the reference's arrays bit for bit (kids holds each
 * job's first position, kstart_stride 1); the execution pieces, compact partial
 * slots and the query-tile, keys-in-lanes and SIMT task lists follow them.
 *
 * Job j (in the caller's order: the reference's small-first stable sort) is the
 * requests job_reqs[job_req_offsets[j] .. job_req_offsets[j+1]) over the
 * contiguous positions [job_k0[j], job_k0[j] + job_keys[j]).  groups = query
 * heads per KV head; use_tc selects the tcgen05 routes (head_dim 128), else
 * every job runs on the SIMT kernel; sms is the SM count the task lists are
 * balanced for; jobs with job_k0 >= no_split_from stay one piece each (the
 * growing decode tails; no_split_from < 0: none).
 *
 * meta receives the int32 buffer, every array on a 16-byte boundary at the
 * layout's off_* offsets.  On TA_ERR_TOO_LARGE (meta_capacity below the
 * need) nothing is written to meta; *meta_size and *layout are set either way.
 * TA_ERR_ARG: an empty job, a request outside [0, num_requests), a
 * non-positive count.  TA_ERR_UNSUPPORTED: a keys-in-lanes task above 64 rows.
 * Pure host code: needs no GPU.
 */
int ta_plan_build(const int32_t* job_req_offsets, const int32_t* job_reqs, const int32_t* job_k0,
                  const int32_t* job_keys, int32_t num_jobs, int32_t num_requests, int32_t groups,
                  int32_t use_tc, int32_t num_kv_heads, int32_t sms, int64_t no_split_from, int32_t* meta,
                  int64_t meta_capacity, int64_t* meta_size, ta_plan_layout* layout);

/* Roofline constants of the tree scheduler's cost model (reference
   schedule.py:29-39): bytes and FLOP per microsecond, per-task and per-partial
   overheads, the small-group row and key tiles, the longest KV segment of a
   job, and the large-group query-row tile (also the per-job request cap). */
typedef struct ta_cost_model {
  double bandwidth;
  double cube_flops;
  double task_us;
  double merge_us;
  int32_t cube_rows;
  int32_t key_tile;
  int32_t kv_split;
  int32_t max_query_rows;
} ta_cost_model;

#define TA_SCHEDULE_GREEDY 1
#define TA_SCHEDULE_CUBE 2

/*
 * Host-side tree scheduler: the greedy or subset-DP ("cube") recursion of the
 * reference (schedule.py:96-143) with its job cost (schedule.py:41-52), run to
 * the decisions its materialisation needs.  Node n (0 = root; children after
 * their parent) has children children[child_offsets[n] .. child_offsets[n+1]),
 * node_requests[n] requests passing through it, and its positions as maximal
 * runs (first, length) = runs[2r], runs[2r+1] for r in [run_offsets[n],
 * run_offsets[n+1]).  On return pushed[n] = 1 where the plan pushes the
 * parent's inherited positions down into node n (the node's requests read them
 * in its own jobs), else 0; *root_cost (may be NULL) is the root's estimated
 * cost.  Every cost is computed as the reference's Python computes it (float
 * sums compensated as CPython's sum() does), so plans, ties included, match.
 * TA_ERR_ARG: a malformed tree or model; TA_ERR_UNSUPPORTED: a tree deeper
 * than 2000 levels.  Pure host code: needs no GPU.
 */
int ta_schedule_tree(const int32_t* child_offsets, const int32_t* children, const int32_t* node_requests,
                     const int32_t* run_offsets, const int64_t* runs, int32_t num_nodes, int32_t method,
                     const ta_cost_model* model, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                     uint8_t* pushed, double* root_cost);

#ifdef __cplusplus
}
#endif

#endif /* TREE_ATTN_H */
