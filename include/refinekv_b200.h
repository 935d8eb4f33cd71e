/*
 * refinekv_b200.h -- C ABI of the RefineKV decode hot path on B200 (sm_100a).
 *
 * The reference (Kevin-lkw/RefineKV-release v0.1.2) is a Python package whose
 * GPU backend is a set of Triton kernels behind two launcher functions,
 * src/refinekv/kernels/runtime.py:93 (select_blocks_triton) and :123
 * (sparse_attention_triton), plus the torch-only summarizer
 * src/refinekv/summary.py:46 (build_summary).  This library replaces exactly
 * that seam.  Every entry point takes plain device pointers, element
 * strides, sizes, scalars and a cudaStream_t passed as void*, returns an
 * rkv_status, never allocates device memory, and only enqueues work on the
 * given stream (no host synchronisation), so every call can be captured in a
 * CUDA graph.
 *
 * Data types: K/V pages and summaries are bf16 (an fp32 K/V cache is
 * summarised by rkv_summarize_f32 into bf16 pages); queries are bf16 or
 * fp32 (rounded to bf16 before use, as the reference does); outputs are in
 * the query dtype.  Head dimensions: multiples of 32 up to 256; block sizes 16,
 * 32 and 64; GQA groups of 1..16 query rows per KV head.
 *
 * Caller-owned scratch: rkv_select and rkv_decode take a workspace whose
 * size comes from the matching *_workspace_size function (same arguments,
 * same current device).  It must be zero-filled once when it is allocated;
 * the kernels leave it reusable.  Word 0 of the workspace (int32) is a
 * sticky device status: nonzero bits mean a bounded device wait expired
 * (RKV_DEVICE_TIMEOUT) or a device-side input was out of range
 * (RKV_DEVICE_BAD_INPUT).  Calls that share a workspace must be ordered on
 * one stream.
 */
#ifndef REFINEKV_B200_H_
#define REFINEKV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RKV_ABI_VERSION 2

#if defined(__GNUC__)
#define RKV_API __attribute__((visibility("default")))
#else
#define RKV_API
#endif

typedef enum rkv_status {
  RKV_OK = 0,
  RKV_ERR_INVALID_ARGUMENT = 1, /* shapes, sizes, null pointers, eps, reduction */
  RKV_ERR_UNSUPPORTED = 2,      /* head_dim / block_size / group outside the kernel set */
  RKV_ERR_ALIGNMENT = 3,        /* a pointer or stride is not 16-byte aligned */
  RKV_ERR_WORKSPACE = 4,        /* workspace missing, too small or misaligned */
  RKV_ERR_CUDA = 5              /* a CUDA runtime call failed; see rkv_last_error() */
} rkv_status;

/* Bits of the device status word (int32 at workspace offset 0). */
#define RKV_DEVICE_TIMEOUT 1
#define RKV_DEVICE_BAD_INPUT 2

/* GQA reductions, RefineKVConfig.gqa_reduction (reference config.py:18). */
#define RKV_GQA_MEAN 0
#define RKV_GQA_MAX 1
#define RKV_GQA_ANY 2

/* Query / output dtypes. */
#define RKV_DTYPE_BF16 0
#define RKV_DTYPE_F32 1

/* Phases of rkv_decode (bit mask; RKV_PHASE_ALL for a normal call). */
#define RKV_PHASE_STATS 1  /* selector phase A: scores, deltas, LSE partials */
#define RKV_PHASE_FINAL 2  /* selector phase B: mask, compaction, representatives */
#define RKV_PHASE_ATTEND 4  /* refined pages + suffix: one partial per attention warp */
#define RKV_PHASE_COMBINE 8 /* LSE combine of all partials into the output */
#define RKV_PHASE_ALL 15

/*
 * Device view of a BlockSummary (reference summary.py:10-32).
 *   key_pages / value_pages: (heads, blocks, block_size, head_dim) bf16 with
 *     contiguous pages (page stride block_size*head_dim, row stride
 *     head_dim) and a free head stride (they may alias the KV cache).
 *   counts: (blocks,) int64 tokens per block (block_size, tail for the last).
 *   key_mean / value_mean / ellipsoid: (heads, blocks, head_dim) bf16, contiguous.
 *   value_norm: (heads, blocks) fp32; max_value_norm: (heads,) fp32.
 *
 * Batched decode (no reference counterpart: the reference decodes one
 * sequence, transformers.py:448-449).  With sequences > 1 the summary holds
 * several prompts that decode in lockstep: the head axis is sequence-major
 * (heads = sequences x KV heads, row = sequence * (heads / sequences) +
 * head), prompt_lengths is a (sequences,) int64 device array, prompt_length
 * is their maximum and blocks = ceil(prompt_length / block_size); counts is
 * (sequences, blocks) with 0 for the blocks past a sequence's prompt, whose
 * summary rows must be zero.  Such padding blocks are never selected,
 * represented or read; their mask bytes are written 0.  Queries, suffix
 * K/V, anchors, masks and outputs use the same sequence-major head axis, and
 * every sequence sees the same suffix length.  sequences 0 or 1 is one prompt
 * (prompt_lengths unused).
 *
 * Paged K/V (no reference counterpart; the layout of a vLLM-style page
 * pool).  With page_table non-null, key_pages / value_pages are pools of
 * pool_pages physical pages of block_size rows: the row t of KV head h in
 * physical page p is at p * page_stride + h * page_head_stride +
 * t * token_stride elements (HND pools [pages, heads, block, dim]: page
 * stride heads*block*dim, head stride block*dim, token stride dim; NHD pools
 * [pages, block, heads, dim]: block*heads*dim, dim, heads*dim).  Logical
 * block b of the sequence that KV-head row r belongs to is physical page
 * page_table[(r / (heads / sequences)) * page_table_stride + b]; entries
 * outside [0, pool_pages) set the status word's range bit and read zeros.
 * The summaries (means, ellipsoid, norms, counts) stay per sequence in
 * logical block order.  Only the decode attention reads pages, so
 * rkv_select ignores the page fields.
 */
typedef struct rkv_summary {
  const void* key_pages;
  const void* value_pages;
  int64_t key_page_head_stride;   /* elements */
  int64_t value_page_head_stride; /* elements */
  const int64_t* counts;
  const void* key_mean;
  const void* value_mean;
  const void* ellipsoid;
  const float* value_norm;
  const float* max_value_norm;
  int64_t heads;
  int64_t blocks;
  int64_t block_size;
  int64_t head_dim;
  int64_t prompt_length;
  int64_t sequences;              /* batched decode: see above; 0 or 1 for one prompt */
  const int64_t* prompt_lengths;  /* (sequences,) device array when sequences > 1 */
  /* Paged K/V (see below); all ignored when page_table is null. */
  const int32_t* page_table;      /* (sequences, page_table_stride) physical page per block */
  int64_t page_table_stride;      /* entries between sequences' rows of page_table */
  int64_t pool_pages;             /* physical pages in the pools */
  int64_t key_page_stride;        /* elements between consecutive physical pages */
  int64_t value_page_stride;
  int64_t key_token_stride;       /* elements between a page's rows (tokens) */
  int64_t value_token_stride;
} rkv_summary;

/*
 * Block summaries of one prompt (replaces reference summary.py:46-113,
 * build_summary; the page view of summary.py:35-43 is the optional copy).
 *   keys / values: (heads, tokens, head_dim) bf16, element strides given,
 *     innermost stride 1, 16-byte aligned rows.
 *   key_pages_out / value_pages_out: optional (heads, blocks, block_size,
 *     head_dim) contiguous destinations; when non-null the kernel also
 *     writes the zero-padded page copy (needed when tokens % block_size != 0
 *     or the cache rows are not page-contiguous).  Pass null for both or
 *     neither.
 *   Outputs as in rkv_summary; max_value_norm is zeroed by this call.
 */
RKV_API int rkv_summarize(const void* keys, const void* values, int64_t heads, int64_t tokens,
                  int64_t head_dim, int64_t key_head_stride, int64_t key_token_stride,
                  int64_t value_head_stride, int64_t value_token_stride, int64_t block_size,
                  void* key_pages_out, void* value_pages_out, void* key_mean, void* value_mean,
                  void* ellipsoid, float* value_norm, float* max_value_norm, int64_t* counts,
                  void* stream);

/*
 * rkv_summarize for an fp32 K/V cache (the reference's build_summary takes any
 * floating cache, summary.py:46-60; config 0 of its benchmarks is fp32).
 *   keys / values: (heads, tokens, head_dim) fp32, element strides given,
 *     innermost stride 1, 16-byte aligned rows.  The summaries are computed
 *     from the fp32 values, exactly as rkv_summarize does from bf16 ones.
 *   key_pages_out / value_pages_out: required (heads, blocks, block_size,
 *     head_dim) bf16 destinations for the zero-padded page copy rounded to
 *     bf16 -- the values the reference's attention uses, since it rounds the
 *     prompt K/V to bf16 before use (reference.py:57, :63-66).  The summary
 *     handed to rkv_select / rkv_decode points at these bf16 pages.
 */
RKV_API int rkv_summarize_f32(const float* keys, const float* values, int64_t heads,
                              int64_t tokens, int64_t head_dim, int64_t key_head_stride,
                              int64_t key_token_stride, int64_t value_head_stride,
                              int64_t value_token_stride, int64_t block_size, void* key_pages_out,
                              void* value_pages_out, void* key_mean, void* value_mean,
                              void* ellipsoid, float* value_norm, float* max_value_norm,
                              int64_t* counts, void* stream);

/*
 * rkv_summarize fused with the prefill's cache write (replaces the
 * reference's prefill sequence transformers.py:529-536, which writes the
 * prompt into the cache and then summarises it from there with
 * summary.py:46-113): reads the prompt K/V once and writes them, as the
 * zero-padded page copy, into rows [0, ceil(tokens / block_size) *
 * block_size) of each head of a cache whose head h starts
 * h * *_cache_head_stride elements after its base (rows of head_dim
 * elements, contiguous), plus the summaries.  The cache then holds the
 * prompt and is the summary's page view.  The head strides must hold the
 * padded prompt.  Rows past the prompt in its last page are written as
 * zeros by this call, but they are cache rows: a decoder that appends its
 * generated tokens to the cache overwrites them later.  The decode kernels
 * never read them as prompt rows (each page's valid rows come from its
 * count), so nothing may rely on them staying zero.
 */
RKV_API int rkv_summarize_into(const void* keys, const void* values, int64_t heads, int64_t tokens,
                       int64_t head_dim, int64_t key_head_stride, int64_t key_token_stride,
                       int64_t value_head_stride, int64_t value_token_stride, int64_t block_size,
                       void* key_cache, int64_t key_cache_head_stride, void* value_cache,
                       int64_t value_cache_head_stride, void* key_mean, void* value_mean,
                       void* ellipsoid, float* value_norm, float* max_value_norm,
                       int64_t* counts, void* stream);

/*
 * Workspace bytes for rkv_select with `queries` query instances.
 */
RKV_API size_t rkv_select_workspace_size(int64_t heads, int64_t group, int64_t blocks, int64_t head_dim,
                                 int64_t queries);

/*
 * Block selection for one or more queries (replaces reference
 * kernels/runtime.py:93 select_blocks_triton; math of reference.py:10-47).
 *   queries: (queries, heads, group, head_dim) contiguous, dtype query_dtype.
 *   mask: (heads, blocks) uint8 (0/1, usable as a bool tensor).  With
 *     accumulate == 0 and queries == 1 the mask is overwritten; otherwise
 *     (accumulate != 0, or several queries) the union of the selections is
 *     ORed into it -- several queries with accumulate == 0 first clear it.
 *     Several queries give the prompt-anchor union of reference
 *     integrations/transformers.py:543-552 in one pair of launches.
 */
RKV_API int rkv_select(const rkv_summary* summary, const void* queries, int query_dtype, int64_t queries_n,
               int64_t group, float eps, int reduction, uint8_t* mask, int accumulate,
               void* workspace, size_t workspace_size, void* stream);

/*
 * Workspace bytes for rkv_decode.
 */
RKV_API size_t rkv_decode_workspace_size(int64_t heads, int64_t group, int64_t blocks, int64_t head_dim,
                                 int64_t block_size);

/*
 * One decode step of one layer: selection, representatives, refined pages,
 * suffix and combine (replaces reference kernels/runtime.py:123
 * sparse_attention_triton; math of reference.py:50-73).
 *   query: (heads, group, head_dim) contiguous, dtype query_dtype.
 *   key_suffix / value_suffix: (heads, suffix_capacity, head_dim) bf16 with
 *     element strides; may be null when suffix_capacity == 0.
 *   suffix_length: device int32 scalar with the visible suffix length (CUDA
 *     graph replay), or null to use suffix_length_host.
 *   anchor_mask: (heads, blocks) uint8 or null; ORed into the selection.
 *   output: (heads, group, head_dim) in query_dtype.
 *   selected: (heads, blocks) uint8 mask written by the call.
 *   phases: RKV_PHASE_ALL, or a subset for timing individual kernels (the
 *     phases must still run in order on the stream); a subset always runs
 *     the four-kernel form (stats, final, attention, combine).
 * RKV_PHASE_ALL runs one kernel (the default for up to 480 KV-head rows,
 * see rkv_decode_kernel_count): heads x parts CTAs, at most one per SM,
 * whose parts of a row wait for one another at bounded barriers.  Decode
 * calls that run concurrently on different streams of one GPU can keep each
 * other's CTAs from becoming resident; their barriers then give up after 1 s
 * with RKV_DEVICE_TIMEOUT in the status word.  Order such calls on one
 * stream (one decode step of a batch of sequences is one call: see the
 * batched summary above), or switch to the four-kernel form with
 * rkv_set_fused_selector(0).
 */
RKV_API int rkv_decode(const rkv_summary* summary, const void* query, int query_dtype, int64_t group,
               const void* key_suffix, const void* value_suffix, int64_t suffix_capacity,
               int64_t key_suffix_head_stride, int64_t key_suffix_token_stride,
               int64_t value_suffix_head_stride, int64_t value_suffix_token_stride,
               const int32_t* suffix_length, int64_t suffix_length_host,
               const uint8_t* anchor_mask, float eps, int reduction, void* output,
               uint8_t* selected, void* workspace, size_t workspace_size, unsigned phases,
               void* stream);

/*
 * rkv_decode without a workspace, for callers that cannot allocate device
 * memory on the decode path: hosts that reach this library only through its
 * C ABI (an FFI from a language with no CUDA allocator of its own), or serving
 * stacks that hand out all device memory before decoding starts and may not
 * allocate afterwards.  This entry point has
 * no counterpart in the reference.
 *   Same arguments and results as rkv_decode with phases = RKV_PHASE_ALL,
 *   minus the workspace.  Scratch comes from one array of
 *   RKV_DECODE_STATIC_SCRATCH_BYTES inside the library's device image, which
 *   every GPU that loads the library holds until the process exits;
 *   geometries whose rkv_decode_workspace_size exceeds it are rejected with
 *   RKV_ERR_WORKSPACE.  All calls on a device share that array and it keeps
 *   the last call's contents (the status word is cleared at the start of each
 *   call), so calls that can overlap on the GPU race: order them on one
 *   stream.  The first call on each device looks up the array's address, with
 *   that device current; make it before any stream capture.  The address is
 *   kept for the life of the process and belongs to the context current at
 *   that first call: after cudaDeviceReset, or any other teardown of the
 *   device's primary context, do not call this entry point on that device
 *   again.  Allocates nothing.
 */
#define RKV_DECODE_STATIC_SCRATCH_BYTES ((size_t)32 << 20)
RKV_API int rkv_decode_static(const rkv_summary* summary, const void* query, int query_dtype,
                              int64_t group, const void* key_suffix, const void* value_suffix,
                              int64_t suffix_capacity, int64_t key_suffix_head_stride,
                              int64_t key_suffix_token_stride, int64_t value_suffix_head_stride,
                              int64_t value_suffix_token_stride, const int32_t* suffix_length,
                              int64_t suffix_length_host, const uint8_t* anchor_mask, float eps,
                              int reduction, void* output, uint8_t* selected, void* stream);

/*
 * Device status word of the last rkv_decode_static call on the current device
 * (0, or the RKV_DEVICE_* bits: a bounded wait that ran out, a device-side
 * input out of range), copied to `out` -- a host or device int32 -- on
 * `stream`, ordered after the calls already issued on it.  With a host
 * pointer, read `*out` after synchronising the stream.  Like
 * rkv_decode_static it allocates nothing and has no counterpart in the
 * reference.
 */
RKV_API int rkv_decode_static_status(int32_t* out, void* stream);

/*
 * Dense decode attention over every page of a prompt plus the suffix, on the
 * same streaming kernel as rkv_decode's refinement (no selector, no
 * representatives): the attention of the adapter's full_attention_layers
 * (reference transformers.py:510-520, dense SDPA over the visible cache)
 * without a mask over a fixed-capacity cache, so that dense layers decode
 * from a CUDA graph at streaming speed.
 *   pages: only the page fields of rkv_summary are read -- key_pages /
 *     value_pages and their strides (contiguous pages, a page pool, or a
 *     batch), heads, blocks, block_size, head_dim, prompt_length, sequences /
 *     prompt_lengths; every row of block b past the prompt is ignored, so the
 *     pages may be a page view of a KV cache whose later rows hold other
 *     tokens.  The summary pointers may be null.
 *   Other arguments as rkv_decode (phases are attention + combine); the
 *   workspace comes from rkv_decode_dense_workspace_size and follows the
 *   same rules.  Results: output (heads, group, head_dim) in query_dtype.
 */
RKV_API size_t rkv_decode_dense_workspace_size(int64_t heads, int64_t group, int64_t blocks,
                                               int64_t head_dim, int64_t block_size);
RKV_API int rkv_decode_dense(const rkv_summary* pages, const void* query, int query_dtype,
                             int64_t group, const void* key_suffix, const void* value_suffix,
                             int64_t suffix_capacity, int64_t key_suffix_head_stride,
                             int64_t key_suffix_token_stride, int64_t value_suffix_head_stride,
                             int64_t value_suffix_token_stride, const int32_t* suffix_length,
                             int64_t suffix_length_host, void* output, void* workspace,
                             size_t workspace_size, void* stream);

/* Kernel launches one rkv_decode call makes for the given phases in the
 * four-kernel form (4 for RKV_PHASE_ALL). */
RKV_API int rkv_decode_launch_count(unsigned phases);

/*
 * Kernel launches of one rkv_decode call (RKV_PHASE_ALL) for this geometry on
 * the current device: 1 when the one-kernel decode runs (selector, every
 * page, the representatives and the combine in one launch), else 4 (stats,
 * final, attention, combine); 0 for an unsupported geometry.
 */
RKV_API int rkv_decode_kernel_count(int64_t heads, int64_t group, int64_t blocks,
                                    int64_t head_dim, int64_t block_size);

/*
 * Process-wide switch of rkv_decode's one-kernel form (on by default; the
 * name is kept from when only the selector was fused).  With 0, rkv_decode
 * runs four kernels (stats, final, attention, combine) and the attention
 * kernel streams every selected page, anchored or not -- for measurement and
 * cross-checks; the results agree within the summation-order tolerance.
 * Set it before planning a workspace: workspace sizes depend on it.  No
 * reference counterpart.
 */
RKV_API void rkv_set_fused_selector(int enable);

/*
 * Sequence split: the prompt blocks of each KV head are spread over `ranks`
 * GPUs (contiguous block ranges; the generated-token suffix on one of them),
 * for when GPUs outnumber KV heads.  The reference runs one GPU per sequence
 * and has no such mode; the math is the same decode step (reference.py:50-73)
 * with its two row-global reductions -- the selector normalisers log Z and
 * log C (reference.py:15-17) and the softmax denominator -- merged across
 * ranks.  A split step is three calls with two all-gathers between them,
 * issued by the host over its own communicator (NCCL in refinekv_b200.parallel):
 *
 *   rkv_decode_split(..., RKV_SPLIT_STATS)   selector phase A; writes this
 *                                            rank's stats slab
 *   all-gather of the stats region           (ranks x stats_slab bytes, in place)
 *   rkv_decode_split(..., RKV_SPLIT_ATTEND)  selector phase B over all ranks'
 *                                            slabs, attention, combine into this
 *                                            rank's output slab (m, l, o per row)
 *   all-gather of the output region          (ranks x output_slab bytes, in place)
 *   rkv_decode_split(..., RKV_SPLIT_MERGE)   LSE merge of the ranks' rows into
 *                                            `output` (every rank gets it)
 *
 * The exchange buffer holds the stats region (ranks stats slabs) followed by
 * the output region (ranks output slabs).  Every rank of a group must pass the
 * same heads, group, head_dim, ranks and max_blocks (the largest block count
 * of any rank), which fix the slab sizes.  Each rank's summary covers only its
 * own blocks, except max_value_norm, which must hold the maximum over all
 * ranks (one all-reduce after summarising).  The workspace is the one
 * rkv_decode_workspace_size gives for this rank's blocks; the same workspace
 * and exchange buffer must be passed to the three calls of a step.
 */
#define RKV_SPLIT_STATS 1
#define RKV_SPLIT_ATTEND 2
#define RKV_SPLIT_MERGE 4
#define RKV_SPLIT_FINAL 2 /* rkv_select_split: phase B over all ranks' slabs */

/*
 * Block selection of rkv_select under a sequence split (the prompt-anchor
 * union at prefill): the same two-step exchange without attention.
 *   rkv_select_split(..., RKV_SPLIT_STATS)  phase A into this rank's slab
 *   all-gather of the exchange buffer        (ranks x slab bytes, in place)
 *   rkv_select_split(..., RKV_SPLIT_FINAL)  phase B over all slabs; writes
 *                                           `mask` for this rank's blocks
 * Slab bytes come from rkv_select_split_slab (0 for an invalid geometry);
 * queries_n and max_blocks must be equal on all ranks.  `mask`, `accumulate`
 * and the workspace are as for rkv_select.
 */
RKV_API size_t rkv_select_split_slab(int64_t heads, int64_t group, int64_t max_blocks,
                                     int64_t queries);
RKV_API int rkv_select_split(const rkv_summary* summary, const void* queries, int query_dtype,
                             int64_t queries_n, int64_t group, float eps, int reduction,
                             uint8_t* mask, int accumulate, void* workspace,
                             size_t workspace_size, int64_t ranks, int64_t rank,
                             int64_t max_blocks, void* exchange, size_t exchange_size,
                             unsigned stage, void* stream);

/* Slab sizes (bytes, multiples of 256) of one rank in the two exchange regions. */
RKV_API int rkv_split_exchange_slabs(int64_t heads, int64_t group, int64_t max_blocks,
                                     int64_t head_dim, size_t* stats_slab, size_t* output_slab);

/*
 * One stage of a sequence-split decode step (arguments as rkv_decode, plus
 * the split geometry).  `selected` covers this rank's blocks; `output` is
 * written by RKV_SPLIT_MERGE only.  `exchange` must be 256-byte aligned and
 * hold ranks * (stats_slab + output_slab) bytes.
 */
RKV_API int rkv_decode_split(const rkv_summary* summary, const void* query, int query_dtype,
                             int64_t group, const void* key_suffix, const void* value_suffix,
                             int64_t suffix_capacity, int64_t key_suffix_head_stride,
                             int64_t key_suffix_token_stride, int64_t value_suffix_head_stride,
                             int64_t value_suffix_token_stride, const int32_t* suffix_length,
                             int64_t suffix_length_host, const uint8_t* anchor_mask, float eps,
                             int reduction, void* output, uint8_t* selected, void* workspace,
                             size_t workspace_size, int64_t ranks, int64_t rank,
                             int64_t max_blocks, void* exchange, size_t exchange_size,
                             unsigned stage, void* stream);

/*
 * Diagnostic: one bounded device wait on an mbarrier that nothing completes,
 * with a limit of `limit_ns` (0 < limit_ns <= 1e9) instead of the kernels'
 * 1 s; it ORs RKV_DEVICE_TIMEOUT into the device int32 *status and returns,
 * the path every kernel takes when a wait runs out.  No counterpart in the
 * reference (which has no device waits); used by the failure-handling tests.
 */
RKV_API int rkv_selftest_wait_timeout(int32_t* status, int64_t limit_ns, void* stream);

/* Message of the last failing call on this host thread ("" if none). */
RKV_API const char* rkv_last_error(void);
RKV_API const char* rkv_status_string(int status);
RKV_API int rkv_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* REFINEKV_B200_H_ */
