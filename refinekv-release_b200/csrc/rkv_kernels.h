// Launch parameters shared by the host entry points (rkv_capi.cu) and the
// kernels.  Plain structs: pointers, sizes, scalars.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rkv {

constexpr int kSelectTile = 32;  // summary blocks per selector tile
constexpr int kMaxGroup = 16;    // GQA rows per KV head (two n8 tiles)
constexpr int kStatsSlots = 8;   // phase-A partials per CTA under a sequence split (one per warp)

enum Reduction { kMean = 0, kMax = 1, kAny = 2 };

// Batched decode: the KV-head rows of several prompts decoding in lockstep,
// sequence-major (row = sequence * heads_per_seq + head), all padded to the
// longest prompt's block count.  seq_prompt is null for a single prompt.
struct SeqLayout {
  const int64_t* seq_prompt;  // (sequences,) prompt lengths, or null
  int heads_per_seq;
  int page;  // tokens per block

  __device__ __forceinline__ int sequence(int row) const {
    return seq_prompt != nullptr ? row / heads_per_seq : 0;
  }
  // Prompt length of row's sequence (`single` for one prompt).
  __device__ __forceinline__ int prompt(int row, int single) const {
    return seq_prompt != nullptr ? static_cast<int>(__ldg(seq_prompt + row / heads_per_seq))
                                 : single;
  }
  // Real blocks of row's sequence (`single` for one prompt).
  __device__ __forceinline__ int blocks(int row, int single) const {
    return seq_prompt != nullptr ? (prompt(row, 0) + page - 1) / page : single;
  }
};

struct SummarizeMaps {
  CUtensorMap keys;    // (dim, tokens, heads), [block_size x 128 bytes] boxes, 128B swizzle
  CUtensorMap values;
};

struct SummarizeParams {
  int heads, tokens, blocks, block_size;
  int f32;            // the caches are fp32 (else bf16); pages are copied out as bf16
  int dim;            // real head dim (the kernel's D is dim rounded up to 64)
  int stages;         // TMA stages per warp
  void* key_pages;    // optional (heads, blocks, block, dim) copy, zero padded
  void* value_pages;  // optional
  int64_t key_pages_head_stride;    // elements between heads' page copies
  int64_t value_pages_head_stride;
  void* key_mean;     // bf16 (heads, blocks, dim)
  void* value_mean;
  void* ellipsoid;
  float* value_norm;      // (heads, blocks)
  float* max_value_norm;  // (heads,), zero on entry
  int64_t* counts;        // (blocks,)
};

struct StatsMaps {
  CUtensorMap key_mean;
  CUtensorMap ellipsoid;
};

struct StatsParams {
  const void* query;  // (instances, heads, group, dim)
  int query_f32;
  int dim;            // real head dim (the kernel's D is dim rounded up to 64)
  const int64_t* counts;
  int heads, group, blocks, instances;
  int tiles, tiles_per_cta, parts;
  int slots;     // partials per CTA: the warp count, or kStatsSlots under a split
  int stages;
  float scale;
  float* z;      // (instances*heads*group, blocks)
  float* delta;  // (instances*heads*group, blocks)
  float* lse;    // (instances*heads*group, parts * slots, 4): z max, z sum, c max, c sum
  SeqLayout seq;  // counts is (sequences, blocks) when batched
  int* status;
};

struct FinalMaps {
  CUtensorMap value_mean;
};

struct FinalParams {
  int heads, group, blocks, instances;
  int tiles, tiles_per_cta, parts_a, parts;
  int stages;
  float eps;
  int reduction;
  const float* z;
  const float* delta;
  // Phase-A partials: lse_slabs slabs of (instances*heads*group, parts_a, 4)
  // (parts_a = phase-A CTAs per row x partials per CTA),
  // lse_slab_floats apart (one slab per rank of a sequence split, else one).
  const float* lse;
  int lse_slabs;
  size_t lse_slab_floats;
  const float* value_norm;
  const float* max_value_norm;
  const uint8_t* anchor;  // (heads, blocks) or null
  uint8_t* mask;          // (heads, blocks)
  int accumulate;         // OR into mask instead of overwriting it
  int decode;             // also compact ids and accumulate representatives
  int split_probs;        // FP32-query mode: hi/lo bf16 split of the probabilities
  int* seg_count;         // (heads, parts)
  int* sel_ids;           // (heads, parts, seg_cap)
  int seg_cap;
  float* rep_m;  // (heads, parts, G8)
  float* rep_l;
  float* rep_o;  // (heads, parts, dim, G8): o^T, group rows innermost
  SeqLayout seq;
  int* status;
};

// One-kernel decode (rkv_fused.cu): for a (KV-head row, part) tile range, in
// one CTA, the selector's two phases (a per-row barrier between them), the
// attention of every page the range needs (anchored, selected, the part's
// share of the suffix) and its representatives, and -- after a second
// per-row barrier -- the row's output channels of this part merged from all
// parts' partials.  Row h has parts_base + 1 parts if h < parts_extra, else
// parts_base; CTA c is part c - first(h) of its row.
struct FusedMaps {
  CUtensorMap key_mean;     // [32 x 64] bf16 boxes, like StatsMaps / FinalMaps
  CUtensorMap ellipsoid;
  CUtensorMap value_mean;
  CUtensorMap key_pages;    // 4-D page maps, like AttendMaps
  CUtensorMap value_pages;
  CUtensorMap key_suffix;   // 3-D row maps, like AttendMaps
  CUtensorMap value_suffix;
};

struct FusedParams {
  const void* query;  // (heads, group, dim)
  int query_f32;
  int dim;            // real head dim
  void* out;          // (heads, group, dim) in the query dtype
  const int64_t* counts;
  int heads, group, blocks, tiles;
  int parts_base, parts_extra;  // parts per row (see above)
  int tcap;           // the largest tile count of a part (shared-memory tables)
  int zd_group;       // > 0: z and delta stay in shared memory (else the workspace's z, delta)
  float scale, eps;
  int reduction;
  float* z;           // (heads*group, blocks)
  float* delta;
  float* lse;         // (heads*group, (parts_base + 1) * warps, 4)
  const float* value_norm;
  const float* max_value_norm;
  const uint8_t* anchor;  // (heads, blocks) or null
  uint8_t* mask;
  int split_probs;
  float* part_m;          // (grid, G8): one softmax partial per CTA
  float* part_l;
  float* part_o;          // (grid, dim, G8)
  unsigned* bar_words;    // per row: arrivals A, generations A, arrivals B, generations B
  int bar_stride;         // words between those four arrays
  SeqLayout seq;
  int page, prompt_length;
  const int32_t* page_table;
  int page_table_stride;
  int pool_pages;
  int has_suffix, suffix_capacity;
  const int* suffix_len_ptr;
  int suffix_len_host;
  int* status;
};

struct AttendMaps {
  CUtensorMap key_pages;
  CUtensorMap value_pages;
  CUtensorMap key_suffix;
  CUtensorMap value_suffix;
};

struct AttendParams {
  const void* query;  // (heads, group, dim)
  int query_f32;
  int dim;            // real head dim (the kernel's D is dim rounded up to 64)
  const int64_t* counts;
  int heads, group, blocks, page;
  int prompt_length;  // rows of block b: min(page, prompt_length - b * page)
  SeqLayout seq;      // batched: each row's own prompt length
  // Paged K/V: physical page of (sequence, block) (null: page = block).
  const int32_t* page_table;
  int page_table_stride;
  int pool_pages;
  int has_suffix;
  int suffix_capacity;
  const int* suffix_len_ptr;  // device scalar or null
  int suffix_len_host;
  const int* seg_count;
  const int* sel_ids;
  int parts_b, seg_cap;
  // Dense decode (rkv_decode_dense): every block of a row is attended, in
  // order, with no selector (seg_count / sel_ids unused, parts_b 1).
  int dense;
  // One partial per (head, CTA, warp), (head, CTA) pairs indexed by head +
  // cta: m, l ((heads + ctas) * warps, G8) and o^T ((heads + ctas) * warps,
  // dim, G8).
  float* att_m;
  float* att_l;
  float* att_o;
  int ctas;
  int stages;
  int* status;
  float scale;
};

struct CombineParams {
  int query_f32;
  int dim;    // real head dim; one CTA column per 32 real channels
  void* out;  // (heads, group, dim) in the query dtype
  int heads, group, page;
  int has_suffix, suffix_capacity;
  const int* suffix_len_ptr;
  int suffix_len_host;
  const int* seg_count;
  int parts_b;
  int dense;           // rkv_decode_dense: no representatives; every block of a row attended
  SeqLayout seq;       // dense: each row's own block count
  int blocks;          // dense: blocks of a single prompt
  const float* rep_m;  // (heads, parts_b, G8)
  const float* rep_l;
  const float* rep_o;  // (heads, parts_b, dim, G8)
  const float* att_m;  // ((heads + ctas) * warps, G8)
  const float* att_l;
  const float* att_o;  // ((heads + ctas) * warps, dim, G8)
  int ctas, warps;     // the attention launch's grid
  int max_sources;     // capacity of the shared-memory source table
  // Sequence split: when non-null, each row's merged (max, sum) goes to
  // part_ml[row * 2 + {0, 1}] and its normalised output to part_o[row * dim
  // + d] (FP32, real dim) instead of `out`.
  float* part_ml;
  float* part_o;
  int* status;
};

// LSE merge of the ranks' rows of a sequence split (rkv_decode_split).
struct MergeParams {
  int query_f32;
  int dim;    // real head dim
  void* out;  // (heads, group, dim) in the query dtype
  int heads, group;
  int ranks;
  const float* part_ml;  // slab r: part_ml + r * slab_floats, (rows, 2)
  const float* part_o;   // slab r: part_o + r * slab_floats, (rows, dim)
  size_t slab_floats;
};

// Host launchers (defined in the .cu files); return a cudaError_t.
cudaError_t launch_summarize(const SummarizeMaps& maps, const SummarizeParams& p, int dim,
                             int ctas, int warps, size_t smem, cudaStream_t stream);
cudaError_t launch_stats(const StatsMaps& maps, const StatsParams& p, int dim, int warps,
                         size_t smem, cudaStream_t stream, bool pdl);
cudaError_t launch_final(const FinalMaps& maps, const FinalParams& p, int dim, int warps,
                         size_t smem, cudaStream_t stream, bool pdl);
cudaError_t launch_attend(const AttendMaps& maps, const AttendParams& p, int dim, int warps,
                          size_t smem, cudaStream_t stream, bool pdl);
cudaError_t launch_combine(const CombineParams& p, int dim, cudaStream_t stream, bool pdl);
cudaError_t launch_fused(const FusedMaps& maps, const FusedParams& p, int dim, int warps,
                         size_t smem, cudaStream_t stream, bool pdl);
cudaError_t launch_merge(const MergeParams& p, int dim, cudaStream_t stream, bool pdl);

// Raise `func`'s dynamic shared-memory limit to at least `bytes` on the
// current device.  Done once per (kernel, device): later calls, including
// those made while a CUDA graph is being captured, only read a cache.
cudaError_t ensure_smem_limit(const void* func, size_t bytes);

// Shared-memory footprint of each kernel for a given stage count.
size_t summarize_smem_bytes(int dim, int block, int warps, int stages, int elem_bytes);
size_t stats_smem_bytes(int dim, int warps, int stages, int group);
size_t final_smem_bytes(int dim, int warps, int stages, int group, int tiles_per_cta);
size_t attend_smem_bytes(int dim, int page, int warps, int stages, int group, int heads,
                         int parts_b);
size_t combine_smem_bytes(int heads, int parts_b, int group, int max_sources);
// zd_group > 0: the part's z and delta kept in shared memory for that many group rows.
size_t fused_smem_bytes(int dim, int page, int warps, int tcap, int zd_group);
int fused_grid(int heads, int parts_base, int parts_extra);

}  // namespace rkv
