// extern "C" entry points of librefinekv_b200.so (declared in
// include/refinekv_b200.h): argument checks, the launch plan shared by the
// workspace-size functions and the launches, TMA descriptor encoding, and the
// kernel launches.  No device memory is allocated here.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <mutex>
#include <string>
#include <vector>

#include "refinekv_b200.h"
#include "rkv_kernels.h"

namespace rkv {
namespace {

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t err, const char* what) {
  return fail(RKV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

// Head dims: multiples of 32 up to 256 (the reference's GPU limits,
// attention.py:29-39).  Kernels compute on the width rounded up to 64, the
// TMA boxes' width; loads past the real width read zeros.
bool supported_dim(int64_t d) { return d >= 32 && d <= 256 && d % 32 == 0; }
int padded_dim(int64_t d) { return static_cast<int>((d + 63) / 64 * 64); }
bool supported_block(int64_t b) { return b == 16 || b == 32 || b == 64; }
bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// Workspace header: status word at 0; the one-kernel decode's per-row barrier
// words from kRowWords -- arrivals A, generations A, arrivals B, generations B,
// kMaxFusedRows words each -- at a fixed place for every geometry.
constexpr size_t kHeaderBytes = 8192;
constexpr size_t kRowWords = 256;
constexpr int64_t kMaxFusedRows = 480;

struct DeviceInfo {
  int sms = 0;
  int smem_optin = 0;
};

int device_info(DeviceInfo* info) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
  static std::mutex mu;
  static DeviceInfo cache[64];
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64) return fail(RKV_ERR_CUDA, "device index out of range");
  if (cache[dev].sms == 0) {
    int sms = 0, optin = 0;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute(SM count)");
    err = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaDeviceGetAttribute(shared memory)");
    cache[dev].sms = sms;
    cache[dev].smem_optin = optin;
  }
  *info = cache[dev];
  return RKV_OK;
}

// ---------------------------------------------------------------------------
// Launch plan: grid splits, pipeline depths, shared memory, workspace layout.
// ---------------------------------------------------------------------------
struct Plan {
  int tiles = 0;
  int warps_a = 8, parts_a = 1, tpc_a = 1, stages_a = 1, slots_a = 8;
  size_t smem_a = 0;
  int warps_b = 8, parts_b = 1, tpc_b = 1, stages_b = 2, seg_cap = 0;
  size_t smem_b = 0;
  int warps_c = 4, stages_c = 2, ctas = 1;
  size_t smem_c = 0;
  int g8 = 8, max_sources = 0;
  size_t smem_d = 0;  // combine
  // One-kernel decode (rkv_fused.cu), used for RKV_PHASE_ALL: parts_base /
  // parts_extra parts per row, tcap_f the largest tile range of a part; its
  // own workspace regions (the same allocation, another layout).
  bool fused = false;
  int warps_f = 8, parts_base = 1, parts_extra = 0, tcap_f = 1, grid_f = 0, zd_f = 0;
  size_t smem_f = 0;
  size_t f_lse = 0, f_z = 0, f_delta = 0, f_part_m = 0, f_part_l = 0, f_part_o = 0;
  // workspace offsets (bytes)
  size_t status = 0, lse = 0, z = 0, delta = 0, seg_count = 0, sel_ids = 0;
  size_t rep_m = 0, rep_l = 0, rep_o = 0, att_m = 0, att_l = 0, att_o = 0, bytes = 0;
};

void split(int tiles, int target_parts, int* parts, int* per) {
  int p = std::max(1, std::min(tiles, target_parts));
  *per = static_cast<int>(cdiv(tiles, p));
  *parts = static_cast<int>(cdiv(tiles, *per));
}

// Attention and combine launch shapes for a plan whose parts_b is set (the
// selector's segment count, or 1 for dense decode).  `dim` is padded.
int plan_attention(Plan* pl, const DeviceInfo& dev, int64_t heads, int64_t group, int64_t dim,
                   int64_t block_size) {
  // Attention: one CTA per SM with about 128 KB of TMA ring, split over as
  // many warps as possible (3..8) with one stage each (more for small
  // stages).  Measured on B200: fewer bytes in flight per SM and more
  // warps beat deeper per-warp rings (6-8 warps x 1 stage: ~91 us per
  // 128K layer vs ~101 us for 4 warps x 3 stages).
  const int64_t stage = 2 * block_size * dim * 2;
  const int64_t ring = 128 * 1024;
  pl->warps_c = static_cast<int>(std::max<int64_t>(3, std::min<int64_t>(8, ring / stage)));
  pl->stages_c =
      static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(4, ring / (pl->warps_c * stage))));
  // The CTA merge parks each warp's (m, l, o^T) in that warp's ring slice.
  const int64_t g8 = group <= 8 ? 8 : 16;
  const int64_t stash = (2 * g8 + g8 * dim) * 4;
  while (pl->stages_c * stage < stash) ++pl->stages_c;
  while (attend_smem_bytes(static_cast<int>(dim), static_cast<int>(block_size), pl->warps_c,
                           pl->stages_c, static_cast<int>(group), static_cast<int>(heads),
                           pl->parts_b) > static_cast<size_t>(dev.smem_optin)) {
    if (pl->stages_c > 1 && (pl->stages_c - 1) * stage >= stash) {
      --pl->stages_c;
    } else if (pl->warps_c > 1) {
      --pl->warps_c;
    } else {
      return fail(RKV_ERR_UNSUPPORTED, "attention stages do not fit");
    }
  }
  pl->smem_c = attend_smem_bytes(static_cast<int>(dim), static_cast<int>(block_size),
                                 pl->warps_c, pl->stages_c, static_cast<int>(group),
                                 static_cast<int>(heads), pl->parts_b);
  pl->ctas = dev.sms;
  pl->g8 = group <= 8 ? 8 : 16;
  pl->max_sources = pl->parts_b + pl->ctas * pl->warps_c;
  pl->smem_d = combine_smem_bytes(static_cast<int>(heads), pl->parts_b, static_cast<int>(group),
                                  pl->max_sources);
  if (pl->smem_d > static_cast<size_t>(dev.smem_optin)) {
    return fail(RKV_ERR_UNSUPPORTED, "combine source table does not fit in shared memory");
  }
  return RKV_OK;
}

// rkv_decode_dense: attention and combine only (one segment per row, no
// representatives); workspace = status word + attention partials.
int make_dense_plan(Plan* pl, int64_t heads, int64_t group, int64_t dim, int64_t block_size) {
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc != RKV_OK) return rc;
  dim = padded_dim(dim);
  pl->parts_b = 1;
  rc = plan_attention(pl, dev, heads, group, dim, block_size);
  if (rc != RKV_OK) return rc;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = up256(off + bytes);
    return at;
  };
  const size_t slots_c = static_cast<size_t>(heads + pl->ctas) * pl->warps_c;
  pl->status = take(kHeaderBytes);
  pl->att_m = take(slots_c * pl->g8 * 4);
  pl->att_l = take(slots_c * pl->g8 * 4);
  pl->att_o = take(slots_c * pl->g8 * dim * 4);
  pl->bytes = off;
  return RKV_OK;
}

// Whether rkv_decode runs the one-kernel decode (switched off process-wide by
// rkv_set_fused_selector(0), for measurement and cross-checks).
std::atomic<int> g_fused_selector{1};

// The one-kernel decode's shape: every SM gets one CTA (uneven parts per row:
// the first `extra` rows one more), never more CTAs than SMs unless each row
// has a single part (then no CTA waits for another); warps of one slice each
// (a K|V page or a key-mean|ellipsoid tile pair).
bool plan_fused(Plan* pl, const DeviceInfo& dev, int64_t heads, int64_t group, int64_t blocks,
                int64_t dim, int64_t block_size) {
  if (!g_fused_selector.load() || heads > kMaxFusedRows) return false;
  // Parts hold an equal share of a row's blocks, at least 16 each.
  const int64_t max_parts = std::max<int64_t>(1, blocks / 16);
  int base, extra;
  if (heads >= dev.sms) {
    base = 1;
    extra = 0;
  } else {
    base = static_cast<int>(dev.sms / heads);
    extra = static_cast<int>(dev.sms % heads);
    if (base >= max_parts) {
      base = static_cast<int>(max_parts);
      extra = 0;
    }
  }
  const int most = base + (extra > 0 ? 1 : 0);
  if (most > 320) return false;  // the combine's lanes hold up to 10 parts each
  // Selector tiles a part touches: its blocks may start inside a tile.
  const int tcap = static_cast<int>(cdiv(cdiv(blocks, base), kSelectTile)) + 1;
  if (tcap > 128) return false;  // the per-part tables live in shared memory
  const int64_t slice = std::max<int64_t>(2LL * kSelectTile * dim * 2, 2LL * block_size * dim * 2);
  const int warps = static_cast<int>(std::min<int64_t>(8, 196608 / slice));
  if (warps < 2) return false;
  // z and delta of the part's tiles stay in shared memory when they fit.
  int zd = static_cast<int>(group);
  size_t smem = fused_smem_bytes(static_cast<int>(dim), static_cast<int>(block_size), warps, tcap,
                                 zd);
  if (smem > static_cast<size_t>(dev.smem_optin)) {
    zd = 0;
    smem = fused_smem_bytes(static_cast<int>(dim), static_cast<int>(block_size), warps, tcap, 0);
  }
  if (smem > static_cast<size_t>(dev.smem_optin)) return false;
  pl->fused = true;
  pl->warps_f = warps;
  pl->smem_f = smem;
  pl->parts_base = base;
  pl->parts_extra = extra;
  pl->tcap_f = tcap;
  pl->zd_f = zd;
  pl->grid_f = fused_grid(static_cast<int>(heads), base, extra);
  return true;
}

// `decode` plans rkv_decode (one query instance); otherwise rkv_select.
// `fixed_parts_a` > 0 pins the phase-A grid (a sequence split needs the same
// partial count on every rank; CTAs past the last tile write empty partials).
int make_plan(Plan* pl, int64_t heads, int64_t group, int64_t blocks, int64_t dim,
              int64_t block_size, int64_t instances, bool decode, int fixed_parts_a = 0) {
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc != RKV_OK) return rc;
  dim = padded_dim(dim);  // shared memory and scratch hold padded rows
  pl->tiles = static_cast<int>(cdiv(blocks, kSelectTile));
  const int64_t rows = heads * instances;
  // Both selector kernels run one wave of at most one CTA per SM: a grid a
  // few CTAs larger than the SM count doubles the work of the SMs that take
  // two.  Phase A: one 16 KB stage (key-mean + ellipsoid tile) per warp.
  const int one_wave = static_cast<int>(std::max<int64_t>(1, dev.sms / rows));
  if (fixed_parts_a > 0) {
    pl->parts_a = fixed_parts_a;
    pl->tpc_a = static_cast<int>(cdiv(pl->tiles, fixed_parts_a));
  } else {
    split(pl->tiles, one_wave, &pl->parts_a, &pl->tpc_a);
  }
  pl->stages_a = 1;
  const int64_t stage_a = 2LL * kSelectTile * dim * 2;
  // No more warps than tiles per CTA (one head per GPU leaves one tile each);
  // up to 12 warps (a 192 KB ring) for groups of at most 8 rows, whose
  // kernels fit 384 threads' registers, 8 under a sequence split (its
  // fixed partial slots per CTA).
  const int64_t max_warps = group <= 8 ? 12 : 8;
  pl->warps_a = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>({fixed_parts_a > 0 ? int64_t{kStatsSlots} : max_warps,
                            196608 / stage_a, static_cast<int64_t>(pl->tpc_a)})));
  // One LSE partial per warp; a sequence split fixes the count so that every
  // rank's slab has the same layout.
  pl->slots_a = fixed_parts_a > 0 ? kStatsSlots : pl->warps_a;
  pl->smem_a = stats_smem_bytes(static_cast<int>(dim), pl->warps_a, pl->stages_a,
                                static_cast<int>(group));
  // Phase B: at least four tiles per CTA -- each CTA leaves one
  // representative partial per row that the combine merges, so a few heads
  // over many one-tile CTAs would flood it.  Segment capacity = blocks per CTA.
  split(pl->tiles, std::min(one_wave, std::max(1, pl->tiles / 4)), &pl->parts_b, &pl->tpc_b);
  pl->seg_cap = pl->tpc_b * kSelectTile;
  // One value-mean stage per warp and up to 12 warps: the decisions and the
  // representative softmax are latency-bound, so warps beat stages (a 1M
  // layer's final kernel measured ~3 us faster than 8 warps x 2 stages).
  pl->stages_b = decode ? 1 : 0;  // select mode stages no value tiles
  const int64_t g8b = group <= 8 ? 8 : 16;
  const int64_t per_warp_b = pl->stages_b * kSelectTile * dim * 2 + g8b * dim * 4;
  pl->warps_b = static_cast<int>(std::max<int64_t>(
      1, std::min<int64_t>({max_warps, 200000 / per_warp_b, static_cast<int64_t>(pl->tpc_b)})));
  pl->smem_b = final_smem_bytes(static_cast<int>(dim), pl->warps_b, pl->stages_b,
                                static_cast<int>(group), pl->tpc_b);
  if (pl->smem_a > static_cast<size_t>(dev.smem_optin) ||
      pl->smem_b > static_cast<size_t>(dev.smem_optin)) {
    return fail(RKV_ERR_UNSUPPORTED, "selector tiles do not fit in shared memory");
  }
  if (decode) {
    rc = plan_attention(pl, dev, heads, group, dim, block_size);
    if (rc != RKV_OK) return rc;
    if (fixed_parts_a == 0 && instances == 1) {
      plan_fused(pl, dev, heads, group, blocks, dim, block_size);
    }
  }
  // Workspace layout.
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = up256(off + bytes);
    return at;
  };
  const size_t rowsg = static_cast<size_t>(rows) * group;
  // A fixed 4 KB header for every geometry: the status word, and the fused
  // selector's per-row barrier words at a fixed place, where no other region
  // of any geometry writes (they clean themselves after every round, so a
  // workspace reused for another geometry finds them consistent).
  pl->status = take(kHeaderBytes);
  // (Under a sequence split phase A writes into the exchange slab instead.)
  pl->lse = take(fixed_parts_a > 0 ? 0 : rowsg * pl->parts_a * pl->slots_a * 4 * 4);
  pl->z = take(rowsg * blocks * 4);
  pl->delta = take(rowsg * blocks * 4);
  if (decode) {
    const size_t slots_b = static_cast<size_t>(heads) * pl->parts_b;
    // (head, cta) pairs that own items are indexed by head + cta.
    const size_t slots_c = static_cast<size_t>(heads + pl->ctas) * pl->warps_c;
    pl->seg_count = take(slots_b * 4);
    pl->sel_ids = take(slots_b * pl->seg_cap * 4);
    pl->rep_m = take(slots_b * pl->g8 * 4);
    pl->rep_l = take(slots_b * pl->g8 * 4);
    pl->rep_o = take(slots_b * pl->g8 * dim * 4);
    pl->att_m = take(slots_c * pl->g8 * 4);
    pl->att_l = take(slots_c * pl->g8 * 4);
    pl->att_o = take(slots_c * pl->g8 * dim * 4);
  }
  pl->bytes = off;
  if (pl->fused) {  // the one-kernel decode's regions, after the same header
    off = kHeaderBytes;
    const int most = pl->parts_base + (pl->parts_extra > 0 ? 1 : 0);
    pl->f_lse = take(rowsg * most * 4 * 4);  // one (max, sum) pair of z and of c per part
    pl->f_z = take(rowsg * blocks * 4);
    pl->f_delta = take(rowsg * blocks * 4);
    pl->f_part_m = take(static_cast<size_t>(pl->grid_f) * pl->g8 * 4);
    pl->f_part_l = take(static_cast<size_t>(pl->grid_f) * pl->g8 * 4);
    pl->f_part_o = take(static_cast<size_t>(pl->grid_f) * pl->g8 * dim * 4);
    pl->bytes = std::max(pl->bytes, off);
  }
  return RKV_OK;
}

// Sequence split: phase-A partials per row on every rank (fixed by the
// largest rank's block count, not by the device, so that all ranks agree) and
// the slab sizes of the exchange buffer.
constexpr int kSplitStatsCtas = 148;  // one wave on a B200 (fixed so that all ranks agree)

struct SplitGeometry {
  int parts_a = 1;
  size_t stats_slab = 0;   // bytes: (heads * group, parts_a, 4) fp32
  size_t ml_bytes = 0;     // bytes of the (rows, 2) block at the start of an output slab
  size_t output_slab = 0;  // bytes: (rows, 2) then (rows, dim) fp32
};

// `instances` query instances per rank (rkv_select_split); dim == 0 for
// selection only (no output slab).
SplitGeometry split_geometry(int64_t heads, int64_t group, int64_t max_blocks, int64_t dim,
                             int64_t instances = 1) {
  SplitGeometry g;
  int per = 1;
  split(static_cast<int>(cdiv(max_blocks, kSelectTile)),
        static_cast<int>(std::max<int64_t>(1, kSplitStatsCtas / (heads * instances))), &g.parts_a,
        &per);
  const size_t rows = static_cast<size_t>(heads) * group;
  g.stats_slab = up256(rows * instances * g.parts_a * kStatsSlots * 16);
  g.ml_bytes = dim > 0 ? up256(rows * 8) : 0;
  g.output_slab = dim > 0 ? g.ml_bytes + up256(rows * dim * 4) : 0;
  return g;
}

// Where the kernels of one rank of a split step read and write.
struct SplitTarget {
  int ranks = 1, rank = 0;
  SplitGeometry geo;
  char* exchange = nullptr;
  float* stats_slab(int r) const { return reinterpret_cast<float*>(exchange + r * geo.stats_slab); }
  float* output_ml(int r) const {
    return reinterpret_cast<float*>(exchange + ranks * geo.stats_slab + r * geo.output_slab);
  }
  float* output_o(int r) const {
    return reinterpret_cast<float*>(reinterpret_cast<char*>(output_ml(r)) + geo.ml_bytes);
  }
};

// ---------------------------------------------------------------------------
// TMA descriptors
// ---------------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                 const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                 const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult found;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &found) ==
            cudaSuccess &&
        found == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiled>(ptr);
    }
  });
  return fn;
}

// 3-D map (dim, rows, heads) of bf16 (elem_bytes 2) or fp32 (4) elements read
// in [box_rows x 128 bytes] boxes (64 bf16 or 32 fp32 columns), 128B swizzle.
int rows_map(CUtensorMap* map, const void* base, int64_t dim, int64_t rows, int64_t heads,
             int64_t row_stride, int64_t head_stride, int box_rows, const char* what,
             int elem_bytes = 2) {
  EncodeTiled encode = encoder();
  if (encode == nullptr) return fail(RKV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int64_t w = elem_bytes;
  if (!aligned16(base) || (row_stride * w) % 16 != 0 ||
      (heads > 1 && (head_stride * w) % 16 != 0)) {
    return fail(RKV_ERR_ALIGNMENT, std::string(what) + ": base and strides must be 16-byte aligned");
  }
  if (heads > 1 && head_stride <= 0) {
    return fail(RKV_ERR_INVALID_ARGUMENT, std::string(what) + ": head stride must be positive");
  }
  cuuint64_t gdim[3] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(heads)};
  cuuint64_t gstride[2] = {static_cast<cuuint64_t>(row_stride * w),
                           static_cast<cuuint64_t>(heads > 1 ? head_stride * w
                                                             : rows * row_stride * w)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / w), static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estride[3] = {1, 1, 1};
  const CUresult r = encode(map,
                            w == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                            3, const_cast<void*>(base), gdim,
                            gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(RKV_ERR_INVALID_ARGUMENT,
                std::string(what) + ": cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  }
  return RKV_OK;
}

// 4-D bf16 map of K/V pages (dim, row in page, head, page), read one
// [block x 64] box per page and column half (the same shared-memory tile as
// rows_map's boxes).  Contiguous pages and HND / NHD page pools are the
// same map with different strides.
int pages_map(CUtensorMap* map, const void* base, int64_t dim, int64_t block, int64_t heads,
              int64_t pages, int64_t token_stride, int64_t head_stride, int64_t page_stride,
              const char* what) {
  EncodeTiled encode = encoder();
  if (encode == nullptr) return fail(RKV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  if (!aligned16(base) || (token_stride * 2) % 16 != 0 || (head_stride * 2) % 16 != 0 ||
      (page_stride * 2) % 16 != 0) {
    return fail(RKV_ERR_ALIGNMENT, std::string(what) + ": base and strides must be 16-byte aligned");
  }
  if (token_stride <= 0 || (heads > 1 && head_stride <= 0) || (pages > 1 && page_stride <= 0)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, std::string(what) + ": strides must be positive");
  }
  cuuint64_t gdim[4] = {static_cast<cuuint64_t>(dim), static_cast<cuuint64_t>(block),
                        static_cast<cuuint64_t>(heads), static_cast<cuuint64_t>(pages)};
  cuuint64_t gstride[3] = {static_cast<cuuint64_t>(token_stride * 2),
                           static_cast<cuuint64_t>((heads > 1 ? head_stride : block * token_stride) * 2),
                           static_cast<cuuint64_t>((pages > 1 ? page_stride : heads * block * token_stride) * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(block), 1, 1};
  cuuint32_t estride[4] = {1, 1, 1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), gdim,
                            gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(RKV_ERR_INVALID_ARGUMENT,
                std::string(what) + ": cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  }
  return RKV_OK;
}

// The page geometry of a summary (all that rkv_decode_dense reads);
// check_summary adds the summary fields.
int check_pages(const rkv_summary* s) {
  if (s == nullptr) return fail(RKV_ERR_INVALID_ARGUMENT, "summary is null");
  if (s->heads <= 0 || s->blocks <= 0 || s->prompt_length <= 0) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "summary sizes must be positive");
  }
  if (!supported_block(s->block_size)) {
    return fail(RKV_ERR_UNSUPPORTED, "block_size must be 16, 32 or 64");
  }
  if (!supported_dim(s->head_dim)) {
    return fail(RKV_ERR_UNSUPPORTED, "head_dim must be a multiple of 32 in [32, 256]");
  }
  if (cdiv(s->prompt_length, s->block_size) != s->blocks) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "blocks must equal ceil(prompt_length / block_size)");
  }
  if (!s->key_pages || !s->value_pages) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "summary has a null page pointer");
  }
  if (s->heads > (1 << 16) || s->blocks > (1LL << 26)) {
    return fail(RKV_ERR_UNSUPPORTED, "summary is larger than the kernels index");
  }
  if (s->sequences < 0 || s->sequences > s->heads ||
      (s->sequences > 1 && (s->heads % s->sequences != 0 || s->prompt_lengths == nullptr))) {
    return fail(RKV_ERR_INVALID_ARGUMENT,
                "sequences must divide heads, with prompt_lengths for a batch");
  }
  if (s->page_table != nullptr &&
      (s->pool_pages <= 0 || s->pool_pages > (1LL << 31) - 1 || s->page_table_stride < s->blocks ||
       s->key_page_stride <= 0 || s->value_page_stride <= 0 || s->key_token_stride <= 0 ||
       s->value_token_stride <= 0)) {
    return fail(RKV_ERR_INVALID_ARGUMENT,
                "a page table needs pool_pages, a stride of at least blocks and positive strides");
  }
  return RKV_OK;
}

int check_summary(const rkv_summary* s) {
  int rc = check_pages(s);
  if (rc != RKV_OK) return rc;
  if (!s->counts || !s->key_mean || !s->value_mean || !s->ellipsoid || !s->value_norm ||
      !s->max_value_norm) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "summary has a null pointer");
  }
  return RKV_OK;
}

// Row-to-sequence layout of a (possibly batched) summary for the kernels.
SeqLayout seq_layout(const rkv_summary* s) {
  SeqLayout l = {};
  const bool batched = s->sequences > 1;
  l.seq_prompt = batched ? s->prompt_lengths : nullptr;
  l.heads_per_seq = static_cast<int>(batched ? s->heads / s->sequences : s->heads);
  l.page = static_cast<int>(s->block_size);
  return l;
}

int check_selection_args(const rkv_summary* s, const void* q, int qdtype, int64_t group,
                         float eps, int reduction) {
  int rc = check_summary(s);
  if (rc != RKV_OK) return rc;
  if (q == nullptr) return fail(RKV_ERR_INVALID_ARGUMENT, "query is null");
  if (qdtype != RKV_DTYPE_BF16 && qdtype != RKV_DTYPE_F32) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "query dtype must be bf16 or fp32");
  }
  if (group < 1 || group > kMaxGroup) return fail(RKV_ERR_UNSUPPORTED, "group must be 1..16");
  if (!std::isfinite(eps) || eps < 0.f) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "eps must be finite and nonnegative");
  }
  if (reduction != RKV_GQA_MEAN && reduction != RKV_GQA_MAX && reduction != RKV_GQA_ANY) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "reduction must be mean, max or any");
  }
  return RKV_OK;
}

int summary_maps(const rkv_summary* s, CUtensorMap* key_mean, CUtensorMap* ellipsoid,
                 CUtensorMap* value_mean) {
  const int64_t H = s->heads, nb = s->blocks, D = s->head_dim;
  int rc = RKV_OK;
  if (key_mean && (rc = rows_map(key_mean, s->key_mean, D, nb, H, D, nb * D, kSelectTile,
                                 "key_mean")) != RKV_OK)
    return rc;
  if (ellipsoid && (rc = rows_map(ellipsoid, s->ellipsoid, D, nb, H, D, nb * D, kSelectTile,
                                  "ellipsoid")) != RKV_OK)
    return rc;
  if (value_mean && (rc = rows_map(value_mean, s->value_mean, D, nb, H, D, nb * D, kSelectTile,
                                   "value_mean")) != RKV_OK)
    return rc;
  return RKV_OK;
}

int check_workspace(const Plan& pl, void* ws, size_t size) {
  if (ws == nullptr || size < pl.bytes) {
    return fail(RKV_ERR_WORKSPACE, "workspace is missing or smaller than the required size " +
                                       std::to_string(pl.bytes));
  }
  if ((reinterpret_cast<uintptr_t>(ws) & 255u) != 0) {
    return fail(RKV_ERR_WORKSPACE, "workspace must be 256-byte aligned");
  }
  return RKV_OK;
}

template <typename T>
T* at(void* ws, size_t off) {
  return reinterpret_cast<T*>(static_cast<char*>(ws) + off);
}

// rkv_decode (RKV_PHASE_ALL) as one launch: selector, every page, the
// representatives and the combine (rkv_fused.cu).
int run_fused_decode(const Plan& pl, const rkv_summary* s, const void* q, int qdtype,
                     int64_t group, const void* key_suffix, const void* value_suffix,
                     int64_t suffix_capacity, int64_t key_suffix_head_stride,
                     int64_t key_suffix_token_stride, int64_t value_suffix_head_stride,
                     int64_t value_suffix_token_stride, const int32_t* suffix_length,
                     int64_t suffix_length_host, float eps, int reduction, const uint8_t* anchor,
                     uint8_t* mask, void* output, void* ws, cudaStream_t stream) {
  const int D = static_cast<int>(s->head_dim);
  const int DP = padded_dim(D);
  const int64_t H = s->heads, B = s->block_size;
  FusedMaps maps;
  int rc = summary_maps(s, &maps.key_mean, &maps.ellipsoid, &maps.value_mean);
  if (rc != RKV_OK) return rc;
  const bool paged = s->page_table != nullptr;
  const int64_t pool_heads = paged ? H / std::max<int64_t>(1, s->sequences) : H;
  rc = pages_map(&maps.key_pages, s->key_pages, D, B, pool_heads, paged ? s->pool_pages : s->blocks,
                 paged ? s->key_token_stride : D, s->key_page_head_stride,
                 paged ? s->key_page_stride : B * D, "key_pages");
  if (rc != RKV_OK) return rc;
  rc = pages_map(&maps.value_pages, s->value_pages, D, B, pool_heads,
                 paged ? s->pool_pages : s->blocks, paged ? s->value_token_stride : D,
                 s->value_page_head_stride, paged ? s->value_page_stride : B * D, "value_pages");
  if (rc != RKV_OK) return rc;
  if (suffix_capacity > 0) {
    rc = rows_map(&maps.key_suffix, key_suffix, D, suffix_capacity, H, key_suffix_token_stride,
                  key_suffix_head_stride, static_cast<int>(B), "key_suffix");
    if (rc != RKV_OK) return rc;
    rc = rows_map(&maps.value_suffix, value_suffix, D, suffix_capacity, H,
                  value_suffix_token_stride, value_suffix_head_stride, static_cast<int>(B),
                  "value_suffix");
    if (rc != RKV_OK) return rc;
  } else {
    maps.key_suffix = maps.key_pages;
    maps.value_suffix = maps.value_pages;
  }
  FusedParams p = {};
  p.query = q;
  p.query_f32 = qdtype == RKV_DTYPE_F32;
  p.dim = D;
  p.out = output;
  p.counts = s->counts;
  p.heads = static_cast<int>(H);
  p.group = static_cast<int>(group);
  p.blocks = static_cast<int>(s->blocks);
  p.tiles = pl.tiles;
  p.parts_base = pl.parts_base;
  p.parts_extra = pl.parts_extra;
  p.tcap = pl.tcap_f;
  p.zd_group = pl.zd_f;
  p.scale = static_cast<float>(std::pow(static_cast<double>(D), -0.5));
  p.eps = eps;
  p.reduction = reduction;
  p.z = at<float>(ws, pl.f_z);
  p.delta = at<float>(ws, pl.f_delta);
  p.lse = at<float>(ws, pl.f_lse);
  p.value_norm = s->value_norm;
  p.max_value_norm = s->max_value_norm;
  p.anchor = anchor;
  p.mask = mask;
  p.split_probs = qdtype == RKV_DTYPE_F32;
  p.part_m = at<float>(ws, pl.f_part_m);
  p.part_l = at<float>(ws, pl.f_part_l);
  p.part_o = at<float>(ws, pl.f_part_o);
  p.bar_words = at<unsigned>(ws, kRowWords);
  p.bar_stride = static_cast<int>(kMaxFusedRows);
  p.seq = seq_layout(s);
  p.page = static_cast<int>(B);
  p.prompt_length = static_cast<int>(s->prompt_length);
  p.page_table = s->page_table;
  p.page_table_stride = static_cast<int>(paged ? s->page_table_stride : 0);
  p.pool_pages = static_cast<int>(paged ? s->pool_pages : s->blocks);
  p.has_suffix = suffix_capacity > 0;
  p.suffix_capacity = static_cast<int>(suffix_capacity);
  p.suffix_len_ptr = suffix_length;
  p.suffix_len_host = static_cast<int>(suffix_length_host);
  p.status = at<int>(ws, pl.status);
  const cudaError_t err = launch_fused(maps, p, DP, pl.warps_f, pl.smem_f, stream, true);
  if (err != cudaSuccess) return cuda_fail(err, "decode launch");
  return RKV_OK;
}

// Phases A and B shared by rkv_select and rkv_decode.
// With `split`, phase A writes this rank's stats slab and phase B reads all
// ranks' slabs.
int run_selector(const Plan& pl, const rkv_summary* s, const void* q, int qdtype, int64_t inst,
                 int64_t group, float eps, int reduction, const uint8_t* anchor, uint8_t* mask,
                 int accumulate, void* ws, bool decode, unsigned phases, cudaStream_t stream,
                 const SplitTarget* split = nullptr) {
  const int D = static_cast<int>(s->head_dim);
  const int DP = padded_dim(D);
  if (phases & RKV_PHASE_STATS) {
    StatsMaps maps;
    int rc = summary_maps(s, &maps.key_mean, &maps.ellipsoid, nullptr);
    if (rc != RKV_OK) return rc;
    StatsParams p = {};
    p.query = q;
    p.query_f32 = qdtype == RKV_DTYPE_F32;
    p.dim = D;
    p.counts = s->counts;
    p.seq = seq_layout(s);
    p.heads = static_cast<int>(s->heads);
    p.group = static_cast<int>(group);
    p.blocks = static_cast<int>(s->blocks);
    p.instances = static_cast<int>(inst);
    p.tiles = pl.tiles;
    p.tiles_per_cta = pl.tpc_a;
    p.parts = pl.parts_a;
    p.slots = pl.slots_a;
    p.stages = pl.stages_a;
    p.scale = static_cast<float>(std::pow(static_cast<double>(D), -0.5));
    p.z = at<float>(ws, pl.z);
    p.delta = at<float>(ws, pl.delta);
    p.lse = split ? split->stats_slab(split->rank) : at<float>(ws, pl.lse);
    p.status = at<int>(ws, pl.status);
    cudaError_t err = launch_stats(maps, p, DP, pl.warps_a, pl.smem_a, stream, true);
    if (err != cudaSuccess) return cuda_fail(err, "selector stats launch");
  }
  if (phases & RKV_PHASE_FINAL) {
    FinalMaps maps;
    int rc = summary_maps(s, nullptr, nullptr, &maps.value_mean);
    if (rc != RKV_OK) return rc;
    FinalParams p = {};
    p.seq = seq_layout(s);
    p.heads = static_cast<int>(s->heads);
    p.group = static_cast<int>(group);
    p.blocks = static_cast<int>(s->blocks);
    p.instances = static_cast<int>(inst);
    p.tiles = pl.tiles;
    p.tiles_per_cta = pl.tpc_b;
    p.parts_a = pl.parts_a * pl.slots_a;  // phase-A partials per row
    p.parts = pl.parts_b;
    p.stages = pl.stages_b;
    p.eps = eps;
    p.reduction = reduction;
    p.z = at<float>(ws, pl.z);
    p.delta = at<float>(ws, pl.delta);
    p.lse = split ? split->stats_slab(0) : at<float>(ws, pl.lse);
    p.lse_slabs = split ? split->ranks : 1;
    p.lse_slab_floats = split ? split->geo.stats_slab / 4 : 0;
    p.value_norm = s->value_norm;
    p.max_value_norm = s->max_value_norm;
    p.anchor = anchor;
    p.mask = mask;
    p.accumulate = accumulate;
    p.decode = decode ? 1 : 0;
    p.split_probs = qdtype == RKV_DTYPE_F32;
    if (decode) {
      p.seg_count = at<int>(ws, pl.seg_count);
      p.sel_ids = at<int>(ws, pl.sel_ids);
      p.seg_cap = pl.seg_cap;
      p.rep_m = at<float>(ws, pl.rep_m);
      p.rep_l = at<float>(ws, pl.rep_l);
      p.rep_o = at<float>(ws, pl.rep_o);
    }
    p.status = at<int>(ws, pl.status);
    cudaError_t err = launch_final(maps, p, DP, pl.warps_b, pl.smem_b, stream, true);
    if (err != cudaSuccess) return cuda_fail(err, "selector final launch");
  }
  return RKV_OK;
}

}  // namespace

void set_last_error(const std::string& message) { g_last_error = message; }

cudaError_t ensure_smem_limit(const void* func, size_t bytes) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  struct Entry {
    const void* func;
    int dev;
    size_t bytes;
  };
  static std::mutex mu;
  static std::vector<Entry> done;
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : done) {
    if (e.func == func && e.dev == dev && e.bytes >= bytes) return cudaSuccess;
  }
  err = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(bytes));
  if (err != cudaSuccess) return err;
  for (Entry& e : done) {
    if (e.func == func && e.dev == dev) {
      e.bytes = bytes;
      return cudaSuccess;
    }
  }
  done.push_back({func, dev, bytes});
  return cudaSuccess;
}

}  // namespace rkv

using namespace rkv;

extern "C" {

int rkv_abi_version(void) { return RKV_ABI_VERSION; }

const char* rkv_last_error(void) { return g_last_error.c_str(); }

const char* rkv_status_string(int status) {
  switch (status) {
    case RKV_OK: return "ok";
    case RKV_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RKV_ERR_UNSUPPORTED: return "unsupported shape";
    case RKV_ERR_ALIGNMENT: return "misaligned pointer or stride";
    case RKV_ERR_WORKSPACE: return "bad workspace";
    case RKV_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

}  // extern "C"

namespace rkv {
namespace {

// rkv_summarize and rkv_summarize_into: the page copy of head h starts
// `*_pages_head_stride` elements after head h - 1's (0: packed pages).
int summarize_impl(const void* keys, const void* values, bool f32, int64_t heads, int64_t tokens,
                   int64_t head_dim, int64_t key_head_stride, int64_t key_token_stride,
                   int64_t value_head_stride, int64_t value_token_stride, int64_t block_size,
                   void* key_pages_out, int64_t key_pages_head_stride, void* value_pages_out,
                   int64_t value_pages_head_stride, void* key_mean, void* value_mean,
                   void* ellipsoid, float* value_norm, float* max_value_norm, int64_t* counts,
                   void* stream) {
  if (heads <= 0 || tokens <= 0) return fail(RKV_ERR_INVALID_ARGUMENT, "empty keys/values");
  if (!supported_dim(head_dim)) return fail(RKV_ERR_UNSUPPORTED, "head_dim must be a multiple of 32 in [32, 256]");
  if (!supported_block(block_size)) return fail(RKV_ERR_UNSUPPORTED, "block_size must be 16, 32 or 64");
  if (!keys || !values || !key_mean || !value_mean || !ellipsoid || !value_norm ||
      !max_value_norm || !counts) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "null pointer");
  }
  if ((key_pages_out == nullptr) != (value_pages_out == nullptr)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "pass both page copies or neither");
  }
  if (f32 && key_pages_out == nullptr) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "an fp32 cache needs the bf16 page copies");
  }
  const int64_t w = f32 ? 4 : 2;
  if (!aligned16(keys) || !aligned16(values) || (key_token_stride * w) % 16 ||
      (value_token_stride * w) % 16 || (key_head_stride * w) % 16 ||
      (value_head_stride * w) % 16) {
    return fail(RKV_ERR_ALIGNMENT, "keys/values rows must be 16-byte aligned");
  }
  if ((key_pages_out && !aligned16(key_pages_out)) || (value_pages_out && !aligned16(value_pages_out)) ||
      !aligned16(key_mean) || !aligned16(value_mean) || !aligned16(ellipsoid)) {
    return fail(RKV_ERR_ALIGNMENT, "outputs must be 16-byte aligned");
  }
  if (tokens > (1LL << 31) - 1 || heads > (1 << 16)) {
    return fail(RKV_ERR_UNSUPPORTED, "prompt is larger than the kernels index");
  }
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc != RKV_OK) return rc;
  SummarizeMaps maps;
  rc = rows_map(&maps.keys, keys, head_dim, tokens, heads, key_token_stride, key_head_stride,
                static_cast<int>(block_size), "keys", static_cast<int>(w));
  if (rc != RKV_OK) return rc;
  rc = rows_map(&maps.values, values, head_dim, tokens, heads, value_token_stride,
                value_head_stride, static_cast<int>(block_size), "values", static_cast<int>(w));
  if (rc != RKV_OK) return rc;
  // Persistent grid: one CTA per SM with about 192 KB of TMA ring per CTA,
  // as many warps as fit (3..12) with one or more stages each.  The pages
  // cost ~2K instructions each, so the kernel is bound by instruction
  // latency: 12 warps at 128 dims measured 182 us per 128K-token layer of 8
  // heads against 208 us for 8 warps (and 199 us for 13).  (fp32 caches
  // have twice the stage bytes, so fewer warps; that path is not tuned.)
  const int64_t stage = 2 * block_size * padded_dim(head_dim) * w;
  const int64_t ring = 192 * 1024;
  const int warps = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(12, ring / stage)));
  const int stages =
      static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(4, ring / (warps * stage))));
  const size_t smem = summarize_smem_bytes(padded_dim(head_dim), static_cast<int>(block_size),
                                           warps, stages, static_cast<int>(w));
  if (smem > static_cast<size_t>(dev.smem_optin)) {
    return fail(RKV_ERR_UNSUPPORTED, "summarizer stages do not fit in shared memory");
  }
  const int64_t blocks = cdiv(tokens, block_size);
  const int ctas = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>(dev.sms, cdiv(heads * blocks, warps))));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t err = cudaMemsetAsync(max_value_norm, 0, static_cast<size_t>(heads) * 4, st);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemsetAsync");
  SummarizeParams p = {};
  p.heads = static_cast<int>(heads);
  p.tokens = static_cast<int>(tokens);
  p.block_size = static_cast<int>(block_size);
  p.blocks = static_cast<int>(blocks);
  p.f32 = f32 ? 1 : 0;
  p.stages = stages;
  p.dim = static_cast<int>(head_dim);
  p.key_pages = key_pages_out;
  p.value_pages = value_pages_out;
  const int64_t packed = blocks * block_size * head_dim;
  p.key_pages_head_stride = key_pages_head_stride > 0 ? key_pages_head_stride : packed;
  p.value_pages_head_stride = value_pages_head_stride > 0 ? value_pages_head_stride : packed;
  p.key_mean = key_mean;
  p.value_mean = value_mean;
  p.ellipsoid = ellipsoid;
  p.value_norm = value_norm;
  p.max_value_norm = max_value_norm;
  p.counts = counts;
  err = launch_summarize(maps, p, padded_dim(head_dim), ctas, warps, smem, st);
  if (err != cudaSuccess) return cuda_fail(err, "summarize launch");
  return RKV_OK;
}

}  // namespace
}  // namespace rkv

extern "C" {

int rkv_summarize(const void* keys, const void* values, int64_t heads, int64_t tokens,
                  int64_t head_dim, int64_t key_head_stride, int64_t key_token_stride,
                  int64_t value_head_stride, int64_t value_token_stride, int64_t block_size,
                  void* key_pages_out, void* value_pages_out, void* key_mean, void* value_mean,
                  void* ellipsoid, float* value_norm, float* max_value_norm, int64_t* counts,
                  void* stream) {
  g_last_error.clear();
  return summarize_impl(keys, values, false, heads, tokens, head_dim, key_head_stride,
                        key_token_stride, value_head_stride, value_token_stride, block_size,
                        key_pages_out, 0, value_pages_out, 0, key_mean, value_mean, ellipsoid,
                        value_norm, max_value_norm, counts, stream);
}

int rkv_summarize_f32(const float* keys, const float* values, int64_t heads, int64_t tokens,
                      int64_t head_dim, int64_t key_head_stride, int64_t key_token_stride,
                      int64_t value_head_stride, int64_t value_token_stride, int64_t block_size,
                      void* key_pages_out, void* value_pages_out, void* key_mean,
                      void* value_mean, void* ellipsoid, float* value_norm,
                      float* max_value_norm, int64_t* counts, void* stream) {
  g_last_error.clear();
  return summarize_impl(keys, values, true, heads, tokens, head_dim, key_head_stride,
                        key_token_stride, value_head_stride, value_token_stride, block_size,
                        key_pages_out, 0, value_pages_out, 0, key_mean, value_mean, ellipsoid,
                        value_norm, max_value_norm, counts, stream);
}

int rkv_summarize_into(const void* keys, const void* values, int64_t heads, int64_t tokens,
                       int64_t head_dim, int64_t key_head_stride, int64_t key_token_stride,
                       int64_t value_head_stride, int64_t value_token_stride, int64_t block_size,
                       void* key_cache, int64_t key_cache_head_stride, void* value_cache,
                       int64_t value_cache_head_stride, void* key_mean, void* value_mean,
                       void* ellipsoid, float* value_norm, float* max_value_norm,
                       int64_t* counts, void* stream) {
  g_last_error.clear();
  if (key_cache == nullptr || value_cache == nullptr) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "null cache");
  }
  if (block_size > 0 && head_dim > 0 && tokens > 0) {
    const int64_t rows = cdiv(tokens, block_size) * block_size * head_dim;
    if (key_cache_head_stride < rows || value_cache_head_stride < rows ||
        (key_cache_head_stride * 2) % 16 || (value_cache_head_stride * 2) % 16) {
      return fail(RKV_ERR_INVALID_ARGUMENT,
                  "cache head strides must hold the padded prompt and be 16-byte multiples");
    }
  }
  return summarize_impl(keys, values, false, heads, tokens, head_dim, key_head_stride,
                        key_token_stride, value_head_stride, value_token_stride, block_size,
                        key_cache, key_cache_head_stride, value_cache, value_cache_head_stride,
                        key_mean, value_mean, ellipsoid, value_norm, max_value_norm, counts,
                        stream);
}

size_t rkv_select_workspace_size(int64_t heads, int64_t group, int64_t blocks, int64_t head_dim,
                                 int64_t queries) {
  if (heads <= 0 || group <= 0 || blocks <= 0 || queries <= 0 || !supported_dim(head_dim)) return 0;
  Plan pl;
  if (make_plan(&pl, heads, group, blocks, head_dim, 32, queries, false) != RKV_OK) return 0;
  return pl.bytes;
}

}  // extern "C"

namespace {

// rkv_select, or one rank's stage of rkv_select_split when `split` is given.
int select_impl(const rkv_summary* summary, const void* queries, int query_dtype,
                int64_t queries_n, int64_t group, float eps, int reduction, uint8_t* mask,
                int accumulate, void* workspace, size_t workspace_size, unsigned phases,
                void* stream, const SplitTarget* split) {
  int rc = check_selection_args(summary, queries, query_dtype, group, eps, reduction);
  if (rc != RKV_OK) return rc;
  if (queries_n < 1 || queries_n * summary->heads > 65535) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "queries must be 1..65535/heads");
  }
  if (mask == nullptr) return fail(RKV_ERR_INVALID_ARGUMENT, "mask is null");
  Plan pl;
  rc = make_plan(&pl, summary->heads, group, summary->blocks, summary->head_dim,
                 summary->block_size, queries_n, false, split ? split->geo.parts_a : 0);
  if (rc != RKV_OK) return rc;
  if ((rc = check_workspace(pl, workspace, workspace_size)) != RKV_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int or_mode = accumulate;
  if (!accumulate && queries_n > 1) {
    if (phases & RKV_PHASE_FINAL) {
      cudaError_t err =
          cudaMemsetAsync(mask, 0, static_cast<size_t>(summary->heads) * summary->blocks, st);
      if (err != cudaSuccess) return cuda_fail(err, "cudaMemsetAsync");
    }
    or_mode = 1;
  }
  return run_selector(pl, summary, queries, query_dtype, queries_n, group, eps, reduction, nullptr,
                      mask, or_mode, workspace, false, phases, st, split);
}

}  // namespace

extern "C" {

int rkv_select(const rkv_summary* summary, const void* queries, int query_dtype, int64_t queries_n,
               int64_t group, float eps, int reduction, uint8_t* mask, int accumulate,
               void* workspace, size_t workspace_size, void* stream) {
  g_last_error.clear();
  return select_impl(summary, queries, query_dtype, queries_n, group, eps, reduction, mask,
                     accumulate, workspace, workspace_size, RKV_PHASE_STATS | RKV_PHASE_FINAL,
                     stream, nullptr);
}

size_t rkv_select_split_slab(int64_t heads, int64_t group, int64_t max_blocks, int64_t queries) {
  if (heads <= 0 || heads > (1 << 16) || group < 1 || group > kMaxGroup || max_blocks <= 0 ||
      max_blocks > (1LL << 26) || queries < 1 || queries * heads > 65535) {
    return 0;
  }
  return split_geometry(heads, group, max_blocks, 0, queries).stats_slab;
}

int rkv_select_split(const rkv_summary* summary, const void* queries, int query_dtype,
                     int64_t queries_n, int64_t group, float eps, int reduction, uint8_t* mask,
                     int accumulate, void* workspace, size_t workspace_size, int64_t ranks,
                     int64_t rank, int64_t max_blocks, void* exchange, size_t exchange_size,
                     unsigned stage, void* stream) {
  g_last_error.clear();
  if (summary == nullptr) return fail(RKV_ERR_INVALID_ARGUMENT, "summary is null");
  if (summary->sequences > 1 || summary->page_table != nullptr) {
    return fail(RKV_ERR_UNSUPPORTED,
                "a sequence split takes one prompt in contiguous pages, not a batch or a page pool");
  }
  if (ranks < 1 || ranks > 64 || rank < 0 || rank >= ranks) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "need 1 <= ranks <= 64 and 0 <= rank < ranks");
  }
  if (max_blocks < summary->blocks || max_blocks > (1LL << 26)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "max_blocks must be at least this rank's block count");
  }
  if (queries_n < 1 || queries_n * summary->heads > 65535) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "queries must be 1..65535/heads");
  }
  if (stage == 0 || stage > (RKV_SPLIT_STATS | RKV_SPLIT_FINAL)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "bad split stage");
  }
  SplitTarget target;
  target.ranks = static_cast<int>(ranks);
  target.rank = static_cast<int>(rank);
  target.geo = split_geometry(summary->heads, group, max_blocks, 0, queries_n);
  target.exchange = static_cast<char*>(exchange);
  const size_t need = static_cast<size_t>(ranks) * target.geo.stats_slab;
  if (exchange == nullptr || exchange_size < need) {
    return fail(RKV_ERR_WORKSPACE, "exchange buffer is missing or smaller than the required size " +
                                       std::to_string(need));
  }
  if ((reinterpret_cast<uintptr_t>(exchange) & 255u) != 0) {
    return fail(RKV_ERR_ALIGNMENT, "exchange buffer must be 256-byte aligned");
  }
  const unsigned phases = ((stage & RKV_SPLIT_STATS) ? RKV_PHASE_STATS : 0u) |
                          ((stage & RKV_SPLIT_FINAL) ? RKV_PHASE_FINAL : 0u);
  return select_impl(summary, queries, query_dtype, queries_n, group, eps, reduction, mask,
                     accumulate, workspace, workspace_size, phases, stream, &target);
}

size_t rkv_decode_workspace_size(int64_t heads, int64_t group, int64_t blocks, int64_t head_dim,
                                 int64_t block_size) {
  if (heads <= 0 || group <= 0 || group > kMaxGroup || blocks <= 0 || !supported_dim(head_dim) ||
      !supported_block(block_size))
    return 0;
  Plan pl;
  if (make_plan(&pl, heads, group, blocks, head_dim, block_size, 1, true) != RKV_OK) return 0;
  return pl.bytes;
}

int rkv_decode_launch_count(unsigned phases) {
  return ((phases & RKV_PHASE_STATS) ? 1 : 0) + ((phases & RKV_PHASE_FINAL) ? 1 : 0) +
         ((phases & RKV_PHASE_ATTEND) ? 1 : 0) + ((phases & RKV_PHASE_COMBINE) ? 1 : 0);
}

}  // extern "C"

namespace {

// The attention and combine launches of rkv_decode (after the selector) and
// of rkv_decode_dense (no selector: every block attended).
int attend_and_combine(const Plan& pl, const rkv_summary* summary, const void* query,
                       int query_dtype, int64_t group, const void* key_suffix,
                       const void* value_suffix, int64_t suffix_capacity,
                       int64_t key_suffix_head_stride, int64_t key_suffix_token_stride,
                       int64_t value_suffix_head_stride, int64_t value_suffix_token_stride,
                       const int32_t* suffix_length, int64_t suffix_length_host, void* output,
                       void* workspace, unsigned phases, bool dense, cudaStream_t st,
                       const SplitTarget* split) {
  int rc = RKV_OK;
  const int64_t H = summary->heads, D = summary->head_dim, B = summary->block_size;
  const int* suffix_ptr = suffix_length;
  if (phases & RKV_PHASE_ATTEND) {
    AttendMaps maps;
    const bool paged = summary->page_table != nullptr;
    const int64_t pool_heads = paged ? H / std::max<int64_t>(1, summary->sequences) : H;
    rc = pages_map(&maps.key_pages, summary->key_pages, D, B, pool_heads,
                   paged ? summary->pool_pages : summary->blocks,
                   paged ? summary->key_token_stride : D, summary->key_page_head_stride,
                   paged ? summary->key_page_stride : B * D, "key_pages");
    if (rc != RKV_OK) return rc;
    rc = pages_map(&maps.value_pages, summary->value_pages, D, B, pool_heads,
                   paged ? summary->pool_pages : summary->blocks,
                   paged ? summary->value_token_stride : D, summary->value_page_head_stride,
                   paged ? summary->value_page_stride : B * D, "value_pages");
    if (rc != RKV_OK) return rc;
    if (suffix_capacity > 0) {
      rc = rows_map(&maps.key_suffix, key_suffix, D, suffix_capacity, H, key_suffix_token_stride,
                    key_suffix_head_stride, static_cast<int>(B), "key_suffix");
      if (rc != RKV_OK) return rc;
      rc = rows_map(&maps.value_suffix, value_suffix, D, suffix_capacity, H,
                    value_suffix_token_stride, value_suffix_head_stride, static_cast<int>(B),
                    "value_suffix");
      if (rc != RKV_OK) return rc;
    } else {
      maps.key_suffix = maps.key_pages;
      maps.value_suffix = maps.value_pages;
    }
    AttendParams p = {};
    p.seq = seq_layout(summary);
    p.query = query;
    p.query_f32 = query_dtype == RKV_DTYPE_F32;
    p.dim = static_cast<int>(D);
    p.counts = summary->counts;
    p.heads = static_cast<int>(H);
    p.group = static_cast<int>(group);
    p.blocks = static_cast<int>(summary->blocks);
    p.page = static_cast<int>(B);
    p.prompt_length = static_cast<int>(summary->prompt_length);
    p.page_table = summary->page_table;
    p.page_table_stride = static_cast<int>(paged ? summary->page_table_stride : 0);
    p.pool_pages = static_cast<int>(paged ? summary->pool_pages : summary->blocks);
    p.has_suffix = suffix_capacity > 0;
    p.suffix_capacity = static_cast<int>(suffix_capacity);
    p.suffix_len_ptr = suffix_ptr;
    p.suffix_len_host = static_cast<int>(suffix_length_host);
    p.seg_count = at<int>(workspace, pl.seg_count);
    p.sel_ids = at<int>(workspace, pl.sel_ids);
    p.parts_b = pl.parts_b;
    p.seg_cap = pl.seg_cap;
    p.dense = dense ? 1 : 0;
    p.att_m = at<float>(workspace, pl.att_m);
    p.att_l = at<float>(workspace, pl.att_l);
    p.att_o = at<float>(workspace, pl.att_o);
    p.ctas = pl.ctas;
    p.stages = pl.stages_c;
    p.status = at<int>(workspace, pl.status);
    p.scale = static_cast<float>(std::pow(static_cast<double>(D), -0.5));
    cudaError_t err = launch_attend(maps, p, padded_dim(D), pl.warps_c, pl.smem_c, st, true);
    if (err != cudaSuccess) return cuda_fail(err, "attention launch");
  }
  if (phases & RKV_PHASE_COMBINE) {
    CombineParams c = {};
    c.query_f32 = query_dtype == RKV_DTYPE_F32;
    c.dim = static_cast<int>(D);
    c.out = output;
    c.heads = static_cast<int>(H);
    c.group = static_cast<int>(group);
    c.page = static_cast<int>(B);
    c.has_suffix = suffix_capacity > 0;
    c.suffix_capacity = static_cast<int>(suffix_capacity);
    c.suffix_len_ptr = suffix_ptr;
    c.suffix_len_host = static_cast<int>(suffix_length_host);
    c.seg_count = at<int>(workspace, pl.seg_count);
    c.parts_b = pl.parts_b;
    c.dense = dense ? 1 : 0;
    c.seq = seq_layout(summary);
    c.blocks = static_cast<int>(summary->blocks);
    c.rep_m = at<float>(workspace, pl.rep_m);
    c.rep_l = at<float>(workspace, pl.rep_l);
    c.rep_o = at<float>(workspace, pl.rep_o);
    c.att_m = at<float>(workspace, pl.att_m);
    c.att_l = at<float>(workspace, pl.att_l);
    c.att_o = at<float>(workspace, pl.att_o);
    c.ctas = pl.ctas;
    c.warps = pl.warps_c;
    c.max_sources = pl.max_sources;
    c.part_ml = split ? split->output_ml(split->rank) : nullptr;
    c.part_o = split ? split->output_o(split->rank) : nullptr;
    c.status = at<int>(workspace, pl.status);
    cudaError_t err = launch_combine(c, padded_dim(D), st, true);
    if (err != cudaSuccess) return cuda_fail(err, "combine launch");
  }
  return RKV_OK;
}

// rkv_decode, and one rank's share of a sequence-split step when `split` is
// given (phase A into the rank's stats slab, phase B over all slabs, combine
// into the rank's output slab).
int decode_impl(const rkv_summary* summary, const void* query, int query_dtype, int64_t group,
                const void* key_suffix, const void* value_suffix, int64_t suffix_capacity,
                int64_t key_suffix_head_stride, int64_t key_suffix_token_stride,
                int64_t value_suffix_head_stride, int64_t value_suffix_token_stride,
                const int32_t* suffix_length, int64_t suffix_length_host,
                const uint8_t* anchor_mask, float eps, int reduction, void* output,
                uint8_t* selected, void* workspace, size_t workspace_size, unsigned phases,
                void* stream, const SplitTarget* split) {
  int rc = check_selection_args(summary, query, query_dtype, group, eps, reduction);
  if (rc != RKV_OK) return rc;
  if (output == nullptr || selected == nullptr) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "output and selected must be non-null");
  }
  if (suffix_capacity < 0 || suffix_capacity > (1LL << 30)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "suffix_capacity out of range");
  }
  if (suffix_capacity > 0 && (key_suffix == nullptr || value_suffix == nullptr)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "suffix K/V are null");
  }
  if (suffix_length == nullptr && (suffix_length_host < 0 || suffix_length_host > suffix_capacity)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "suffix_length_host must be in [0, suffix_capacity]");
  }
  if (phases == 0 || phases > RKV_PHASE_ALL) return fail(RKV_ERR_INVALID_ARGUMENT, "bad phases");
  Plan pl;
  rc = make_plan(&pl, summary->heads, group, summary->blocks, summary->head_dim,
                 summary->block_size, 1, true, split ? split->geo.parts_a : 0);
  if (rc != RKV_OK) return rc;
  if ((rc = check_workspace(pl, workspace, workspace_size)) != RKV_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pl.fused && phases == RKV_PHASE_ALL && split == nullptr) {
    return run_fused_decode(pl, summary, query, query_dtype, group, key_suffix, value_suffix,
                            suffix_capacity, key_suffix_head_stride, key_suffix_token_stride,
                            value_suffix_head_stride, value_suffix_token_stride, suffix_length,
                            suffix_length_host, eps, reduction, anchor_mask, selected, output,
                            workspace, st);
  }
  rc = run_selector(pl, summary, query, query_dtype, 1, group, eps, reduction, anchor_mask,
                    selected, 0, workspace, true, phases, st, split);
  if (rc != RKV_OK) return rc;
  return attend_and_combine(pl, summary, query, query_dtype, group, key_suffix, value_suffix,
                            suffix_capacity, key_suffix_head_stride, key_suffix_token_stride,
                            value_suffix_head_stride, value_suffix_token_stride, suffix_length,
                            suffix_length_host, output, workspace, phases, false, st, split);
}

}  // namespace

extern "C" {

int rkv_decode(const rkv_summary* summary, const void* query, int query_dtype, int64_t group,
               const void* key_suffix, const void* value_suffix, int64_t suffix_capacity,
               int64_t key_suffix_head_stride, int64_t key_suffix_token_stride,
               int64_t value_suffix_head_stride, int64_t value_suffix_token_stride,
               const int32_t* suffix_length, int64_t suffix_length_host,
               const uint8_t* anchor_mask, float eps, int reduction, void* output,
               uint8_t* selected, void* workspace, size_t workspace_size, unsigned phases,
               void* stream) {
  g_last_error.clear();
  return decode_impl(summary, query, query_dtype, group, key_suffix, value_suffix,
                     suffix_capacity, key_suffix_head_stride, key_suffix_token_stride,
                     value_suffix_head_stride, value_suffix_token_stride, suffix_length,
                     suffix_length_host, anchor_mask, eps, reduction, output, selected,
                     workspace, workspace_size, phases, stream, nullptr);
}

int rkv_split_exchange_slabs(int64_t heads, int64_t group, int64_t max_blocks, int64_t head_dim,
                             size_t* stats_slab, size_t* output_slab) {
  g_last_error.clear();
  if (heads <= 0 || heads > (1 << 16) || group < 1 || group > kMaxGroup || max_blocks <= 0 ||
      max_blocks > (1LL << 26)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "split geometry out of range");
  }
  if (!supported_dim(head_dim)) return fail(RKV_ERR_UNSUPPORTED, "head_dim must be a multiple of 32 in [32, 256]");
  if (stats_slab == nullptr || output_slab == nullptr) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "null output pointer");
  }
  const SplitGeometry geo = split_geometry(heads, group, max_blocks, head_dim);
  *stats_slab = geo.stats_slab;
  *output_slab = geo.output_slab;
  return RKV_OK;
}

int rkv_decode_split(const rkv_summary* summary, const void* query, int query_dtype, int64_t group,
                     const void* key_suffix, const void* value_suffix, int64_t suffix_capacity,
                     int64_t key_suffix_head_stride, int64_t key_suffix_token_stride,
                     int64_t value_suffix_head_stride, int64_t value_suffix_token_stride,
                     const int32_t* suffix_length, int64_t suffix_length_host,
                     const uint8_t* anchor_mask, float eps, int reduction, void* output,
                     uint8_t* selected, void* workspace, size_t workspace_size, int64_t ranks,
                     int64_t rank, int64_t max_blocks, void* exchange, size_t exchange_size,
                     unsigned stage, void* stream) {
  g_last_error.clear();
  int rc = check_selection_args(summary, query, query_dtype, group, eps, reduction);
  if (rc != RKV_OK) return rc;
  if (summary->sequences > 1 || summary->page_table != nullptr) {
    return fail(RKV_ERR_UNSUPPORTED,
                "a sequence split takes one prompt in contiguous pages, not a batch or a page pool");
  }
  if (ranks < 1 || ranks > 64 || rank < 0 || rank >= ranks) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "need 1 <= ranks <= 64 and 0 <= rank < ranks");
  }
  if (max_blocks < summary->blocks || max_blocks > (1LL << 26)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "max_blocks must be at least this rank's block count");
  }
  if (stage == 0 || stage > (RKV_SPLIT_STATS | RKV_SPLIT_ATTEND | RKV_SPLIT_MERGE)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "bad split stage");
  }
  SplitTarget target;
  target.ranks = static_cast<int>(ranks);
  target.rank = static_cast<int>(rank);
  target.geo = split_geometry(summary->heads, group, max_blocks, summary->head_dim);
  target.exchange = static_cast<char*>(exchange);
  const size_t need = static_cast<size_t>(ranks) * (target.geo.stats_slab + target.geo.output_slab);
  if (exchange == nullptr || exchange_size < need) {
    return fail(RKV_ERR_WORKSPACE, "exchange buffer is missing or smaller than the required size " +
                                       std::to_string(need));
  }
  if ((reinterpret_cast<uintptr_t>(exchange) & 255u) != 0) {
    return fail(RKV_ERR_ALIGNMENT, "exchange buffer must be 256-byte aligned");
  }
  if (output == nullptr) return fail(RKV_ERR_INVALID_ARGUMENT, "output must be non-null");
  if (stage & RKV_SPLIT_STATS) {
    rc = decode_impl(summary, query, query_dtype, group, key_suffix, value_suffix,
                     suffix_capacity, key_suffix_head_stride, key_suffix_token_stride,
                     value_suffix_head_stride, value_suffix_token_stride, suffix_length,
                     suffix_length_host, anchor_mask, eps, reduction, output, selected, workspace,
                     workspace_size, RKV_PHASE_STATS, stream, &target);
    if (rc != RKV_OK) return rc;
  }
  if (stage & RKV_SPLIT_ATTEND) {
    rc = decode_impl(summary, query, query_dtype, group, key_suffix, value_suffix,
                     suffix_capacity, key_suffix_head_stride, key_suffix_token_stride,
                     value_suffix_head_stride, value_suffix_token_stride, suffix_length,
                     suffix_length_host, anchor_mask, eps, reduction, output, selected, workspace,
                     workspace_size, RKV_PHASE_FINAL | RKV_PHASE_ATTEND | RKV_PHASE_COMBINE,
                     stream, &target);
    if (rc != RKV_OK) return rc;
  }
  if (stage & RKV_SPLIT_MERGE) {
    MergeParams m = {};
    m.query_f32 = query_dtype == RKV_DTYPE_F32;
    m.dim = static_cast<int>(summary->head_dim);
    m.out = output;
    m.heads = static_cast<int>(summary->heads);
    m.group = static_cast<int>(group);
    m.ranks = target.ranks;
    m.part_ml = target.output_ml(0);
    m.part_o = target.output_o(0);
    m.slab_floats = target.geo.output_slab / 4;
    const cudaError_t err = launch_merge(m, static_cast<int>(summary->head_dim),
                                         static_cast<cudaStream_t>(stream), true);
    if (err != cudaSuccess) return cuda_fail(err, "split merge launch");
  }
  return RKV_OK;
}

}  // extern "C"

extern "C" {

size_t rkv_decode_dense_workspace_size(int64_t heads, int64_t group, int64_t blocks,
                                       int64_t head_dim, int64_t block_size) {
  if (heads <= 0 || group <= 0 || group > kMaxGroup || blocks <= 0 || !supported_dim(head_dim) ||
      !supported_block(block_size))
    return 0;
  Plan pl;
  if (make_dense_plan(&pl, heads, group, head_dim, block_size) != RKV_OK) return 0;
  return pl.bytes;
}

int rkv_decode_dense(const rkv_summary* pages, const void* query, int query_dtype, int64_t group,
                     const void* key_suffix, const void* value_suffix, int64_t suffix_capacity,
                     int64_t key_suffix_head_stride, int64_t key_suffix_token_stride,
                     int64_t value_suffix_head_stride, int64_t value_suffix_token_stride,
                     const int32_t* suffix_length, int64_t suffix_length_host, void* output,
                     void* workspace, size_t workspace_size, void* stream) {
  g_last_error.clear();
  int rc = check_pages(pages);
  if (rc != RKV_OK) return rc;
  if (query == nullptr || output == nullptr) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "query and output must be non-null");
  }
  if (query_dtype != RKV_DTYPE_BF16 && query_dtype != RKV_DTYPE_F32) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "query dtype must be bf16 or fp32");
  }
  if (group < 1 || group > kMaxGroup) return fail(RKV_ERR_UNSUPPORTED, "group must be 1..16");
  if (suffix_capacity < 0 || suffix_capacity > (1LL << 30)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "suffix_capacity out of range");
  }
  if (suffix_capacity > 0 && (key_suffix == nullptr || value_suffix == nullptr)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "suffix K/V are null");
  }
  if (suffix_length == nullptr && (suffix_length_host < 0 || suffix_length_host > suffix_capacity)) {
    return fail(RKV_ERR_INVALID_ARGUMENT, "suffix_length_host must be in [0, suffix_capacity]");
  }
  Plan pl;
  rc = make_dense_plan(&pl, pages->heads, group, pages->head_dim, pages->block_size);
  if (rc != RKV_OK) return rc;
  if ((rc = check_workspace(pl, workspace, workspace_size)) != RKV_OK) return rc;
  return attend_and_combine(pl, pages, query, query_dtype, group, key_suffix, value_suffix,
                            suffix_capacity, key_suffix_head_stride, key_suffix_token_stride,
                            value_suffix_head_stride, value_suffix_token_stride, suffix_length,
                            suffix_length_host, output, workspace,
                            RKV_PHASE_ATTEND | RKV_PHASE_COMBINE, true,
                            static_cast<cudaStream_t>(stream), nullptr);
}

}  // extern "C"

extern "C" {

void rkv_set_fused_selector(int enable) { g_fused_selector.store(enable ? 1 : 0); }

int rkv_decode_kernel_count(int64_t heads, int64_t group, int64_t blocks, int64_t head_dim,
                            int64_t block_size) {
  if (heads <= 0 || group <= 0 || group > kMaxGroup || blocks <= 0 || !supported_dim(head_dim) ||
      !supported_block(block_size))
    return 0;
  Plan pl;
  if (make_plan(&pl, heads, group, blocks, head_dim, block_size, 1, true) != RKV_OK) return 0;
  return pl.fused ? 1 : 4;
}

}  // extern "C"
