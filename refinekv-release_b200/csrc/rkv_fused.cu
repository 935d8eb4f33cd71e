// One-kernel decode step of a layer (reference: src/refinekv/reference.py:10-73;
// the reference's GPU form is six Triton kernels, kernels/selection.py:47-223
// and kernels/attention.py:13-329).
//
// One CTA per (KV-head row, part); a row's parts split its blocks into equal
// contiguous ranges, and the grid never has more CTAs than SMs (unless every
// row has a single part), so all parts of a row are resident together (the
// host sizes it; one CTA per SM by shared memory).  A CTA:
//   0. reads its row's anchor bytes once: its own blocks' anchor bits, and
//      whether every block of the row is anchored (then no part of the row
//      needs the selector statistics, and steps 1 and 3 are skipped);
//   1. phase A: z and delta of every (group row, block) of its tiles from the
//      key-mean and ellipsoid tiles (TMA, mma.sync), kept for phase B, and
//      one log-sum-exp partial per part; arrives at the row's barrier A;
//   2. streams, without waiting, the pages whose attention is known before
//      any decision: its anchored blocks (selected whatever the risk,
//      reference.py:54-55) and its share of the generated suffix;
//   3. unless every block of its range is anchored: waits at barrier A (by
//      then normally passed), merges the row's partials into log Z / log C,
//      decides every block of its tiles (risk, GQA reduction, non-finite
//      override) and writes the mask, each tile's representatives (value
//      means, logit z) joining the softmax while the next tile is decided,
//      then streams its selected non-anchored pages;
//   4. merges its warps into one softmax partial; in a row of at most
//      kLastParts parts the part that arrives last writes the row's output
//      from all parts' partials, in a longer row the parts meet at barrier B
//      and each writes its slice of the output channels.
// Every wait is bounded (status bit on timeout).  The order of the work is
// static (block order, warps round-robin), so results are deterministic.
// The page arithmetic is the attention kernel's (rkv_attend.cu): the same
// helpers of rkv_device.cuh; only the order in which partials merge differs.
#include "rkv_device.cuh"
#include "rkv_kernels.h"
#include "rkv_risk.cuh"

namespace rkv {
namespace {

// Shared-memory layout (also sized by the host): a TMA slice per warp, two
// mbarriers per warp, row normalisers, flags, the warps' phase-A (max, sum)
// pairs, per-tile bit masks and offsets, one block list (anchored blocks,
// then the selected non-anchored ones) and, when they fit, the part's z,
// delta and value norms.  The warps' final partials, then the row's parts'
// weights, are parked in the slices.
struct FusedLayout {
  size_t bars, norms, flags, lse, sel_bits, anc_bits, offsets, anc_off,
      anchored, zs, ds, vs, bytes;
  // zd_group > 0: z and delta of the part's tiles stay in shared memory,
  // [tcap][zd_group][32] each, instead of the workspace, with the blocks'
  // value norms [tcap][32].
  __host__ __device__ FusedLayout(int warps, int slice, int tcap, int zd_group) {
    const size_t t = static_cast<size_t>(tcap);
    size_t off = static_cast<size_t>(warps) * slice;
    auto take = [&](size_t bytes_) {
      const size_t at_ = off;
      off += round16(bytes_);
      return at_;
    };
    bars = take(static_cast<size_t>(warps) * 2 * 8);
    norms = take(2 * kMaxGroup * 4);
    flags = take(8 * 4);
    lse = take(static_cast<size_t>(warps) * kMaxGroup * 16);  // [warps][16] float4
    sel_bits = take(t * 4);        // [tcap] uint32
    anc_bits = take(t * 4);        // [tcap] uint32
    offsets = take((t + 1) * 4);   // [tcap + 1] int
    anc_off = take((t + 1) * 4);   // [tcap + 1] int
    anchored = take(t * kSelectTile * 4);  // [tcap * 32] int
    const size_t zd = t * static_cast<size_t>(zd_group) * kSelectTile * 4;
    zs = take(zd);
    ds = take(zd);
    vs = take(zd_group > 0 ? t * kSelectTile * 4 : 0);
    bytes = off + kSmemSlack;
  }
};

template <int D, int R>
struct FusedShape {
  static constexpr int kSel = kSelectTile * D * 2;  // one key-mean / ellipsoid / value-mean tile
  static constexpr int kPage = R * D * 2;           // one K or V page
  static constexpr int kSlice = (2 * kSel > 2 * kPage ? 2 * kSel : 2 * kPage);
};

// Bounded wait for a generation word to move past `seen`; false on timeout.
__device__ __forceinline__ bool wait_generation(const unsigned* word, unsigned seen) {
  const unsigned long long start = global_ns();
  while (true) {
    unsigned now;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(now) : "l"(word) : "memory");
    if (now != seen) return true;
    if (global_ns() - start > kWaitLimitNs) return false;
    __nanosleep(64);
  }
}

// Release/acquire at GPU scope: an arrival publishes the writes that precede
// it (its own and, through a CTA or warp barrier, its CTA's), and the last
// arrival acquires everyone's before it moves the generation on.
__device__ __forceinline__ unsigned atom_add_acq_rel(unsigned* word, unsigned v) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old) : "l"(word), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void red_add_release(unsigned* word, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(word), "r"(v) : "memory");
}

__device__ __forceinline__ void store_relaxed(unsigned* word, unsigned v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(word), "r"(v) : "memory");
}

// Arrival of one part at a row barrier (one thread, after a CTA or warp
// barrier that follows the writes it publishes): the last of `parts`
// arrivals resets the count and moves the generation on, so the words are
// clean for the next call (which starts after this grid has completed).
// Returns whether this was the last arrival.
__device__ __forceinline__ bool arrive(unsigned* count, unsigned* gen, int parts) {
  const unsigned before = atom_add_acq_rel(count, 1u);
  if (before != static_cast<unsigned>(parts) - 1u) return false;
  store_relaxed(count, 0u);
  if (gen != nullptr) red_add_release(gen, 1u);
  return true;
}

__device__ __forceinline__ unsigned read_generation(const unsigned* word) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(word) : "memory");
  return v;
}

// Streams `count` items of one warp -- K|V pages or suffix chunks of R rows --
// through the warp's slice with separate K and V barriers (K refilled as soon
// as the scores are done), into the running softmax (m, l, o).  item(j)
// returns {suffix?, page or first suffix row, valid rows, head coordinate};
// pre() runs once, after the first page's copies are issued (or at once when
// there is nothing to stream).
// False on a timeout, after the copies in flight have landed.
template <int R, int D, int NT, typename ItemFn, typename PreFn>
__device__ __forceinline__ bool stream_items(int count, ItemFn item, PreFn pre, const FusedMaps& maps,
                                             uint8_t* slice, uint64_t* bar_a, uint64_t* bar_b,
                                             uint32_t& uses_a, uint32_t& uses_b,
                                             const uint32_t (&qb)[D / 16][NT][2], float scale,
                                             bool split, float (&m)[NT][2], float (&l)[NT][2],
                                             float (&o)[D / 16][NT][4], uint64_t policy,
                                             int lane) {
  if (count <= 0) {
    pre();
    return true;
  }
  constexpr int kPage = R * D * 2;
  auto issue = [&](const int4& it, bool value) {
    if (lane == 0) {
      uint64_t* bar = value ? bar_b : bar_a;
      uint8_t* dst = slice + (value ? kPage : 0);
      fence_proxy_async();
      mbar_expect_tx(bar, kPage);
      if (it.x) {
        tma_tile_hint<D>(dst, value ? &maps.value_suffix : &maps.key_suffix, bar, it.y, it.w, R,
                         policy);
      } else {
        tma_page_hint<D>(dst, value ? &maps.value_pages : &maps.key_pages, bar, it.w, it.y, R,
                         policy);
      }
    }
  };
  int4 cur = item(0);
  issue(cur, false);
  issue(cur, true);
  pre();  // runs while the first page lands
  uint32_t issued_a = uses_a + 1, issued_b = uses_b + 1;
  bool ok = true;
  for (int j = 0; j < count; ++j) {
    if (!warp_wait(bar_a, uses_a & 1)) {
      ok = false;
      break;
    }
    ++uses_a;
    float logit[R / 16][NT][4];
    score_tile<R, D, NT>(smem_addr(slice), qb, logit, lane);
#pragma unroll
    for (int mt = 0; mt < R / 16; ++mt)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int r = mt * 16 + (lane >> 2) + (c >> 1) * 8;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          logit[mt][nt][c] = r < cur.z ? logit[mt][nt][c] * scale : -INFINITY;
      }
    __syncwarp();
    int4 next = make_int4(0, 0, 0, 0);
    const bool more = j + 1 < count;
    if (more) {
      next = item(j + 1);
      issue(next, false);
      ++issued_a;
    }
    softmax_update<R, D, NT>(logit, m, l, o);
    uint32_t hi[R / 16][NT][2], lo[R / 16][NT][2];
    prob_frags<R, NT>(logit, hi, lo, split);
    if (!warp_wait(bar_b, uses_b & 1)) {
      ok = false;
      break;
    }
    ++uses_b;
    accumulate_values<R, D, NT>(smem_addr(slice + kPage), hi, o, lane);
    if (split) accumulate_values<R, D, NT>(smem_addr(slice + kPage), lo, o, lane);
    __syncwarp();
    if (more) {
      issue(next, true);
      ++issued_b;
    }
    cur = next;
  }
  for (; uses_a < issued_a; ++uses_a) mbar_wait(bar_a, uses_a & 1);
  for (; uses_b < issued_b; ++uses_b) mbar_wait(bar_b, uses_b & 1);
  return ok;
}

// Rows of at most this many parts are merged by the part that arrives last.
constexpr int kLastParts = 32;

// Row stride of a stashed warp partial: 4 floats of padding keep the stash's
// stores (lanes 2 group rows apart) and the merge's loads (lanes one group row
// apart) on distinct banks.
template <int D>
constexpr int kStashStride = D + 4;

// A warp's final (m, l, o^T) into shared memory: m[W][G8], l[W][G8] and
// o[W][G8][kStashStride].
template <int D, int NT>
__device__ __forceinline__ void stash_padded(float* sm_m, float* sm_l, float* sm_o, int warp,
                                             int lane, const float (&m)[NT][2],
                                             const float (&l)[NT][2],
                                             const float (&o)[D / 16][NT][4]) {
  constexpr int G8 = NT * 8;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int g = nt * 8 + 2 * (lane & 3) + j;
      if (lane < 4) {
        sm_m[warp * G8 + g] = m[nt][j];
        sm_l[warp * G8 + g] = l[nt][j];
      }
      float* row = sm_o + (warp * G8 + g) * kStashStride<D>;
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        const int d0 = dt * 16 + (lane >> 2);
        row[d0] = o[dt][nt][j];
        row[d0 + 8] = o[dt][nt][2 + j];
      }
    }
  }
}

// PACK4: group of at most 4 rows (q and q^2 share one n8 tile); GM: group
// rows evaluated per block in phase B (padded to 4, 8 or 16).
template <int D, int R, int NT, bool PACK4, int GM>
__global__ void __launch_bounds__(256, 1) fused_kernel(const __grid_constant__ FusedMaps maps,
                                                       const FusedParams p) {
  constexpr int T = kSelectTile;
  constexpr int kSel = FusedShape<D, R>::kSel;
  constexpr int kSlice = FusedShape<D, R>::kSlice;
  constexpr int G8 = NT * 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  const int W = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const FusedLayout lay(W, kSlice, p.tcap, p.zd_group);
  uint8_t* slice = smem + static_cast<size_t>(warp) * kSlice;
  uint64_t* bar_a = reinterpret_cast<uint64_t*>(smem + lay.bars) + warp * 2;
  uint64_t* bar_b = bar_a + 1;
  float* lz = reinterpret_cast<float*>(smem + lay.norms);
  float* lc = lz + kMaxGroup;
  int* flags = reinterpret_cast<int*>(smem + lay.flags);  // 0 bad row stat, 2 listed, 3 last
  float4* lse_s = reinterpret_cast<float4*>(smem + lay.lse);              // [W][kMaxGroup]
  uint32_t* sel_bits = reinterpret_cast<uint32_t*>(smem + lay.sel_bits);  // [tcap]
  uint32_t* anc_bits = reinterpret_cast<uint32_t*>(smem + lay.anc_bits);  // [tcap]
  int* offsets = reinterpret_cast<int*>(smem + lay.offsets);             // [tcap + 1]
  int* anc_off = reinterpret_cast<int*>(smem + lay.anc_off);             // [tcap + 1]
  int* blist = reinterpret_cast<int*>(smem + lay.anchored);              // [tcap * 32]
  float* zsm = reinterpret_cast<float*>(smem + lay.zs);  // [tcap][group][32] when p.zd_group
  float* dsm = reinterpret_cast<float*>(smem + lay.ds);
  float* vsm = reinterpret_cast<float*>(smem + lay.vs);  // [tcap][32] when p.zd_group
  const bool zd_local = p.zd_group != 0;

  // This CTA's row and part.
  const int c = blockIdx.x;
  const int P = p.parts_base, X = p.parts_extra;
  int h, part, parts_h;
  if (c < X * (P + 1)) {
    h = c / (P + 1);
    part = c - h * (P + 1);
    parts_h = P + 1;
  } else {
    const int c2 = c - X * (P + 1);
    h = X + c2 / P;
    part = c2 - (c2 / P) * P;
    parts_h = P;
  }
  const int first_cta = c - part;
  const int lse_parts = P + (X > 0 ? 1 : 0);
  // This part's blocks: an equal share of the row's real blocks (so every part
  // streams as many pages as the others), and the selector tiles they touch.
  const int blocks_h = p.seq.blocks(h, p.blocks);
  const int b_lo = static_cast<int>(static_cast<long long>(blocks_h) * part / parts_h);
  const int b_hi = static_cast<int>(static_cast<long long>(blocks_h) * (part + 1) / parts_h);
  const int t_lo = b_lo / T;
  const int t_hi = b_hi > b_lo ? (b_hi + T - 1) / T : t_lo;
  const int n_t = t_hi - t_lo;
  auto mine = [&](int b) { return b >= b_lo && b < b_hi; };
  const int64_t* counts = p.counts + static_cast<size_t>(p.seq.sequence(h)) * p.blocks;
  const char* q = static_cast<const char*>(p.query) +
                  static_cast<size_t>(h) * p.group * p.dim * (p.query_f32 ? 4 : 2);
  unsigned* arrive_a = p.bar_words + h;
  unsigned* gen_a = arrive_a + p.bar_stride;
  unsigned* arrive_b = gen_a + p.bar_stride;
  unsigned* gen_b = arrive_b + p.bar_stride;

  if (lane == 0) {
    mbar_init(bar_a, 1);
    mbar_init(bar_b, 1);
    mbar_fence_init();
    // The summaries do not change during decode: this warp's first tile goes
    // to L2 before the dependency wait.
    if (warp < n_t) {
      tma_prefetch_tile<D>(&maps.key_mean, (t_lo + warp) * T, h);
      tma_prefetch_tile<D>(&maps.ellipsoid, (t_lo + warp) * T, h);
    }
    // So does the warp's first page when the anchor mask marks it -- a hint
    // only: the mask is read again after the wait, and that read decides.
    const int b_first = b_lo + warp;
    if (p.anchor != nullptr && p.page_table == nullptr && b_first < b_hi &&
        __ldcg(p.anchor + static_cast<size_t>(h) * p.blocks + b_first) != 0) {
      tma_prefetch_page<D>(&maps.key_pages, h, b_first);
      tma_prefetch_page<D>(&maps.value_pages, h, b_first);
    }
  }
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&maps.key_mean);
    tma_prefetch_desc(&maps.ellipsoid);
    tma_prefetch_desc(&maps.value_mean);
    tma_prefetch_desc(&maps.key_pages);
    tma_prefetch_desc(&maps.value_pages);
    if (p.has_suffix) {
      tma_prefetch_desc(&maps.key_suffix);
      tma_prefetch_desc(&maps.value_suffix);
    }
    for (int i = 0; i < 8; ++i) flags[i] = 0;
  }
  for (int k = threadIdx.x; k < n_t; k += blockDim.x) anc_bits[k] = 0u;
  for (int i = threadIdx.x; i * 128 < p.group * p.dim * (p.query_f32 ? 4 : 2); i += blockDim.x) {
    prefetch_l2(q + i * 128);
  }
  // The part's value norms, counts and anchor bytes, read one tile at a time
  // by the decisions and phase A, go to L2 now (prefetches only).
  if (b_hi > b_lo) {
    const int nvn = (b_hi - b_lo) * 4, ncn = (b_hi - b_lo) * 8, nan_ = b_hi - b_lo;
    const char* vn = reinterpret_cast<const char*>(p.value_norm + static_cast<size_t>(h) * p.blocks + b_lo);
    const char* cn = reinterpret_cast<const char*>(counts + b_lo);
    const char* an = p.anchor != nullptr
                         ? reinterpret_cast<const char*>(p.anchor + static_cast<size_t>(h) * p.blocks + b_lo)
                         : nullptr;
    const int lines_vn = (nvn + 127) / 128, lines_cn = (ncn + 127) / 128;
    const int lines_an = an != nullptr ? (nan_ + 127) / 128 : 0;
    for (int i = threadIdx.x; i < lines_vn + lines_cn + lines_an; i += blockDim.x) {
      if (i < lines_vn) {
        prefetch_l2(vn + i * 128);
      } else if (i < lines_vn + lines_cn) {
        prefetch_l2(cn + (i - lines_vn) * 128);
      } else {
        prefetch_l2(an + (i - lines_vn - lines_cn) * 128);
      }
    }
  }
  __syncthreads();
  pdl_wait();
  // Every CTA of this grid has started once all have passed here, so a grid
  // launched early behind this one can never hold an SM one of ours needs.
  pdl_launch_dependents();
  const uint64_t policy = l2_evict_first_policy();
  // The row's barrier generations before this part's arrivals (they move only
  // once every part, this one included, has arrived).
  unsigned seen_a = 0, seen_b = 0;
  if (threadIdx.x == 0) {
    seen_a = read_generation(gen_a);
    seen_b = read_generation(gen_b);
  }
  int suffix_len = 0;
  if (p.has_suffix) {
    suffix_len = p.suffix_len_ptr != nullptr ? *p.suffix_len_ptr : p.suffix_len_host;
    if (suffix_len < 0 || suffix_len > p.suffix_capacity) {
      if (threadIdx.x == 0) atomicOr(p.status, kStatusBadInput);
      suffix_len = suffix_len < 0 ? 0 : p.suffix_capacity;
    }
  }
  const int prompt_h = p.seq.prompt(h, p.prompt_length);
  const int pool_head = p.page_table != nullptr ? h - p.seq.sequence(h) * p.seq.heads_per_seq : h;
  uint32_t uses_a = 0, uses_b = 0;  // completed waits per barrier (parity = uses & 1)
  bool aborted = false;
  auto timeout = [&]() {
    if (lane == 0) atomicOr(p.status, kStatusTimeout);
    aborted = true;
  };

  // Anchored blocks of the range, one bit per block (known before any
  // statistics), and whether every block of the row is anchored: a row whose
  // every block is anchored needs no statistics at all -- all its blocks are
  // selected whatever the risk (reference.py:54-55) and none is represented
  // -- so every part of it skips phase A and barrier A (they all find the
  // same, from the same mask).  One pass over the row's anchor bytes, 16 per
  // thread (one round trip; from L2 after the first part's).
  int row_ok = p.anchor != nullptr && blocks_h > 0;
  const uint8_t* arow = p.anchor != nullptr ? p.anchor + static_cast<size_t>(h) * p.blocks : nullptr;
  // A 16-block group's anchored bits into this part's tile words.
  auto own_bits = [&](int b0, uint32_t bits16) {
    const int lo = max(b0, b_lo), hi = min(b0 + 16, b_hi);
    if (lo >= hi) return;
    const uint32_t span = ((hi - lo) == 32 ? ~0u : ((1u << (hi - lo)) - 1u)) << (lo - b0);
    const uint32_t mine16 = bits16 & span;
    if (mine16 != 0u) atomicOr(&anc_bits[b0 / T - t_lo], mine16 << (b0 % T));
  };
  if (arow != nullptr && (reinterpret_cast<uintptr_t>(arow) & 15u) == 0) {
    const int n16 = blocks_h >> 4;
    for (int i0 = 0; i0 < n16; i0 += 8 * blockDim.x) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * blockDim.x + threadIdx.x;
        v[u] = i < n16 ? __ldg(reinterpret_cast<const uint4*>(arow) + i) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i = i0 + u * blockDim.x + threadIdx.x;
        if (i >= n16) continue;
        const uint32_t w4[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
        uint32_t bits16 = 0u;
#pragma unroll
        for (int e = 0; e < 4; ++e) {  // one bit per nonzero byte
          uint32_t t = w4[e] | (w4[e] >> 4);
          t |= t >> 2;
          t |= t >> 1;
          t &= 0x01010101u;
          bits16 |= ((t * 0x01020408u) >> 24) << (4 * e);
        }
        row_ok &= bits16 == 0xffffu;
        own_bits(16 * i, bits16);
      }
    }
    for (int b = (n16 << 4) + threadIdx.x; b < blocks_h; b += blockDim.x) {
      const bool a = arow[b] != 0;
      row_ok &= a;
      if (a && b >= b_lo && b < b_hi) atomicOr(&anc_bits[b / T - t_lo], 1u << (b % T));
    }
  } else if (arow != nullptr) {
    for (int b = threadIdx.x; b < blocks_h; b += blockDim.x) {
      const bool a = arow[b] != 0;
      row_ok &= a;
      if (a && b >= b_lo && b < b_hi) atomicOr(&anc_bits[b / T - t_lo], 1u << (b % T));
    }
  }
  const bool row_anchored = __syncthreads_and(row_ok) != 0;
  // The anchored list (block order).
  if (warp == (W > 1 ? 1 : 0)) {
    int acc = 0;
    for (int k0 = 0; k0 < n_t; k0 += 32) {
      const int k = k0 + lane;
      const int cnt = k < n_t ? __popc(anc_bits[k]) : 0;
      int incl = cnt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      if (k < n_t) anc_off[k] = acc + incl - cnt;
      acc += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) flags[2] = acc;
  }
  __syncthreads();
  for (int k = warp; k < n_t; k += W) {
    const uint32_t ab = anc_bits[k];
    if ((ab >> lane) & 1u) blist[anc_off[k] + __popc(ab & ((1u << lane) - 1u))] = (t_lo + k) * T + lane;
  }

  // ---------------- phase A: statistics of this warp's tiles ----------------
  if (!row_anchored) {
    int lane_rows[T / 16][2];
    constexpr int kHalves = PACK4 ? 1 : 2;
#pragma unroll
    for (int mt = 0; mt < T / 16; ++mt) {
      lane_rows[mt][0] = mt * 16 + (lane >> 2) + (PACK4 && ((lane >> 1) & 1) ? 8 : 0);
      lane_rows[mt][1] = lane_rows[mt][0] + 8;
    }
    uint32_t qk[D / 16][NT][2], q2[D / 16][NT][2];
    uint32_t packed[PACK4 ? 2 * D / 16 : 1][2];
    if constexpr (PACK4) {
      uint32_t q1[D / 16][1][2];
      load_query_frags<D, 1>(q1, q, p.query_f32, p.group, p.dim, lane & 15, false);
      pack4_frags<D>(q1, packed, lane);
    } else {
      load_query_frags<D, NT>(qk, q, p.query_f32, p.group, p.dim, lane, false);
      square_frags<D, NT>(qk, q2);
    }
    float zm[NT][2], zs[NT][2], cm[NT][2], cs[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        zm[nt][j] = cm[nt][j] = -INFINITY;
        zs[nt][j] = cs[nt][j] = 0.f;
      }
    for (int k = warp; k < n_t && !aborted; k += W) {
      const int tile = t_lo + k;
      if (lane == 0) {
        fence_proxy_async();
        mbar_expect_tx(bar_a, 2 * kSel);
        tma_tile_hint<D>(slice, &maps.key_mean, bar_a, tile * T, h, T, policy);
        tma_tile_hint<D>(slice + kSel, &maps.ellipsoid, bar_a, tile * T, h, T, policy);
        if (k + W < n_t) {  // one stage per warp: warm L2 with the next tile meanwhile
          tma_prefetch_tile<D>(&maps.key_mean, (tile + W) * T, h);
          tma_prefetch_tile<D>(&maps.ellipsoid, (tile + W) * T, h);
        }
      }
      long long cnt[T / 16][2];
#pragma unroll
      for (int mt = 0; mt < T / 16; ++mt)
#pragma unroll
        for (int hf = 0; hf < kHalves; ++hf) {
          const int b = tile * T + lane_rows[mt][hf];
          cnt[mt][hf] = mine(b) ? __ldg(counts + b) : 1;
        }
      if (zd_local) {  // the decisions' value norms, while the tile lands
        const int b = tile * T + lane;
        vsm[k * T + lane] =
            mine(b) ? __ldg(p.value_norm + static_cast<size_t>(h) * p.blocks + b) : 0.f;
      }
      if (!warp_wait(bar_a, uses_a & 1)) {
        timeout();
        mbar_wait(bar_a, uses_a & 1);  // bounded: the copy must land before the CTA exits
        break;
      }
      ++uses_a;
      const uint32_t base = smem_addr(slice);
      float sc[T / 16][NT][4], pr[T / 16][NT][4];
      int row_of[T / 16][2];
      int g_base;
      if constexpr (PACK4) {
        float acc[T / 16][4];
        score_tile_pair<T, D>(base, base + kSel, packed, acc, lane);
        const bool upper = (lane >> 1) & 1;
#pragma unroll
        for (int mt = 0; mt < T / 16; ++mt) {
          const float send0 = upper ? acc[mt][0] : acc[mt][2];
          const float send1 = upper ? acc[mt][1] : acc[mt][3];
          const float recv0 = __shfl_xor_sync(0xffffffffu, send0, 2);
          const float recv1 = __shfl_xor_sync(0xffffffffu, send1, 2);
          sc[mt][0][0] = upper ? recv0 : acc[mt][0];
          sc[mt][0][1] = upper ? recv1 : acc[mt][1];
          pr[mt][0][0] = upper ? acc[mt][2] : recv0;
          pr[mt][0][1] = upper ? acc[mt][3] : recv1;
          row_of[mt][0] = mt * 16 + (lane >> 2) + (upper ? 8 : 0);
        }
        g_base = 2 * (lane & 1);
      } else {
        score_tile<T, D, NT>(base, qk, sc, lane);
        score_tile<T, D, NT>(base + kSel, q2, pr, lane);
#pragma unroll
        for (int mt = 0; mt < T / 16; ++mt) {
          row_of[mt][0] = mt * 16 + (lane >> 2);
          row_of[mt][1] = row_of[mt][0] + 8;
        }
        g_base = 0;
      }
      __syncwarp();
      float zv[T / 16][NT][4], cv[T / 16][NT][4];
#pragma unroll
      for (int mt = 0; mt < T / 16; ++mt) {
#pragma unroll
        for (int hf = 0; hf < kHalves; ++hf) {
          const int b = tile * T + row_of[mt][hf];
          const float log_count = mine(b) ? flog(static_cast<float>(cnt[mt][hf])) : 0.f;
#pragma unroll
          for (int jc = 0; jc < 2; ++jc) {
            const int c = 2 * hf + jc;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const int g = PACK4 ? g_base + jc : nt * 8 + 2 * (lane & 3) + jc;
              zv[mt][nt][c] = -INFINITY;
              cv[mt][nt][c] = -INFINITY;
              if (!mine(b) || g >= p.group) continue;
              const float score = sc[mt][nt][c] * p.scale;
              const float proj = pr[mt][nt][c];
              const float delta = (sqrtf(proj < 0.f ? 0.f : proj) * p.scale) * kInflate;
              const float z = score + log_count;
              if (zd_local) {
                const int at_ = ((tile - t_lo) * p.group + g) * T + row_of[mt][hf];
                zsm[at_] = z;
                dsm[at_] = delta;
              } else {
                const size_t rowg = static_cast<size_t>(h) * p.group + g;
                p.z[rowg * p.blocks + b] = z;
                p.delta[rowg * p.blocks + b] = delta;
              }
              zv[mt][nt][c] = z;
              cv[mt][nt][c] = z + log_cosh(delta);
            }
          }
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int jc = 0; jc < 2; ++jc) {
          float tz = -INFINITY, tc = -INFINITY;
          bool nan = false;
#pragma unroll
          for (int mt = 0; mt < T / 16; ++mt)
#pragma unroll
            for (int hf = 0; hf < kHalves; ++hf) {
              const float a = zv[mt][nt][2 * hf + jc], b = cv[mt][nt][2 * hf + jc];
              tz = fmaxf(tz, a);
              tc = fmaxf(tc, b);
              nan |= (a != a) || (b != b);
            }
          float sz = 0.f, sc2 = 0.f;
          const float rz = tz == -INFINITY ? 0.f : tz, rc = tc == -INFINITY ? 0.f : tc;
#pragma unroll
          for (int mt = 0; mt < T / 16; ++mt)
#pragma unroll
            for (int hf = 0; hf < kHalves; ++hf) {
              sz += fexp(zv[mt][nt][2 * hf + jc] - rz);
              sc2 += fexp(cv[mt][nt][2 * hf + jc] - rc);
            }
          if (nan) sz = sc2 = NAN;
          lse_merge(zm[nt][jc], zs[nt][jc], tz, sz);
          lse_merge(cm[nt][jc], cs[nt][jc], tc, sc2);
        }
    }
    // One (max, sum) pair per warp and row (empty for a warp without tiles).
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float mz = zm[nt][j], mc = cm[nt][j];
#pragma unroll
        for (int off = PACK4 ? 2 : 4; off < 32; off <<= 1) {
          mz = fmaxf(mz, __shfl_xor_sync(0xffffffffu, mz, off));
          mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, off));
        }
        const float rz = mz == -INFINITY ? 0.f : mz, rc = mc == -INFINITY ? 0.f : mc;
        float sz = zs[nt][j] == 0.f ? 0.f : zs[nt][j] * fexp(zm[nt][j] - rz);
        float sc = cs[nt][j] == 0.f ? 0.f : cs[nt][j] * fexp(cm[nt][j] - rc);
#pragma unroll
        for (int off = PACK4 ? 2 : 4; off < 32; off <<= 1) {
          sz += __shfl_xor_sync(0xffffffffu, sz, off);
          sc += __shfl_xor_sync(0xffffffffu, sc, off);
        }
        const bool writer = PACK4 ? lane < 2 : lane < 4;
        const int g = PACK4 ? 2 * lane + j : nt * 8 + 2 * lane + j;
        if (writer && g < p.group) lse_s[warp * kMaxGroup + g] = make_float4(mz, sz, mc, sc);
      }
  }
  __syncthreads();
  // One partial per part and group row, the warps' pairs merged in warp order
  // (warps without tiles hold empty pairs), by the last warp, which then
  // arrives at barrier A -- while its first page lands.
  auto publish_stats = [&]() {
    if (warp != W - 1 || row_anchored) return;
    if (lane < p.group) {
      float4 acc = lse_s[lane];
      for (int w = 1; w < W; ++w) {
        const float4 v = lse_s[w * kMaxGroup + lane];
        lse_merge(acc.x, acc.y, v.x, v.y);
        lse_merge(acc.z, acc.w, v.z, v.w);
      }
      *reinterpret_cast<float4*>(
          p.lse + ((static_cast<size_t>(h) * p.group + lane) * lse_parts + part) * 4) = acc;
    }
    __syncwarp();
    if (lane == 0) arrive(arrive_a, gen_a, parts_h);
  };

  // ---------------- attention known before the decisions -------------------
  float m[NT][2], l[NT][2], o[D / 16][NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m[nt][0] = m[nt][1] = -INFINITY;
    l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
    for (int dt = 0; dt < D / 16; ++dt) o[dt][nt][0] = o[dt][nt][1] = o[dt][nt][2] = o[dt][nt][3] = 0.f;
  }
  const bool split = p.split_probs != 0;
  uint32_t qb[D / 16][NT][2];
  load_query_frags<D, NT>(qb, q, p.query_f32, p.group, p.dim, lane, false);
  // A page of block `block`: physical page (page table), valid rows.
  auto page_item = [&](int block) {
    int page = block;
    if (p.page_table != nullptr) {
      page = __ldg(p.page_table + static_cast<size_t>(p.seq.sequence(h)) * p.page_table_stride +
                   block);
      if (page < 0 || page >= p.pool_pages) {  // flag the call; read page 0 instead
        if (lane == 0) atomicOr(p.status, kStatusBadInput);
        page = 0;
      }
    }
    return make_int4(0, page, min(R, prompt_h - block * R), pool_head);
  };
  const int n_anc = flags[2];
  const int n_suffix = (suffix_len + R - 1) / R;                          // chunks of the row
  const int my_suffix = n_suffix > part ? (n_suffix - part + parts_h - 1) / parts_h : 0;
  {
    const int n1 = n_anc + my_suffix;
    const int mine = n1 > warp ? (n1 - warp + W - 1) / W : 0;
    auto item = [&](int j) {
      const int i = warp + j * W;
      if (i < n_anc) return page_item(blist[i]);
      const int chunk = part + (i - n_anc) * parts_h;
      return make_int4(1, chunk * R, min(R, suffix_len - chunk * R), h);
    };
    if (aborted) {
      publish_stats();
    } else if (!stream_items<R, D, NT>(mine, item, publish_stats, maps, slice, bar_a, bar_b,
                                       uses_a, uses_b, qb, p.scale, split, m, l, o, policy,
                                       lane)) {
      timeout();
    }
  }

  // ---------------- phase B: row normalisers, decisions ---------------------
  // A part whose every block is anchored decides nothing: its blocks are
  // selected whatever the risk (reference.py:54-55) and it holds no
  // representatives, so it neither waits for the row's normalisers nor reads
  // its statistics back.
  const bool all_anchored = n_anc == b_hi - b_lo;
  if (all_anchored) {
    for (int k = warp; k < n_t; k += W) {
      const int b = (t_lo + k) * T + lane;
      if (mine(b)) p.mask[static_cast<size_t>(h) * p.blocks + b] = 1;
    }
  } else {
    if (threadIdx.x == 0 && !wait_generation(gen_a, seen_a)) atomicOr(p.status, kStatusTimeout);
    __syncthreads();
    for (int g = warp; g < p.group; g += W) {
      const float* in = p.lse + (static_cast<size_t>(h) * p.group + g) * lse_parts * 4;
      float m0 = -INFINITY, s0 = 0.f, m1 = -INFINITY, s1 = 0.f;
      for (int k0 = lane; k0 < parts_h; k0 += 32 * 8) {
        float4 v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int k = k0 + 32 * u;
          v[u] = k < parts_h ? __ldcg(reinterpret_cast<const float4*>(in + 4 * k))
                             : make_float4(-INFINITY, 0.f, -INFINITY, 0.f);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          lse_merge(m0, s0, v[u].x, v[u].y);
          lse_merge(m1, s1, v[u].z, v[u].w);
        }
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) {
        const float om = __shfl_xor_sync(0xffffffffu, m0, off);
        const float os = __shfl_xor_sync(0xffffffffu, s0, off);
        const float pm = __shfl_xor_sync(0xffffffffu, m1, off);
        const float ps = __shfl_xor_sync(0xffffffffu, s1, off);
        lse_merge(m0, s0, om, os);
        lse_merge(m1, s1, pm, ps);
      }
      if (lane == 0) {
        const float zl = m0 + flog(s0), cl = m1 + flog(s1);
        lz[g] = zl;
        lc[g] = cl;
        if (!finite(zl) || !finite(cl)) atomicOr(&flags[0], 1);
      }
    }
    __syncthreads();
    const bool bad_global = flags[0] != 0;
    const float vmax = __ldg(p.max_value_norm + h);
    // A lane's block of tile k needs a decision when it is this part's and not
    // anchored; its statistics come from shared memory (or the workspace when
    // they did not fit there).
    float zr[GM], dr[GM], vn = 0.f;
    auto load_stats = [&](int k, float (&zs)[GM], float (&ds)[GM], float& v) {
      const int b = (t_lo + k) * T + lane;
      const bool need = k < n_t && mine(b) && !((anc_bits[k] >> lane) & 1u);
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        const size_t row = static_cast<size_t>(h) * p.group + g;
        const bool live = need && g < p.group;
        if (zd_local) {
          zs[g] = live ? zsm[(k * p.group + g) * T + lane] : 0.f;
          ds[g] = live ? dsm[(k * p.group + g) * T + lane] : 0.f;
        } else {
          zs[g] = live ? __ldcg(p.z + row * p.blocks + b) : 0.f;
          ds[g] = live ? __ldcg(p.delta + row * p.blocks + b) : 0.f;
        }
      }
      v = !need ? 0.f
                : zd_local ? vsm[k * T + lane]
                           : __ldg(p.value_norm + static_cast<size_t>(h) * p.blocks + b);
    };
    // The representatives of a decided tile join the running softmax while the
    // warp decides its next one: its value-mean tile loads on one barrier (two
    // tiles in flight at most, one per barrier); logit z, value the block's
    // value mean.
    auto rep_logits = [&](int k, uint32_t reps, float (&lg)[T / 16][NT][4]) {
      const int tile = t_lo + k;
#pragma unroll
      for (int mt = 0; mt < T / 16; ++mt)
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const int r = mt * 16 + (lane >> 2) + (cc >> 1) * 8;
          const bool rep = (reps >> r) & 1u;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int g = nt * 8 + 2 * (lane & 3) + (cc & 1);
            if (!(rep && g < p.group)) {
              lg[mt][nt][cc] = -INFINITY;
            } else if (zd_local) {
              lg[mt][nt][cc] = zsm[(k * p.group + g) * T + r];
            } else {
              lg[mt][nt][cc] =
                  __ldcg(p.z + (static_cast<size_t>(h) * p.group + g) * p.blocks + tile * T + r);
            }
          }
        }
    };
    int pend_k = -1, pend_half = 0;
    uint32_t pend_reps = 0u;
    auto finish_pending = [&]() {
      if (pend_k < 0) return;
      uint64_t* bar = pend_half ? bar_b : bar_a;
      uint32_t& uses = pend_half ? uses_b : uses_a;
      if (!warp_wait(bar, uses & 1)) {
        timeout();
        mbar_wait(bar, uses & 1);  // bounded: the copy must land before the slice is reused
      }
      ++uses;
      if (!aborted) {
        float lg[T / 16][NT][4];
        rep_logits(pend_k, pend_reps, lg);
        attend_tile<T, D, NT>(lg, smem_addr(slice + pend_half * kSel), m, l, o, split, lane);
      }
      __syncwarp();
      pend_k = -1;
    };
    for (int k = warp; k < n_t; k += W) {
      load_stats(k, zr, dr, vn);
      const int b = (t_lo + k) * T + lane;
      const bool valid = mine(b);
      const bool anc = (anc_bits[k] >> lane) & 1u;
      bool sel = anc;
      if (valid && !anc) {
        float agg = p.reduction == kMax ? -INFINITY : 0.f;
        bool any = false, bad = false;
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          if (g >= p.group) continue;
          const float r = block_risk(zr[g], dr[g], lz[g], lc[g], vn, vmax);
          bad |= !finite(r);
          if (p.reduction == kMean) {
            agg += r;
          } else if (p.reduction == kMax) {
            agg = (r > agg || r != r) ? r : agg;
          } else {
            any |= r > p.eps;
          }
        }
        bool dec;
        if (p.reduction == kMean) {
          dec = agg / static_cast<float>(p.group) > p.eps;
        } else if (p.reduction == kMax) {
          dec = agg > p.eps;
        } else {
          dec = any;
        }
        sel = dec || bad || bad_global;
      }
      if (valid) p.mask[static_cast<size_t>(h) * p.blocks + b] = sel ? 1 : 0;
      const uint32_t listed = __ballot_sync(0xffffffffu, valid && sel && !anc);
      const uint32_t reps = __ballot_sync(0xffffffffu, valid && !sel);
      if (lane == 0) sel_bits[k] = listed;
      if (reps != 0u && !aborted) {
        const int half = pend_k >= 0 ? pend_half ^ 1 : 0;
        if (lane == 0) {
          uint64_t* bar = half ? bar_b : bar_a;
          fence_proxy_async();
          mbar_expect_tx(bar, kSel);
          tma_tile_hint<D>(slice + half * kSel, &maps.value_mean, bar, (t_lo + k) * T, h, T, policy);
        }
        finish_pending();  // the previous tile's representatives while this one lands
        pend_k = k;
        pend_reps = reps;
        pend_half = half;
      }
    }
    finish_pending();
    __syncthreads();
    // Compaction (block order): the selected blocks that are not anchored.
    if (warp == 0) {
      int acc = 0;
      for (int k0 = 0; k0 < n_t; k0 += 32) {
        const int k = k0 + lane;
        const int cnt = k < n_t ? __popc(sel_bits[k]) : 0;
        int incl = cnt;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int y = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += y;
        }
        if (k < n_t) offsets[k] = acc + incl - cnt;
        acc += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) flags[2] = acc;
    }
    __syncthreads();
    for (int k = warp; k < n_t; k += W) {
      const uint32_t sb = sel_bits[k];
      if ((sb >> lane) & 1u) blist[offsets[k] + __popc(sb & ((1u << lane) - 1u))] = (t_lo + k) * T + lane;
    }
    __syncthreads();
  }
  // A batched row's blocks past its prompt belong to no part: the last part
  // writes their mask bytes 0.
  if (part == parts_h - 1) {
    for (int b = blocks_h + threadIdx.x; b < p.blocks; b += blockDim.x) {
      p.mask[static_cast<size_t>(h) * p.blocks + b] = 0;
    }
  }

  // ---------------- selected non-anchored pages ------------------------------
  const int n_sel = all_anchored ? 0 : flags[2];
  {
    const int mine = n_sel > warp ? (n_sel - warp + W - 1) / W : 0;
    auto item = [&](int j) { return page_item(blist[warp + j * W]); };
    if (!aborted && !stream_items<R, D, NT>(mine, item, [] {}, maps, slice, bar_a, bar_b, uses_a,
                                            uses_b, qb, p.scale, split, m, l, o, policy, lane)) {
      timeout();
    }
  }

  // ---------------- this part's partial, then the row's output ---------------
  reduce_l<NT>(l);
  __syncthreads();  // every slice is idle: park the warps' partials there
  {
    float* st_m = reinterpret_cast<float*>(smem);      // [W][G8]
    float* st_l = st_m + W * G8;                       // [W][G8]
    float* st_o = st_l + W * G8;                       // [W][G8][kStashStride]
    stash_padded<D, NT>(st_m, st_l, st_o, warp, lane, m, l, o);
    __syncthreads();
    // All of a thread's outputs share one group row (the block is a multiple
    // of G8 threads): its warps' weights exp(m - max m), once.
    const int g = threadIdx.x % G8;
    float wts[8];
    float top = -INFINITY;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      if (w < W) top = fmaxf(top, st_m[w * G8 + g]);
    }
    const float ref = top == -INFINITY ? 0.f : top;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float mw = w < W ? st_m[w * G8 + g] : -INFINITY;
      wts[w] = mw == -INFINITY ? 0.f : __expf(mw - ref);
    }
    if (threadIdx.x < G8) {  // the part's max and sum per group row
      float den = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        if (w < W) den += wts[w] * st_l[w * G8 + g];
      }
      p.part_m[static_cast<size_t>(c) * G8 + g] = top;
      p.part_l[static_cast<size_t>(c) * G8 + g] = den;
    }
    float* out_o = p.part_o + static_cast<size_t>(c) * G8 * D;
    for (int idx = threadIdx.x; idx < G8 * D; idx += blockDim.x) {
      const int d = idx / G8;
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < 8; ++w) {
        if (w < W) acc += wts[w] * st_o[(w * G8 + g) * kStashStride<D> + d];
      }
      out_o[idx] = acc;  // o^T: [d][g]
    }
  }
  __syncthreads();
  // Rows of at most kLastParts parts: the part that arrives last merges the
  // whole row (no part waits for another).  Longer rows meet at barrier B and
  // every part writes its slice of the channels.
  int c0 = 0, c1 = p.dim;
  if (parts_h <= kLastParts) {
    if (threadIdx.x == 0) flags[3] = arrive(arrive_b, nullptr, parts_h) ? 1 : 0;
    __syncthreads();
    if (flags[3] == 0) return;
  } else {
    if (threadIdx.x == 0) {
      arrive(arrive_b, gen_b, parts_h);
      if (!wait_generation(gen_b, seen_b)) atomicOr(p.status, kStatusTimeout);
    }
    __syncthreads();
    c0 = p.dim * part / parts_h;
    c1 = p.dim * (part + 1) / parts_h;
  }
  // The row's output from its parts' partials: teams of tp threads per
  // (channel, 4 group rows), each thread over every tp-th part.  The first
  // pass's partial rows load first, then the parts' (max, sum) pairs are
  // staged in shared memory as weights w = exp(m - max m) and sums w * l.
  const int g4s = (p.group + 3) >> 2;
  const int items = (c1 - c0) * g4s;
  int tp = 32;
  while (tp > 1 && tp * items > static_cast<int>(blockDim.x)) tp >>= 1;
  const int teams = blockDim.x / tp, t_in = threadIdx.x % tp;
  constexpr int kAheadParts = 16;  // partial rows a thread holds while the weights are staged
  float4 ahead[kAheadParts];
  {
    const int item = threadIdx.x / tp;
    const bool ok = item < items;
    const int d = c0 + (ok ? item / g4s : 0), g0 = ok ? 4 * (item % g4s) : 0;
#pragma unroll
    for (int u = 0; u < kAheadParts; ++u) {
      const int k = u * tp + t_in;
      ahead[u] = ok && k < parts_h
                     ? __ldcg(reinterpret_cast<const float4*>(
                           p.part_o + (static_cast<size_t>(first_cta + k) * D + d) * G8 + g0))
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  // The parts' (max, sum) pairs staged in shared memory with vector loads by
  // all threads (in a long row every part reads them all: one request per 16
  // bytes keeps those few L2 lines from becoming a hot spot), then one warp
  // per group row: weights w = exp(m - max m) in place, denominator
  // sum(w * l).
  float* wgt = reinterpret_cast<float*>(smem);  // [parts_h][G8] m, then weights
  float* lsum = wgt + parts_h * G8;             // [parts_h][G8] l
  float* den = lsum + parts_h * G8;             // [G8] denominators
  {
    const int n4 = parts_h * G8 / 4;
    const float4* m4 = reinterpret_cast<const float4*>(p.part_m + static_cast<size_t>(first_cta) * G8);
    const float4* l4 = reinterpret_cast<const float4*>(p.part_l + static_cast<size_t>(first_cta) * G8);
    for (int i0 = 0; i0 < n4; i0 += 4 * blockDim.x) {
      float4 mv[4], lv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * blockDim.x + threadIdx.x;
        mv[u] = i < n4 ? __ldcg(m4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        lv[u] = i < n4 ? __ldcg(l4 + i) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * blockDim.x + threadIdx.x;
        if (i < n4) {
          reinterpret_cast<float4*>(wgt)[i] = mv[u];
          reinterpret_cast<float4*>(lsum)[i] = lv[u];
        }
      }
    }
  }
  __syncthreads();
  for (int g = warp; g < G8; g += W) {
    if (g >= p.group) {  // padding group rows: weight 0 (read by the float4 loads below)
      for (int k = lane; k < parts_h; k += 32) wgt[k * G8 + g] = 0.f;
      continue;
    }
    float mx = -INFINITY;
    for (int k = lane; k < parts_h; k += 32) mx = fmaxf(mx, wgt[k * G8 + g]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float ref = mx == -INFINITY ? 0.f : mx;
    float sum = 0.f;
    for (int k = lane; k < parts_h; k += 32) {
      const float mk = wgt[k * G8 + g];
      const float w = mk == -INFINITY ? 0.f : fexp(mk - ref);
      wgt[k * G8 + g] = w;
      sum += w == 0.f ? 0.f : w * lsum[k * G8 + g];
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) den[g] = sum;
  }
  __syncthreads();
  auto add_part = [&](float4& acc, int k, int g0, const float4& v) {
    const float4 w = *reinterpret_cast<const float4*>(wgt + k * G8 + g0);
    acc.x += w.x != 0.f ? w.x * v.x : 0.f;
    acc.y += w.y != 0.f ? w.y * v.y : 0.f;
    acc.z += w.z != 0.f ? w.z * v.z : 0.f;
    acc.w += w.w != 0.f ? w.w * v.w : 0.f;
  };
  for (int base = 0; base < items; base += teams) {  // uniform trip count: shuffles below
    const int item = base + threadIdx.x / tp;
    const bool ok = item < items;
    const int d = c0 + (ok ? item / g4s : 0), g0 = ok ? 4 * (item % g4s) : 0;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    int k_from = 0;
    if (base == 0) {  // the rows loaded ahead
#pragma unroll
      for (int u = 0; u < kAheadParts; ++u) {
        const int k = u * tp + t_in;
        if (ok && k < parts_h) add_part(acc, k, g0, ahead[u]);
      }
      k_from = kAheadParts * tp;
    }
    for (int k0 = k_from; k0 < parts_h; k0 += 8 * tp) {
      float4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int k = k0 + u * tp + t_in;
        v[u] = ok && k < parts_h
                   ? __ldcg(reinterpret_cast<const float4*>(
                         p.part_o + (static_cast<size_t>(first_cta + k) * D + d) * G8 + g0))
                   : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int k = k0 + u * tp + t_in;
        if (ok && k < parts_h) add_part(acc, k, g0, v[u]);
      }
    }
    for (int off = tp >> 1; off > 0; off >>= 1) {
      acc.x += __shfl_xor_sync(0xffffffffu, acc.x, off);
      acc.y += __shfl_xor_sync(0xffffffffu, acc.y, off);
      acc.z += __shfl_xor_sync(0xffffffffu, acc.z, off);
      acc.w += __shfl_xor_sync(0xffffffffu, acc.w, off);
    }
    if (ok && t_in == 0) {
      const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int g = g0 + j;
        if (g >= p.group) break;
        const float out = a4[j] / fmaxf(den[g], 1e-30f);
        const size_t at_ = (static_cast<size_t>(h) * p.group + g) * p.dim + d;
        if (p.query_f32) {
          static_cast<float*>(p.out)[at_] = out;
        } else {
          static_cast<__nv_bfloat16*>(p.out)[at_] = __float2bfloat16_rn(out);
        }
      }
    }
  }
}

template <int D, int R, int NT, bool PACK4, int GM>
cudaError_t launch_t(const FusedMaps& maps, const FusedParams& p, int warps, size_t smem,
                     cudaStream_t stream, bool pdl) {
  auto kernel = fused_kernel<D, R, NT, PACK4, GM>;
  cudaError_t err = ensure_smem_limit(reinterpret_cast<const void*>(kernel), smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(fused_grid(p.heads, p.parts_base, p.parts_extra));
  cfg.blockDim = dim3(warps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, maps, p);
}

template <int D, int R>
cudaError_t launch_g(const FusedMaps& maps, const FusedParams& p, int warps, size_t smem,
                     cudaStream_t stream, bool pdl) {
  if (p.group <= 4) return launch_t<D, R, 1, true, 4>(maps, p, warps, smem, stream, pdl);
  if (p.group <= 8) return launch_t<D, R, 1, false, 8>(maps, p, warps, smem, stream, pdl);
  return launch_t<D, R, 2, false, 16>(maps, p, warps, smem, stream, pdl);
}

template <int D>
cudaError_t launch_r(const FusedMaps& maps, const FusedParams& p, int warps, size_t smem,
                     cudaStream_t stream, bool pdl) {
  switch (p.page) {
    case 16: return launch_g<D, 16>(maps, p, warps, smem, stream, pdl);
    case 32: return launch_g<D, 32>(maps, p, warps, smem, stream, pdl);
    case 64: return launch_g<D, 64>(maps, p, warps, smem, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

int fused_grid(int heads, int parts_base, int parts_extra) {
  return heads * parts_base + parts_extra;
}

size_t fused_smem_bytes(int dim, int page, int warps, int tcap, int zd_group) {
  const int sel = kSelectTile * dim * 2, pg = page * dim * 2;
  const int slice = 2 * sel > 2 * pg ? 2 * sel : 2 * pg;
  return FusedLayout(warps, slice, tcap, zd_group).bytes;
}

cudaError_t launch_fused(const FusedMaps& maps, const FusedParams& p, int dim, int warps,
                         size_t smem, cudaStream_t stream, bool pdl) {
  switch (dim) {
    case 64: return launch_r<64>(maps, p, warps, smem, stream, pdl);
    case 128: return launch_r<128>(maps, p, warps, smem, stream, pdl);
    case 192: return launch_r<192>(maps, p, warps, smem, stream, pdl);
    case 256: return launch_r<256>(maps, p, warps, smem, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace rkv
