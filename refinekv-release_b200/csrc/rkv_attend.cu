// Split decode attention over refined pages and the generated suffix, and the
// LSE combine with the representative partials (reference:
// src/refinekv/reference.py:50-73; the reference's GPU form is
// kernels/attention.py:166-329).
//
// Work list.  For KV head h the items are its selected pages (in the
// deterministic block order written by the selector) followed by its suffix
// chunks of `page` tokens.  All heads' items form one list of T entries that
// is cut into C equal contiguous ranges, one per CTA, so a head that refines
// many pages is spread over many CTAs and the grid stays balanced whatever
// the per-head selection counts are.  Everything is read from device memory
// (selection counts, suffix length), so the launch is graph-safe.
//
// attend_kernel: one CTA per SM, independent warps.  Warp w of a CTA takes
// the CTA's items k = lo + w + j*warps and streams them through its own ring
// of TMA stages (K page | V page, with separate barriers so K is refilled as
// soon as the scores are done).  Per item: S^T = K . q^T (tokens on M, group
// rows on N) with mma.sync, mask rows past the item's token count, online
// softmax, probabilities -> P^T operand by movmatrix, O^T += V^T . P^T.  At
// each head boundary in its range the warp writes its own (m, l, o^T)
// partial and goes on streaming: there is no CTA barrier in the loop; the
// warps' partials for the CTA's last head are merged into one at the end.
//
// combine_kernel: per (head, 32 channels), merges the selector's
// representative partials with the attention warps' partials of that head
// and writes the output rows in the query dtype.
#include "rkv_device.cuh"
#include "rkv_kernels.h"

namespace rkv {
namespace {

// Which CTA holds global item x when T items are cut into C ranges
// (ranges are nonempty because C <= T).
struct WorkList {
  long long T;
  long long C;
  __device__ long long cta_of(long long x) const { return ((x + 1) * C + T - 1) / T - 1; }
};

// Partial slots are indexed by (head, CTA) pairs that own items.  Along the
// CTAs' contiguous ranges a CTA covers heads h_a..h_b and the next CTA starts
// at head h_b or later, so head + cta strictly increases over the owned pairs:
// it is a collision-free index below heads + ctas.
__device__ __forceinline__ size_t pair_slot(long long head, long long cta) {
  return static_cast<size_t>(head + cta);
}

__device__ __forceinline__ int visible_suffix(int has_suffix, const int* len_ptr, int len_host,
                                              int capacity, int* status) {
  if (!has_suffix) return 0;
  int len = len_ptr != nullptr ? *len_ptr : len_host;
  if (len < 0 || len > capacity) {
    if (threadIdx.x == 0) atomicOr(status, kStatusBadInput);
    len = len < 0 ? 0 : capacity;
  }
  return len;
}

// seg_pre[h][0..PB] = prefix sums of the selected-page counts over the
// selector segments of head h; hstart[0..H] = first global item of each
// head.  Called by every thread of the CTA.  Dense decode (`dense_blocks`
// non-null): one segment per row holding all of its blocks (PB must be 1).
__device__ __forceinline__ void build_work_list(const int* seg_count, int H, int PB, int n_suffix,
                                                int* seg_pre, long long* hstart,
                                                const SeqLayout* dense_blocks = nullptr,
                                                int blocks = 0) {
  if (dense_blocks != nullptr) {
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
      seg_pre[2 * h] = 0;
      seg_pre[2 * h + 1] = dense_blocks->blocks(h, blocks);
    }
  } else {
    for (int i = threadIdx.x; i < H * PB; i += blockDim.x) {
      seg_pre[(i / PB) * (PB + 1) + (i % PB) + 1] = __ldcg(seg_count + i);
    }
    __syncthreads();
    for (int h = threadIdx.x; h < H; h += blockDim.x) {
      int* pre = seg_pre + h * (PB + 1);
      pre[0] = 0;
      for (int k = 1; k <= PB; ++k) pre[k] += pre[k - 1];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    long long acc = 0;
    hstart[0] = 0;
    for (int h = 0; h < H; ++h) {
      acc += seg_pre[h * (PB + 1) + PB] + n_suffix;
      hstart[h + 1] = acc;
    }
  }
  __syncthreads();
}

template <int R, int D, int NT>
__global__ void __launch_bounds__(256, 1) attend_kernel(const __grid_constant__ AttendMaps maps,
                                                        const AttendParams p) {
  constexpr int kTile = R * D * 2;
  constexpr int kStage = 2 * kTile;
  constexpr int G8 = NT * 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  const int H = p.heads, PB = p.parts_b;
  size_t off = 0;
  uint8_t* ring = smem;  // [warp][stage][K | V]
  off += static_cast<size_t>(warps) * S * kStage;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + off);  // [warp][stage][K, V]
  off += round16(static_cast<size_t>(warps) * S * 16);
  int* valid_rows = reinterpret_cast<int*>(smem + off);  // [warp][stage]
  off += round16(static_cast<size_t>(warps) * S * 4);
  long long* hstart = reinterpret_cast<long long*>(smem + off);  // [H + 1]
  off += round16(static_cast<size_t>(H + 1) * 8);
  int* seg_pre = reinterpret_cast<int*>(smem + off);  // [H][PB + 1]

  if (lane == 0) {
    for (int s = 0; s < 2 * S; ++s) mbar_init(&bars[warp * 2 * S + s], 1);
    mbar_fence_init();
  }
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&maps.key_pages);
    tma_prefetch_desc(&maps.value_pages);
    if (p.has_suffix) {
      tma_prefetch_desc(&maps.key_suffix);
      tma_prefetch_desc(&maps.value_suffix);
    }
    if (p.suffix_len_ptr != nullptr) prefetch_l2(p.suffix_len_ptr);
  }
  // The query lines (all heads', spread over the CTAs) go to L2 before the
  // dependency wait; a prefetch returns no data, so a query the previous
  // kernel is still writing is read correctly after the wait.
  {
    const int q_lines = (H * p.group * p.dim * (p.query_f32 ? 4 : 2) + 127) / 128;
    for (int i = blockIdx.x + threadIdx.x * gridDim.x; i < q_lines; i += blockDim.x * gridDim.x) {
      prefetch_l2(static_cast<const char*>(p.query) + static_cast<size_t>(i) * 128);
    }
  }
  pdl_wait();
  pdl_launch_dependents();
  // K/V pages are read once per step: evict them first so that the selector's
  // outputs and the partials the combine reads stay in L2.
  const uint64_t stream_policy = l2_evict_first_policy();

  const int suffix_len = visible_suffix(p.has_suffix, p.suffix_len_ptr, p.suffix_len_host,
                                        p.suffix_capacity, p.status);
  build_work_list(p.seg_count, H, PB, (suffix_len + R - 1) / R, seg_pre, hstart,
                  p.dense ? &p.seq : nullptr, p.blocks);
  WorkList wl;
  wl.T = hstart[H];
  wl.C = wl.T < p.ctas ? wl.T : p.ctas;
  const long long cta = blockIdx.x;
  if (cta >= wl.C) return;  // no items: this CTA owns no partial
  const long long lo = wl.T * cta / wl.C, hi = wl.T * (cta + 1) / wl.C;
  const int count_w = hi - lo > warp ? static_cast<int>((hi - lo - warp + warps - 1) / warps) : 0;

  // Item descriptors {head, physical page or first suffix row, valid rows,
  // is_suffix} are decoded 32 at a time, one per lane, one batch ahead of
  // use, so the loads of the selected ids are off the issue path.  Each
  // lane's head cursor only moves forward because batches are decoded in
  // order.
  int lane_head = 0;
  auto decode = [&](int base) {
    const int j = base + lane;
    int4 d = make_int4(0, 0, 0, 0);
    if (j >= count_w) return d;
    const long long k = lo + warp + static_cast<long long>(j) * warps;
    while (hstart[lane_head + 1] <= k) ++lane_head;
    const int h = lane_head;
    const int pos = static_cast<int>(k - hstart[h]);
    const int* pre = seg_pre + h * (PB + 1);
    if (pos < pre[PB]) {
      int a = 0, b = PB;  // segment with pre[a] <= pos < pre[a + 1]
      while (b - a > 1) {
        const int mid = (a + b) >> 1;
        if (pre[mid] <= pos) a = mid; else b = mid;
      }
      const int block = p.dense ? pos
                                : __ldg(p.sel_ids + (static_cast<size_t>(h) * PB + a) * p.seg_cap +
                                        (pos - pre[a]));
      int page = block;  // physical page: the page table's entry when paged
      if (p.page_table != nullptr) {
        page = __ldg(p.page_table + static_cast<size_t>(p.seq.sequence(h)) * p.page_table_stride +
                     block);
        if (page < 0 || page >= p.pool_pages) {  // flag the call; read page 0 instead
          atomicOr(p.status, kStatusBadInput);
          page = 0;
        }
      }
      d = make_int4(h, page, min(R, p.seq.prompt(h, p.prompt_length) - block * R), 0);
    } else {
      const int c = pos - pre[PB];
      d = make_int4(h, c * R, min(R, suffix_len - c * R), 1);
    }
    return d;
  };
  int batch_base = 0;
  int4 cur = decode(0);
  int4 nxt = decode(32);
  auto item = [&](int j) {  // whole warp; j advances by one per call
    if (j >= batch_base + 32) {
      batch_base += 32;
      cur = nxt;
      nxt = decode(batch_base + 32);
    }
    const int src = j - batch_base;
    return make_int4(__shfl_sync(0xffffffffu, cur.x, src), __shfl_sync(0xffffffffu, cur.y, src),
                     __shfl_sync(0xffffffffu, cur.z, src), __shfl_sync(0xffffffffu, cur.w, src));
  };
  // Head coordinate of row h in the page maps: a page pool holds each
  // sequence's KV heads, contiguous or batched pages hold every row.
  auto pool_head = [&](int h) {
    return p.page_table != nullptr ? h - p.seq.sequence(h) * p.seq.heads_per_seq : h;
  };
  // K and V of a stage have their own barriers: K is refilled as soon as the
  // scores are computed, V after the value product.
  auto issue_k = [&](int j, const int4& d) {
    if (lane == 0) {
      const int s = j % S;
      valid_rows[warp * S + s] = d.z;
      uint64_t* bk = &bars[(warp * S + s) * 2];
      mbar_expect_tx(bk, kTile);
      if (d.w) {
        tma_tile_hint<D>(ring + (warp * S + s) * kStage, &maps.key_suffix, bk, d.y, d.x, R,
                         stream_policy);
      } else {
        tma_page_hint<D>(ring + (warp * S + s) * kStage, &maps.key_pages, bk, pool_head(d.x), d.y,
                         R, stream_policy);
      }
    }
  };
  auto issue_v = [&](int j, const int4& d) {
    if (lane == 0) {
      const int s = j % S;
      uint64_t* bv = &bars[(warp * S + s) * 2 + 1];
      mbar_expect_tx(bv, kTile);
      if (d.w) {
        tma_tile_hint<D>(ring + (warp * S + s) * kStage + kTile, &maps.value_suffix, bv, d.y,
                         d.x, R, stream_policy);
      } else {
        tma_page_hint<D>(ring + (warp * S + s) * kStage + kTile, &maps.value_pages, bv,
                         pool_head(d.x), d.y, R, stream_policy);
      }
    }
  };
  const int first_fill = min(S, count_w);
  for (int j = 0; j < first_fill; ++j) {
    const int4 d = item(j);
    issue_k(j, d);
    issue_v(j, d);
  }
  int issued_k = first_fill, issued_v = first_fill;

  bool aborted = false;
  int jj = 0;  // next local item to consume
  int last_head = -1;
  int h = 0;
  while (hstart[h + 1] <= lo) ++h;
  for (; h < H && hstart[h] < hi; ++h) {
    if (hstart[h + 1] == hstart[h]) continue;
    const long long seg_hi = hi < hstart[h + 1] ? hi : hstart[h + 1];
    const int j_end =
        seg_hi - lo > warp ? static_cast<int>((seg_hi - lo - warp + warps - 1) / warps) : 0;
    uint32_t qb[D / 16][NT][2];
    load_query_frags<D, NT>(
        qb,
        static_cast<const char*>(p.query) +
            static_cast<size_t>(h) * p.group * p.dim * (p.query_f32 ? 4 : 2),
        p.query_f32, p.group, p.dim, lane, false);
    float m[NT][2], l[NT][2], o[D / 16][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = -INFINITY;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt)
        o[dt][nt][0] = o[dt][nt][1] = o[dt][nt][2] = o[dt][nt][3] = 0.f;
    }
    for (; jj < j_end; ++jj) {
      if (aborted) continue;
      const int s = jj % S;
      const uint32_t par = (jj / S) & 1;
      uint64_t* bk = &bars[(warp * S + s) * 2];
      if (!warp_wait(bk, par)) {
        if (lane == 0) atomicOr(p.status, kStatusTimeout);
        drain_pending(bars + warp * S * 2, S, jj, issued_k, issued_v);
        aborted = true;
        continue;
      }
      const int valid = valid_rows[warp * S + s];
      const uint32_t base = smem_addr(ring + (warp * S + s) * kStage);
      float logit[R / 16][NT][4];
      score_tile<R, D, NT>(base, qb, logit, lane);
#pragma unroll
      for (int mt = 0; mt < R / 16; ++mt)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int r = mt * 16 + (lane >> 2) + (c >> 1) * 8;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            logit[mt][nt][c] = r < valid ? logit[mt][nt][c] * p.scale : -INFINITY;
        }
      __syncwarp();
      const bool refill = jj + S < count_w;
      int4 next = make_int4(0, 0, 0, 0);
      if (refill) {
        next = item(jj + S);
        if (lane == 0) fence_proxy_async();
        issue_k(jj + S, next);
        ++issued_k;
      }
      softmax_update<R, D, NT>(logit, m, l, o);
      uint32_t hi_frag[R / 16][NT][2], lo_frag[R / 16][NT][2];
      prob_frags<R, NT>(logit, hi_frag, lo_frag, p.query_f32 != 0);
      if (!warp_wait(bk + 1, par)) {
        if (lane == 0) atomicOr(p.status, kStatusTimeout);
        drain_pending(bars + warp * S * 2, S, jj, issued_k, issued_v);
        aborted = true;
        continue;
      }
      accumulate_values<R, D, NT>(base + kTile, hi_frag, o, lane);
      if (p.query_f32) accumulate_values<R, D, NT>(base + kTile, lo_frag, o, lane);
      __syncwarp();
      if (refill) {
        if (lane == 0) fence_proxy_async();
        issue_v(jj + S, next);
        ++issued_v;
      }
    }
    // This warp's partial for head h (empty, m = -inf, if it had no item).
    reduce_l<NT>(l);
    if (hstart[h + 1] >= hi) {
      // The CTA's last head: park the partial in this warp's own (now idle)
      // ring stage; the warps are merged into one partial after the loop.
      float* st = reinterpret_cast<float*>(ring + static_cast<size_t>(warp) * S * kStage);
      stash_warp_partial<D, NT>(st, st + G8, st + 2 * G8, 0, lane, m, l, o);
      last_head = h;
      continue;
    }
    const size_t slot = pair_slot(h, cta) * warps + warp;
    float* op = p.att_o + slot * D * G8;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int g0 = nt * 8 + 2 * (lane & 3);
      if (lane < 4) {
        *reinterpret_cast<float2*>(p.att_m + slot * G8 + g0) = make_float2(m[nt][0], m[nt][1]);
        *reinterpret_cast<float2*>(p.att_l + slot * G8 + g0) = make_float2(l[nt][0], l[nt][1]);
      }
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        const int d0 = dt * 16 + (lane >> 2);
        *reinterpret_cast<float2*>(op + d0 * G8 + g0) = make_float2(o[dt][nt][0], o[dt][nt][1]);
        *reinterpret_cast<float2*>(op + (d0 + 8) * G8 + g0) =
            make_float2(o[dt][nt][2], o[dt][nt][3]);
      }
    }
  }
  // One partial for the last head of this CTA's range, slot (head, cta, 0):
  // merge the warps' parked partials.
  __syncthreads();
  if (last_head >= 0) {
    const size_t slot = pair_slot(last_head, cta) * warps;
    auto stash = [&](int w) {
      return reinterpret_cast<const float*>(ring + static_cast<size_t>(w) * S * kStage);
    };
    for (int idx = threadIdx.x; idx < G8 * D; idx += blockDim.x) {
      const int d = idx / G8, g = idx - d * G8;
      float top = -INFINITY;
      for (int w = 0; w < warps; ++w) top = fmaxf(top, stash(w)[g]);
      const float ref = top == -INFINITY ? 0.f : top;
      float acc = 0.f, den = 0.f;
      for (int w = 0; w < warps; ++w) {
        const float* st = stash(w);
        const float mw = st[g];
        const float sc = mw == -INFINITY ? 0.f : __expf(mw - ref);
        acc += sc * st[2 * G8 + g * D + d];
        den += sc * st[G8 + g];
      }
      p.att_o[slot * D * G8 + d * G8 + g] = acc;
      if (d == 0) {
        p.att_m[slot * G8 + g] = top;
        p.att_l[slot * G8 + g] = den;
      }
    }
  }
}

// Shared-memory layout of combine_kernel (also sized by the host).
struct CombineLayout {
  size_t hstart, seg_pre, stats, wgt, lsum, red, bytes;
  __host__ __device__ CombineLayout(int H, int PB, int G8, int max_sources) {
    size_t off = 0;
    hstart = off;
    off += round16(static_cast<size_t>(H + 1) * 8);
    seg_pre = off;
    off += round16(static_cast<size_t>(H) * (PB + 1) * 4);
    stats = off;
    off += round16(static_cast<size_t>(2) * G8 * 4);
    wgt = off;
    off += round16(static_cast<size_t>(max_sources) * G8 * 4);
    lsum = off;
    off += round16(static_cast<size_t>(max_sources) * G8 * 4);
    red = off;
    off += static_cast<size_t>(8) * 32 * G8 * 4;
    bytes = off + kSmemSlack;
  }
};

// grid (heads, dim / 32), 8 warps; lane = output channel.  After the work
// list (one round of loads), every load of the combine is issued at once:
// the m and l of every partial of the head (staged in shared memory and
// turned into weights exp(m - M_g)) and this warp's o^T rows (every 8th
// partial, kBatch per round, kept in registers).  The warps' sums are then
// added in shared memory.
// QN: the 16-byte pieces of each (source, channel) o^T row that hold real
// group rows (ceil(group / 4)); only those are loaded.
template <int D, int G8, int QN>
__global__ void __launch_bounds__(256) combine_kernel(const CombineParams p) {
  constexpr int kWarps = 8;
  constexpr int kBatch = 24 / QN;  // sources per warp and round (24 float4 in flight)
  constexpr int kStage = 4;  // m/l entries staged per thread per round
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x, d = blockIdx.y * 32 + lane;
  const int H = p.heads, PB = p.parts_b;
  const int n_rep = p.dense ? 0 : PB;  // representative sources (none in dense decode)
  const CombineLayout lay(H, PB, G8, p.max_sources);
  long long* hstart = reinterpret_cast<long long*>(smem + lay.hstart);
  int* seg_pre = reinterpret_cast<int*>(smem + lay.seg_pre);
  float* top = reinterpret_cast<float*>(smem + lay.stats);  // [G8] row maxima
  float* den = top + G8;                                    // [G8] denominators
  float* wgt = reinterpret_cast<float*>(smem + lay.wgt);    // [sources][G8]
  float* lsum = reinterpret_cast<float*>(smem + lay.lsum);  // [sources][G8]
  float* red = reinterpret_cast<float*>(smem + lay.red);    // [warps][32][G8]

  // Everything but the attention partials was complete before the attention
  // kernel passed its own dependency wait (the suffix length, the selector's
  // page counts and representative partials), and this grid launches only
  // after every attention CTA has passed it: the work list and the
  // representative rows are read before this grid's wait, off the critical
  // path behind the attention kernel.
  const int suffix_len = visible_suffix(p.has_suffix, p.suffix_len_ptr, p.suffix_len_host,
                                        p.suffix_capacity, p.status);
  build_work_list(p.seg_count, H, PB, (suffix_len + p.page - 1) / p.page, seg_pre, hstart,
                  p.dense ? &p.seq : nullptr, p.blocks);
  WorkList wl;
  wl.T = hstart[H];
  wl.C = wl.T < p.ctas ? wl.T : p.ctas;
  // Attention partials of head h: CTAs [first, last] of its items.  A CTA
  // whose range ends inside head h merged its warps into slot warp 0; only
  // the last of them can run on into the next head and then left one
  // partial per warp.
  int n_att = 0, n_merged = 0;
  long long first = 0;
  if (hstart[h + 1] > hstart[h]) {
    first = wl.cta_of(hstart[h]);
    const long long last = wl.cta_of(hstart[h + 1] - 1);
    const long long last_hi = wl.T * (last + 1) / wl.C;
    n_merged = static_cast<int>(last - first);
    n_att = n_merged + (last_hi > hstart[h + 1] ? p.warps : 1);
  }
  const int nsrc = n_rep + n_att;
  if (nsrc > p.max_sources) {  // cannot happen with the host's plan; never read past the table
    if (threadIdx.x == 0) atomicOr(p.status, kStatusBadInput);
    pdl_wait();
    pdl_launch_dependents();
    return;
  }
  auto src_index = [&](int k) -> size_t {
    if (k < n_rep) return static_cast<size_t>(h) * PB + k;
    const int a = k - n_rep;  // merged CTAs first, then the last CTA's slots
    const long long c = first + (a < n_merged ? a : n_merged);
    const int w = a < n_merged ? 0 : a - n_merged;
    return pair_slot(h, c) * p.warps + w;
  };
  auto o_row = [&](int k) {
    return reinterpret_cast<const float4*>((k < n_rep ? p.rep_o : p.att_o) + src_index(k) * D * G8 +
                                           d * G8);
  };
  // This warp's first round of o rows: sources [k_lo, k_hi) of it (the
  // representative rows before the wait, the attention rows after it).
  float4 v[kBatch][QN];
  auto load_round = [&](int k0, int k_lo, int k_hi) {
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int k = k0 + u * kWarps;
#pragma unroll
      for (int q = 0; q < QN; ++q) {
        if (k >= k_lo && k < k_hi) v[u][q] = __ldcg(o_row(k) + q);
        else if (k_lo == 0) v[u][q] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  };
  // m and l of sources [k_lo, k_hi), loaded kStage at a time per thread.
  auto stage_ml = [&](int k_lo, int k_hi) {
    for (int i0 = k_lo * G8 + threadIdx.x; i0 < k_hi * G8; i0 += blockDim.x * kStage) {
      float mv[kStage], lv[kStage];
#pragma unroll
      for (int u = 0; u < kStage; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < k_hi * G8) {
          const int k = i / G8, g = i - k * G8;
          const size_t at = src_index(k) * G8 + g;
          mv[u] = __ldcg((k < n_rep ? p.rep_m : p.att_m) + at);
          lv[u] = __ldcg((k < n_rep ? p.rep_l : p.att_l) + at);
        }
      }
#pragma unroll
      for (int u = 0; u < kStage; ++u) {
        const int i = i0 + u * blockDim.x;
        if (i < k_hi * G8) {
          wgt[i] = mv[u];
          lsum[i] = lv[u];
        }
      }
    }
  };
  load_round(warp, 0, n_rep);
  stage_ml(0, n_rep);
  pdl_wait();
  pdl_launch_dependents();
  load_round(warp, n_rep, nsrc);
  stage_ml(n_rep, nsrc);
  __syncthreads();
  for (int g = warp; g < G8; g += kWarps) {
    float mx = -INFINITY;
    for (int k = lane; k < nsrc; k += 32) mx = fmaxf(mx, wgt[k * G8 + g]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) top[g] = mx == -INFINITY ? 0.f : mx;
  }
  __syncthreads();
  // Weights; an empty partial (m = -inf) gets weight 0 and contributes nothing.
  for (int i = threadIdx.x; i < nsrc * G8; i += blockDim.x) {
    const float m = wgt[i];
    const float w = m == -INFINITY ? 0.f : __expf(m - top[i % G8]);
    wgt[i] = w;
    lsum[i] = w == 0.f ? 0.f : lsum[i] * w;
  }
  __syncthreads();
  for (int g = warp; g < G8; g += kWarps) {
    float s = 0.f;
    for (int k = lane; k < nsrc; k += 32) s += lsum[k * G8 + g];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) den[g] = s;
  }
  float acc[G8];
#pragma unroll
  for (int g = 0; g < G8; ++g) acc[g] = 0.f;
  for (int k0 = warp;; k0 += kBatch * kWarps) {
#pragma unroll
    for (int u = 0; u < kBatch; ++u) {
      const int k = k0 + u * kWarps;
      if (k >= nsrc) continue;
#pragma unroll
      for (int q = 0; q < QN; ++q) {
        const float* w = wgt + k * G8 + 4 * q;
        // An unused slot may hold a stale value: weight 0 must not multiply it.
        if (w[0] != 0.f) acc[4 * q + 0] += w[0] * v[u][q].x;
        if (w[1] != 0.f) acc[4 * q + 1] += w[1] * v[u][q].y;
        if (w[2] != 0.f) acc[4 * q + 2] += w[2] * v[u][q].z;
        if (w[3] != 0.f) acc[4 * q + 3] += w[3] * v[u][q].w;
      }
    }
    if (k0 + kBatch * kWarps >= nsrc) break;
    load_round(k0 + kBatch * kWarps, 0, nsrc);
  }
#pragma unroll
  for (int g = 0; g < G8; ++g) red[(warp * 32 + lane) * G8 + g] = acc[g];
  __syncthreads();
  for (int i = threadIdx.x; i < 32 * G8; i += blockDim.x) {
    const int ln = i / G8, g = i - ln * G8;
    if (g >= p.group) continue;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[(w * 32 + ln) * G8 + g];
    const float out = s / fmaxf(den[g], 1e-30f);
    const size_t row = static_cast<size_t>(h) * p.group + g;
    const size_t o = row * p.dim + blockIdx.y * 32 + ln;
    if (p.part_o != nullptr) {  // sequence split: this rank's row partial
      p.part_o[o] = out;
      if (blockIdx.y == 0 && ln == 0) {
        p.part_ml[row * 2] = top[g];
        p.part_ml[row * 2 + 1] = den[g];
      }
    } else if (p.query_f32) {
      static_cast<float*>(p.out)[o] = out;
    } else {
      static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(out);
    }
  }
}

// Sequence split: out[row, d] = sum_r w_r o_r[row, d] / sum_r w_r with
// w_r = l_r exp(m_r - max_r m_r) over the ranks whose row is non-empty.
// One CTA per KV head, one thread per (group row, dim) element.
__global__ void __launch_bounds__(256) merge_kernel(const MergeParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const int h = blockIdx.x;
  const int dim = p.dim;
  for (int i = threadIdx.x; i < p.group * dim; i += blockDim.x) {
    const int g = i / dim, d = i - g * dim;
    const size_t row = static_cast<size_t>(h) * p.group + g;
    float top = -INFINITY;
    for (int r = 0; r < p.ranks; ++r) {
      const float* ml = p.part_ml + r * p.slab_floats + row * 2;
      if (ml[1] > 0.f) top = fmaxf(top, ml[0]);
    }
    float num = 0.f, den = 0.f;
    for (int r = 0; r < p.ranks; ++r) {
      const float* ml = p.part_ml + r * p.slab_floats + row * 2;
      if (!(ml[1] > 0.f)) continue;
      const float w = ml[1] * __expf(ml[0] - top);
      den += w;
      num += w * p.part_o[r * p.slab_floats + row * dim + d];
    }
    const float out = num / fmaxf(den, 1e-30f);
    if (p.query_f32) {
      static_cast<float*>(p.out)[row * dim + d] = out;
    } else {
      static_cast<__nv_bfloat16*>(p.out)[row * dim + d] = __float2bfloat16_rn(out);
    }
  }
}

cudaError_t launch_pdl(const void* kernel, dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, bool pdl, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

template <int R, int D, int NT>
cudaError_t launch_attend_t(const AttendMaps& maps, const AttendParams& p, int warps, size_t smem,
                            cudaStream_t stream, bool pdl) {
  const void* kernel = reinterpret_cast<const void*>(attend_kernel<R, D, NT>);
  cudaError_t err = ensure_smem_limit(kernel, smem);
  if (err != cudaSuccess) return err;
  void* args[] = {const_cast<AttendMaps*>(&maps), const_cast<AttendParams*>(&p)};
  return launch_pdl(kernel, dim3(p.ctas), dim3(warps * 32), smem, stream, pdl, args);
}

template <int R, int D>
cudaError_t attend_nt(const AttendMaps& maps, const AttendParams& p, int warps, size_t smem,
                      cudaStream_t stream, bool pdl) {
  if (p.group <= 8) return launch_attend_t<R, D, 1>(maps, p, warps, smem, stream, pdl);
  return launch_attend_t<R, D, 2>(maps, p, warps, smem, stream, pdl);
}

template <int R>
cudaError_t attend_dim(const AttendMaps& maps, const AttendParams& p, int dim, int warps,
                       size_t smem, cudaStream_t stream, bool pdl) {
  switch (dim) {
    case 64: return attend_nt<R, 64>(maps, p, warps, smem, stream, pdl);
    case 128: return attend_nt<R, 128>(maps, p, warps, smem, stream, pdl);
    case 192: return attend_nt<R, 192>(maps, p, warps, smem, stream, pdl);
    case 256: return attend_nt<R, 256>(maps, p, warps, smem, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <int D, int G8, int QN>
cudaError_t launch_combine_t(const CombineParams& p, cudaStream_t stream, bool pdl) {
  const void* kernel = reinterpret_cast<const void*>(combine_kernel<D, G8, QN>);
  const size_t smem = CombineLayout(p.heads, p.parts_b, G8, p.max_sources).bytes;
  cudaError_t err = ensure_smem_limit(kernel, smem);
  if (err != cudaSuccess) return err;
  void* args[] = {const_cast<CombineParams*>(&p)};
  return launch_pdl(kernel, dim3(p.heads, p.dim / 32), dim3(256), smem, stream, pdl, args);
}

template <int D>
cudaError_t combine_g(const CombineParams& p, cudaStream_t stream, bool pdl) {
  switch ((p.group + 3) / 4) {
    case 1: return launch_combine_t<D, 8, 1>(p, stream, pdl);
    case 2: return launch_combine_t<D, 8, 2>(p, stream, pdl);
    case 3: return launch_combine_t<D, 16, 3>(p, stream, pdl);
    default: return launch_combine_t<D, 16, 4>(p, stream, pdl);
  }
}


}  // namespace

size_t attend_smem_bytes(int dim, int page, int warps, int stages, int group, int heads,
                         int parts_b) {
  (void)group;
  size_t bytes = kSmemSlack;
  bytes += static_cast<size_t>(warps) * stages * 2 * page * dim * 2;  // TMA ring
  bytes += round16(static_cast<size_t>(warps) * stages * 16);          // K and V barriers
  bytes += round16(static_cast<size_t>(warps) * stages * 4);           // valid rows
  bytes += round16(static_cast<size_t>(heads + 1) * 8);
  bytes += round16(static_cast<size_t>(heads) * (parts_b + 1) * 4);
  return bytes;
}

size_t combine_smem_bytes(int heads, int parts_b, int group, int max_sources) {
  return CombineLayout(heads, parts_b, group <= 8 ? 8 : 16, max_sources).bytes;
}

cudaError_t launch_attend(const AttendMaps& maps, const AttendParams& p, int dim, int warps,
                          size_t smem, cudaStream_t stream, bool pdl) {
  switch (p.page) {
    case 16: return attend_dim<16>(maps, p, dim, warps, smem, stream, pdl);
    case 32: return attend_dim<32>(maps, p, dim, warps, smem, stream, pdl);
    case 64: return attend_dim<64>(maps, p, dim, warps, smem, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_combine(const CombineParams& p, int dim, cudaStream_t stream, bool pdl) {
  switch (dim) {
    case 64: return combine_g<64>(p, stream, pdl);
    case 128: return combine_g<128>(p, stream, pdl);
    case 192: return combine_g<192>(p, stream, pdl);
    case 256: return combine_g<256>(p, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_merge(const MergeParams& p, int dim, cudaStream_t stream, bool pdl) {
  (void)dim;  // the merge works on the real width in p.dim
  void* args[] = {const_cast<MergeParams*>(&p)};
  return launch_pdl(reinterpret_cast<const void*>(merge_kernel), dim3(p.heads), dim3(256), 0,
                    stream, pdl, args);
}

}  // namespace rkv
