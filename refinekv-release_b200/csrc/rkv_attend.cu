// Split decode attention over refined pages and the generated suffix, plus
// the LSE combine with the representative partials (reference:
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
// Per CTA: 4 warps, each streaming its own items (k = lo + warp + j*4)
// through a private ring of TMA stages [K page | V page].  For an item the
// warp computes S^T = K . q^T (tokens on M, group rows on N) with mma.sync,
// masks rows past the page's token count, updates its online softmax, turns
// the probabilities into the P^T operand with movmatrix and accumulates
// O^T += V^T . P^T.  At each head boundary inside its range the CTA merges
// its warps and writes one (m, l, o) partial.  The CTA that completes a head
// last (atomic ticket) merges that head's partials with the selector's
// representative partials and writes the output row in the query dtype.
#include "rkv_device.cuh"
#include "rkv_kernels.h"

namespace rkv {
namespace {

template <int R, int D, int NT>
__global__ void __launch_bounds__(128, 1) attend_kernel(const __grid_constant__ AttendMaps maps,
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
  off += round16(static_cast<size_t>(H) * (PB + 1) * 4);
  int* flags = reinterpret_cast<int*>(smem + off);  // [4]
  off += 16;
  int* pending = reinterpret_cast<int*>(smem + off);  // [H][3] heads this CTA combines
  off += round16(static_cast<size_t>(H) * 12);
  float* st_m = reinterpret_cast<float*>(smem + off);  // [warps][G8]
  float* st_l = st_m + warps * G8;
  float* st_o = st_l + warps * G8;  // [warps][G8][D]

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
  }
  pdl_wait();

  int suffix_len = 0;
  if (p.has_suffix) {
    suffix_len = p.suffix_len_ptr != nullptr ? *p.suffix_len_ptr : p.suffix_len_host;
    if (suffix_len < 0 || suffix_len > p.suffix_capacity) {
      if (threadIdx.x == 0) atomicOr(p.status, kStatusBadInput);
      suffix_len = suffix_len < 0 ? 0 : p.suffix_capacity;
    }
  }
  const int n_suffix = (suffix_len + R - 1) / R;

  // Selected-page counts of every (head, selector segment), loaded in
  // parallel, then prefix sums per head.
  for (int i = threadIdx.x; i < H * PB; i += blockDim.x) {
    seg_pre[(i / PB) * (PB + 1) + (i % PB) + 1] = __ldcg(p.seg_count + i);
  }
  __syncthreads();
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    int* pre = seg_pre + h * (PB + 1);
    pre[0] = 0;
    for (int k = 1; k <= PB; ++k) pre[k] += pre[k - 1];
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

  const long long T = hstart[H];
  const long long C = T < p.ctas ? T : p.ctas;  // CTAs that own a nonempty range
  const long long cta = blockIdx.x;
  long long lo = 0, hi = 0;
  if (cta < C) {
    lo = T * cta / C;
    hi = T * (cta + 1) / C;
  }
  // CTA whose range holds global item x (ranges are nonempty when C <= T).
  auto cta_of = [&](long long x) { return ((x + 1) * C + T - 1) / T - 1; };

  const int count_w = hi - lo > warp ? static_cast<int>((hi - lo - warp + warps - 1) / warps) : 0;

  // Item descriptors {head, first row, valid rows, is_suffix} are decoded 32
  // at a time, one per lane, one batch ahead of use, so the loads of the
  // selected ids and counts are off the issue path.  Each lane's head
  // cursor only moves forward because batches are decoded in order.
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
      const int block = __ldg(p.sel_ids + (static_cast<size_t>(h) * PB + a) * p.seg_cap +
                              (pos - pre[a]));
      d = make_int4(h, block * R, min(R, p.prompt_length - block * R), 0);
    } else {
      const int c = pos - pre[PB];
      d = make_int4(h, c * R, min(R, suffix_len - c * R), 1);
    }
    return d;
  };
  int batch_base = 0;
  int4 cur = decode(0);
  int4 nxt = decode(32);
  auto item = [&](int j) {  // whole warp; j never skips ahead of the batch
    if (j >= batch_base + 32) {
      batch_base += 32;
      cur = nxt;
      nxt = decode(batch_base + 32);
    }
    const int src = j - batch_base;
    return make_int4(__shfl_sync(0xffffffffu, cur.x, src), __shfl_sync(0xffffffffu, cur.y, src),
                     __shfl_sync(0xffffffffu, cur.z, src), __shfl_sync(0xffffffffu, cur.w, src));
  };
  // K and V of a stage have their own barriers: K is refilled as soon as the
  // scores are computed, V after the value product.
  auto issue_k = [&](int j, const int4& d) {
    if (lane == 0) {
      const int s = j % S;
      valid_rows[warp * S + s] = d.z;
      uint64_t* bk = &bars[(warp * S + s) * 2];
      mbar_expect_tx(bk, kTile);
      tma_tile<D>(ring + (warp * S + s) * kStage, d.w ? &maps.key_suffix : &maps.key_pages, bk,
                  d.y, d.x, R);
    }
  };
  auto issue_v = [&](int j, const int4& d) {
    if (lane == 0) {
      const int s = j % S;
      uint64_t* bv = &bars[(warp * S + s) * 2 + 1];
      mbar_expect_tx(bv, kTile);
      tma_tile<D>(ring + (warp * S + s) * kStage + kTile,
                  d.w ? &maps.value_suffix : &maps.value_pages, bv, d.y, d.x, R);
    }
  };
  const int first_fill = min(S, count_w);
  for (int j = 0; j < first_fill; ++j) {
    const int4 d = item(j);
    issue_k(j, d);
    issue_v(j, d);
  }
  int issued_k = first_fill, issued_v = first_fill;

  // Merge head h's partials (selector representatives + attention CTAs
  // [first, last]) and write its output rows.  Row maxima and denominators
  // first (one warp per row), then one float4 of output per thread, with the
  // partial loads issued 16 at a time so they overlap.
  float* comb = st_m;  // reuses the stash: [2][G]
  auto combine = [&](int h, int first, int last) {
    const int G = p.group;
    const int n_att = last - first + 1;
    const int nsrc = PB + n_att;
    auto slot_of = [&](int k) {
      return k < PB ? static_cast<size_t>(h * PB + k) * G
                    : static_cast<size_t>(h * p.ctas + first + k - PB) * G;
    };
    for (int g = warp; g < G; g += warps) {
      float top = -INFINITY;
      for (int k = lane; k < nsrc; k += 32) {
        top = fmaxf(top, __ldcg((k < PB ? p.rep_m : p.att_m) + slot_of(k) + g));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, o));
      const float ref = top == -INFINITY ? 0.f : top;
      float den = 0.f;
      for (int k = lane; k < nsrc; k += 32) {
        const size_t slot = slot_of(k) + g;
        den += __ldcg((k < PB ? p.rep_l : p.att_l) + slot) *
               __expf(__ldcg((k < PB ? p.rep_m : p.att_m) + slot) - ref);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
      if (lane == 0) {
        comb[g] = ref;
        comb[G + g] = fmaxf(den, 1e-30f);
      }
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * (D / 4); idx += blockDim.x) {
      const int g = idx / (D / 4), d4 = idx - g * (D / 4);
      const float ref = comb[g];
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k0 = 0; k0 < nsrc; k0 += 16) {
        float w[16];
        float4 v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int k = k0 + u;
          w[u] = -INFINITY;
          v[u] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (k < nsrc) {
            const size_t slot = slot_of(k) + g;
            w[u] = __ldcg((k < PB ? p.rep_m : p.att_m) + slot);
            v[u] = __ldcg(reinterpret_cast<const float4*>((k < PB ? p.rep_o : p.att_o) +
                                                          slot * D) + d4);
          }
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const float e = __expf(w[u] - ref);
          acc.x += e * v[u].x;
          acc.y += e * v[u].y;
          acc.z += e * v[u].z;
          acc.w += e * v[u].w;
        }
      }
      const float inv = 1.f / comb[G + g];
      const size_t o = (static_cast<size_t>(h) * G + g) * D + d4 * 4;
      if (p.query_f32) {
        *reinterpret_cast<float4*>(static_cast<float*>(p.out) + o) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      } else {
        __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out) + o;
        *reinterpret_cast<uint2*>(out) =
            make_uint2(pack_bf16(acc.x * inv, acc.y * inv), pack_bf16(acc.z * inv, acc.w * inv));
      }
    }
    __syncthreads();
  };
  // Count this CTA's contribution to head h.  The last of `expected`
  // arrivals owns the head's combine, which runs after this CTA's own pages
  // so that a combine never delays the streaming of other pages.
  if (threadIdx.x == 0) flags[1] = 0;
  auto arrive = [&](int h, int expected, int first, int last) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(p.done + h, 1) == expected - 1) {
      int* e = pending + 3 * flags[1]++;
      e[0] = h;
      e[1] = first;
      e[2] = last;
    }
    __syncthreads();
  };

  bool aborted = false;
  int jj = 0;  // next local item to consume
  if (lo < hi) {
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
              static_cast<size_t>(h) * p.group * D * (p.query_f32 ? 4 : 2),
          p.query_f32, p.group, lane, false);
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
      reduce_l<NT>(l);
      stash_warp_partial<D, NT>(st_m, st_l, st_o, warp, lane, m, l, o);
      __syncthreads();
      const size_t slot = static_cast<size_t>(h) * p.ctas + cta;
      merge_stashed<D>(st_m, st_l, st_o, warps, G8, p.group, p.att_m + slot * p.group,
                       p.att_l + slot * p.group, p.att_o + slot * p.group * D, threadIdx.x,
                       blockDim.x);
      const int first = static_cast<int>(cta_of(hstart[h]));
      const int last = static_cast<int>(cta_of(hstart[h + 1] - 1));
      arrive(h, last - first + 1, first, last);
    }
  }
  pdl_launch_dependents();

  // Heads with no item (nothing refined, empty suffix) still need their
  // representative partials combined: one owner CTA per such head.
  for (int h = 0; h < H; ++h) {
    if (hstart[h + 1] != hstart[h]) continue;
    const long long owner = T == 0 ? h % p.ctas : cta_of(hstart[h] < T ? hstart[h] : T - 1);
    if (owner == cta) arrive(h, 1, 0, -1);
  }
  __threadfence();
  __syncthreads();
  for (int i = 0; i < flags[1]; ++i) {
    const int* e = pending + 3 * i;
    combine(e[0], e[1], e[2]);
    if (threadIdx.x == 0) p.done[e[0]] = 0;
  }
}

template <int R, int D, int NT>
cudaError_t launch_attend_t(const AttendMaps& maps, const AttendParams& p, int warps, size_t smem,
                            cudaStream_t stream, bool pdl) {
  auto kernel = attend_kernel<R, D, NT>;
  cudaError_t err = ensure_smem_limit(reinterpret_cast<const void*>(kernel), smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.ctas);
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

}  // namespace

size_t attend_smem_bytes(int dim, int page, int warps, int stages, int group, int heads,
                         int parts_b) {
  const int g8 = group <= 8 ? 8 : 16;
  size_t bytes = kSmemSlack;
  bytes += static_cast<size_t>(warps) * stages * 2 * page * dim * 2;  // TMA ring
  bytes += round16(static_cast<size_t>(warps) * stages * 16);          // K and V barriers
  bytes += round16(static_cast<size_t>(warps) * stages * 4);           // valid rows
  bytes += round16(static_cast<size_t>(heads + 1) * 8);
  bytes += round16(static_cast<size_t>(heads) * (parts_b + 1) * 4) + 16;
  bytes += round16(static_cast<size_t>(heads) * 12);  // pending combines
  bytes += static_cast<size_t>(warps) * g8 * 4 * 2 + static_cast<size_t>(warps) * g8 * dim * 4;
  return bytes;
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

}  // namespace rkv
