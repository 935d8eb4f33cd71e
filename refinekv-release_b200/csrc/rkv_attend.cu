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
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + off);
  off += round16(static_cast<size_t>(warps) * S * 8);
  int4* desc = reinterpret_cast<int4*>(smem + off);  // {head, row, valid, suffix}
  off += static_cast<size_t>(warps) * S * 16;
  long long* hstart = reinterpret_cast<long long*>(smem + off);  // [H + 1]
  off += round16(static_cast<size_t>(H + 1) * 8);
  int* seg_pre = reinterpret_cast<int*>(smem + off);  // [H][PB + 1]
  off += round16(static_cast<size_t>(H) * (PB + 1) * 4);
  int* flags = reinterpret_cast<int*>(smem + off);  // [4]
  off += 16;
  float* st_m = reinterpret_cast<float*>(smem + off);  // [warps][G8]
  float* st_l = st_m + warps * G8;
  float* st_o = st_l + warps * G8;  // [warps][G8][D]

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[warp * S + s], 1);
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

  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    int acc = 0;
    seg_pre[h * (PB + 1)] = 0;
    for (int k = 0; k < PB; ++k) {
      acc += p.seg_count[h * PB + k];
      seg_pre[h * (PB + 1) + k + 1] = acc;
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

  // Lane 0 decodes and issues local item j of this warp.  Its head cursor
  // only moves forward because the warp's items are issued in order.
  int issue_head = 0;
  auto issue = [&](int j) {
    const long long k = lo + warp + static_cast<long long>(j) * warps;
    while (hstart[issue_head + 1] <= k) ++issue_head;
    const int h = issue_head;
    const int pos = static_cast<int>(k - hstart[h]);
    const int* pre = seg_pre + h * (PB + 1);
    int row, valid, is_suffix;
    if (pos < pre[PB]) {
      int a = 0, b = PB;  // find seg with pre[seg] <= pos < pre[seg + 1]
      while (b - a > 1) {
        const int mid = (a + b) >> 1;
        if (pre[mid] <= pos) a = mid; else b = mid;
      }
      const int block = p.sel_ids[(static_cast<size_t>(h) * PB + a) * p.seg_cap + (pos - pre[a])];
      row = block * R;
      valid = static_cast<int>(p.counts[block]);
      is_suffix = 0;
    } else {
      const int c = pos - pre[PB];
      row = c * R;
      valid = min(R, suffix_len - c * R);
      is_suffix = 1;
    }
    const int s = j % S;
    desc[warp * S + s] = make_int4(h, row, valid, is_suffix);
    uint8_t* dst = ring + (warp * S + s) * kStage;
    mbar_expect_tx(&bars[warp * S + s], kStage);
    tma_tile<D>(dst, is_suffix ? &maps.key_suffix : &maps.key_pages, &bars[warp * S + s], row, h,
                R);
    tma_tile<D>(dst + kTile, is_suffix ? &maps.value_suffix : &maps.value_pages,
                &bars[warp * S + s], row, h, R);
  };
  int issued = min(S, count_w);
  if (lane == 0) {
    for (int j = 0; j < issued; ++j) issue(j);
  }

  // Merge this head's partials (selector representatives + attention CTAs
  // [first, last]) and write the output rows.
  auto combine = [&](int h, long long first, long long last) {
    const int G = p.group;
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
      const int g = idx / D, d = idx - g * D;
      float top = -INFINITY;
      for (int k = 0; k < PB; ++k) top = fmaxf(top, __ldcg(p.rep_m + (h * PB + k) * G + g));
      for (long long c = first; c <= last; ++c)
        top = fmaxf(top, __ldcg(p.att_m + (h * p.ctas + c) * G + g));
      const float ref = top == -INFINITY ? 0.f : top;
      float acc = 0.f, den = 0.f;
      for (int k = 0; k < PB; ++k) {
        const size_t slot = static_cast<size_t>(h * PB + k) * G + g;
        const float w = __expf(__ldcg(p.rep_m + slot) - ref);
        acc += w * __ldcg(p.rep_o + slot * D + d);
        den += w * __ldcg(p.rep_l + slot);
      }
      for (long long c = first; c <= last; ++c) {
        const size_t slot = static_cast<size_t>(h * p.ctas + c) * G + g;
        const float w = __expf(__ldcg(p.att_m + slot) - ref);
        acc += w * __ldcg(p.att_o + slot * D + d);
        den += w * __ldcg(p.att_l + slot);
      }
      const float out = acc / fmaxf(den, 1e-30f);
      const size_t o = (static_cast<size_t>(h) * G + g) * D + d;
      if (p.query_f32) {
        static_cast<float*>(p.out)[o] = out;
      } else {
        static_cast<__nv_bfloat16*>(p.out)[o] = __float2bfloat16_rn(out);
      }
    }
  };
  // Count this CTA's contribution to head h; the last of `expected` combines.
  auto arrive = [&](int h, int expected, long long first, long long last) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) flags[0] = atomicAdd(p.done + h, 1) == expected - 1;
    __syncthreads();
    if (flags[0]) {
      __threadfence();
      combine(h, first, last);
      if (threadIdx.x == 0) p.done[h] = 0;
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
        if (!warp_wait(&bars[warp * S + s], (jj / S) & 1)) {
          if (lane == 0) atomicOr(p.status, kStatusTimeout);
          drain_pending(bars + warp * S, S, jj, issued);
          aborted = true;
          continue;
        }
        const int valid = desc[warp * S + s].z;
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
        attend_tile<R, D, NT>(logit, base + kTile, m, l, o, p.query_f32 != 0, lane);
        __syncwarp();
        if (jj + S < count_w) {
          if (lane == 0) {
            fence_proxy_async();
            issue(jj + S);
          }
          ++issued;
        }
      }
      reduce_l<NT>(l);
      stash_warp_partial<D, NT>(st_m, st_l, st_o, warp, lane, m, l, o);
      __syncthreads();
      const size_t slot = static_cast<size_t>(h) * p.ctas + cta;
      merge_stashed<D>(st_m, st_l, st_o, warps, G8, p.group, p.att_m + slot * p.group,
                       p.att_l + slot * p.group, p.att_o + slot * p.group * D, threadIdx.x,
                       blockDim.x);
      const long long first = cta_of(hstart[h]);
      const long long last = cta_of(hstart[h + 1] - 1);
      arrive(h, static_cast<int>(last - first + 1), first, last);
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
  bytes += round16(static_cast<size_t>(warps) * stages * 8);           // barriers
  bytes += static_cast<size_t>(warps) * stages * 16;                   // item descriptors
  bytes += round16(static_cast<size_t>(heads + 1) * 8);
  bytes += round16(static_cast<size_t>(heads) * (parts_b + 1) * 4) + 16;
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
