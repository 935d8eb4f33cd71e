// Post-prefill block summarizer (reference: src/refinekv/summary.py:46-113).
//
// Persistent grid, one CTA per SM; the (head, page) list is cut into equal
// contiguous ranges, one per CTA, and warp w of a CTA takes pages
// lo + w + j * warps.  Each warp streams its pages through its own ring of
// TMA stages (K page | V page, [rows x 64] boxes, 128-byte swizzle; rows past
// the prompt read as zeros) and computes everything from shared memory, so
// HBM sees K and V exactly once:
//   * lane per 16-byte channel chunk: FP32 sums of K and V, per-channel K
//     range -> bf16 means, squared half widths, 1/width;
//   * lane per row: V row norms and the centred, width-normalised squared
//     distance of every real K row -> the page's value norm and radius;
//   * the bf16 ellipsoid (radius^2 * width^2 * (1 + 2^-8)), the optional
//     zero-padded page copy, counts and the per-head maximum value norm.
// The K/V sums follow the reference's FP32 summation order (bit-identical
// means); the centred radius and the value norms reduce over channels in a
// different order than torch's vectorised CPU kernels, so the ellipsoid can
// differ from the reference's by an ulp and the norms by an FP32 rounding.
//
// K/V caches may be bf16 or fp32 (the reference's build_summary takes any
// floating cache, summary.py:46-60).  An fp32 cache is summarised from its
// fp32 values, and its pages are always copied out rounded to bf16: the
// reference's attention rounds the prompt K/V to bf16 before use
// (reference.py:57, :63-66), so the decode kernels read the same values.
#include "rkv_device.cuh"
#include "rkv_kernels.h"

namespace rkv {
namespace {

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  return u;
}

// Eight consecutive channels (8 * v .. 8 * v + 7) of row r of a swizzled fp32
// tile (two 16-byte chunks).
template <typename T>
__device__ __forceinline__ void load8(const uint8_t* tile, int r, int v, int rows, float (&f)[8]);

template <>
__device__ __forceinline__ void load8<float>(const uint8_t* tile, int r, int v, int rows,
                                             float (&f)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(tile + swz(r, 2 * v, rows));
  const float4 b = *reinterpret_cast<const float4*>(tile + swz(r, 2 * v + 1, rows));
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
  f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

// Eight consecutive channels of row r as four float2 pairs (packed-FP32 math).
template <typename T>
__device__ __forceinline__ void load8x2(const uint8_t* tile, int r, int v, int rows,
                                        float2 (&f)[4]) {
  if constexpr (sizeof(T) == 2) {
    const uint4 u = *reinterpret_cast<const uint4*>(tile + swz(r, v, rows));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
    }
  } else {
    const float4 a = *reinterpret_cast<const float4*>(tile + swz(r, 2 * v, rows));
    const float4 b = *reinterpret_cast<const float4*>(tile + swz(r, 2 * v + 1, rows));
    f[0] = make_float2(a.x, a.y);
    f[1] = make_float2(a.z, a.w);
    f[2] = make_float2(b.x, b.y);
    f[3] = make_float2(b.z, b.w);
  }
}

// The same eight channels as a bf16 page-copy chunk (bf16: the stored bits).
template <typename T>
__device__ __forceinline__ uint4 page_chunk(const uint8_t* tile, int r, int v, int rows) {
  if constexpr (sizeof(T) == 2) {
    return *reinterpret_cast<const uint4*>(tile + swz(r, v, rows));
  } else {
    float f[8];
    load8<T>(tile, r, v, rows, f);
    return pack8(f);
  }
}

// max/min that keep a NaN once seen, like torch.amax / torch.maximum.
__device__ __forceinline__ float nan_max(float a, float b) { return (b > a || b != b) ? b : a; }
__device__ __forceinline__ float nan_min(float a, float b) { return (b < a || b != b) ? b : a; }

// D: the tile width (the real head dim p.dim rounded up to 64; TMA fills the
// padding columns with zeros and nothing reads them).  T: the cache's element
// type (bf16 or fp32); each lane of the per-channel pass owns 8 channels.
template <int D, int R, typename T>
__global__ void __launch_bounds__(384, 1) summarize_kernel(const __grid_constant__ SummarizeMaps maps,
                                                           const SummarizeParams p) {
  constexpr int kTile = R * D * static_cast<int>(sizeof(T));
  constexpr int kStage = 2 * kTile;
  const int kChunks = p.dim / 8;                              // real 8-channel chunks per row
  const int kLpc = 32 % kChunks == 0 ? 32 / kChunks : 1;      // lanes per chunk (row interleave)
  const int kActive = kChunks * kLpc;                         // lanes of the per-chunk pass
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  uint8_t* ring = smem;  // [warp][stage][K | V]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(warps) * S * kStage);
  float* scratch = reinterpret_cast<float*>(smem + static_cast<size_t>(warps) * S * kStage +
                                            round16(static_cast<size_t>(warps) * S * 8));
  float* kmean_s = scratch + warp * 2 * D;  // this warp's [D] negated bf16-rounded K means
  float* rscale_s = kmean_s + D;            // and [D] reciprocal half widths

  const long long pages = static_cast<long long>(p.heads) * p.blocks;
  const long long lo = pages * blockIdx.x / gridDim.x;
  const long long hi = pages * (blockIdx.x + 1) / gridDim.x;
  const int mine = hi - lo > warp ? static_cast<int>((hi - lo - warp + warps - 1) / warps) : 0;

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[warp * S + s], 1);
    mbar_fence_init();
  }
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&maps.keys);
    tma_prefetch_desc(&maps.values);
  }
  __syncwarp();
  pdl_wait();
  pdl_launch_dependents();
  const uint64_t policy = l2_evict_first_policy();

  auto page_of = [&](int j) { return lo + warp + static_cast<long long>(j) * warps; };
  auto issue = [&](int j) {  // lane 0
    const long long pg = page_of(j);
    const int h = static_cast<int>(pg / p.blocks), b = static_cast<int>(pg % p.blocks);
    const int s = j % S;
    uint8_t* dst = ring + static_cast<size_t>(warp * S + s) * kStage;
    mbar_expect_tx(&bars[warp * S + s], kStage);
    tma_tile_hint_w<D, sizeof(T)>(dst, &maps.keys, &bars[warp * S + s], b * R, h, R, policy);
    tma_tile_hint_w<D, sizeof(T)>(dst + kTile, &maps.values, &bars[warp * S + s], b * R, h, R,
                                  policy);
  };
  const int first = min(S, mine);
  if (lane == 0) {
    for (int j = 0; j < first; ++j) issue(j);
  }
  int issued = first;

  for (int j = 0; j < mine; ++j) {
    const int s = j % S;
    const long long pg = page_of(j);
    const int h = static_cast<int>(pg / p.blocks), b = static_cast<int>(pg % p.blocks);
    const int count = min(R, p.tokens - b * R);
    if (!warp_wait(&bars[warp * S + s], (j / S) & 1)) {
      // A wait that ran out: mark the head's value-norm bound NaN (the
      // selector then expands every page of it) and stop this warp.
      if (lane == 0) atomicMax(reinterpret_cast<int*>(p.max_value_norm + h), 0x7fffffff);
      drain_pending(bars + warp * S, S, j, issued);
      break;
    }
    const uint8_t* kt = ring + static_cast<size_t>(warp * S + s) * kStage;
    const uint8_t* vt = kt + kTile;

    // Lane per channel chunk: sums and K range over the real rows.  The sums
    // follow the reference's order exactly: torch's CPU sum over the rows of
    // a page (summary.py:72-74) adds 16-row chunks one after another, each
    // summed row by row from zero (padding rows add +0).  Lane group u of a
    // chunk of channels sums row chunks u, u + kLpc, ...; the chunk sums are
    // then added in chunk order, so the FP32 sums -- and the bf16 means --
    // are bit-identical to the reference's for bf16 and fp32 caches alike.
    constexpr int kRowChunks = R / 16;
    // Sums as float2 pairs (packed FP32 adds: each channel's adds stay in row
    // order); the K range of a bf16 cache as packed bf16 max / min, which
    // propagate a NaN like torch.amax / amin (a bf16 max is exact).
    float2 kpart[kRowChunks][4], vpart[kRowChunks][4];
    __nv_bfloat162 kmx2[4], kmn2[4];
    float kmax[8], kmin[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      kmax[i] = -INFINITY;
      kmin[i] = INFINITY;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      kmx2[i] = __floats2bfloat162_rn(-INFINITY, -INFINITY);
      kmn2[i] = __floats2bfloat162_rn(INFINITY, INFINITY);
#pragma unroll
      for (int s2 = 0; s2 < kRowChunks; ++s2) kpart[s2][i] = vpart[s2][i] = make_float2(0.f, 0.f);
    }
    const int c16 = lane % kChunks;
    if (lane < kActive) {
#pragma unroll
      for (int s2 = 0; s2 < kRowChunks; ++s2) {
        const int chunk = lane / kChunks + s2 * kLpc;
        if (chunk >= kRowChunks) break;
        const int r_end = min(chunk * 16 + 16, count);
        auto add_row = [&](int r) {
          float2 kf[4], vf[4];
          load8x2<T>(vt, r, c16, R, vf);
          if constexpr (sizeof(T) == 2) {
            // One 16-byte load of the K chunk serves both the sums and the range.
            const uint4 u = *reinterpret_cast<const uint4*>(kt + swz(r, c16, R));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              __nv_bfloat162 kb;
              *reinterpret_cast<uint32_t*>(&kb) = w[i];
              kmx2[i] = __hmax2_nan(kmx2[i], kb);
              kmn2[i] = __hmin2_nan(kmn2[i], kb);
              kf[i] = make_float2(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xffff0000u));
            }
          } else {
            load8x2<T>(kt, r, c16, R, kf);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              kmax[2 * i] = nan_max(kmax[2 * i], kf[i].x);
              kmax[2 * i + 1] = nan_max(kmax[2 * i + 1], kf[i].y);
              kmin[2 * i] = nan_min(kmin[2 * i], kf[i].x);
              kmin[2 * i + 1] = nan_min(kmin[2 * i + 1], kf[i].y);
            }
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            kpart[s2][i] = __fadd2_rn(kpart[s2][i], kf[i]);
            vpart[s2][i] = __fadd2_rn(vpart[s2][i], vf[i]);
          }
        };
        if (r_end == chunk * 16 + 16) {  // a full chunk: row offsets known at compile time
#pragma unroll
          for (int i = 0; i < 16; ++i) add_row(chunk * 16 + i);
        } else {
          for (int r = chunk * 16; r < r_end; ++r) add_row(r);
        }
        if (r_end < chunk * 16 + 16) {  // zero padding rows: x + 0 turns a -0 sum into +0
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            kpart[s2][i] = __fadd2_rn(kpart[s2][i], make_float2(0.f, 0.f));
            vpart[s2][i] = __fadd2_rn(vpart[s2][i], make_float2(0.f, 0.f));
          }
        }
      }
    }
    if constexpr (sizeof(T) == 2) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 hi = __bfloat1622float2(kmx2[i]), lo = __bfloat1622float2(kmn2[i]);
        kmax[2 * i] = hi.x;
        kmax[2 * i + 1] = hi.y;
        kmin[2 * i] = lo.x;
        kmin[2 * i + 1] = lo.y;
      }
    }
    for (int off = kChunks; off < kActive; off <<= 1) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        kmax[i] = nan_max(kmax[i], __shfl_xor_sync(0xffffffffu, kmax[i], off));
        kmin[i] = nan_min(kmin[i], __shfl_xor_sync(0xffffffffu, kmin[i], off));
      }
    }
    // Chunk k lives in slot k / kLpc of lane group k % kLpc.
    float ksum[8], vsum[8];
#pragma unroll
    for (int s2 = 0; s2 < kRowChunks; ++s2) {
      for (int g = 0; g < kLpc; ++g) {
        const int chunk = s2 * kLpc + g;
        if (chunk >= kRowChunks) break;
        const int src = g * kChunks + c16;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float k0 = __shfl_sync(0xffffffffu, kpart[s2][i].x, src);
          const float k1 = __shfl_sync(0xffffffffu, kpart[s2][i].y, src);
          const float v0 = __shfl_sync(0xffffffffu, vpart[s2][i].x, src);
          const float v1 = __shfl_sync(0xffffffffu, vpart[s2][i].y, src);
          ksum[2 * i] = chunk == 0 ? k0 : ksum[2 * i] + k0;
          ksum[2 * i + 1] = chunk == 0 ? k1 : ksum[2 * i + 1] + k1;
          vsum[2 * i] = chunk == 0 ? v0 : vsum[2 * i] + v0;
          vsum[2 * i + 1] = chunk == 0 ? v1 : vsum[2 * i + 1] + v1;
        }
      }
    }
    const float cnt = static_cast<float>(count);
    // A full page holds a power-of-two count: x * 2^-k is the correctly
    // rounded x / 2^k (both round the same real number), so the means take a
    // multiply there and the IEEE division only on a partial last page.
    if ((count & (count - 1)) == 0) {
      const float inv = __frcp_rn(cnt);  // exact: cnt is a power of two
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ksum[i] *= inv;
        vsum[i] *= inv;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ksum[i] /= cnt;
        vsum[i] /= cnt;
      }
    }
    float width2[8];
    if (lane < kChunks) {
      float kmean[8], vmean[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        kmean[i] = bf16_round(ksum[i]);
        vmean[i] = bf16_round(vsum[i]);
        float w = nan_max(kmax[i] - kmean[i], kmean[i] - kmin[i]);
        w = w < 1e-6f ? 1e-6f : w;
        width2[i] = bf16_round(w * w);
        kmean_s[c16 * 8 + i] = -kmean[i];
        rscale_s[c16 * 8 + i] = __frsqrt_rn(width2[i]);
      }
      const size_t off = static_cast<size_t>(pg) * p.dim + c16 * 8;
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.key_mean) + off) = pack8(kmean);
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.value_mean) + off) = pack8(vmean);
    }
    __syncwarp();

    // Lane per row: V row norm and the centred, normalised K distance.
    float vnorm = -INFINITY, dmax = -INFINITY;
    for (int r = lane; r < count; r += 32) {
      // Packed FP32: (k - mean) * scale, its square and v^2 accumulated as
      // channel pairs, summed at the end (the reference's channel order is not
      // reproducible anyway: torch vectorises the sum).
      float2 sq2 = make_float2(0.f, 0.f), dist2 = make_float2(0.f, 0.f);
      auto add_chunk = [&](int c) {
        float2 kf[4], vf[4];
        load8x2<T>(kt, r, c, R, kf);
        load8x2<T>(vt, r, c, R, vf);
        const float4 m0 = *reinterpret_cast<const float4*>(kmean_s + c * 8);
        const float4 m1 = *reinterpret_cast<const float4*>(kmean_s + c * 8 + 4);
        const float4 s0 = *reinterpret_cast<const float4*>(rscale_s + c * 8);
        const float4 s1 = *reinterpret_cast<const float4*>(rscale_s + c * 8 + 4);
        const float2 neg_mean[4] = {make_float2(m0.x, m0.y), make_float2(m0.z, m0.w),
                                    make_float2(m1.x, m1.y), make_float2(m1.z, m1.w)};
        const float2 scale[4] = {make_float2(s0.x, s0.y), make_float2(s0.z, s0.w),
                                 make_float2(s1.x, s1.y), make_float2(s1.z, s1.w)};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          sq2 = __ffma2_rn(vf[i], vf[i], sq2);
          const float2 x = __fmul2_rn(__fadd2_rn(kf[i], neg_mean[i]), scale[i]);
          dist2 = __ffma2_rn(x, x, dist2);
        }
      };
      if (kChunks == D / 8) {  // the full tile width: chunk offsets known at compile time
#pragma unroll
        for (int c = 0; c < D / 8; ++c) add_chunk(c);
      } else {
#pragma unroll 4
        for (int c = 0; c < kChunks; ++c) add_chunk(c);
      }
      vnorm = nan_max(vnorm, sqrtf(sq2.x + sq2.y));
      dmax = nan_max(dmax, dist2.x + dist2.y);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      vnorm = nan_max(vnorm, __shfl_xor_sync(0xffffffffu, vnorm, off));
      dmax = nan_max(dmax, __shfl_xor_sync(0xffffffffu, dmax, off));
    }
    float rho2 = dmax < 0.f ? 0.f : dmax;
    rho2 = sqrtf(rho2);
    rho2 = rho2 * rho2;
    if (lane < kChunks) {
      float ell[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) ell[i] = (rho2 * width2[i]) * 1.00390625f;
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.ellipsoid) +
                                static_cast<size_t>(pg) * p.dim + c16 * 8) = pack8(ell);
    }
    if (lane == 0) {
      p.value_norm[pg] = vnorm;
      // Norms are >= 0 (or a positive NaN), so their bit patterns order as ints.
      atomicMax(reinterpret_cast<int*>(p.max_value_norm + h), __float_as_int(vnorm));
      if (h == 0) p.counts[b] = count;
    }
    // Zero-padded page copy: the rows past the prompt are written as zeros
    // here; a decoder may later append generated tokens there, and the
    // decode kernels mask them out by the page's count, never by their value.
    if (p.key_pages != nullptr) {
      const size_t row0 = static_cast<size_t>(b) * R * p.dim;  // page b of head h
      uint4* kdst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.key_pages) +
                                             h * p.key_pages_head_stride + row0);
      uint4* vdst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.value_pages) +
                                             h * p.value_pages_head_stride + row0);
      for (int i = lane; i < R * kChunks; i += 32) {
        const int r = i / kChunks, c = i - r * kChunks;
        kdst[i] = page_chunk<T>(kt, r, c, R);
        vdst[i] = page_chunk<T>(vt, r, c, R);
      }
    }
    __syncwarp();
    if (j + S < mine) {
      if (lane == 0) {
        fence_proxy_async();
        issue(j + S);
      }
      ++issued;
    }
  }
}

template <int D, int R, typename T>
cudaError_t launch_t(const SummarizeMaps& maps, const SummarizeParams& p, int ctas, int warps,
                     size_t smem, cudaStream_t stream) {
  const void* kernel = reinterpret_cast<const void*>(summarize_kernel<D, R, T>);
  cudaError_t err = ensure_smem_limit(kernel, smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(warps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, summarize_kernel<D, R, T>, maps, p);
}

template <int D, typename T>
cudaError_t launch_r(const SummarizeMaps& maps, const SummarizeParams& p, int ctas, int warps,
                     size_t smem, cudaStream_t stream) {
  switch (p.block_size) {
    case 16: return launch_t<D, 16, T>(maps, p, ctas, warps, smem, stream);
    case 32: return launch_t<D, 32, T>(maps, p, ctas, warps, smem, stream);
    case 64: return launch_t<D, 64, T>(maps, p, ctas, warps, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

template <int D>
cudaError_t launch_d(const SummarizeMaps& maps, const SummarizeParams& p, int ctas, int warps,
                     size_t smem, cudaStream_t stream) {
  return p.f32 ? launch_r<D, float>(maps, p, ctas, warps, smem, stream)
               : launch_r<D, __nv_bfloat16>(maps, p, ctas, warps, smem, stream);
}

}  // namespace

size_t summarize_smem_bytes(int dim, int block, int warps, int stages, int elem_bytes) {
  return kSmemSlack + static_cast<size_t>(warps) * stages * 2 * block * dim * elem_bytes +
         round16(static_cast<size_t>(warps) * stages * 8) + static_cast<size_t>(warps) * 2 * dim * 4;
}

cudaError_t launch_summarize(const SummarizeMaps& maps, const SummarizeParams& p, int dim,
                             int ctas, int warps, size_t smem, cudaStream_t stream) {
  switch (dim) {
    case 64: return launch_d<64>(maps, p, ctas, warps, smem, stream);
    case 128: return launch_d<128>(maps, p, ctas, warps, smem, stream);
    case 192: return launch_d<192>(maps, p, ctas, warps, smem, stream);
    case 256: return launch_d<256>(maps, p, ctas, warps, smem, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace rkv
