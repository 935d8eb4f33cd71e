// Post-prefill block summarizer (reference: src/refinekv/summary.py:46-113).
//
// One lane group per (head, page): each lane owns 8 channels (one 16-byte
// vector) of every row of the page.  Pass 1 streams the page once from HBM
// and accumulates FP32 sums of K and V, the per-channel K range and the
// largest V row norm; it also writes the zero-padded page copy when the
// caller needs one.  Pass 2 re-reads the (now L2-resident) K rows for the
// centred radius.  HBM traffic: K and V once, plus the optional page copy
// and the ~5% of summaries written.
#include "rkv_device.cuh"
#include "rkv_kernels.h"

namespace rkv {
namespace {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __low2float(p[i]);
    f[2 * i + 1] = __high2float(p[i]);
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  u.x = pack_bf16(f[0], f[1]);
  u.y = pack_bf16(f[2], f[3]);
  u.z = pack_bf16(f[4], f[5]);
  u.w = pack_bf16(f[6], f[7]);
  return u;
}

// max/min that keep a NaN once seen, like torch.amax / torch.maximum.
__device__ __forceinline__ float nan_max(float a, float b) { return (b > a || b != b) ? b : a; }
__device__ __forceinline__ float nan_min(float a, float b) { return (b < a || b != b) ? b : a; }

template <int D>
__global__ void __launch_bounds__(256, 2) summarize_kernel(const SummarizeParams p) {
  constexpr int kChunks = D / 8;
  constexpr int kLanes = kChunks <= 8 ? 8 : (kChunks <= 16 ? 16 : 32);
  constexpr int kPagesPerWarp = 32 / kLanes;
  const int lane = threadIdx.x & 31;
  const int sub = lane / kLanes, cl = lane % kLanes;
  const long long page =
      (static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) *
          kPagesPerWarp +
      sub;
  const bool page_ok = page < static_cast<long long>(p.heads) * p.blocks;
  const bool lane_ok = page_ok && cl < kChunks;
  const int h = page_ok ? static_cast<int>(page / p.blocks) : 0;
  const int b = page_ok ? static_cast<int>(page % p.blocks) : 0;
  const int B = p.block_size;
  const int count = page_ok ? min(B, p.tokens - b * B) : 0;

  pdl_wait();
  pdl_launch_dependents();

  const __nv_bfloat16* __restrict__ kbase =
      static_cast<const __nv_bfloat16*>(p.keys) + h * p.key_head_stride +
      static_cast<long long>(b) * B * p.key_token_stride + cl * 8;
  const __nv_bfloat16* __restrict__ vbase =
      static_cast<const __nv_bfloat16*>(p.values) + h * p.value_head_stride +
      static_cast<long long>(b) * B * p.value_token_stride + cl * 8;
  uint4* __restrict__ kpage =
      p.key_pages ? reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.key_pages) +
                                             page * B * D + cl * 8)
                  : nullptr;
  uint4* __restrict__ vpage =
      p.value_pages ? reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.value_pages) +
                                               page * B * D + cl * 8)
                    : nullptr;

  float ksum[8], kmax[8], kmin[8], vsum[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ksum[i] = 0.f;
    vsum[i] = 0.f;
    kmax[i] = -INFINITY;
    kmin[i] = INFINITY;
  }
  float vnorm = -INFINITY;

  // Rows are read kBatch at a time: every load of a batch is in flight
  // before the first is used.
  constexpr int kBatch = 8;
  for (int t0 = 0; t0 < B; t0 += kBatch) {
    uint4 kb[kBatch], vb[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      kb[i] = make_uint4(0, 0, 0, 0);
      vb[i] = make_uint4(0, 0, 0, 0);
      if (lane_ok && t0 + i < count) {
        kb[i] = __ldg(reinterpret_cast<const uint4*>(kbase + (t0 + i) * p.key_token_stride));
        vb[i] = __ldg(reinterpret_cast<const uint4*>(vbase + (t0 + i) * p.value_token_stride));
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int t = t0 + i;
      const bool row = lane_ok && t < count;
      if (kpage != nullptr && lane_ok) {
        kpage[t * (D / 8)] = kb[i];
        vpage[t * (D / 8)] = vb[i];
      }
      float kf[8], vf[8];
      unpack8(kb[i], kf);
      unpack8(vb[i], vf);
      float sq = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (row) {
          ksum[c] += kf[c];
          vsum[c] += vf[c];
          kmax[c] = nan_max(kmax[c], kf[c]);
          kmin[c] = nan_min(kmin[c], kf[c]);
        }
        sq += vf[c] * vf[c];
      }
#pragma unroll
      for (int off = 1; off < kLanes; off <<= 1) sq += __shfl_xor_sync(0xffffffffu, sq, off);
      if (row) vnorm = nan_max(vnorm, sqrtf(sq));
    }
  }

  const float cnt = static_cast<float>(count > 0 ? count : 1);
  float kmean[8], vmean[8], width2[8], rscale[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    kmean[i] = bf16_round(ksum[i] / cnt);
    vmean[i] = bf16_round(vsum[i] / cnt);
    float w = nan_max(kmax[i] - kmean[i], kmean[i] - kmin[i]);
    w = w < 1e-6f ? 1e-6f : w;
    width2[i] = bf16_round(w * w);
    rscale[i] = __frsqrt_rn(width2[i]);
  }

  // Pass 2: largest normalised centred squared distance of a real row
  // (the page was just read, so these loads hit L2).
  float dmax = -INFINITY;
  for (int t0 = 0; t0 < B; t0 += kBatch) {
    uint4 kb[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      kb[i] = make_uint4(0, 0, 0, 0);
      if (lane_ok && t0 + i < count) {
        kb[i] = __ldg(reinterpret_cast<const uint4*>(kbase + (t0 + i) * p.key_token_stride));
      }
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int t = t0 + i;
      float dsum = 0.f;
      if (lane_ok && t < count) {
        float kf[8];
        unpack8(kb[i], kf);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float x = (kf[c] - kmean[c]) * rscale[c];
          dsum += x * x;
        }
      }
#pragma unroll
      for (int off = 1; off < kLanes; off <<= 1) dsum += __shfl_xor_sync(0xffffffffu, dsum, off);
      if (t < count) dmax = nan_max(dmax, dsum);
    }
  }
  float rho2 = dmax < 0.f ? 0.f : dmax;
  rho2 = sqrtf(rho2);
  rho2 = rho2 * rho2;

  if (lane_ok) {
    float ell[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) ell[i] = (rho2 * width2[i]) * 1.00390625f;
    const long long off = page * D + cl * 8;
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.key_mean) + off) = pack8(kmean);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.value_mean) + off) = pack8(vmean);
    *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.ellipsoid) + off) = pack8(ell);
    if (cl == 0) {
      p.value_norm[page] = vnorm;
      // Norms are >= 0 (or a positive NaN), so their bit patterns order as ints.
      atomicMax(reinterpret_cast<int*>(p.max_value_norm + h), __float_as_int(vnorm));
      if (h == 0) p.counts[b] = count;
    }
  }
}

template <int D>
cudaError_t launch_summarize_t(const SummarizeParams& p, cudaStream_t stream) {
  constexpr int kChunks = D / 8;
  constexpr int kLanes = kChunks <= 8 ? 8 : (kChunks <= 16 ? 16 : 32);
  constexpr int kPagesPerWarp = 32 / kLanes;
  constexpr int kWarps = 8;
  const long long pages = static_cast<long long>(p.heads) * p.blocks;
  const long long per_cta = static_cast<long long>(kWarps) * kPagesPerWarp;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((pages + per_cta - 1) / per_cta));
  cfg.blockDim = dim3(kWarps * 32);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, summarize_kernel<D>, p);
}

}  // namespace

cudaError_t launch_summarize(const SummarizeParams& p, int dim, cudaStream_t stream) {
  switch (dim) {
    case 64: return launch_summarize_t<64>(p, stream);
    case 128: return launch_summarize_t<128>(p, stream);
    case 192: return launch_summarize_t<192>(p, stream);
    case 256: return launch_summarize_t<256>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace rkv
