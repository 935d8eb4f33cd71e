// Selector math shared by the selector kernels (rkv_select.cu) and the fused
// select-and-stream kernel (rkv_fused.cu): the log-space risk of a block
// (reference: src/refinekv/reference.py:19-34) and (max, sum) merges of
// log-sum-exp partials.
#pragma once

#include <cuda_runtime.h>

namespace rkv {

constexpr float kInflate = 1.00390625f;  // 1 + 2^-8
constexpr float kDeltaSplit = 10.f;
// exp and log on the special-function unit (__expf / __logf): a few ulp from
// the correctly rounded functions, far inside the 1e-3 relative eps margin
// that decides which blocks are judged against the reference; the
// accurate library calls cost several times as many instructions on the
// selector's latency-bound path.
__device__ __forceinline__ float fexp(float x) { return __expf(x); }
__device__ __forceinline__ float flog(float x) { return __logf(x); }

// log(cosh(delta)) with the reference's two branches (reference.py:19-22).
// Only the branch the reference selects is evaluated (a NaN takes the large
// one, as torch.where does), so the value is the same with half the work.
__device__ __forceinline__ float log_cosh(float delta) {
  if (delta <= kDeltaSplit) return flog((fexp(delta) + fexp(-delta)) * 0.5f);
  return delta + flog((1.f + fexp(-2.f * delta)) * 0.5f);
}

// Risk of one (row, block): distortion ("mass") + importance ("value") terms,
// evaluated in the same operation order as reference.py:25-34.  1/t is the
// correctly rounded reciprocal (the value of the reference's t.reciprocal());
// the tanh quotients take the fast division (within 2 ulp), like the
// exponentials far inside the eps margin.
// Only the branch the reference selects is evaluated (delta <= 10, else the
// large-delta forms; a NaN takes the latter, as torch.where does).
__device__ __forceinline__ float block_risk(float z, float delta, float log_z, float log_c,
                                            float vnorm, float vmax) {
  const float two_vmax = 2.f * vmax;
  float mass, tanh_half;
  if (delta <= kDeltaSplit) {
    const float t = fexp(delta);
    mass = (two_vmax * fexp(z - log_c)) * (0.5f * (t + __frcp_rn(t)) - 1.f);
    tanh_half = __fdividef(t - 1.f, t + 1.f);
  } else {
    const float e_neg = fexp(-delta);
    float one_minus = 1.f - e_neg;
    one_minus = one_minus < 1e-30f ? 1e-30f : one_minus;
    const float lcm1 = (delta + 2.f * flog(one_minus)) - 0.693147182464599609375f;
    mass = two_vmax * fexp((z - log_c) + lcm1);
    tanh_half = __fdividef(1.f - e_neg, 1.f + e_neg);
  }
  const float importance = ((2.f * vnorm) * fexp(z - log_z)) * tanh_half;
  return mass + importance;
}

__device__ __forceinline__ bool finite(float x) { return isfinite(x); }

__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float top = fmaxf(m, m2);
  const float ref = top == -INFINITY ? 0.f : top;
  s = s * fexp(m - ref) + s2 * fexp(m2 - ref);
  m = top;
}

}  // namespace rkv
