// Device-side building blocks shared by the RefineKV sm_100a kernels.
//
// Data movement: TMA tiled loads (cp.async.bulk.tensor, no multicast) of
// [rows x head_dim] bf16 tiles into 128B-swizzled shared memory, completed on
// per-stage mbarriers.  Every mbarrier wait is bounded by the global timer.
//
// Math: mma.sync m16n8k16 bf16 -> fp32 with the token (or block) axis on M
// and the GQA group axis on N, so a group of up to 8 query rows wastes no
// more than half of an n8 tile.  The S^T fragment is turned into the P^T
// operand of the value product with movmatrix (register transpose), so the
// probabilities never touch shared memory.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace rkv {

// ---------------------------------------------------------------------------
// status bits written to the workspace status word
// ---------------------------------------------------------------------------
constexpr int kStatusTimeout = 1;     // an mbarrier wait hit its time limit
constexpr int kStatusBadInput = 2;    // a device-side input failed a range check

constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s per wait

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete; false after
// `limit_ns` (1 s by default).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - start > limit_ns) return false;
  }
}

// Warp-uniform wait: every lane polls; if any lane gave up, all report failure
// so the warp never splits around the .sync.aligned tensor instructions.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity) {
  const bool ok = mbar_wait(bar, parity);
  return __all_sync(0xffffffffu, ok);
}

// After a wait timed out at local item `from`: wait again (bounded) for every
// load this warp issued and has not consumed, so no copy is still landing in
// shared memory when the CTA exits.
__device__ __forceinline__ void drain_pending(uint64_t* bars, int stages, int from, int issued) {
  for (int j = from; j < issued; ++j) mbar_wait(&bars[j % stages], (j / stages) & 1);
}

// Same for rings whose stages hold separate K and V barriers ([stage][2]).
__device__ __forceinline__ void drain_pending(uint64_t* bars, int stages, int from, int issued_k,
                                              int issued_v) {
  for (int j = from; j < issued_k; ++j) mbar_wait(&bars[(j % stages) * 2], (j / stages) & 1);
  for (int j = from; j < issued_v; ++j) mbar_wait(&bars[(j % stages) * 2 + 1], (j / stages) & 1);
}

// ---------------------------------------------------------------------------
// TMA (tiled, 3-D: x = channel, y = row, z = head).  No multicast anywhere.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// Same load with an L2 cache-policy hint (used with an evict-first policy for
// K/V pages that are streamed once per step).
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int x, int y, int z, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar)),
      "l"(policy)
      : "memory");
}

// 4-D form (x = channel, y = row in page, z = head, w = page) for K/V pages.
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                 int x, int y, int z, int w, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_addr(bar)),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  return policy;
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Bring one [rows x D] bf16 tile into L2 (no shared memory, no barrier, no
// data returned): warms L2 and the address translation for a later tma_tile
// of the same rows.  L2 is the point of coherence, so a prefetch issued
// before a dependency wait can never make a later read stale.
template <int D>
__device__ __forceinline__ void tma_prefetch_tile(const CUtensorMap* map, int row, int head) {
#pragma unroll
  for (int i = 0; i < D / 64; ++i) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(i * 64), "r"(row), "r"(head)
                 : "memory");
  }
}

// The same for one page of a 4-D page map (all its rows).
template <int D>
__device__ __forceinline__ void tma_prefetch_page(const CUtensorMap* map, int head, int page) {
#pragma unroll
  for (int i = 0; i < D / 64; ++i) {
    asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(i * 64), "r"(0), "r"(head), "r"(page)
                 : "memory");
  }
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Order this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) writes to the same buffers.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Load one [rows x D] bf16 tile as D/64 boxes of [rows x 64] (128 B rows,
// SWIZZLE_128B).  Box i lands at dst + i * rows * 128.
template <int D>
__device__ __forceinline__ void tma_tile(void* dst, const CUtensorMap* map, uint64_t* bar, int row,
                                         int head, int rows) {
#pragma unroll
  for (int i = 0; i < D / 64; ++i) {
    tma_load_3d(static_cast<char*>(dst) + i * rows * 128, map, bar, i * 64, row, head);
  }
}

// One K or V page (all `rows` rows of KV head `head` in page `page`) from a
// 4-D page map, landing in the same swizzled layout as tma_tile.
template <int D>
__device__ __forceinline__ void tma_page_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                              int head, int page, int rows, uint64_t policy) {
#pragma unroll
  for (int i = 0; i < D / 64; ++i) {
    tma_load_4d_hint(static_cast<char*>(dst) + i * rows * 128, map, bar, i * 64, 0, head, page,
                     policy);
  }
}

template <int D>
__device__ __forceinline__ void tma_tile_hint(void* dst, const CUtensorMap* map, uint64_t* bar,
                                              int row, int head, int rows, uint64_t policy) {
#pragma unroll
  for (int i = 0; i < D / 64; ++i) {
    tma_load_3d_hint(static_cast<char*>(dst) + i * rows * 128, map, bar, i * 64, row, head,
                     policy);
  }
}

// Same for a tile of `W`-byte-wide elements: W == 2 is tma_tile_hint, W == 4
// (fp32) loads D / 32 boxes of [rows x 32] (128-byte rows, the same
// swizzled layout; box i lands at dst + i * rows * 128).
template <int D, int W>
__device__ __forceinline__ void tma_tile_hint_w(void* dst, const CUtensorMap* map, uint64_t* bar,
                                                int row, int head, int rows, uint64_t policy) {
  constexpr int kBoxCols = 128 / W;
#pragma unroll
  for (int i = 0; i < D / kBoxCols; ++i) {
    tma_load_3d_hint(static_cast<char*>(dst) + i * rows * 128, map, bar, i * kBoxCols, row, head,
                     policy);
  }
}

// Byte offset of the 16-byte chunk `c16` (= column / 8) of row `r` inside a
// swizzled tile of `rows` rows.
__device__ __forceinline__ uint32_t swz(int r, int c16, int rows) {
  return static_cast<uint32_t>((c16 >> 3) * rows * 128 + r * 128 + (((c16 & 7) ^ (r & 7)) << 4));
}

// Dynamic shared memory is carved from a 1024-byte aligned base (the 128B
// swizzle atom); every kernel reserves kSmemSlack extra bytes for it.
constexpr int kSmemSlack = 1024;

__device__ __forceinline__ uint8_t* align_smem(uint8_t* p) {
  return p + ((1024u - (smem_addr(p) & 1023u)) & 1023u);
}

__host__ __device__ constexpr size_t round16(size_t x) { return (x + 15) & ~static_cast<size_t>(15); }

// ---------------------------------------------------------------------------
// programmatic dependent launch
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" :::);
}

// ---------------------------------------------------------------------------
// named barrier over the first `threads` threads of the CTA
// ---------------------------------------------------------------------------
__device__ __forceinline__ void named_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// tensor-core fragments
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
      " {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Transpose an 8x8 b16 matrix held one pair per thread (row lane/4,
// columns 2*(lane%4)+{0,1}).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// Query B fragments for S^T = tile . q^T.  Thread lane holds, for n-tile nt
// and k-step ks, q[g][d] with g = nt*8 + lane/4 and
// d = ks*16 + 2*(lane%4) + {0,1} (b0) and + 8 (b1).  Rows g >= group and
// channels d >= dim are 0.  `square` builds the fragments of bf16(q^2)
// instead (the ellipsoid term).  Every load is issued unconditionally from a
// clamped in-range address before any value is used, so the whole query
// arrives in one memory round trip.
template <int D, int NT>
__device__ __forceinline__ void load_query_frags(uint32_t (&qb)[D / 16][NT][2], const void* q,
                                                 int q_is_f32, int group, int dim, int lane,
                                                 bool square) {
  auto finish = [&](int nt, int ks, int half, float x0, float x1) {
    const int g = nt * 8 + (lane >> 2);
    const int d = ks * 16 + half * 8 + 2 * (lane & 3);
    if (!(g < group && d < dim)) x0 = x1 = 0.f;
    if (square) {
      x0 = x0 * x0;
      x1 = x1 * x1;
    }
    qb[ks][nt][half] = pack_bf16(x0, x1);
  };
  auto offset = [&](int nt, int ks, int half) {
    const int g = min(nt * 8 + (lane >> 2), group - 1);
    const int d = min(ks * 16 + half * 8 + 2 * (lane & 3), dim - 2);
    return g * dim + d;
  };
  if (q_is_f32) {
    const float* qf = static_cast<const float*>(q);
    float2 raw[NT][D / 16][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
        for (int half = 0; half < 2; ++half)
          raw[nt][ks][half] = *reinterpret_cast<const float2*>(qf + offset(nt, ks, half));
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
        for (int half = 0; half < 2; ++half)
          finish(nt, ks, half, bf16_round(raw[nt][ks][half].x), bf16_round(raw[nt][ks][half].y));
  } else {
    const __nv_bfloat16* qh = static_cast<const __nv_bfloat16*>(q);
    __nv_bfloat162 raw[NT][D / 16][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
        for (int half = 0; half < 2; ++half)
          raw[nt][ks][half] = *reinterpret_cast<const __nv_bfloat162*>(qh + offset(nt, ks, half));
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
        for (int half = 0; half < 2; ++half)
          finish(nt, ks, half, __low2float(raw[nt][ks][half]), __high2float(raw[nt][ks][half]));
  }
}

// bf16(q^2) fragments from the bf16 q fragments (the ellipsoid term).
template <int D, int NT>
__device__ __forceinline__ void square_frags(const uint32_t (&qb)[D / 16][NT][2],
                                             uint32_t (&q2)[D / 16][NT][2]) {
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&qb[ks][nt][half]);
        const float x0 = __low2float(v), x1 = __high2float(v);
        q2[ks][nt][half] = pack_bf16(x0 * x0, x1 * x1);
      }
}

// Groups of at most 4 rows: one n8 tile carries [q | q^2] and the reduction
// runs over 2*D (first the key-mean tile against q, then the ellipsoid tile
// against q^2).  Columns 0-3 of the result are q.kbar, columns 4-7 are
// q^2.W2, so every lane of the epilogue holds useful values.
template <int D>
__device__ __forceinline__ void pack4_frags(const uint32_t (&qb)[D / 16][1][2],
                                            uint32_t (&packed)[2 * D / 16][2], int lane) {
  const bool upper = (lane >> 2) >= 4;  // columns 4-7 hold q^2
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks)
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&qb[ks][0][half]);
      const float x0 = __low2float(v), x1 = __high2float(v);
      packed[ks][half] = upper ? 0u : qb[ks][0][half];
      packed[D / 16 + ks][half] = upper ? pack_bf16(x0 * x0, x1 * x1) : 0u;
    }
}

template <int R, int D>
__device__ __forceinline__ void score_tile_pair(uint32_t tile_a, uint32_t tile_b,
                                                const uint32_t (&packed)[2 * D / 16][2],
                                                float (&acc)[R / 16][4], int lane) {
#pragma unroll
  for (int mt = 0; mt < R / 16; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
  const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int ks = 0; ks < 2 * D / 16; ++ks) {
    const uint32_t tile = ks < D / 16 ? tile_a : tile_b;
    const int kk = ks < D / 16 ? ks : ks - D / 16;
#pragma unroll
    for (int mt = 0; mt < R / 16; ++mt) {
      uint32_t a[4];
      ldsm_x4(tile + swz(mt * 16 + row, kk * 2 + (lane >> 4), R), a);
      mma_bf16(acc[mt], a, packed[ks][0], packed[ks][1]);
    }
  }
}

// acc[mt][nt] = tile[mt*16 .. +16) . q^T for a swizzled [R x D] tile.  The
// k-steps are the outer loop so the R/16 independent accumulator chains
// interleave.
template <int R, int D, int NT>
__device__ __forceinline__ void score_tile(uint32_t tile, const uint32_t (&qb)[D / 16][NT][2],
                                           float (&acc)[R / 16][NT][4], int lane) {
#pragma unroll
  for (int mt = 0; mt < R / 16; ++mt)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
      acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.f;
  const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
  for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
    for (int mt = 0; mt < R / 16; ++mt) {
      uint32_t a[4];
      ldsm_x4(tile + swz(mt * 16 + row, ks * 2 + (lane >> 4), R), a);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_bf16(acc[mt][nt], a, qb[ks][nt][0], qb[ks][nt][1]);
    }
  }
}

// o[dt][nt] += V^T[dt*16 .. +16) . P^T for a swizzled [R x D] value tile.
template <int R, int D, int NT>
__device__ __forceinline__ void accumulate_values(uint32_t tile,
                                                  const uint32_t (&pb)[R / 16][NT][2],
                                                  float (&o)[D / 16][NT][4], int lane) {
  const int trow = (lane & 7) + ((lane >> 4) & 1) * 8;
  const int cadd = (lane >> 3) & 1;
#pragma unroll
  for (int dt = 0; dt < D / 16; ++dt) {
#pragma unroll
    for (int kt = 0; kt < R / 16; ++kt) {
      uint32_t a[4];
      ldsm_x4_trans(tile + swz(kt * 16 + trow, dt * 2 + cadd, R), a);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_bf16(o[dt][nt], a, pb[kt][nt][0], pb[kt][nt][1]);
    }
  }
}

// ---------------------------------------------------------------------------
// Online softmax over one tile whose logits sit in the S^T C-fragment layout
// (row = token, column = group row).  Thread lane owns group rows
// g = nt*8 + 2*(lane%4) + j (j = 0, 1) in m[nt][j], l[nt][j] (l is a
// per-thread partial sum, reduced across the 8 lanes of a column at the end).
// `logit` holds natural-log logits, -inf for masked entries; on return it
// holds the FP32 probabilities exp(logit - m_new) and o has been rescaled.
// ---------------------------------------------------------------------------
template <int R, int D, int NT>
__device__ __forceinline__ void softmax_update(float (&logit)[R / 16][NT][4], float (&m)[NT][2],
                                               float (&l)[NT][2], float (&o)[D / 16][NT][4]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float mx = -INFINITY;
#pragma unroll
      for (int mt = 0; mt < R / 16; ++mt) mx = fmaxf(mx, fmaxf(logit[mt][nt][j], logit[mt][nt][2 + j]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
      const float m_new = fmaxf(m[nt][j], mx);
      const float ref = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = __expf(m[nt][j] - ref);
      m[nt][j] = m_new;
      float sum = 0.f;
#pragma unroll
      for (int mt = 0; mt < R / 16; ++mt) {
        const float p0 = __expf(logit[mt][nt][j] - ref);
        const float p1 = __expf(logit[mt][nt][2 + j] - ref);
        logit[mt][nt][j] = p0;
        logit[mt][nt][2 + j] = p1;
        sum += p0 + p1;
      }
      l[nt][j] = l[nt][j] * alpha + sum;
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        o[dt][nt][j] *= alpha;
        o[dt][nt][2 + j] *= alpha;
      }
    }
  }
}

// Probabilities (C layout) -> P^T B fragments via movmatrix.  `hi` holds the
// bf16 rounding of p; with `split`, `lo` holds bf16(p - hi) so that
// V.hi + V.lo carries p to ~2^-16 relative (the FP32-query mode).
template <int R, int NT>
__device__ __forceinline__ void prob_frags(const float (&p)[R / 16][NT][4],
                                           uint32_t (&hi)[R / 16][NT][2],
                                           uint32_t (&lo)[R / 16][NT][2], bool split) {
#pragma unroll
  for (int mt = 0; mt < R / 16; ++mt) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const float a = p[mt][nt][2 * half], b = p[mt][nt][2 * half + 1];
        const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        hi[mt][nt][half] = movmatrix_trans(*reinterpret_cast<const uint32_t*>(&h));
        if (split) {
          lo[mt][nt][half] =
              movmatrix_trans(pack_bf16(a - __low2float(h), b - __high2float(h)));
        }
      }
    }
  }
}

// Online-softmax step + value accumulation for one staged value tile.
template <int R, int D, int NT>
__device__ __forceinline__ void attend_tile(float (&logit)[R / 16][NT][4], uint32_t value_tile,
                                            float (&m)[NT][2], float (&l)[NT][2],
                                            float (&o)[D / 16][NT][4], bool split, int lane) {
  softmax_update<R, D, NT>(logit, m, l, o);
  uint32_t hi[R / 16][NT][2], lo[R / 16][NT][2];
  prob_frags<R, NT>(logit, hi, lo, split);
  accumulate_values<R, D, NT>(value_tile, hi, o, lane);
  if (split) accumulate_values<R, D, NT>(value_tile, lo, o, lane);
}

// Sum the per-thread partial l over the 8 lanes sharing a column pair.
template <int NT>
__device__ __forceinline__ void reduce_l(float (&l)[NT][2]) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v = l[nt][j];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 8);
      v += __shfl_xor_sync(0xffffffffu, v, 16);
      l[nt][j] = v;
    }
  }
}

// ---------------------------------------------------------------------------
// Warp partials -> one partial per CTA.  Each warp stores m, l (per group
// row) and o^T (per row x channel) to shared memory; after a barrier the CTA
// merges them.  Layout of the scratch: m[W][G8], l[W][G8], o[W][G8][D].
// ---------------------------------------------------------------------------
template <int D, int NT>
__device__ __forceinline__ void stash_warp_partial(float* sm_m, float* sm_l, float* sm_o, int warp,
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
#pragma unroll
      for (int dt = 0; dt < D / 16; ++dt) {
        const int d0 = dt * 16 + (lane >> 2);
        sm_o[(warp * G8 + g) * D + d0] = o[dt][nt][j];
        sm_o[(warp * G8 + g) * D + d0 + 8] = o[dt][nt][2 + j];
      }
    }
  }
}

// Merge `warps` stashed partials and write all g8 rows to global as one
// partial: m_out[g], l_out[g] and o^T in o_out[d * g8 + g].  Called by
// `threads` threads.
template <int D>
__device__ __forceinline__ void merge_stashed(const float* sm_m, const float* sm_l,
                                              const float* sm_o, int warps, int g8, float* m_out,
                                              float* l_out, float* o_out, int tid, int threads) {
  for (int idx = tid; idx < g8 * D; idx += threads) {
    const int d = idx / g8, g = idx - d * g8;
    float top = -INFINITY;
    for (int w = 0; w < warps; ++w) top = fmaxf(top, sm_m[w * g8 + g]);
    const float ref = top == -INFINITY ? 0.f : top;
    float acc = 0.f, den = 0.f;
    for (int w = 0; w < warps; ++w) {
      const float m = sm_m[w * g8 + g];
      const float s = m == -INFINITY ? 0.f : __expf(m - ref);
      acc += s * sm_o[(w * g8 + g) * D + d];
      den += s * sm_l[w * g8 + g];
    }
    o_out[d * g8 + g] = acc;
    if (d == 0) {
      m_out[g] = top;
      l_out[g] = den;
    }
  }
}

}  // namespace rkv
