// Per-step block selector (reference: src/refinekv/reference.py:10-47; the
// reference's GPU form is kernels/selection.py:47-223 and
// kernels/attention.py:13-137).
//
// Phase A (stats): per (query instance, KV head) and per tile of 32 blocks,
// TMA stages the key-mean and ellipsoid tiles (bf16, swizzled) and computes
//   s = (q . kbar) * D^-1/2,  delta = sqrt(max(q^2 . W2, 0)) * D^-1/2 * (1+2^-8)
// with mma.sync (blocks on M, group rows on N).  It stores z = s + log(count)
// and delta for phase B and keeps running (max, sum) pairs for
// LSE_b(z) and LSE_b(z + log cosh delta), one pair per CTA and row.
//
// Phase B (final): merges those pairs into the row-global log Z / log C,
// evaluates the risk of every (row, block), reduces over the group
// (mean / max / any), forces blocks with non-finite statistics, ORs the
// anchors, and writes the byte mask.  In decode mode it also writes the
// selected block ids compacted in block order (one segment per CTA, so the
// order is deterministic) and runs the representative softmax over the
// unselected blocks of its range (logit z, value = value_mean, staged by TMA),
// leaving one (m, l, o) partial per CTA for the combine.
#include "rkv_device.cuh"
#include "rkv_kernels.h"
#include "rkv_risk.cuh"

namespace rkv {
namespace {

// Summary tiles per warp fetched into L2 ahead of the stats kernel's
// dependency wait (two per warp: about 38 MB over a full B200 at D 128).
constexpr int kStatsPrefetch = 2;
// Normaliser partials each lane loads before merging any of them.
constexpr int kNormBatch = 8;

// ------------------------------- phase A ----------------------------------

// PACK4 (groups of at most 4 rows): q and q^2 share one n8 tile, see
// score_tile_pair; each lane then finishes 4 (block, row) elements.
template <int D, int NT, bool PACK4>
__global__ void __launch_bounds__(NT == 1 ? 384 : 256) stats_kernel(const __grid_constant__ StatsMaps maps,
                                                    const StatsParams p) {
  constexpr int R = kSelectTile;
  constexpr int kTile = R * D * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  uint8_t* tiles = smem;  // [warp][stage][key_mean | ellipsoid]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + warps * S * 2 * kTile);

  const int ih = blockIdx.x;  // instance * heads + head
  const int inst = ih / p.heads, h = ih - inst * p.heads;
  const int t0 = blockIdx.y * p.tiles_per_cta;
  const int t1_all = min(p.tiles, t0 + p.tiles_per_cta);
  const int mine_all = t1_all - t0 > warp ? (t1_all - t0 - warp + warps - 1) / warps : 0;
  const int64_t* counts = p.counts + static_cast<size_t>(p.seq.sequence(h)) * p.blocks;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&maps.key_mean);
    tma_prefetch_desc(&maps.ellipsoid);
  }
  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[warp * S + s], 1);
    mbar_fence_init();
    // The summaries do not change during decode: this warp's first tiles go
    // to L2 before the dependency wait, so their first-touch latency
    // overlaps the previous kernel's tail (nothing is consumed before it).
    for (int j = 0; j < min(kStatsPrefetch, mine_all); ++j) {
      const int row = (t0 + warp + j * warps) * R;
      tma_prefetch_tile<D>(&maps.key_mean, row, h);
      tma_prefetch_tile<D>(&maps.ellipsoid, row, h);
    }
  }
  // Token counts of the same tiles (lanes 0, 16 and 31 cover a tile's
  // 256 bytes) and the query rows (which the previous kernel may still be
  // writing: a prefetch only warms L2 and the translation, it returns no data).
  if (lane == 0 || lane == 16 || lane == 31) {
    for (int j = 0; j < min(kStatsPrefetch, mine_all); ++j) {
      prefetch_l2(counts + min((t0 + warp + j * warps) * R + lane, p.blocks - 1));
    }
  }
  const char* q = static_cast<const char*>(p.query) +
                  static_cast<size_t>(ih) * p.group * p.dim * (p.query_f32 ? 4 : 2);
  for (int i = threadIdx.x; i * 128 < p.group * p.dim * (p.query_f32 ? 4 : 2); i += blockDim.x) {
    prefetch_l2(q + i * 128);
  }
  __syncwarp();
  pdl_wait();
  pdl_launch_dependents();
  // A batched row stops at its own sequence's blocks (tiles wholly past them
  // are skipped; their partial slots stay empty).
  const int blocks_h = p.seq.blocks(h, p.blocks);
  const int t1 = max(t0, min(t1_all, (blocks_h + R - 1) / R));
  const int mine = t1 - t0 > warp ? (t1 - t0 - warp + warps - 1) / warps : 0;

  // Key-mean and ellipsoid tiles are read once per step: evict them first so
  // that z and delta, which the next kernel reads, stay in L2 at long
  // contexts (the tiles of a 1M-token layer outsize L2).
  const uint64_t stream_policy = l2_evict_first_policy();
  auto issue = [&](int j) {
    const int s = j % S;
    uint8_t* dst = tiles + (warp * S + s) * 2 * kTile;
    const int row = (t0 + warp + j * warps) * R;
    mbar_expect_tx(&bars[warp * S + s], 2 * kTile);
    tma_tile_hint<D>(dst, &maps.key_mean, &bars[warp * S + s], row, h, R, stream_policy);
    tma_tile_hint<D>(dst + kTile, &maps.ellipsoid, &bars[warp * S + s], row, h, R, stream_policy);
  };
  if (lane == 0) {
    for (int j = 0; j < min(S, mine); ++j) issue(j);
  }

  // This lane's block rows within a tile (the C-fragment rows it finishes).
  constexpr int kHalves = PACK4 ? 1 : 2;
  int lane_rows[R / 16][2];
#pragma unroll
  for (int mt = 0; mt < R / 16; ++mt) {
    lane_rows[mt][0] = mt * 16 + (lane >> 2) + (PACK4 && ((lane >> 1) & 1) ? 8 : 0);
    lane_rows[mt][1] = lane_rows[mt][0] + 8;
  }
  // Token counts of this lane's blocks in tile j; the first tile's are
  // requested before the query, then each next tile's one step ahead.
  auto load_counts = [&](int j, long long (&c)[R / 16][2]) {
    const int tile = t0 + warp + j * warps;
#pragma unroll
    for (int mt = 0; mt < R / 16; ++mt)
#pragma unroll
      for (int hf = 0; hf < kHalves; ++hf) {
        const int b = tile * R + lane_rows[mt][hf];
        c[mt][hf] = (j < mine && b < blocks_h) ? __ldg(counts + b) : 1;
      }
  };
  long long cnt_next[R / 16][2];
  load_counts(0, cnt_next);

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

  int issued = min(S, mine);
  for (int j = 0; j < mine; ++j) {
    const int s = j % S;
    const int tile = t0 + warp + j * warps;
    long long cnt[R / 16][2];
#pragma unroll
    for (int mt = 0; mt < R / 16; ++mt)
#pragma unroll
      for (int hf = 0; hf < kHalves; ++hf) cnt[mt][hf] = cnt_next[mt][hf];
    load_counts(j + 1, cnt_next);
    if (!warp_wait(&bars[warp * S + s], (j / S) & 1)) {
      if (lane == 0) atomicOr(p.status, kStatusTimeout);
      drain_pending(bars + warp * S, S, j, issued);
      break;
    }
    const uint32_t base = smem_addr(tiles + (warp * S + s) * 2 * kTile);
    // Per element: score (q.kbar) and projection (q^2.W2) of (block row, group row).
    float sc[R / 16][NT][4], pr[R / 16][NT][4];
    int row_of[R / 16][2];  // this lane's block rows per m-tile and half
    int g_base;             // group row of element column j is g_base + j (PACK4)
    if constexpr (PACK4) {
      float acc[R / 16][4];
      score_tile_pair<R, D>(base, base + kTile, packed, acc, lane);
      const bool upper = (lane >> 1) & 1;  // holds q^2.W2 before the exchange
#pragma unroll
      for (int mt = 0; mt < R / 16; ++mt) {
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
      score_tile<R, D, NT>(base, qk, sc, lane);
      score_tile<R, D, NT>(base + kTile, q2, pr, lane);
#pragma unroll
      for (int mt = 0; mt < R / 16; ++mt) {
        row_of[mt][0] = mt * 16 + (lane >> 2);
        row_of[mt][1] = row_of[mt][0] + 8;
      }
      g_base = 0;
    }
    __syncwarp();
    if (j + S < mine) {
      if (lane == 0) {
        fence_proxy_async();
        issue(j + S);
      }
      ++issued;
    }
    // z and z + log cosh(delta) of every element first (independent), then
    // one (max, sum) update per column: no serial exp chain.
    float zv[R / 16][NT][4], cv[R / 16][NT][4];
#pragma unroll
    for (int mt = 0; mt < R / 16; ++mt) {
#pragma unroll
      for (int hf = 0; hf < kHalves; ++hf) {
        const int b = tile * R + row_of[mt][hf];
        const float log_count = b < blocks_h ? flog(static_cast<float>(cnt[mt][hf])) : 0.f;
#pragma unroll
        for (int jc = 0; jc < 2; ++jc) {
          const int c = 2 * hf + jc;
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int g = PACK4 ? g_base + jc : nt * 8 + 2 * (lane & 3) + jc;
            zv[mt][nt][c] = -INFINITY;
            cv[mt][nt][c] = -INFINITY;
            if (b >= blocks_h || g >= p.group) continue;
            const float score = sc[mt][nt][c] * p.scale;
            const float proj = pr[mt][nt][c];
            const float delta = (sqrtf(proj < 0.f ? 0.f : proj) * p.scale) * kInflate;
            const float z = score + log_count;
            const size_t rowg = static_cast<size_t>(ih) * p.group + g;
            p.z[rowg * p.blocks + b] = z;
            p.delta[rowg * p.blocks + b] = delta;
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
        for (int mt = 0; mt < R / 16; ++mt)
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
        for (int mt = 0; mt < R / 16; ++mt)
#pragma unroll
          for (int hf = 0; hf < kHalves; ++hf) {
            sz += fexp(zv[mt][nt][2 * hf + jc] - rz);
            sc2 += fexp(cv[mt][nt][2 * hf + jc] - rc);
          }
        if (nan) sz = sc2 = NAN;  // a NaN row statistic must stay non-finite
        lse_merge(zm[nt][jc], zs[nt][jc], tz, sz);
        lse_merge(cm[nt][jc], cs[nt][jc], tc, sc2);
      }
  }

  // One (max, sum) pair per warp and column: reduce the maxima over the
  // lanes that share a column (8 lanes; 16 with PACK4), rescale each lane's
  // sum once, add the sums.  Each warp writes its own partial (slot
  // part * slots + warp), so there is no CTA barrier; slots past the CTA's
  // warp count (a fixed count under a sequence split) are left empty.
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
      if (writer && g < p.group) {
        float* out = p.lse + ((static_cast<size_t>(ih) * p.group + g) * p.parts * p.slots +
                              static_cast<size_t>(blockIdx.y) * p.slots + warp) * 4;
        *reinterpret_cast<float4*>(out) = make_float4(mz, sz, mc, sc);
      }
    }
  if (warp == 0 && p.slots > warps) {
    for (int i = lane; i < p.group * (p.slots - warps); i += 32) {
      const int g = i / (p.slots - warps), w = warps + i % (p.slots - warps);
      float* out = p.lse + ((static_cast<size_t>(ih) * p.group + g) * p.parts * p.slots +
                            static_cast<size_t>(blockIdx.y) * p.slots + w) * 4;
      *reinterpret_cast<float4*>(out) = make_float4(-INFINITY, 0.f, -INFINITY, 0.f);
    }
  }
}

// ------------------------------- phase B ----------------------------------

// GM = group rows evaluated per block (the group padded to 4, 8 or 16); the
// padding rows repeat row 0 and are masked out of the reduction, which keeps
// the per-row risk evaluations branch-free and independent.
template <int D, int NT, int GM>
__global__ void __launch_bounds__(NT == 1 ? 384 : 256) final_kernel(const __grid_constant__ FinalMaps maps,
                                                    const FinalParams p) {
  constexpr int R = kSelectTile;
  constexpr int kTile = R * D * 2;
  constexpr int G8 = NT * 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem(smem_raw);
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = p.stages;
  const int ntiles = p.tiles_per_cta;
  uint8_t* tiles = smem;  // [warp][stage] value_mean tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + warps * S * kTile);
  float* log_z = reinterpret_cast<float*>(smem + warps * S * kTile +
                                          round16(static_cast<size_t>(warps) * S * 8));
  float* log_c = log_z + kMaxGroup;
  uint32_t* sel_bits = reinterpret_cast<uint32_t*>(log_c + kMaxGroup);  // [ntiles]
  uint32_t* rep_bits = sel_bits + ntiles;                               // [ntiles]
  int* offsets = reinterpret_cast<int*>(rep_bits + ntiles);             // [ntiles + 1]
  int* rep_list = offsets + ntiles + 1;                                 // [ntiles]
  int* flags = rep_list + ntiles;                                       // [4]
  float* st_m = reinterpret_cast<float*>(flags + 4);                    // [warps][G8]
  float* st_l = st_m + warps * G8;
  float* st_o = st_l + warps * G8;  // [warps][G8][D]

  const int ih = blockIdx.x;
  const int inst = ih / p.heads, h = ih - inst * p.heads;
  (void)inst;
  const int part = blockIdx.y;
  const int t0 = part * p.tiles_per_cta;
  const int t1 = min(p.tiles, t0 + p.tiles_per_cta);

  if (p.decode && lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[warp * S + s], 1);
    mbar_fence_init();
  }
  if (threadIdx.x == 0) {
    flags[0] = 0;
    if (p.decode) tma_prefetch_desc(&maps.value_mean);
  }
  // The value-mean tiles of the CTA's range (read by the representative
  // softmax after the decisions) go to L2 before the dependency wait, while
  // DRAM idles through the stats kernel's tail and the decisions.
  if (p.decode && lane == 0) {
    for (int t = t0 + warp; t < t1; t += warps) tma_prefetch_tile<D>(&maps.value_mean, t * R, h);
  }
  // Value norms and anchor bits do not change during decode: the lines of
  // this warp's first two tiles go to L2 before the dependency wait (the
  // first and last lane's addresses cover a tile's lines).
  if (lane == 0 || lane == 31) {
    for (int j = 0; j < 2; ++j) {
      const int t = t0 + warp + j * warps;
      const int b = min(t * R + lane, p.blocks - 1);
      if (t < t1) {
        prefetch_l2(p.value_norm + static_cast<size_t>(h) * p.blocks + b);
        if (p.anchor != nullptr) prefetch_l2(p.anchor + static_cast<size_t>(h) * p.blocks + b);
      }
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_launch_dependents();
  // A batched row's blocks past its own prompt are padding: never selected
  // or represented, their mask bytes written 0.
  const int blocks_h = p.seq.blocks(h, p.blocks);

  // Pass-1 inputs of a tile (one lane per block): z and delta of every row,
  // the value norm and the anchor bit.  Three buffers rotate by name through
  // a loop unrolled three times, so the loads of the tile two steps ahead
  // are in flight while the current tile is decided (a register copy at the
  // end of each iteration would wait for them).
  struct TileIn {
    float z[GM], d[GM], vn;
    bool anc;
  };
  auto load_tile = [&](int t, TileIn& in) {
    const int b = t * R + lane;
    if (t < t1 && b < blocks_h) {
      in.vn = p.value_norm[static_cast<size_t>(h) * p.blocks + b];
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        const size_t row = static_cast<size_t>(ih) * p.group + (g < p.group ? g : 0);
        in.z[g] = p.z[row * p.blocks + b];
        in.d[g] = p.delta[row * p.blocks + b];
      }
      in.anc = p.anchor != nullptr && p.anchor[static_cast<size_t>(h) * p.blocks + b] != 0;
    }
  };
  TileIn buf_a, buf_b, buf_c;
  load_tile(t0 + warp, buf_a);
  load_tile(t0 + warp + warps, buf_b);

  // Row-global normalisers from the phase-A partials (of every rank's slab
  // under a sequence split): one warp per row, lanes load partials in
  // parallel and merge them with shuffles.
  for (int g = warp; g < p.group; g += warps) {
    const float* in = p.lse + (static_cast<size_t>(ih) * p.group + g) * p.parts_a * 4;
    float m0 = -INFINITY, s0 = 0.f, m1 = -INFINITY, s1 = 0.f;
    const int n_part = p.parts_a * p.lse_slabs;
    for (int k0 = lane; k0 < n_part; k0 += 32 * kNormBatch) {
      float4 v[kNormBatch];  // all of a batch's loads in flight before any merge
#pragma unroll
      for (int u = 0; u < kNormBatch; ++u) {
        const int k = k0 + 32 * u;
        const int slab = k / p.parts_a, part_k = k - slab * p.parts_a;
        v[u] = k < n_part
                   ? *reinterpret_cast<const float4*>(in + slab * p.lse_slab_floats + 4 * part_k)
                   : make_float4(-INFINITY, 0.f, -INFINITY, 0.f);
      }
#pragma unroll
      for (int u = 0; u < kNormBatch; ++u) {
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
      const float lz = m0 + flog(s0);
      const float lc = m1 + flog(s1);
      log_z[g] = lz;
      log_c[g] = lc;
      if (!finite(lz) || !finite(lc)) atomicOr(&flags[0], 1);
    }
  }
  __syncthreads();
  const bool bad_global = flags[0] != 0;
  const float vmax = p.max_value_norm[h];

  // Pass 1: decisions, one lane per block.
  auto decide = [&](int t, const TileIn& in) {
    const int b = t * R + lane;
    const bool valid = b < blocks_h;
    bool sel = false;
    if (valid) {
      float lz[GM], lc[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        const int gg = g < p.group ? g : 0;
        lz[g] = log_z[gg];
        lc[g] = log_c[gg];
      }
      float risk[GM];
#pragma unroll
      for (int g = 0; g < GM; ++g)
        risk[g] = block_risk(in.z[g], in.d[g], lz[g], lc[g], in.vn, vmax);
      float agg = p.reduction == kMax ? -INFINITY : 0.f;
      bool any = false, bad = false;
#pragma unroll
      for (int g = 0; g < GM; ++g) {
        if (g >= p.group) continue;
        const float r = risk[g];
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
      sel = dec || bad || bad_global || in.anc;
    }
    if (b < p.blocks) {
      uint8_t* mk = p.mask + static_cast<size_t>(h) * p.blocks + b;
      if (p.accumulate) {
        if (sel) *mk = 1;
      } else {
        *mk = sel ? 1 : 0;
      }
    }
    const uint32_t sb = __ballot_sync(0xffffffffu, sel);
    const uint32_t vb = __ballot_sync(0xffffffffu, valid);
    if (lane == 0) {
      sel_bits[t - t0] = sb;
      rep_bits[t - t0] = vb & ~sb;
    }
  };
  for (int t = t0 + warp; t < t1; t += 3 * warps) {
    load_tile(t + 2 * warps, buf_c);
    decide(t, buf_a);
    if (t + warps >= t1) break;
    load_tile(t + 3 * warps, buf_a);
    decide(t + warps, buf_b);
    if (t + 2 * warps >= t1) break;
    load_tile(t + 4 * warps, buf_b);
    decide(t + 2 * warps, buf_c);
  }
  if (!p.decode) return;
  __syncthreads();

  // Deterministic compaction: tile offsets in block order, and the list of
  // tiles holding at least one representative (rank k goes to warp k % warps).
  // Warp 0 scans 32 tiles at a time: a shuffle prefix sum of the selected
  // counts and a ballot rank for the representative list.
  if (warp == 0) {
    const int n_t = t1 - t0;
    int acc = 0, reps = 0;
    for (int k0 = 0; k0 < n_t; k0 += 32) {
      const int k = k0 + lane;
      const int c = k < n_t ? __popc(sel_bits[k]) : 0;
      const bool has_rep = k < n_t && rep_bits[k] != 0u;
      int incl = c;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      if (k < n_t) offsets[k] = acc + incl - c;
      acc += __shfl_sync(0xffffffffu, incl, 31);
      const uint32_t rb = __ballot_sync(0xffffffffu, has_rep);
      if (has_rep) rep_list[reps + __popc(rb & ((1u << lane) - 1u))] = k;
      reps += __popc(rb);
    }
    if (lane == 0) {
      offsets[n_t] = acc;
      flags[1] = reps;
      p.seg_count[h * p.parts + part] = acc;
    }
  }
  __syncthreads();
  int* ids = p.sel_ids + (static_cast<size_t>(h) * p.parts + part) * p.seg_cap;
  for (int t = t0 + warp; t < t1; t += warps) {
    const uint32_t sb = sel_bits[t - t0];
    if ((sb >> lane) & 1u) ids[offsets[t - t0] + __popc(sb & ((1u << lane) - 1u))] = t * R + lane;
  }

  const int n_reps = flags[1];
  const size_t slot = static_cast<size_t>(h) * p.parts + part;
  if (n_reps == 0) {  // nothing to represent: an empty partial (weight 0 in the combine)
    if (threadIdx.x < G8) {
      p.rep_m[slot * G8 + threadIdx.x] = -INFINITY;
      p.rep_l[slot * G8 + threadIdx.x] = 0.f;
    }
    return;
  }
  const int mine = n_reps > warp ? (n_reps - warp + warps - 1) / warps : 0;
  const uint64_t stream_policy = l2_evict_first_policy();
  auto issue = [&](int j) {
    const int s = j % S;
    mbar_expect_tx(&bars[warp * S + s], kTile);
    tma_tile_hint<D>(tiles + (warp * S + s) * kTile, &maps.value_mean, &bars[warp * S + s],
                     (t0 + rep_list[warp + j * warps]) * R, h, R, stream_policy);
  };
  // Logits (z) of the representatives of this warp's j-th tile; loaded one
  // tile ahead so their latency overlaps the current tile's work.
  auto load_logits = [&](int j, float (&lg)[R / 16][NT][4]) {
    const bool have = j < mine;
    const int k = have ? rep_list[warp + j * warps] : 0;
    const uint32_t reps = have ? rep_bits[k] : 0u;
    const int tile = t0 + k;
#pragma unroll
    for (int mt = 0; mt < R / 16; ++mt)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int r = mt * 16 + (lane >> 2) + (c >> 1) * 8;
        const bool rep = (reps >> r) & 1u;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const int g = nt * 8 + 2 * (lane & 3) + (c & 1);
          lg[mt][nt][c] =
              (rep && g < p.group)
                  ? p.z[(static_cast<size_t>(ih) * p.group + g) * p.blocks + tile * R + r]
                  : -INFINITY;
        }
      }
  };
  int issued = min(S, mine);
  if (lane == 0) {
    for (int j = 0; j < issued; ++j) issue(j);
  }
  float m[NT][2], l[NT][2], o[D / 16][NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    m[nt][0] = m[nt][1] = -INFINITY;
    l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
    for (int dt = 0; dt < D / 16; ++dt) o[dt][nt][0] = o[dt][nt][1] = o[dt][nt][2] = o[dt][nt][3] = 0.f;
  }
  float next_logit[R / 16][NT][4];
  load_logits(0, next_logit);
  for (int j = 0; j < mine; ++j) {
    const int s = j % S;
    if (!warp_wait(&bars[warp * S + s], (j / S) & 1)) {
      if (lane == 0) atomicOr(p.status, kStatusTimeout);
      drain_pending(bars + warp * S, S, j, issued);
      break;
    }
    float logit[R / 16][NT][4];
#pragma unroll
    for (int mt = 0; mt < R / 16; ++mt)
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) logit[mt][nt][c] = next_logit[mt][nt][c];
    load_logits(j + 1, next_logit);
    attend_tile<R, D, NT>(logit, smem_addr(tiles + (warp * S + s) * kTile), m, l, o,
                          p.split_probs != 0, lane);
    __syncwarp();
    if (j + S < mine) {
      if (lane == 0) {
        fence_proxy_async();
        issue(j + S);
      }
      ++issued;
    }
  }
  reduce_l<NT>(l);
  stash_warp_partial<D, NT>(st_m, st_l, st_o, warp, lane, m, l, o);
  __syncthreads();
  merge_stashed<D>(st_m, st_l, st_o, warps, G8, p.rep_m + slot * G8, p.rep_l + slot * G8,
                   p.rep_o + slot * G8 * D, threadIdx.x, blockDim.x);
}

template <typename Kernel, typename Maps, typename Params>
cudaError_t launch_k(Kernel kernel, const Maps& maps, const Params& p, dim3 grid, int warps,
                     size_t smem, cudaStream_t stream, bool pdl) {
  cudaError_t err = ensure_smem_limit(reinterpret_cast<const void*>(kernel), smem);
  if (err != cudaSuccess) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
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

template <int D>
cudaError_t stats_dispatch(const StatsMaps& maps, const StatsParams& p, int warps, size_t smem,
                           cudaStream_t stream, bool pdl) {
  const dim3 grid(p.instances * p.heads, p.parts);
  if (p.group <= 4) {
    return launch_k(stats_kernel<D, 1, true>, maps, p, grid, warps, smem, stream, pdl);
  }
  if (p.group <= 8) {
    return launch_k(stats_kernel<D, 1, false>, maps, p, grid, warps, smem, stream, pdl);
  }
  return launch_k(stats_kernel<D, 2, false>, maps, p, grid, warps, smem, stream, pdl);
}

template <int D>
cudaError_t final_dispatch(const FinalMaps& maps, const FinalParams& p, int warps, size_t smem,
                           cudaStream_t stream, bool pdl) {
  const dim3 grid(p.instances * p.heads, p.parts);
  if (p.group <= 4) return launch_k(final_kernel<D, 1, 4>, maps, p, grid, warps, smem, stream, pdl);
  if (p.group <= 8) return launch_k(final_kernel<D, 1, 8>, maps, p, grid, warps, smem, stream, pdl);
  return launch_k(final_kernel<D, 2, 16>, maps, p, grid, warps, smem, stream, pdl);
}

}  // namespace

size_t stats_smem_bytes(int dim, int warps, int stages, int group) {
  (void)group;
  return kSmemSlack + static_cast<size_t>(warps) * stages * 2 * kSelectTile * dim * 2 +
         round16(static_cast<size_t>(warps) * stages * 8);
}

size_t final_smem_bytes(int dim, int warps, int stages, int group, int tiles_per_cta) {
  const int g8 = group <= 8 ? 8 : 16;
  size_t bytes = kSmemSlack + static_cast<size_t>(warps) * stages * kSelectTile * dim * 2;
  bytes += round16(static_cast<size_t>(warps) * stages * 8);
  bytes += 2 * kMaxGroup * 4;
  bytes += static_cast<size_t>(tiles_per_cta) * 4 * 4 + 4 + 16;
  bytes += static_cast<size_t>(warps) * g8 * 4 * 2 + static_cast<size_t>(warps) * g8 * dim * 4;
  return bytes;
}

cudaError_t launch_stats(const StatsMaps& maps, const StatsParams& p, int dim, int warps,
                         size_t smem, cudaStream_t stream, bool pdl) {
  switch (dim) {
    case 64: return stats_dispatch<64>(maps, p, warps, smem, stream, pdl);
    case 128: return stats_dispatch<128>(maps, p, warps, smem, stream, pdl);
    case 192: return stats_dispatch<192>(maps, p, warps, smem, stream, pdl);
    case 256: return stats_dispatch<256>(maps, p, warps, smem, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_final(const FinalMaps& maps, const FinalParams& p, int dim, int warps,
                         size_t smem, cudaStream_t stream, bool pdl) {
  switch (dim) {
    case 64: return final_dispatch<64>(maps, p, warps, smem, stream, pdl);
    case 128: return final_dispatch<128>(maps, p, warps, smem, stream, pdl);
    case 192: return final_dispatch<192>(maps, p, warps, smem, stream, pdl);
    case 256: return final_dispatch<256>(maps, p, warps, smem, stream, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace rkv
