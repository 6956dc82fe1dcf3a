// Training kernels for the oblivious-tree hot path on sm_100a.
//
// Per boosting round (src/booster.rs:349-501 is the reference's sequence):
//   k_grad / GOSS           gradients, row sampling, per-round max |g| and max h
//   [ncclAllReduce max]     multi-GPU: global maxima (the fixed-point scales)
//   k_quant                 per-row fixed-point q(g), q(h), excluded flag, level-0 slots
//   per level d:
//     k_hist                exact fixed-point histogram of the built nodes
//     [ncclAllReduce]       multi-GPU: sum of the built histograms (int64, exact)
//     k_split               derive sibling nodes, f64 gain scan, argmax, model write,
//                           leaf values at the last level (no separate leaf pass)
//     k_apply               leaf = 2*leaf + (bin > t) and the next level's build slot;
//                           at the last level pred += leafval[leaf]
//
// Exactness: histogram cells are int64 sums of per-row fixed-point values
// q = round(x * 2^e) (rw_expf.h). Shared memory holds the low 32 bits of each cell as
// an int32 atomic accumulator biased by 2^31; the rare carries out of the low word are
// added to the global int64 cell as +-2^32, and the low words are flushed at the end.
// The result equals the int64 sum of q over the contributing rows regardless of
// scheduling, so histograms, splits and leaf values are bit-identical run to run and
// at every GPU count.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "rw_expf.h"
#include "rw_internal.cuh"

#define RW_INF __longlong_as_double(0x7ff0000000000000LL)

namespace {

constexpr int kHistThreads = 512;
constexpr uint32_t kBias = 0x80000000u;
constexpr int kHistSmemBudget = 112 * 1024;  // two CTAs per SM
constexpr int kTargetCtas = 2 * 148;
constexpr int kMaxCluster = 8;

namespace cg = cooperative_groups;

struct HistArgs {
  const uint8_t* bins;
  uint64_t ld;
  const int16_t* slot;
  const int32_t* qg;
  const int32_t* qh;
  uint64_t n_pad;
  uint32_t nf, nb;
  uint32_t gchunk;  // groups per CTA (blockIdx.z selects the chunk)
  long long* out;
  uint64_t rows_per_cta;
};

// Adds ±2^32 to the global cell when the 32-bit shared accumulator wrapped in the add
// of q that returned `old` (the shared word holds the cell's low 32 bits + 2^31).
__device__ __forceinline__ void carry_out(uint32_t old, int32_t q, long long* gcell) {
  const uint32_t nw = old + (uint32_t)q;
  const int delta = (nw < old ? 1 : 0) - (q < 0 ? 1 : 0);
  if (delta != 0)
    atomicAdd(reinterpret_cast<unsigned long long*>(gcell),
              (unsigned long long)((long long)delta * 4294967296LL));
}

// A wrap is only possible when the returned low word is within 2^26 (>= |q|) of the
// 32-bit boundary, i.e. old + 2^26 (mod 2^32) < 2^27.
__device__ __forceinline__ bool near_edge(uint32_t og, uint32_t oh) {
  return min(og + (1u << 26), oh + (1u << 26)) < (1u << 27);
}

// One CTA: feature tile [blockIdx.y*FT, +FT) x group chunk x row range, in a cluster of
// CTAs along the row ranges. Lane (k, j) handles feature j of the tile for row slot k;
// each thread covers 4 consecutive rows per step (one u32 of u8 bins, or one u16 of
// 4-bit bins). Shared cells are laid out [group][bin][FT]: the FT lanes of one row hit
// FT distinct banks. After the rows, the cluster's CTAs sum their shared histograms
// through distributed shared memory, each CTA flushing a slice to the global int64
// histogram, so a cell costs one global atomic per cluster rather than per CTA.
template <int FT, bool PACKED>
__global__ void __launch_bounds__(kHistThreads, 2) k_hist(HistArgs a) {
  extern __shared__ uint32_t smem[];
  const uint32_t G = a.gchunk, nb = a.nb;
  const uint32_t cells = G * nb * FT;
  uint32_t* lo_g = smem;
  uint32_t* lo_h = smem + cells;
  for (uint32_t i = threadIdx.x; i < 2 * cells; i += kHistThreads) smem[i] = kBias;
  __syncthreads();

  constexpr int RW = 32 / FT;
  constexpr int kStep = (kHistThreads / 32) * RW * 4;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = lane % FT, k = lane / FT;
  const uint32_t f0 = blockIdx.y * FT;
  const uint32_t f = f0 + j;
  const bool fvalid = f < a.nf;
  const int g0 = (int)(blockIdx.z * a.gchunk);
  const uint8_t* col = a.bins + (size_t)(fvalid ? f : 0) * a.ld;
  long long* outf = a.out + (size_t)(fvalid ? f : 0) * nb * 2;
  const size_t gstride = (size_t)a.nf * nb * 2;

  const uint64_t r_begin = (uint64_t)blockIdx.x * a.rows_per_cta;
  uint64_t r_end = r_begin + a.rows_per_cta;
  if (r_end > a.n_pad) r_end = a.n_pad;

  for (uint64_t rb = r_begin + (uint64_t)(warp * RW + k) * 4; rb < r_end; rb += kStep) {
    const uint2 sl2 = *reinterpret_cast<const uint2*>(a.slot + rb);
    const int4 qg4 = *reinterpret_cast<const int4*>(a.qg + rb);
    const int4 qh4 = *reinterpret_cast<const int4*>(a.qh + rb);
    uint32_t b4;
    if (PACKED) {
      const uint32_t p = *reinterpret_cast<const uint16_t*>(col + (rb >> 1));
      b4 = (p & 0xfu) | ((p & 0xf0u) << 4) | ((p & 0xf00u) << 8) | ((p & 0xf000u) << 12);
    } else {
      b4 = *reinterpret_cast<const uint32_t*>(col + rb);
    }
    const int sl[4] = {(int)(int16_t)(sl2.x & 0xffffu), (int)(int16_t)(sl2.x >> 16),
                       (int)(int16_t)(sl2.y & 0xffffu), (int)(int16_t)(sl2.y >> 16)};
    const int32_t qg[4] = {qg4.x, qg4.y, qg4.z, qg4.w};
    const int32_t qh[4] = {qh4.x, qh4.y, qh4.z, qh4.w};
    uint32_t og[4], oh[4], cell[4];
    bool act[4];
#pragma unroll
    for (int s = 0; s < 4; s++) {
      const uint32_t grp = (uint32_t)(sl[s] - g0);
      act[s] = fvalid && grp < G;
      cell[s] = (grp * nb + ((b4 >> (8 * s)) & 0xffu)) * FT + j;
      if (act[s]) {
        og[s] = atomicAdd(&lo_g[cell[s]], (uint32_t)qg[s]);
        oh[s] = atomicAdd(&lo_h[cell[s]], (uint32_t)qh[s]);
      }
    }
#pragma unroll
    for (int s = 0; s < 4; s++) {
      if (act[s] && near_edge(og[s], oh[s])) {
        const uint32_t bin = (b4 >> (8 * s)) & 0xffu;
        long long* gc = outf + (size_t)sl[s] * gstride + (size_t)bin * 2;
        carry_out(og[s], qg[s], gc);
        carry_out(oh[s], qh[s], gc + 1);
      }
    }
  }

  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const uint32_t cn = cluster.num_blocks(), cr = cluster.block_rank();
  const uint32_t words = 2 * cells;
  const uint32_t per = (words + cn - 1) / cn;
  const uint32_t w_begin = cr * per, w_end = min(words, w_begin + per);
  for (uint32_t w = w_begin + threadIdx.x; w < w_end; w += kHistThreads) {
    long long v = 0;
    for (uint32_t r = 0; r < cn; r++) {
      const uint32_t* remote = cluster.map_shared_rank(smem, (int)r);
      v += (long long)remote[w] - (long long)kBias;
    }
    if (v == 0) continue;
    const uint32_t c = w < cells ? w : w - cells;
    const uint32_t jj = c % FT, rest = c / FT, bin = rest % nb, grp = rest / nb;
    const uint32_t ff = f0 + jj;
    if (ff >= a.nf) continue;
    long long* gc = a.out + (size_t)(g0 + grp) * gstride + ((size_t)ff * nb + bin) * 2 +
                    (w < cells ? 0 : 1);
    atomicAdd(reinterpret_cast<unsigned long long*>(gc), (unsigned long long)v);
  }
  cluster.sync();  // keep this CTA's shared memory alive until every reader is done
}

template <int FT, bool PACKED>
cudaError_t launch_hist_t(const HistArgs& args, dim3 grid, int cluster, size_t smem,
                          cudaStream_t s) {
  cudaError_t e = cudaFuncSetAttribute(k_hist<FT, PACKED>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kHistThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k_hist<FT, PACKED>, args);
}

template <bool PACKED>
cudaError_t launch_hist_ft(int ft, const HistArgs& args, dim3 grid, int cluster, size_t smem,
                           cudaStream_t s) {
  switch (ft) {
    case 32: return launch_hist_t<32, PACKED>(args, grid, cluster, smem, s);
    case 16: return launch_hist_t<16, PACKED>(args, grid, cluster, smem, s);
    case 8: return launch_hist_t<8, PACKED>(args, grid, cluster, smem, s);
    case 4: return launch_hist_t<4, PACKED>(args, grid, cluster, smem, s);
    case 2: return launch_hist_t<2, PACKED>(args, grid, cluster, smem, s);
    default: return launch_hist_t<1, PACKED>(args, grid, cluster, smem, s);
  }
}

// --------------------------------------------------------------------------------
// Split scan: one CTA per feature; its 32 warps take 32 nodes at a time (one node per
// warp), lanes take 8 consecutive bins. Per-node gain terms go to shared memory and
// each bin's thread adds them in node order, as src/cpu.rs:242-259 does.

constexpr int kSplitThreads = 1024;
constexpr int kSplitWarps = kSplitThreads / 32;

struct SplitSmem {
  double term[kSplitWarps][256];
  long long mono[4][256];  // exact left/right (g, h) totals over nodes (monotone only)
  double red_g[kSplitWarps];
  uint32_t red_i[kSplitWarps];
  int last;
  uint32_t s_f, s_b;
};

__device__ __forceinline__ long long shfl_up_ll(long long v, int d) {
  return __shfl_up_sync(0xffffffffu, v, d);
}

__device__ __forceinline__ uint32_t hash01_bits(uint32_t id, uint32_t seed) {
  // src/gpu_kernels.rs hash01 (salted integer hash of (id, seed)).
  uint32_t x = id * 2654435761u + (seed ^ 0x455A4B41u);
  x ^= x >> 15;
  x *= 2246822519u;
  x ^= x >> 13;
  return x & 0x00FFFFFFu;
}

// Keep (g1, i1) if strictly greater, ties to the lower index.
__device__ __forceinline__ void argmax_merge(double& g, uint32_t& i, double g2, uint32_t i2) {
  if (g2 > g || (g2 == g && i2 < i)) {
    g = g2;
    i = i2;
  }
}

// Block-wide argmax; the result is valid in thread 0.
__device__ void block_argmax(double& g, uint32_t& i, SplitSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double g2 = __shfl_down_sync(0xffffffffu, g, off);
    const uint32_t i2 = __shfl_down_sync(0xffffffffu, i, off);
    if (lane + off < 32) argmax_merge(g, i, g2, i2);
  }
  if (lane == 0) {
    sm.red_g[warp] = g;
    sm.red_i[warp] = i;
  }
  __syncthreads();
  if (warp == 0) {
    g = lane < kSplitWarps ? sm.red_g[lane] : -RW_INF;
    i = lane < kSplitWarps ? sm.red_i[lane] : 0xffffffffu;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const double g2 = __shfl_down_sync(0xffffffffu, g, off);
      const uint32_t i2 = __shfl_down_sync(0xffffffffu, i, off);
      if (lane + off < 32) argmax_merge(g, i, g2, i2);
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kSplitThreads) k_split(SplitLaunch a) {
  extern __shared__ __align__(16) unsigned char split_raw[];
  SplitSmem& sm = *reinterpret_cast<SplitSmem*>(split_raw);
  const uint32_t f = blockIdx.x;
  const uint32_t nf = a.nf, nb = a.nb, nsplit = nb - 1;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const double inv_g = 1.0 / (double)rw_pow2f(rw_qscale_exp(a.maxbits[0]));
  const double inv_h = 1.0 / (double)rw_pow2f(rw_qscale_exp(a.maxbits[1]));
  const double lambda = a.lambda, mc = a.min_child;
  const int mono = a.monotone ? a.monotone[f] : 0;

  // The next level's built-histogram buffer is zeroed here (this CTA's slice).
  if (a.hb_next) {
    const uint64_t per = (a.hb_next_words + nf - 1) / nf;
    const uint64_t w0 = (uint64_t)f * per;
    const uint64_t w1 = w0 + per < a.hb_next_words ? w0 + per : a.hb_next_words;
    for (uint64_t w = w0 + threadIdx.x; w < w1; w += kSplitThreads) a.hb_next[w] = 0;
  }
  if (mono)
    for (int i = threadIdx.x; i < 4 * 256; i += kSplitThreads) (&sm.mono[0][0])[i] = 0;

  double gain = 0.0;
  const uint32_t b_self = threadIdx.x;

  for (uint32_t c = 0; c < a.n_nodes; c += kSplitWarps) {
    const uint32_t nd = c + warp;
    if (nd < a.n_nodes) {
      long long vg[8], vh[8];
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint32_t b = lane * 8 + i;
        long long xg = 0, xh = 0;
        if (b < nb) {
          if (a.mode == 0) {
            const long long* p = a.hb + (((size_t)nd * nf + f) * nb + b) * 2;
            xg = p[0];
            xh = p[1];
          } else {
            const long long* po = a.hb + (((size_t)(nd >> 1) * nf + f) * nb + b) * 2;
            if (nd & 1u) {
              xg = po[0];
              xh = po[1];
            } else {
              const long long* pp = a.hp + (((size_t)(nd >> 1) * nf + f) * nb + b) * 2;
              xg = pp[0] - po[0];
              xh = pp[1] - po[1];
            }
          }
          long long* q = a.hf + (((size_t)nd * nf + f) * nb + b) * 2;
          q[0] = xg;
          q[1] = xh;
        }
        vg[i] = xg;
        vh[i] = xh;
      }
#pragma unroll
      for (int i = 1; i < 8; i++) {
        vg[i] += vg[i - 1];
        vh[i] += vh[i - 1];
      }
      long long sg = vg[7], sh = vh[7];
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const long long tg = shfl_up_ll(sg, d), th = shfl_up_ll(sh, d);
        if (lane >= d) {
          sg += tg;
          sh += th;
        }
      }
      const long long eg = sg - vg[7], eh = sh - vh[7];
      const long long totg = __shfl_sync(0xffffffffu, sg, 31);
      const long long toth = __shfl_sync(0xffffffffu, sh, 31);
      const double gt = (double)totg * inv_g;
      const double ht = (double)toth * inv_h;
      const double parent = gt * gt / (ht + lambda);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint32_t b = lane * 8 + i;
        if (b < nsplit) {
          const long long pgi = vg[i] + eg, phi = vh[i] + eh;
          const double gl = (double)pgi * inv_g;
          const double hl = (double)phi * inv_h;
          const double gr = gt - gl, hr = ht - hl;
          const double valid = (double)((hl >= mc) & (hr >= mc));
          sm.term[warp][b] = valid * (gl * gl / (hl + lambda) + gr * gr / (hr + lambda) - parent);
          if (mono) {
            atomicAdd(reinterpret_cast<unsigned long long*>(&sm.mono[0][b]), (unsigned long long)pgi);
            atomicAdd(reinterpret_cast<unsigned long long*>(&sm.mono[1][b]), (unsigned long long)phi);
            atomicAdd(reinterpret_cast<unsigned long long*>(&sm.mono[2][b]),
                      (unsigned long long)(totg - pgi));
            atomicAdd(reinterpret_cast<unsigned long long*>(&sm.mono[3][b]),
                      (unsigned long long)(toth - phi));
          }
        }
      }
    }
    __syncthreads();
    if (b_self < nsplit) {
      const uint32_t cnt = (a.n_nodes - c) < (uint32_t)kSplitWarps ? (a.n_nodes - c) : kSplitWarps;
      for (uint32_t w = 0; w < cnt; w++) gain += sm.term[w][b_self];
    }
    __syncthreads();
  }

  // candidate masks (extensions): per-tree column sampling and monotone direction
  const bool dropped = a.colsample < 1.0f &&
                       (float)hash01_bits(f, a.tree_seed ^ 0x5bd1e995u) / 16777215.0f >=
                           a.colsample;
  double key = -RW_INF;
  if (b_self < nsplit) {
    key = gain;
    if (dropped) key = -1e30;
    else if (mono) {
      const double glt = (double)sm.mono[0][b_self] * inv_g;
      const double hlt = (double)sm.mono[1][b_self] * inv_h;
      const double grt = (double)sm.mono[2][b_self] * inv_g;
      const double hrt = (double)sm.mono[3][b_self] * inv_h;
      const double wl = -glt / (hlt + lambda);
      const double wr = -grt / (hrt + lambda);
      if ((mono > 0 && wl > wr) || (mono < 0 && wl < wr)) key = -1e30;
    }
    if (key != key) key = -RW_INF;  // NaN never wins (cpu.rs: `gv > bg`)
  }
  uint32_t idx = b_self;
  block_argmax(key, idx, sm);
  if (threadIdx.x == 0) {
    a.best_gain[f] = key;
    a.best_bin[f] = key == -RW_INF ? 0u : idx;
    __threadfence();
    const uint32_t ticket = atomicAdd(a.counter, 1u);
    sm.last = ticket == nf - 1;
  }
  __syncthreads();
  if (!sm.last) return;
  __threadfence();

  // Last CTA: argmax across features (lowest feature wins ties) and model write.
  double bk = -RW_INF;
  uint32_t bf = 0xffffffffu;
  for (uint32_t ff = threadIdx.x; ff < nf; ff += kSplitThreads)
    argmax_merge(bk, bf, __ldcg(a.best_gain + ff), ff);
  block_argmax(bk, bf, sm);
  if (threadIdx.x == 0) {
    if (bk == -RW_INF) bf = 0;
    const uint32_t bb = __ldcg(a.best_bin + bf);
    sm.s_f = bf;
    sm.s_b = bb;
    a.feat[a.slot] = bf;
    a.thr[a.slot] = a.cuts[(size_t)bf * nsplit + bb];
    if (a.thr_bin) a.thr_bin[a.slot] = (uint16_t)bb;
    a.split_ft[0] = bf;
    a.split_ft[1] = bb;
    a.fi_gain[bf] += (float)(bk > 0.0 ? bk : 0.0);
    a.fi_count[bf] += 1.0f;
    *a.counter = 0u;
  }
  __syncthreads();
  if (a.last_level) {
    const uint32_t fs = sm.s_f, bs = sm.s_b;
    for (uint32_t nd = threadIdx.x; nd < a.n_nodes; nd += kSplitThreads) {
      long long lg = 0, lh = 0, tg = 0, th = 0;
      const long long* p = a.hf + (((size_t)nd * nf + fs) * nb) * 2;
      for (uint32_t b = 0; b < nb; b++) {
        const long long xg = __ldcg(p + 2 * b), xh = __ldcg(p + 2 * b + 1);
        tg += xg;
        th += xh;
        if (b <= bs) {
          lg += xg;
          lh += xh;
        }
      }
      const long long rg = tg - lg, rh = th - lh;
      const double lgd = (double)lg * inv_g, lhd = (double)lh * inv_h;
      const double rgd = (double)rg * inv_g, rhd = (double)rh * inv_h;
      a.leafval[a.leaf_base + 2 * nd] = (float)(-a.lr * lgd / (lhd + lambda));
      a.leafval[a.leaf_base + 2 * nd + 1] = (float)(-a.lr * rgd / (rhd + lambda));
    }
  }
}

// --------------------------------------------------------------------------------

__global__ void k_bin(const float* __restrict__ x, uint64_t n, uint32_t nf,
                      const float* __restrict__ cuts, uint32_t nb1, uint8_t* __restrict__ bins,
                      uint64_t ld, uint32_t f0, uint32_t fcount) {
  extern __shared__ float s_cuts[];
  for (uint32_t i = threadIdx.x; i < fcount * nb1; i += blockDim.x)
    s_cuts[i] = cuts[(size_t)f0 * nb1 + i];
  __syncthreads();
  const uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  for (uint32_t fl = 0; fl < fcount; fl++) {
    const float v = __ldg(x + r * nf + f0 + fl);
    const float* c = s_cuts + (size_t)fl * nb1;
    uint32_t lo = 0, hi = nb1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi) >> 1;
      if (c[mid] < v) lo = mid + 1;
      else hi = mid;
    }
    bins[(size_t)(f0 + fl) * ld + r] = (uint8_t)lo;
  }
}

__global__ void k_pack4(const uint8_t* __restrict__ bins, uint64_t n_pad, uint32_t nf,
                        uint8_t* __restrict__ packed) {
  const uint64_t half = n_pad / 2;
  const uint64_t total = half * nf;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t f = i / half, k = i % half;
    const uint8_t lo = bins[f * n_pad + 2 * k] & 0x0f;
    const uint8_t hi = bins[f * n_pad + 2 * k + 1] & 0x0f;
    packed[i] = (uint8_t)(lo | (hi << 4));
  }
}

__device__ __forceinline__ uint32_t f32_bits_abs(float v) {
  return __float_as_uint(v) & 0x7fffffffu;
}

__device__ void block_max2_atomic(uint32_t mg, uint32_t mh, uint32_t* maxbits) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    mg = max(mg, __shfl_down_sync(0xffffffffu, mg, off));
    mh = max(mh, __shfl_down_sync(0xffffffffu, mh, off));
  }
  __shared__ uint32_t rg[32], rh[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) {
    rg[warp] = mg;
    rh[warp] = mh;
  }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    mg = lane < nw ? rg[lane] : 0u;
    mh = lane < nw ? rh[lane] : 0u;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      mg = max(mg, __shfl_down_sync(0xffffffffu, mg, off));
      mh = max(mh, __shfl_down_sync(0xffffffffu, mh, off));
    }
    if (lane == 0) {
      if (mg) atomicMax(maxbits, mg);
      if (mh) atomicMax(maxbits + 1, mh);
    }
  }
}

// Gradients (src/cpu.rs:181-193), stride row sampling (src/cpu.rs:172-176, 202-204)
// and the round's maxima over the sampled rows. Unsampled and padded rows
// (n <= i < n_pad) get g = h = 0, which removes them from every histogram and leaf sum.
__global__ void k_grad(const float* __restrict__ pred, const float* __restrict__ y,
                       float* __restrict__ g, float* __restrict__ h, uint64_t n, uint64_t n_pad,
                       int logistic, uint64_t stride, uint64_t phase, uint64_t row_offset,
                       int compute_max, uint32_t* maxbits) {
  uint32_t mg = 0, mh = 0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_pad;
       i += (uint64_t)gridDim.x * blockDim.x) {
    float gv = 0.0f, hv = 0.0f;
    if (i < n) {
      if (logistic) rw_logistic_grad(pred[i], y[i], &gv, &hv);
      else {
        gv = pred[i] - y[i];
        hv = 1.0f;
      }
    }
    const bool sampled = i < n && (stride <= 1 || ((row_offset + i) % stride) == phase);
    if (!sampled) {
      gv = 0.0f;
      hv = 0.0f;
    }
    g[i] = gv;
    h[i] = hv;
    mg = max(mg, f32_bits_abs(gv));
    mh = max(mh, f32_bits_abs(hv));
  }
  if (compute_max) block_max2_atomic(mg, mh, maxbits);
}

// Per round: q = round(x * 2^e) for g and h (scales from the final maxima), the row's
// excluded flag (node bit 15; a row whose g and h both quantise to 0 adds nothing to
// any sum), node reset and the level-0 build slot. Also zeroes the level-0 histogram.
constexpr uint16_t kExcluded = 0x8000;

__global__ void k_quant(const float* __restrict__ g, const float* __restrict__ h,
                        const uint32_t* __restrict__ maxbits, uint64_t n_pad,
                        int32_t* __restrict__ qg, int32_t* __restrict__ qh,
                        uint16_t* __restrict__ node, int16_t* __restrict__ slot,
                        long long* __restrict__ hb0, uint64_t hb0_words) {
  const float sg = rw_pow2f(rw_qscale_exp(maxbits[0]));
  const float sh = rw_pow2f(rw_qscale_exp(maxbits[1]));
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t nthr = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t w = tid; w < hb0_words; w += nthr) hb0[w] = 0;
  for (uint64_t i = tid; i < n_pad; i += nthr) {
    const int32_t a = rw_quantize(g[i], sg), b = rw_quantize(h[i], sh);
    const bool excl = (a | b) == 0;
    qg[i] = a;
    qh[i] = b;
    node[i] = excl ? kExcluded : 0;
    slot[i] = excl ? -1 : 0;
  }
}

// leaf = 2*leaf + (bin[f*] > t*) (src/cpu.rs:278-281) for 4 rows per thread, keeping the
// excluded flag; then either the next level's build slot (odd children keyed by the
// parent when subtracting, else the node itself; -1 when excluded or not built), or, at
// the last level, pred += leafval[leaf] (src/cpu.rs:319-320).
__global__ void k_apply(const uint8_t* __restrict__ bins, uint64_t ld, int packed,
                        uint16_t* __restrict__ node, int16_t* __restrict__ slot,
                        const uint32_t* __restrict__ split_ft, uint64_t n4, int next_odd_only,
                        int final_level, const float* __restrict__ leafval, uint32_t leaf_base,
                        float* __restrict__ pred) {
  const uint32_t f = split_ft[0], t = split_ft[1];
  const uint8_t* col = bins + (size_t)f * ld;
  for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
       q += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = q * 4;
    uint32_t b4;
    if (packed) {
      const uint32_t p = *reinterpret_cast<const uint16_t*>(col + (r >> 1));
      b4 = (p & 0xfu) | ((p & 0xf0u) << 4) | ((p & 0xf00u) << 8) | ((p & 0xf000u) << 12);
    } else {
      b4 = *reinterpret_cast<const uint32_t*>(col + r);
    }
    uint2 nd2 = *reinterpret_cast<const uint2*>(node + r);
    uint32_t nds[4] = {nd2.x & 0xffffu, nd2.x >> 16, nd2.y & 0xffffu, nd2.y >> 16};
    int sl[4];
#pragma unroll
    for (int s = 0; s < 4; s++) {
      const uint32_t ex = nds[s] & kExcluded;
      const uint32_t leaf = (nds[s] & 0x7fffu) * 2u + (((b4 >> (8 * s)) & 0xffu) > t ? 1u : 0u);
      nds[s] = ex | leaf;
      if (ex) sl[s] = -1;
      else if (next_odd_only) sl[s] = (leaf & 1u) ? (int)(leaf >> 1) : -1;
      else sl[s] = (int)leaf;
    }
    nd2.x = (nds[0] & 0xffffu) | (nds[1] << 16);
    nd2.y = (nds[2] & 0xffffu) | (nds[3] << 16);
    *reinterpret_cast<uint2*>(node + r) = nd2;
    if (final_level) {
      float4 p4 = *reinterpret_cast<const float4*>(pred + r);
      p4.x += leafval[leaf_base + (nds[0] & 0x7fffu)];
      p4.y += leafval[leaf_base + (nds[1] & 0x7fffu)];
      p4.z += leafval[leaf_base + (nds[2] & 0x7fffu)];
      p4.w += leafval[leaf_base + (nds[3] & 0x7fffu)];
      *reinterpret_cast<float4*>(pred + r) = p4;
    } else {
      uint2 s2;
      s2.x = ((uint32_t)sl[0] & 0xffffu) | ((uint32_t)sl[1] << 16);
      s2.y = ((uint32_t)sl[2] & 0xffffu) | ((uint32_t)sl[3] << 16);
      *reinterpret_cast<uint2*>(slot + r) = s2;
    }
  }
}

__global__ void k_fill(float* p, float v, uint64_t n) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// ---- GOSS (src/cpu.rs:64-110): exact k-th largest |g| by MSB-first radix select ----

__global__ void k_goss_init(uint32_t* sel, uint64_t k) {
  sel[0] = 0u;  // prefix
  sel[1] = 0u;  // mask of decided bits
  sel[2] = (uint32_t)k;
  sel[3] = 0u;
}

__global__ void k_goss_digit_hist(const float* __restrict__ g, uint64_t n,
                                  unsigned long long* counts, const uint32_t* sel, int pass) {
  __shared__ uint32_t sc[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) sc[i] = 0;
  __syncthreads();
  const uint32_t prefix = sel[0], mask = sel[1];
  const int shift = 24 - 8 * pass;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t v = f32_bits_abs(g[i]);
    if ((v & mask) == prefix) atomicAdd(&sc[(v >> shift) & 0xffu], 1u);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    if (sc[i]) atomicAdd(&counts[i], (unsigned long long)sc[i]);
}

// Walk digits from the largest down; the k-th largest (0-based) lies in the first
// digit whose cumulative count exceeds k.
__global__ void k_goss_digit_select(unsigned long long* counts, uint32_t* sel, int pass) {
  if (threadIdx.x != 0) return;
  const int shift = 24 - 8 * pass;
  unsigned long long k = sel[2], cum = 0;
  uint32_t digit = 0;
  for (int d = 255; d >= 0; d--) {
    const unsigned long long c = counts[d];
    if (cum + c > k) {
      digit = (uint32_t)d;
      k -= cum;
      break;
    }
    cum += c;
  }
  sel[0] |= digit << shift;
  sel[1] |= 0xffu << shift;
  sel[2] = (uint32_t)k;
  if (pass == 3) sel[3] = sel[0];
  for (int d = 0; d < 256; d++) counts[d] = 0ull;
}

__global__ void k_goss_apply(float* __restrict__ g, float* __restrict__ h, uint64_t n,
                             uint64_t row_offset, const uint32_t* sel, double keep_prob,
                             float fact, uint64_t seed, uint32_t* maxbits) {
  const float thresh = __uint_as_float(sel[3]);
  uint32_t mg = 0, mh = 0;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    float gv = g[i], hv = 1.0f;
    if (!(fabsf(gv) >= thresh)) {
      const uint64_t r = row_offset + i;
      uint64_t hh = (r ^ (seed * 0x9E3779B97F4A7C15ull) ^ 0x00424552455A4B41ull) *
                    0xD6E8FEB86659FD93ull;
      hh ^= hh >> 32;
      if ((double)(hh >> 11) / 9007199254740992.0 < keep_prob) {
        gv = gv * fact;
        hv = fact;
      } else {
        gv = 0.0f;
        hv = 0.0f;
      }
    }
    g[i] = gv;
    h[i] = hv;
    mg = max(mg, f32_bits_abs(gv));
    mh = max(mh, f32_bits_abs(hv));
  }
  block_max2_atomic(mg, mh, maxbits);
}

__global__ void k_debug_expf(const float* x, uint64_t n, float* o_rw, float* o_cuda) {
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x) {
    o_rw[i] = rw_expf(x[i]);
    o_cuda[i] = expf(x[i]);
  }
}

int grid_for(uint64_t work, int threads) {
  uint64_t b = (work + threads - 1) / threads;
  if (b > (uint64_t)148 * 16) b = (uint64_t)148 * 16;
  if (b < 1) b = 1;
  return (int)b;
}

}  // namespace

// ---------------------------------------------------------------------------------

cudaError_t launch_hist(const HistLaunch& L, cudaStream_t s, int* n_launch) {
  // Feature-tile width FT and group chunk: the CTA's cells 8*G*nb*FT bytes must fit.
  const uint64_t per_ft_group = 8ull * L.nb;
  int ft = 32;
  while (ft > 1 && per_ft_group * L.groups * (uint64_t)ft > (uint64_t)kHistSmemBudget) ft >>= 1;
  uint32_t gchunk = L.groups;
  while (gchunk > 1 && per_ft_group * gchunk * (uint64_t)ft > (uint64_t)kHistSmemBudget)
    gchunk = (gchunk + 1) / 2;
  while ((uint32_t)ft > 1 && (uint32_t)ft / 2 >= L.nf) ft >>= 1;  // no idle tile lanes
  const uint32_t ftiles = (L.nf + ft - 1) / ft;
  const uint32_t gz = (L.groups + gchunk - 1) / gchunk;
  // Row chunks: whole multiples of kRowAlign rows, about two CTAs per SM in total,
  // grouped into clusters of up to kMaxCluster CTAs along the row chunks.
  const uint64_t units = L.n_pad / kRowAlign;
  uint64_t rchunks = (units + 3) / 4;  // >= 8192 rows per CTA
  uint64_t max_r = (uint64_t)kTargetCtas / ((uint64_t)ftiles * gz);
  if (max_r < 1) max_r = 1;
  if (rchunks > max_r) rchunks = max_r;
  if (rchunks > units) rchunks = units;
  if (rchunks < 1) rchunks = 1;
  const uint64_t rows = (units + rchunks - 1) / rchunks * kRowAlign;
  rchunks = (L.n_pad + rows - 1) / rows;
  int cluster = 1;
  while (cluster * 2 <= kMaxCluster && (uint64_t)cluster * 2 <= rchunks) cluster *= 2;
  rchunks = (rchunks + cluster - 1) / cluster * cluster;

  HistArgs a;
  a.bins = L.bins;
  a.ld = L.ld;
  a.slot = L.slot;
  a.qg = L.qg;
  a.qh = L.qh;
  a.n_pad = L.n_pad;
  a.nf = L.nf;
  a.nb = L.nb;
  a.gchunk = gchunk;
  a.out = L.out;
  a.rows_per_cta = rows;
  const size_t smem = 8ull * gchunk * L.nb * (uint64_t)ft;
  dim3 grid((unsigned)rchunks, ftiles, gz);
  if (n_launch) (*n_launch)++;
  return L.packed ? launch_hist_ft<true>(ft, a, grid, cluster, smem, s)
                  : launch_hist_ft<false>(ft, a, grid, cluster, smem, s);
}

cudaError_t launch_split(const SplitLaunch& a, cudaStream_t s) {
  const size_t smem = sizeof(SplitSmem);
  cudaError_t e = cudaFuncSetAttribute(k_split, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  k_split<<<a.nf, kSplitThreads, smem, s>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_bin(const float* x, uint64_t n, uint32_t nf, const float* d_cuts,
                       uint32_t n_bins, uint8_t* d_bins, uint64_t ld, cudaStream_t s, int* nl) {
  const uint32_t nb1 = n_bins - 1;
  const uint32_t per = (48 * 1024) / (4 * (nb1 ? nb1 : 1));
  const uint32_t ftile = per < 1 ? 1 : (per > nf ? nf : per);
  for (uint32_t f0 = 0; f0 < nf; f0 += ftile) {
    const uint32_t fc = nf - f0 < ftile ? nf - f0 : ftile;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    k_bin<<<blocks, 256, (size_t)fc * nb1 * 4, s>>>(x, n, nf, d_cuts, nb1, d_bins, ld, f0, fc);
    if (nl) (*nl)++;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_pack4(const uint8_t* d_bins, uint64_t n_pad, uint32_t nf, uint8_t* d_packed,
                         cudaStream_t s, int* nl) {
  k_pack4<<<grid_for(n_pad / 2 * nf, 256), 256, 0, s>>>(d_bins, n_pad, nf, d_packed);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_grad(const float* pred, const float* y, float* g, float* h, uint64_t n,
                        uint64_t n_pad, int logistic, uint64_t stride, uint64_t phase,
                        uint64_t row_offset, int compute_max, uint32_t* maxbits,
                        cudaStream_t s, int* nl) {
  k_grad<<<grid_for(n_pad, 256), 256, 0, s>>>(pred, y, g, h, n, n_pad, logistic, stride, phase,
                                               row_offset, compute_max, maxbits);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_quant(const float* g, const float* h, const uint32_t* maxbits, uint64_t n_pad,
                         int32_t* qg, int32_t* qh, uint16_t* node, int16_t* slot,
                         long long* hb0, uint64_t hb0_words, cudaStream_t s, int* nl) {
  k_quant<<<grid_for(n_pad, 256), 256, 0, s>>>(g, h, maxbits, n_pad, qg, qh, node, slot, hb0,
                                               hb0_words);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_apply(const uint8_t* bins, uint64_t ld, int packed, uint16_t* node,
                         int16_t* slot, const uint32_t* split_ft, uint64_t n_pad,
                         int next_odd_only, int final_level, const float* leafval,
                         uint32_t leaf_base, float* pred, cudaStream_t s, int* nl) {
  const uint64_t n4 = n_pad / 4;
  k_apply<<<grid_for(n4, 256), 256, 0, s>>>(bins, ld, packed, node, slot, split_ft, n4,
                                             next_odd_only, final_level, leafval, leaf_base, pred);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_fill_f32(float* p, float v, uint64_t n, cudaStream_t s, int* nl) {
  k_fill<<<grid_for(n, 256), 256, 0, s>>>(p, v, n);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_goss_init(const GossState& st, uint64_t k, cudaStream_t s, int* nl) {
  k_goss_init<<<1, 1, 0, s>>>(st.sel, k);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_goss_digit_hist(const float* g, uint64_t n, const GossState& st, int pass,
                                   cudaStream_t s, int* nl) {
  k_goss_digit_hist<<<grid_for(n, 256), 256, 0, s>>>(g, n, st.counts, st.sel, pass);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_goss_digit_select(const GossState& st, int pass, cudaStream_t s, int* nl) {
  k_goss_digit_select<<<1, 32, 0, s>>>(st.counts, st.sel, pass);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_goss_apply(float* g, float* h, uint64_t n, uint64_t row_offset,
                              const GossState& st, double keep_prob, float fact, uint64_t seed,
                              uint32_t* maxbits, cudaStream_t s, int* nl) {
  k_goss_apply<<<grid_for(n, 256), 256, 0, s>>>(g, h, n, row_offset, st.sel, keep_prob, fact,
                                                 seed, maxbits);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_debug_expf(const float* x, uint64_t n, float* out_rw, float* out_cuda,
                              cudaStream_t s) {
  k_debug_expf<<<grid_for(n, 256), 256, 0, s>>>(x, n, out_rw, out_cuda);
  return cudaGetLastError();
}
