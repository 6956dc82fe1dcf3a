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

#include <map>
#include <mutex>
#include <utility>

#include "rw_expf.h"
#include "rw_internal.cuh"

#define RW_INF __longlong_as_double(0x7ff0000000000000LL)

namespace {

constexpr int kHistThreads = 512;
// Rows one histogram CTA may accumulate into its 32-bit shared cells: every |q| is at
// most 2^RW_QBITS, so a cell's partial sum stays within 2^(30) in magnitude and the
// 32-bit word holds it exactly (no carries, no returned values needed).
constexpr uint32_t kMaxRowsPerCta = 1u << (30 - RW_QBITS);
static_assert(kMaxRowsPerCta >= 512, "quantisation too fine for one bin tile per CTA");
constexpr int kMaxCluster = 8;
constexpr int kStages = 2;
constexpr int kSmemPerSm = 227 * 1024;  // usable shared memory per SM (one or two CTAs)

namespace cg = cooperative_groups;

// ---- TMA bulk copies and mbarriers (PTX) -------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// 1D bulk copy global -> this CTA's shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Waits for the mbarrier phase with a ~1 s clock limit; false when the limit passed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > 2000000000LL) return false;
  return true;
}

struct HistArgs {
  const uint8_t* bins;
  BinLayout lay;
  const int16_t* slot;
  const int32_t* qg;
  const int32_t* qh;
  uint64_t n_pad;
  uint32_t nf, nb;
  uint32_t gchunk;  // groups per CTA (blockIdx.z selects the chunk)
  long long* out;
  int* err;
  uint64_t rows_per_cta;  // multiple of kBinTile
  uint32_t stage_bytes;   // bytes per stage
  uint32_t hist_bytes;    // bytes of the shared histogram (stages follow it)
};

// One CTA: a tile of FT*FPL consecutive features x group chunk x row range (at most
// kMaxRowsPerCta rows), in a cluster of CTAs along the row ranges. The row range streams
// through shared memory one bin tile (kBinTile rows) at a time: thread 0 issues TMA bulk
// copies -- the CTA's feature slice of the tile is one contiguous block in the row-tiled
// bin layout, plus the tile's slot/q arrays -- into a double-buffered stage, completing on
// an mbarrier, while the CTA accumulates the previous tile. Lane (k, j) handles features
// j + p*FT (p < FPL) of the tile for row slot k, U consecutive rows at a time. Shared
// words are laid out [group][bin][g|h][FT*FPL]: for each p the FT lanes of one row hit FT
// distinct banks, and a cell's h word is a fixed offset from its g word. Cells are plain
// 32-bit integers updated by reductions whose results are not read back: the row bound
// keeps every partial sum exact. With FT = 32 every lane of a warp works on the same row,
// so rows that are not built are skipped warp-uniformly. After the rows, the cluster's
// CTAs sum their shared histograms through distributed shared memory, each CTA adding a
// slice to the global int64 histogram.
template <int FT, int FPL, bool PACKED>
__global__ void __launch_bounds__(kHistThreads, 1) k_hist(HistArgs a) {
  constexpr uint32_t FTT = FT * FPL;  // features per CTA
  constexpr uint32_t T = kBinTile;
  constexpr int RW = 32 / FT;
  // rows per lane step: 16 (one 16-byte load of u8 bins) when a tile round of
  // 16 warps x RW slots x 16 rows fits the tile, else 4
  constexpr uint32_t U = (16u * (kHistThreads / 32) * RW <= T) ? 16u : 4u;
  extern __shared__ __align__(128) unsigned char hsm[];
  uint32_t* smem = reinterpret_cast<uint32_t*>(hsm);
  const uint32_t G = a.gchunk, nb = a.nb;
  const uint32_t words = 2 * G * nb * FTT;
  unsigned char* stage0 = hsm + a.hist_bytes;
  __shared__ __align__(8) uint64_t bar[kStages];
  __shared__ int abort_flag;
  for (uint32_t i = threadIdx.x; i < words; i += kHistThreads) smem[i] = 0u;
  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; st++) mbar_init(&bar[st], 1);
    mbar_init_fence();
    abort_flag = 0;
  }
  __syncthreads();

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = lane % FT, k = lane / FT;
  const uint32_t f0 = blockIdx.y * FTT;
  const int g0 = (int)(blockIdx.z * a.gchunk);
  const uint32_t rs = a.lay.rs;
  const size_t gstride = (size_t)a.nf * nb * 2;
  const uint32_t nvalid = a.nf - f0 < FTT ? a.nf - f0 : FTT;
  bool fval[FPL];
#pragma unroll
  for (int p = 0; p < FPL; p++) fval[p] = (uint32_t)(p * FT + j) < nvalid;

  const uint64_t r_begin = (uint64_t)blockIdx.x * a.rows_per_cta;
  uint64_t r_end = r_begin + a.rows_per_cta;
  if (r_end > a.n_pad) r_end = a.n_pad;
  const uint32_t ntiles = r_end > r_begin ? (uint32_t)((r_end - r_begin) / T) : 0u;

  auto stage_ptr = [&](int st) { return stage0 + (size_t)st * a.stage_bytes; };
  auto issue = [&](uint32_t t, int st) {  // thread 0
    unsigned char* sp = stage_ptr(st);
    const uint64_t r0 = r_begin + (uint64_t)t * T;
    const uint32_t bbytes = nvalid * rs;
    mbar_expect_tx(&bar[st], bbytes + 10u * T);
    bulk_g2s(sp, a.bins + (r0 / T) * a.lay.tile_bytes + (uint64_t)f0 * rs, bbytes, &bar[st]);
    unsigned char* rowp = sp + (size_t)FTT * rs;
    bulk_g2s(rowp, a.slot + r0, 2u * T, &bar[st]);
    bulk_g2s(rowp + 2u * T, a.qg + r0, 4u * T, &bar[st]);
    bulk_g2s(rowp + 6u * T, a.qh + r0, 4u * T, &bar[st]);
  };

  if (threadIdx.x == 0 && ntiles > 0) issue(0, 0);
  for (uint32_t t = 0; t < ntiles; t++) {
    const int st = t & 1;
    if (threadIdx.x == 0 && t + 1 < ntiles && !abort_flag) {
      fence_proxy_async_smem();  // the stage's last readers finished before the barrier below
      issue(t + 1, st ^ 1);
    }
    // After a wait gave up, no further copies are issued and no further waits are made.
    if (!abort_flag && !mbar_wait_bounded(&bar[st], (t >> 1) & 1u)) abort_flag = 1;
    const unsigned char* sp = stage_ptr(st);
    const int16_t* s_slot = reinterpret_cast<const int16_t*>(sp + (size_t)FTT * rs);
    const int32_t* s_qg = reinterpret_cast<const int32_t*>(sp + (size_t)FTT * rs + 2u * T);
    const int32_t* s_qh = reinterpret_cast<const int32_t*>(sp + (size_t)FTT * rs + 6u * T);
    if (!abort_flag) {
      for (uint32_t rg = warp * RW + k; rg < T / U; rg += (kHistThreads / 32) * RW) {
        const uint32_t r = rg * U;
        uint32_t bw[FPL][U / 4];
#pragma unroll
        for (int p = 0; p < FPL; p++) {
          const unsigned char* sb = sp + (size_t)(p * FT + j) * rs;
          if (U == 16) {
            if (PACKED) {
              const uint2 pk = *reinterpret_cast<const uint2*>(sb + r / 2);
              const uint32_t pw[2] = {pk.x, pk.y};
#pragma unroll
              for (int h2 = 0; h2 < 2; h2++)
#pragma unroll
                for (int q2 = 0; q2 < 2; q2++) {
                  const uint32_t v = pw[h2] >> (16 * q2);
                  bw[p][(2 * h2 + q2) % (U / 4)] = (v & 0xfu) | ((v & 0xf0u) << 4) |
                                                   ((v & 0xf00u) << 8) | ((v & 0xf000u) << 12);
                }
            } else {
              const uint4 pk = *reinterpret_cast<const uint4*>(sb + r);
              const uint32_t pw[4] = {pk.x, pk.y, pk.z, pk.w};
#pragma unroll
              for (int q = 0; q < (int)(U / 4); q++) bw[p][q] = pw[q];
            }
          } else {
            if (PACKED) {
              const uint32_t v = *reinterpret_cast<const uint16_t*>(sb + r / 2);
              bw[p][0] = (v & 0xfu) | ((v & 0xf0u) << 4) | ((v & 0xf00u) << 8) |
                         ((v & 0xf000u) << 12);
            } else {
              bw[p][0] = *reinterpret_cast<const uint32_t*>(sb + r);
            }
          }
        }
#pragma unroll
        for (int q4 = 0; q4 < (int)(U / 4); q4++) {
          const uint2 sl2 = *reinterpret_cast<const uint2*>(s_slot + r + 4 * q4);
          const int4 qg4 = *reinterpret_cast<const int4*>(s_qg + r + 4 * q4);
          const int4 qh4 = *reinterpret_cast<const int4*>(s_qh + r + 4 * q4);
          const int sl[4] = {(int)(int16_t)(sl2.x & 0xffffu), (int)(int16_t)(sl2.x >> 16),
                             (int)(int16_t)(sl2.y & 0xffffu), (int)(int16_t)(sl2.y >> 16)};
          const uint32_t qgr[4] = {(uint32_t)qg4.x, (uint32_t)qg4.y, (uint32_t)qg4.z,
                                   (uint32_t)qg4.w};
          const uint32_t qhr[4] = {(uint32_t)qh4.x, (uint32_t)qh4.y, (uint32_t)qh4.z,
                                   (uint32_t)qh4.w};
#pragma unroll
          for (int s = 0; s < 4; s++) {
            const uint32_t grp = (uint32_t)(sl[s] - g0);
            if (FT == 32 && grp >= G) continue;  // warp-uniform: every lane works on this row
            const uint32_t lb = grp * nb * (2 * FTT) + (uint32_t)j;
#pragma unroll
            for (int p = 0; p < FPL; p++) {
              if (fval[p] && (FT == 32 || grp < G)) {
                const uint32_t bin = __byte_perm(bw[p][q4], 0u, 0x4440u + (uint32_t)s);
                const uint32_t w = lb + bin * (2 * FTT) + (uint32_t)(p * FT);
                atomicAdd(&smem[w], qgr[s]);
                atomicAdd(&smem[w + FTT], qhr[s]);
              }
            }
          }
        }
      }
    }
    __syncthreads();  // every reader of stage `st` is done before it is refilled
  }
  if (abort_flag && threadIdx.x == 0) atomicExch(a.err, 1);

  cg::cluster_group cluster = cg::this_cluster();
  cluster.sync();
  const uint32_t cn = cluster.num_blocks(), cr = cluster.block_rank();
  const uint32_t per = (words + cn - 1) / cn;
  const uint32_t w_begin = cr * per, w_end = min(words, w_begin + per);
  for (uint32_t w = w_begin + threadIdx.x; w < w_end; w += kHistThreads) {
    long long v = 0;
    for (uint32_t r = 0; r < cn; r++) {
      const uint32_t* remote = cluster.map_shared_rank(smem, (int)r);
      v += (long long)(int32_t)remote[w];
    }
    if (v == 0) continue;
    const uint32_t blk = w / (2 * FTT), within = w % (2 * FTT);
    const uint32_t is_h = within >= FTT ? 1u : 0u, fo = within - is_h * FTT;
    const uint32_t bin = blk % nb, grp = blk / nb;
    const uint32_t ff = f0 + fo;
    if (ff >= a.nf) continue;
    long long* gc = a.out + (size_t)(g0 + grp) * gstride + ((size_t)ff * nb + bin) * 2 + is_h;
    atomicAdd(reinterpret_cast<unsigned long long*>(gc), (unsigned long long)v);
  }
  cluster.sync();  // keep this CTA's shared memory alive until every reader is done
}

template <int FT, int FPL, bool PACKED>
const void* hist_fn() {
  return reinterpret_cast<const void*>(&k_hist<FT, FPL, PACKED>);
}

template <bool PACKED>
const void* pick_hist(int ft, int fpl) {
  if (fpl == 2) return hist_fn<32, 2, PACKED>();
  switch (ft) {
    case 32: return hist_fn<32, 1, PACKED>();
    case 16: return hist_fn<16, 1, PACKED>();
    case 8: return hist_fn<8, 1, PACKED>();
    case 4: return hist_fn<4, 1, PACKED>();
    case 2: return hist_fn<2, 1, PACKED>();
    default: return hist_fn<1, 1, PACKED>();
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
                      BinLayout lay, uint32_t f0, uint32_t fcount) {
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
    bins[lay.offset(f0 + fl, r)] = (uint8_t)lo;
  }
}

// 4-bit packing (src/gpu_kernels.rs:628-643): byte = bin(2k) | bin(2k+1) << 4 within each
// feature row of each tile.
__global__ void k_pack4(const uint8_t* __restrict__ bins, BinLayout lu, uint64_t n_pad,
                        uint8_t* __restrict__ packed, BinLayout lp) {
  const uint64_t pairs = n_pad / 2 * lu.nf;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < pairs;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t f = (uint32_t)(i % lu.nf);
    const uint64_t r = (i / lu.nf) * 2;
    const uint8_t lo = bins[lu.offset(f, r)] & 0x0f;
    const uint8_t hi = bins[lu.offset(f, r + 1)] & 0x0f;
    packed[lp.offset(f, r)] = (uint8_t)(lo | (hi << 4));
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
__global__ void k_apply(const uint8_t* __restrict__ bins, BinLayout lay,
                        uint16_t* __restrict__ node, int16_t* __restrict__ slot,
                        const uint32_t* __restrict__ split_ft, uint64_t n4, int next_odd_only,
                        int final_level, const float* __restrict__ leafval, uint32_t leaf_base,
                        float* __restrict__ pred) {
  const uint32_t f = split_ft[0], t = split_ft[1];
  for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
       q += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = q * 4;
    uint32_t b4;
    if (lay.packed) {
      const uint32_t p = *reinterpret_cast<const uint16_t*>(bins + lay.offset(f, r));
      b4 = (p & 0xfu) | ((p & 0xf0u) << 4) | ((p & 0xf00u) << 8) | ((p & 0xf000u) << 12);
    } else {
      b4 = *reinterpret_cast<const uint32_t*>(bins + lay.offset(f, r));
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

int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1)
      n = 148;
  }
  return n;
}

// Shared-memory plan of one histogram CTA: the histogram (8 bytes per cell, FT*FPL
// features) plus dummy cells, plus two stages of (FT*FPL bins rows + 10 bytes of row
// state) x tile rows. Prefers two features per lane at FT = 32 (per-row work shared by
// both features), then one feature per lane with FT halving, then group chunks.
struct HistPlan {
  int ft, fpl;
  uint32_t gchunk, tile, stride, stage_bytes, hist_bytes;
  size_t smem;
};

HistPlan plan_hist(uint32_t nb, uint32_t groups, uint32_t nf, bool packed) {
  const uint64_t budget = kSmemPerSm - 2048;
  struct Cand {
    int ft, fpl;
  };
  const Cand cands[] = {{32, 2}, {32, 1}, {16, 1}, {8, 1}, {4, 1}, {2, 1}, {1, 1}};
  const uint32_t rs = (packed ? kBinTile / 2 : kBinTile) + 16;
  for (uint32_t gchunk = groups; gchunk >= 1; gchunk = gchunk > 1 ? (gchunk + 1) / 2 : 0) {
    for (const Cand& c : cands) {
      if (c.fpl == 2 && nf <= 32) continue;
      if (c.fpl == 1 && c.ft > 1 && (uint32_t)c.ft / 2 >= nf) continue;  // no idle tile lanes
      const uint32_t ftt = (uint32_t)(c.ft * c.fpl);
      const uint32_t stage = ftt * rs + 10u * kBinTile;
      const uint64_t hist = 8ull * gchunk * nb * ftt;
      if (hist + kStages * (uint64_t)stage <= budget) {
        HistPlan p{};
        p.ft = c.ft;
        p.fpl = c.fpl;
        p.gchunk = gchunk;
        p.tile = kBinTile;
        p.stride = rs;
        p.stage_bytes = (stage + 127) / 128 * 128;
        p.hist_bytes = (uint32_t)((hist + 127) / 128 * 128);
        p.smem = p.hist_bytes + kStages * (size_t)p.stage_bytes;
        return p;
      }
    }
    if (gchunk == 1) break;
  }
  HistPlan none{};
  return none;
}

// Occupancy of one histogram kernel configuration, queried once per (kernel, smem):
// co-resident clusters for cluster sizes kMaxCluster, /2, ..., 1 (size 1 = CTAs).
struct HistOcc {
  int max_clusters[4];
};

// The kernel's dynamic shared memory limit only ever grows, so a launch that needs less
// than an earlier one of the same kernel (another level, bin count or dataset) still fits.
const HistOcc* hist_occupancy(const void* kfn, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<std::pair<int, const void*>, size_t>, HistOcc> cache;
  static std::map<std::pair<int, const void*>, size_t> smem_limit;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  const auto kd = std::make_pair(dev, kfn);
  size_t& lim = smem_limit[kd];
  if (smem > lim) {
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return nullptr;
    lim = smem;
  }
  auto key = std::make_pair(kd, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return &it->second;
  HistOcc o{};
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, kHistThreads, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  for (int ci = 0, cl = kMaxCluster; cl >= 1; cl >>= 1, ci++) {
    if (cl == 1) {
      o.max_clusters[ci] = sm_count() * per_sm;
      continue;
    }
    cudaLaunchConfig_t q = {};
    q.gridDim = dim3(cl, 1, 1);
    q.blockDim = dim3(kHistThreads);
    q.dynamicSmemBytes = smem;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = cl;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    q.attrs = qa;
    q.numAttrs = 1;
    int maxc = 0;
    if (cudaOccupancyMaxActiveClusters(&maxc, kfn, &q) != cudaSuccess) maxc = 0;
    o.max_clusters[ci] = maxc;
  }
  return &(cache[key] = o);
}

cudaError_t launch_hist(const HistLaunch& L, cudaStream_t s, int* n_launch) {
  const HistPlan P = plan_hist(L.nb, L.groups, L.nf, L.lay.packed != 0);
  if (P.smem == 0) return cudaErrorInvalidConfiguration;
  const uint32_t ftt = (uint32_t)(P.ft * P.fpl);
  const uint32_t ftiles = (L.nf + ftt - 1) / ftt;
  const uint32_t gz = (L.groups + P.gchunk - 1) / P.gchunk;
  const void* kfn =
      L.lay.packed ? pick_hist<true>(P.ft, P.fpl) : pick_hist<false>(P.ft, P.fpl);
  const HistOcc* occ = hist_occupancy(kfn, P.smem);
  if (!occ) return cudaErrorInvalidConfiguration;
  const uint64_t units = L.n_pad / P.tile;  // n_pad is a multiple of the tile
  const uint64_t tiles_of = (uint64_t)ftiles * gz;
  // One wave: pick the cluster size whose co-resident clusters (clusters must fit inside
  // a GPC, so not every SM can host one) hold the most CTAs, then size the row chunks
  // so that every (feature tile, group chunk) gets the same whole number of clusters.
  uint64_t best_ctas = 0, rchunks = 1;
  int cluster = 1;
  for (int ci = 0, cl = kMaxCluster; cl >= 1; cl >>= 1, ci++) {
    const int maxc = occ->max_clusters[ci];
    if (maxc < 1) continue;
    uint64_t per_tile = (uint64_t)maxc / tiles_of;  // clusters per (feature tile, group)
    if (per_tile < 1) per_tile = 1;
    uint64_t rc = per_tile * (uint64_t)cl;
    if (rc > units) rc = units / cl * cl;
    if (rc < (uint64_t)cl) continue;
    const uint64_t ctas = rc * tiles_of;
    if (ctas > best_ctas + best_ctas / 16) {  // larger clusters unless they cost >6% of CTAs
      best_ctas = ctas;
      rchunks = rc;
      cluster = cl;
    }
  }
  // No CTA accumulates more than kMaxRowsPerCta rows (larger inputs take more waves).
  constexpr uint64_t kMaxTiles = kMaxRowsPerCta / kBinTile;
  if ((units + rchunks - 1) / rchunks > kMaxTiles) {
    rchunks = (units + kMaxTiles - 1) / kMaxTiles;
    rchunks = (rchunks + cluster - 1) / cluster * cluster;
  }
  const uint64_t tiles_per = (units + rchunks - 1) / rchunks;
  const uint64_t rows = tiles_per * P.tile;

  HistArgs a;
  a.bins = L.bins;
  a.lay = L.lay;
  a.slot = L.slot;
  a.qg = L.qg;
  a.qh = L.qh;
  a.n_pad = L.n_pad;
  a.nf = L.nf;
  a.nb = L.nb;
  a.gchunk = P.gchunk;
  a.out = L.out;
  a.err = L.err;
  a.rows_per_cta = rows;
  a.stage_bytes = P.stage_bytes;
  a.hist_bytes = P.hist_bytes;
  dim3 grid((unsigned)rchunks, ftiles, gz);
  if (n_launch) (*n_launch)++;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kHistThreads);
  cfg.dynamicSmemBytes = P.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void* args[] = {&a};
  return cudaLaunchKernelExC(&cfg, kfn, args);
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
                       uint32_t n_bins, uint8_t* d_bins, const BinLayout& lay, cudaStream_t s,
                       int* nl) {
  const uint32_t nb1 = n_bins - 1;
  const uint32_t per = (48 * 1024) / (4 * (nb1 ? nb1 : 1));
  const uint32_t ftile = per < 1 ? 1 : (per > nf ? nf : per);
  for (uint32_t f0 = 0; f0 < nf; f0 += ftile) {
    const uint32_t fc = nf - f0 < ftile ? nf - f0 : ftile;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    k_bin<<<blocks, 256, (size_t)fc * nb1 * 4, s>>>(x, n, nf, d_cuts, nb1, d_bins, lay, f0, fc);
    if (nl) (*nl)++;
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_pack4(const uint8_t* d_bins, const BinLayout& lay_u8, uint64_t n_pad,
                         uint8_t* d_packed, const BinLayout& lay_p, cudaStream_t s, int* nl) {
  k_pack4<<<grid_for(n_pad / 2 * lay_u8.nf, 256), 256, 0, s>>>(d_bins, lay_u8, n_pad, d_packed,
                                                               lay_p);
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

cudaError_t launch_apply(const uint8_t* bins, const BinLayout& lay, uint16_t* node,
                         int16_t* slot, const uint32_t* split_ft, uint64_t n_pad,
                         int next_odd_only, int final_level, const float* leafval,
                         uint32_t leaf_base, float* pred, cudaStream_t s, int* nl) {
  const uint64_t n4 = n_pad / 4;
  k_apply<<<grid_for(n4, 256), 256, 0, s>>>(bins, lay, node, slot, split_ft, n4, next_odd_only,
                                             final_level, leafval, leaf_base, pred);
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
