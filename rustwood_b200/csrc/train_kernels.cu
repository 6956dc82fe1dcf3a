// Training kernels for the oblivious-tree hot path on sm_100a.
//
// Per boosting round (src/booster.rs:349-501 is the reference's sequence):
//   k_grad / GOSS           gradients, row sampling, per-round max |g| and max h
//   [ncclAllReduce max]     multi-GPU: global maxima (the fixed-point scales)
//   k_quant                 per-row fixed-point q = (q(g), q(h)), excluded flag, node reset
//   per level d:
//     k_hist                exact fixed-point histogram of the built nodes, over the
//                           level's row list (all rows at level 0)
//     [ncclAllReduce]       multi-GPU: sum of the built histograms (int64, exact)
//     k_split               derive sibling nodes, f64 gain scan, argmax, model write,
//                           leaf values at the last level (no separate leaf pass)
//     k_apply               leaf = 2*leaf + (bin > t) and the next level's row list
//                           (per node the child with less hessian, or both children
//                           without subtraction; the sibling is parent - built);
//                           at the last level pred += leafval[leaf]
//
// Exactness: histogram cells are int64 sums of per-row fixed-point values
// q = round(x * 2^e) with |q| <= 2^RW_QBITS (rw_expf.h). A histogram CTA accumulates at
// most kMaxRowsPerCta rows into 32-bit shared cells before adding them to the global
// int64 cells, so every partial sum is exact. The result equals the int64 sum of q over
// the contributing rows whatever the scheduling, the row order of the lists or which
// child of a pair is built, so histograms, splits and leaf values are bit-identical run
// to run and at every GPU count.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <utility>

#include "rw_expf.h"
#include "rw_internal.cuh"

#define RW_INF __longlong_as_double(0x7ff0000000000000LL)

namespace {

// Programmatic dependent launch: the level loop is a chain of short kernels, each
// launched with programmatic stream serialization so its launch and CTA setup overlap the
// previous kernel's tail. Every kernel first waits for its predecessor grid to complete
// (and its memory to be visible) and then lets its own successor launch.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// The same in two steps, for kernels that first load data no running grid writes: when
// a kernel starts, the grid two launches back has completed (its successor let this one
// launch only after waiting for it), so only the immediately preceding grid may still
// be writing; loads of anything it does not write may precede the wait.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

constexpr int kHistThreads = 1024;
// Rows one histogram CTA accumulates into its 32-bit shared cells before adding them to
// the global int64 cells: every |q| is at most 2^RW_QBITS, so a cell's partial sum
// stays within 2^30 in magnitude and the 32-bit word holds it exactly.
constexpr uint32_t kMaxRowsPerCta = 1u << (30 - RW_QBITS);
static_assert(kMaxRowsPerCta >= 1024, "quantisation too fine for the histogram row bound");
// A listed level gathers its rows through a ring of kListSlots shared-memory slots of
// kListRows rows: the rows' list entries (row id, q) and their bin runs (cp.async 16-byte
// copies, one per thread), issued kListSlots - 1 slots ahead of the slot being accumulated.
#ifndef RW_LIST_ROWS
#define RW_LIST_ROWS 256
#endif
#ifndef RW_STREAM_ROWS
#define RW_STREAM_ROWS 512
#endif
#ifndef RW_STREAM_STAGES
#define RW_STREAM_STAGES 2
#endif
constexpr uint32_t kListRows = RW_LIST_ROWS;
constexpr int kListSlots = 3;
static_assert(kListRows * 4 <= kHistThreads && kListRows % (kHistThreads / 32) == 0,
              "at most one 16-byte bin chunk per thread per slot, whole rows per warp");
// The all-rows level streams its rows through shared memory in stages of kStreamRows
// (one TMA bulk copy of the stage's bin rows and one of its q values), kStreamStages deep.
constexpr uint32_t kStreamRows = RW_STREAM_ROWS;
constexpr int kStreamStages = RW_STREAM_STAGES;
constexpr uint32_t kStreamRowsPerWarp = kStreamRows / (kHistThreads / 32);
static_assert(kStreamRows % (kHistThreads / 32) == 0, "whole rows per warp per stage");

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
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t bytes) {
  // bytes < 16 zero-fills the rest (bytes == 0: nothing is read)
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Waits for the mbarrier phase with a ~1 s clock limit; false when the limit passed.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity))
    if (clock64() - t0 > 2000000000LL) return false;
  return true;
}

// Adds one row's tile to the shared cells: lane j owns columns j (feature 2j) and 32+j
// (feature 2j+1); `bb` holds the two bins (u8 pair or one byte of 4-bit pairs). A lane
// whose feature is past nf adds into the dummy bin row `nb` (never flushed), which keeps
// the warp free of divergent branches.
template <bool PACKED>
__device__ __forceinline__ void hist_add_row(uint32_t* hs, uint32_t bb, int2 qq, uint32_t lane,
                                             bool v0, bool v1, uint32_t nb) {
  uint32_t b0 = PACKED ? (bb & 0xfu) : (bb & 0xffu);
  uint32_t b1 = PACKED ? ((bb >> 4) & 0xfu) : (bb >> 8);
  b0 = v0 ? b0 : nb;
  b1 = v1 ? b1 : nb;
  const uint32_t c0 = b0 * (2 * kHistFeat) + lane, c1 = b1 * (2 * kHistFeat) + 32 + lane;
  atomicAdd(&hs[c0], (uint32_t)qq.x);
  atomicAdd(&hs[c0 + kHistFeat], (uint32_t)qq.y);
  atomicAdd(&hs[c1], (uint32_t)qq.x);
  atomicAdd(&hs[c1 + kHistFeat], (uint32_t)qq.y);
}

// Exclusive prefix of n (<= 4 * blockDim.x) values into out[0..n], out[n] = the total;
// thread i holds values i * per .. i * per + per - 1 (per = ceil(n / blockDim.x), zero
// past n) in v; warp_sums has 33 words. All threads of the block call it.
__device__ void block_exclusive_scan_vals(const uint32_t (&v)[4], uint32_t n, uint32_t* out,
                                          uint32_t* warp_sums) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x / 32;
  const uint32_t per = (n + blockDim.x - 1) / blockDim.x;
  const uint32_t b0 = threadIdx.x * per;
  uint32_t sum = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) sum += v[k];
  uint32_t incl = sum;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= (uint32_t)d) incl += y;
  }
  if (lane == 31) warp_sums[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t ws = lane < nw ? warp_sums[lane] : 0u, wi = ws;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, wi, d);
      if (lane >= (uint32_t)d) wi += y;
    }
    if (lane < nw) warp_sums[lane] = wi - ws;  // exclusive warp offsets
    if (lane == nw - 1) warp_sums[32] = wi;    // block total
  }
  __syncthreads();
  uint32_t run = warp_sums[warp] + incl - sum;
#pragma unroll
  for (int k = 0; k < 4; k++)
    if (k < (int)per && b0 + k < n) {
      out[b0 + k] = run;
      run += v[k];
    }
  if (threadIdx.x == 0) out[n] = warp_sums[32];
  __syncthreads();
}

// Exclusive prefixes of two arrays at once: in_k[0..n_k) (n_k <= 4 * blockDim.x, global,
// written by an earlier kernel) into out_k[0..n_k], out_k[n_k] = the total. Both arrays'
// loads are issued together and share the block barriers. warp_sums has 66 words. All
// threads of the block call it.
__device__ void block_exclusive_scan2(const uint32_t* in0, uint32_t n0, uint32_t* out0,
                                      const uint32_t* in1, uint32_t n1, uint32_t* out1,
                                      uint32_t* warp_sums) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x / 32;
  const uint32_t per0 = (n0 + blockDim.x - 1) / blockDim.x, per1 = (n1 + blockDim.x - 1) / blockDim.x;
  const uint32_t b0 = threadIdx.x * per0, b1 = threadIdx.x * per1;
  uint32_t v0[4], v1[4], sum0 = 0, sum1 = 0;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    v0[k] = (k < (int)per0 && b0 + k < n0) ? __ldcg(in0 + b0 + k) : 0u;
    v1[k] = (k < (int)per1 && b1 + k < n1) ? __ldcg(in1 + b1 + k) : 0u;
  }
#pragma unroll
  for (int k = 0; k < 4; k++) {
    sum0 += v0[k];
    sum1 += v1[k];
  }
  uint32_t incl0 = sum0, incl1 = sum1;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t y0 = __shfl_up_sync(0xffffffffu, incl0, d);
    const uint32_t y1 = __shfl_up_sync(0xffffffffu, incl1, d);
    if (lane >= (uint32_t)d) {
      incl0 += y0;
      incl1 += y1;
    }
  }
  if (lane == 31) {
    warp_sums[warp] = incl0;
    warp_sums[33 + warp] = incl1;
  }
  __syncthreads();
  if (warp < 2) {
    uint32_t* ws_arr = warp_sums + 33 * warp;
    const uint32_t ws = lane < nw ? ws_arr[lane] : 0u;
    uint32_t wi = ws;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, wi, d);
      if (lane >= (uint32_t)d) wi += y;
    }
    if (lane < nw) ws_arr[lane] = wi - ws;  // exclusive warp offsets
    if (lane == nw - 1) ws_arr[32] = wi;    // block total
  }
  __syncthreads();
  uint32_t run0 = warp_sums[warp] + incl0 - sum0, run1 = warp_sums[33 + warp] + incl1 - sum1;
#pragma unroll
  for (int k = 0; k < 4; k++) {
    if (k < (int)per0 && b0 + k < n0) {
      out0[b0 + k] = run0;
      run0 += v0[k];
    }
    if (k < (int)per1 && b1 + k < n1) {
      out1[b1 + k] = run1;
      run1 += v1[k];
    }
  }
  if (threadIdx.x == 0) {
    out0[n0] = warp_sums[32];
    out1[n1] = warp_sums[65];
  }
  __syncthreads();
}

// Histogram of one level over a row list (or all rows), exact in fixed point.
//
// Row bins are tile-major: tile t's row r is the kHistFeat-byte (u8) or kHistFeat/2-byte
// (4-bit) run at rowbins + (t * n_pad + r) * tile_bytes. The work space is (feature tile
// t, list index i), tile-major; CTA b takes the contiguous slice [b*per, (b+1)*per) and
// walks it in parts that stay inside one (tile, group) and hold at most kMaxRowsPerCta
// rows. Per part the CTA accumulates into shared 32-bit cells laid out
// [bin][g|h][64 columns]: lane j of a warp handles the tile's features 2j and 2j+1
// (columns j and 32+j, so the warp's 32 lanes update 32 distinct banks). With a row list
// the warps gather their rows' runs and q values directly; over all rows (the identity
// list) the part is one contiguous range, streamed through shared memory by TMA bulk
// copies in stages, so HBM sees long sequential reads. The cells are updated by
// reductions whose results are not read back. At the end of a part its nonzero cells
// are added to the global int64 histogram, which has the same cell layout per (group,
// tile) -- [group][tile][bin][g|h][64 columns], column j holding feature 2j and column
// 32+j feature 2j+1 -- and cleared.
template <bool PACKED>
__global__ void __launch_bounds__(kHistThreads) k_hist(HistLaunch a, uint32_t ftiles) {
  extern __shared__ __align__(16) uint32_t hs[];
  __shared__ __align__(8) uint64_t bar[kStreamStages];
  __shared__ int s_abort;
  constexpr uint32_t TB = PACKED ? kHistFeat / 2 : kHistFeat;  // tile bytes per row
  __shared__ uint32_t warp_sums[66];
  const uint32_t nb = a.nb, words = nb * 2 * kHistFeat;
  // the cells are cleared while the preceding grid still runs (shared memory only)
  for (uint32_t c = threadIdx.x; c < words; c += kHistThreads) hs[c] = 0u;
  pdl_enter();
  unsigned char* stage0 = reinterpret_cast<unsigned char*>(hs + words + 2 * kHistFeat);
  // list segments: lpre = prefix of the group lengths (list index -> group), start = each
  // group's first entry in `entries` (from the prefix of the parents' row counts)
  uint32_t* s_lpre = reinterpret_cast<uint32_t*>(stage0 + (size_t)kListSlots * kListRows * (TB + 16));
  uint32_t* s_start = s_lpre + a.groups + 1;
  uint32_t* s_cap = s_start + a.groups;
  if (a.entries) {
    block_exclusive_scan2(a.pcount, a.parents, s_cap, a.glen, a.groups, s_lpre, warp_sums);
    for (uint32_t g = threadIdx.x; g < a.groups; g += kHistThreads) {
      if (a.pairs) {
        s_start[g] = s_cap[g];
      } else {
        // the second child's run starts after the first child's rows of the parent
        const uint32_t k = g >> 1;
        s_start[g] = s_cap[k] + ((g & 1u) ? (s_cap[k + 1] - s_cap[k]) - (s_lpre[g + 1] - s_lpre[g])
                                          : 0u);
      }
    }
    __syncthreads();
  }
  const uint32_t L = a.entries ? s_lpre[a.groups] : a.n_ident;
  const uint64_t total = (uint64_t)L * ftiles;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint64_t w, w_end;
  const uint32_t units = a.entries ? ftiles * a.groups : 0u;  // (tile, group) units
  if (units != 0 && units <= 32 && units * 4 <= gridDim.x &&
      total <= (uint64_t)gridDim.x * 2 * kMaxRowsPerCta) {
    // Few units and short slices: each nonempty unit u gets its own CTAs, 1 + floor(len_u
    // * (grid - units) / total) of them (at most the grid in all), which split it evenly.
    // No CTA straddles two units, so every CTA flushes once; a CTA's share is within
    // total / (grid - units) rows. (With long slices a CTA flushes several times anyway,
    // and the contiguous slices below balance the rows better.)
    __shared__ unsigned long long s_range[2];
    if (warp == 0) {
      uint32_t c = 0;
      uint64_t u_start = 0, u_len = 0;
      if ((uint32_t)lane < units) {
        const uint32_t t = (uint32_t)lane / a.groups, g = (uint32_t)lane % a.groups;
        u_len = s_lpre[g + 1] - s_lpre[g];
        u_start = (uint64_t)t * L + s_lpre[g];
        c = u_len ? (uint32_t)(u_len * (gridDim.x - units) / total) + 1u : 0u;
      }
      uint32_t incl = c;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += y;
      }
      const uint32_t first = incl - c;
      if (lane == 0) s_range[0] = s_range[1] = 0;
      __syncwarp();
      if (blockIdx.x >= first && blockIdx.x < incl) {  // at most one lane
        const uint32_t k = blockIdx.x - first;
        s_range[0] = u_start + u_len * k / c;
        s_range[1] = u_start + u_len * (k + 1) / c;
      }
    }
    __syncthreads();
    w = s_range[0];
    w_end = s_range[1];
  } else {
    // contiguous slices of the work space; identity slices are whole stages (n_ident is
    // a multiple of kStreamRows)
    uint64_t per = (total + gridDim.x - 1) / gridDim.x;
    if (!a.entries) per = (per + kStreamRows - 1) / kStreamRows * kStreamRows;
    w = (uint64_t)blockIdx.x * per;
    w_end = min(total, w + per);
  }
  if (w >= w_end) return;
  constexpr uint32_t kStageBytes = kStreamRows * (TB + 8);
  if (threadIdx.x == 0) {
    s_abort = 0;
    if (!a.entries) {
      for (int st = 0; st < kStreamStages; st++) mbar_init(&bar[st], 1);
      mbar_init_fence();
    }
  }
  uint32_t phase_base = 0;  // stages consumed so far (mbarrier phase bookkeeping)
  while (w < w_end) {
    const uint32_t t = (uint32_t)(w / L);
    const uint32_t i0 = (uint32_t)(w % L);
    // the group holding list index i0: the last k with lpre[k] <= i0
    uint32_t grp = 0, g_end = L, ebase = 0;
    if (a.entries) {
      uint32_t lo = 0, hi = a.groups;
      while (hi - lo > 1) {
        const uint32_t mid = (lo + hi) >> 1;
        if (s_lpre[mid] <= i0) lo = mid;
        else hi = mid;
      }
      grp = lo;
      g_end = s_lpre[lo + 1];
      ebase = s_start[lo] + (i0 - s_lpre[lo]);  // entries of this part start here
    }
    uint64_t i1 = min((uint64_t)g_end, (uint64_t)i0 + kMaxRowsPerCta);
    i1 = min(i1, (uint64_t)i0 + (w_end - w));
    const uint32_t fbase = t * kHistFeat;
    const bool v0 = fbase + 2 * lane < a.nf, v1 = fbase + 2 * lane + 1 < a.nf;
    const unsigned char* tile = a.rowbins + (size_t)t * a.n_pad * TB;
    __syncthreads();  // cleared cells (and barrier init) are visible
    if (!a.entries) {
      // ---- streamed: rows i0 .. i1 in stages of kStreamRows ----
      const uint32_t nst = (uint32_t)((i1 - i0) / kStreamRows);
      auto issue = [&](uint32_t k) {
        const int st = (int)((phase_base + k) % kStreamStages);
        unsigned char* sp = stage0 + (size_t)st * kStageBytes;
        const uint64_t r0 = i0 + (uint64_t)k * kStreamRows;
        mbar_expect_tx(&bar[st], kStageBytes);
        bulk_g2s(sp, tile + r0 * TB, kStreamRows * TB, &bar[st]);
        bulk_g2s(sp + kStreamRows * TB, a.q + r0, kStreamRows * 8, &bar[st]);
      };
      if (threadIdx.x == 0) {
        fence_proxy_async_smem();
        for (uint32_t k = 0; k < nst && k < (uint32_t)kStreamStages; k++) issue(k);
      }
      uint32_t consumed = 0;
      for (uint32_t k = 0; k < nst; k++) {
        const uint32_t gk = phase_base + k;
        const int st = (int)(gk % kStreamStages);
        if (!s_abort && !mbar_wait_bounded(&bar[st], (gk / kStreamStages) & 1u)) s_abort = 1;
        if (!s_abort) {
          const unsigned char* sp = stage0 + (size_t)st * kStageBytes;
          const int2* sq = reinterpret_cast<const int2*>(sp + kStreamRows * TB);
#pragma unroll
          for (int u = 0; u < (int)kStreamRowsPerWarp; u++) {
            const uint32_t r = warp * kStreamRowsPerWarp + u;
            const uint32_t bb = PACKED ? (uint32_t)sp[r * TB + lane]
                                       : (uint32_t)*reinterpret_cast<const uint16_t*>(sp + r * TB + 2 * lane);
            hist_add_row<PACKED>(hs, bb, sq[r], lane, v0, v1, nb);
          }
        }
        __syncthreads();  // every reader of stage st is done
        if (s_abort) break;
        consumed = k + 1;
        if (threadIdx.x == 0 && k + kStreamStages < nst) {
          fence_proxy_async_smem();
          issue(k + kStreamStages);
        }
      }
      if (s_abort) {
        // a wait gave up: let the copies already issued land (bounded) before leaving
        const uint32_t issued = min(nst, consumed + (uint32_t)kStreamStages);
        if (threadIdx.x == 0)
          for (uint32_t k = consumed; k < issued; k++) {
            const uint32_t gk = phase_base + k;
            mbar_wait_bounded(&bar[gk % kStreamStages], (gk / kStreamStages) & 1u);
          }
        __syncthreads();
        break;
      }
      phase_base += nst;
    } else {
      // ---- gathered: the list's rows, through the slot ring ----
      // slot: [kListRows][TB] bin runs, then [kListRows] int4 entries (row, qg, qh, 0)
      constexpr uint32_t kSlotBytes = kListRows * (TB + 16);
      const uint32_t cnt = (uint32_t)(i1 - i0);
      const uint32_t nsl = (cnt + kListRows - 1) / kListRows;
      const uint32_t my_row = threadIdx.x / 4, my_part = threadIdx.x % 4;
      auto load_entry = [&](uint32_t j) {  // this thread's entry of slot j (row my_row)
        const uint32_t li = j * kListRows + my_row;
        return my_row < kListRows && li < cnt && ebase + li < a.n_pad
                   ? __ldcg(a.entries + ebase + li)
                   : make_int4(0, 0, 0, 0);
      };
      auto issue = [&](uint32_t j, int4 e) {
        unsigned char* sp = stage0 + (size_t)(j % kListSlots) * kSlotBytes;
        // rows outside the table never reach memory (defensive: lists hold rows < n_pad)
        const bool live = j * kListRows + my_row < cnt && (uint32_t)e.x < a.n_pad;
        if (my_row < kListRows && my_part * 16 < TB)
          cp_async16(sp + my_row * TB + my_part * 16,
                     tile + (size_t)(live ? (uint32_t)e.x : 0u) * TB + my_part * 16,
                     live ? 16u : 0u);
        if (my_row < kListRows && my_part == 0)
          reinterpret_cast<int4*>(sp + kListRows * TB)[my_row] =
              live ? e : make_int4(0, 0, 0, 0);
        cp_async_commit();
      };
      int4 e_next;
#pragma unroll
      for (uint32_t k = 0; k + 1 < (uint32_t)kListSlots; k++) {
        e_next = load_entry(k);
        if (k < nsl) issue(k, e_next);
        else cp_async_commit();
      }
      e_next = load_entry(kListSlots - 1);
      for (uint32_t j = 0; j < nsl; j++) {
        cp_async_wait<kListSlots - 2>();  // this thread's copies for slot j have landed
        __syncthreads();                  // ... and everyone else's
        const unsigned char* sp = stage0 + (size_t)(j % kListSlots) * kSlotBytes;
        const int4* se = reinterpret_cast<const int4*>(sp + kListRows * TB);
        const uint32_t here = min(kListRows, cnt - j * kListRows);
#pragma unroll
        for (int u = 0; u < (int)(kListRows / (kHistThreads / 32)); u++) {
          const uint32_t r = warp * (kListRows / (kHistThreads / 32)) + u;
          if (r >= here) break;  // warp-uniform
          const int4 e = se[r];
          const uint32_t bb = PACKED ? (uint32_t)sp[r * TB + lane]
                                     : (uint32_t)*reinterpret_cast<const uint16_t*>(sp + r * TB + 2 * lane);
          hist_add_row<PACKED>(hs, bb, make_int2(e.y, e.z), lane, v0, v1, nb);
        }
        __syncthreads();  // slot j is free again
        if (j + kListSlots - 1 < nsl) issue(j + kListSlots - 1, e_next);
        else cp_async_commit();
        e_next = load_entry(j + kListSlots);
      }
      cp_async_wait<0>();
    }
    __syncthreads();
    // the global cells of (grp, t) use the shared layout, so consecutive threads add
    // into consecutive int64 words
    // The CTAs start their passes at different offsets (whole 1024-word steps, so the
    // adds stay coalesced): at any moment they add into different words instead of all
    // contending for the same ones in the L2.
    unsigned long long* gout =
        reinterpret_cast<unsigned long long*>(a.out + ((size_t)grp * ftiles + t) * words);
    // Eight cells per thread are read before their adds are issued, so the pass is not
    // one shared-memory round trip per cell.
    const uint32_t steps = (words + kHistThreads - 1) / kHistThreads;
    const uint32_t rot = blockIdx.x % steps;
    for (uint32_t k0 = 0; k0 < steps; k0 += 8) {
      uint32_t c[8], v[8];
#pragma unroll
      for (int u = 0; u < 8; u++) {
        uint32_t st = k0 + u + rot;
        st = st >= steps ? st - steps : st;
        c[u] = st * kHistThreads + threadIdx.x;
        v[u] = (k0 + u < steps && c[u] < words) ? hs[c[u]] : 0u;
      }
#pragma unroll
      for (int u = 0; u < 8; u++)
        if (v[u] != 0u) {
          hs[c[u]] = 0u;
          atomicAdd(gout + c[u], (unsigned long long)(long long)(int32_t)v[u]);
        }
    }
    w += i1 - i0;
  }
  if (s_abort && threadIdx.x == 0 && a.err) atomicExch(a.err, 1);
}

// --------------------------------------------------------------------------------
// Split scan (src/cpu.rs:235-276), in two kernels:
//   k_gain  one CTA per (node, feature), one thread per bin: the node's histogram
//           (the sibling derived as parent - built child), its exact int64 prefix over
//           bins, and the per-node gain term of every threshold in f64 exactly as
//           src/cpu.rs:242-259 writes it;
//   k_best  one CTA per feature, one thread per threshold: the terms summed in node
//           order (the order src/cpu.rs adds them), the candidate masks, the feature's
//           best threshold (ties to the lowest bin) and, at the last level, the leaf
//           values that threshold would give.
// The cross-feature argmax is taken by the leaf-index update (k_apply).

constexpr int kGainThreads = 256;  // >= n_bins
constexpr int kBestThreads = 256;

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

// Block-wide argmax over kBestThreads threads; the result is valid in thread 0.
__device__ void block_argmax256(double& g, uint32_t& i, double* red_g, uint32_t* red_i) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double g2 = __shfl_down_sync(0xffffffffu, g, off);
    const uint32_t i2 = __shfl_down_sync(0xffffffffu, i, off);
    if (lane + off < 32) argmax_merge(g, i, g2, i2);
  }
  if (lane == 0) {
    red_g[warp] = g;
    red_i[warp] = i;
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int w = 1; w < kBestThreads / 32; w++) argmax_merge(g, i, red_g[w], red_i[w]);
}

// 2^-e for the round's fixed-point exponent e (exact; built from the exponent bits).
__device__ __forceinline__ double q_inv_scale(uint32_t maxbits) {
  return __longlong_as_double((long long)(1023 - rw_qscale_exp(maxbits)) << 52);
}

// One CTA per (node, tile, group of 4 columns); thread b owns bin b of the 4 features in
// those columns. A 32-byte sector of the layout holds exactly 4 columns, so every load
// and store is a whole-sector vector access.
constexpr uint32_t kGainCols = 4;

// One node of k_gain: this thread's bin b of the 4 columns (x: g of the 4, then h), the
// node's full histogram for the next level, the exact prefixes over bins, and the gain
// terms. All threads of the block call it (it synchronises).
__device__ __forceinline__ void gain_node(const SplitLaunch& a, uint32_t nd, const long long* x,
                                          const uint32_t* fq, size_t cell, size_t node_words,
                                          long long (*wsum)[2 * kGainCols], long long* tot) {
  const uint32_t nf = a.nf, nb = a.nb, nsplit = nb - 1, b = threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (!a.last_level && b < nb) {  // the next level's parent histograms
    long long* o = a.hf + nd * node_words + cell;
    reinterpret_cast<longlong2*>(o)[0] = make_longlong2(x[0], x[1]);
    reinterpret_cast<longlong2*>(o)[1] = make_longlong2(x[2], x[3]);
    reinterpret_cast<longlong2*>(o + kHistFeat)[0] = make_longlong2(x[4], x[5]);
    reinterpret_cast<longlong2*>(o + kHistFeat)[1] = make_longlong2(x[6], x[7]);
  }
  // inclusive prefixes over bins (exact int64), 8 at once
  long long p[2 * kGainCols];
#pragma unroll
  for (int i = 0; i < 2 * (int)kGainCols; i++) p[i] = x[i];
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
#pragma unroll
    for (int i = 0; i < 2 * (int)kGainCols; i++) {
      const long long v = __shfl_up_sync(0xffffffffu, p[i], d);
      if (lane >= d) p[i] += v;
    }
  }
  if (lane == 31)
#pragma unroll
    for (int i = 0; i < 2 * (int)kGainCols; i++) wsum[warp][i] = p[i];
  __syncthreads();
  if (threadIdx.x < 2 * kGainCols) {
    long long c = 0;
    for (int w = 0; w < kGainThreads / 32; w++) {
      const long long v = wsum[w][threadIdx.x];
      wsum[w][threadIdx.x] = c;
      c += v;
    }
    tot[threadIdx.x] = c;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2 * (int)kGainCols; i++) p[i] += wsum[warp][i];
  long long tg_[kGainCols], th_[kGainCols];
#pragma unroll
  for (int i = 0; i < (int)kGainCols; i++) {
    tg_[i] = tot[i];
    th_[i] = tot[kGainCols + i];
  }
  __syncthreads();  // wsum and tot are free for the next node
  if (a.prefix && b < nb) {
    // the hessian prefixes k_best reads for the next level's built-child choice
#pragma unroll
    for (int i = 0; i < (int)kGainCols; i++)
      if (fq[i] < nf) a.prefix[((size_t)fq[i] * a.n_nodes + nd) * nb + b] = p[kGainCols + i];
  }
  if (b >= nsplit) return;
  const double inv_g = q_inv_scale(a.maxbits[0]), inv_h = q_inv_scale(a.maxbits[1]);
  const double lambda = a.lambda, mc = a.min_child;
#pragma unroll
  for (int i = 0; i < (int)kGainCols; i++) {
    const uint32_t f = fq[i];
    if (f >= nf) continue;
    const long long pgi = p[i], phi = p[kGainCols + i];
    const long long tg = tg_[i], th = th_[i];
    const double gt = (double)tg * inv_g, ht = (double)th * inv_h;
    const double parent = gt * gt / (ht + lambda);
    const double gl = (double)pgi * inv_g, hl = (double)phi * inv_h;
    const double gr = gt - gl, hr = ht - hl;
    const double dl = hl + lambda, dr = hr + lambda;
    // src/cpu.rs writes valid * (gl^2/(hl+lambda) + gr^2/(hr+lambda) - parent). FP64
    // division is the costly part on this GPU, so an invalid threshold skips it when
    // that product is a zero: both denominators nonzero (the quotients of these finite
    // fixed-point sums are then finite). Its +0 in place of a possible -0 leaves the
    // node-order sum unchanged (the sum starts at +0 and never becomes -0).
    double term;
    if ((hl >= mc) & (hr >= mc)) term = gl * gl / dl + gr * gr / dr - parent;
    else if (dl != 0.0 && dr != 0.0 && parent - parent == 0.0) term = 0.0;
    else term = 0.0 * (gl * gl / dl + gr * gr / dr - parent);
    a.term[((size_t)f * a.n_nodes + nd) * nsplit + b] = term;
    if (a.mono && a.monotone[f] != 0) {
      // exact left/right (g, h) totals over all nodes for the monotone rule
      unsigned long long* m =
          reinterpret_cast<unsigned long long*>(a.mono + ((size_t)f * nsplit + b) * 4);
      atomicAdd(m + 0, (unsigned long long)pgi);
      atomicAdd(m + 1, (unsigned long long)phi);
      atomicAdd(m + 2, (unsigned long long)(tg - pgi));
      atomicAdd(m + 3, (unsigned long long)(th - phi));
    }
  }
}

// One CTA per (node, 4-column sector); with subtraction the node's histogram is its
// pair's built child (hb, keyed by the parent) or the sibling parent - built. Thread b
// owns bin b of the 4 features in those columns; a 32-byte sector of the layout holds
// exactly 4 columns, so every load and store is a whole-sector vector access. (One CTA
// per node pair, loading the pair once for both children, measured slower: half the
// CTAs, each twice as long.)
__global__ void __launch_bounds__(kGainThreads) k_gain(SplitLaunch a) {
  __shared__ long long wsum[kGainThreads / 32][2 * kGainCols];
  __shared__ long long tot[2 * kGainCols];
  const uint32_t nd = blockIdx.x;
  const uint32_t t = blockIdx.y / (kHistFeat / kGainCols);
  const uint32_t c0 = (blockIdx.y % (kHistFeat / kGainCols)) * kGainCols;
  const uint32_t nf = a.nf, nb = a.nb, b = threadIdx.x;
  const uint32_t ftiles = (nf + kHistFeat - 1) / kHistFeat;
  uint32_t fq[kGainCols];
  bool any = false;
#pragma unroll
  for (int i = 0; i < (int)kGainCols; i++) {
    const uint32_t c = c0 + i;  // column -> feature: j -> 2j, 32 + j -> 2j + 1
    fq[i] = t * kHistFeat + 2 * (c % 32) + c / 32;
    any |= fq[i] < nf;
  }
  if (!any) {  // uniform per CTA
    pdl_wait();
    pdl_trigger();
    return;
  }
  // 4 consecutive int64 columns (one 32-byte sector) for g and for h
  auto load4 = [](const long long* src, long long* dst) {
    const longlong2 u = __ldcg(reinterpret_cast<const longlong2*>(src));
    const longlong2 v = __ldcg(reinterpret_cast<const longlong2*>(src + 2));
    dst[0] = u.x;
    dst[1] = u.y;
    dst[2] = v.x;
    dst[3] = v.y;
  };
  const size_t cell = ((size_t)t * nb + (b < nb ? b : 0)) * (2 * kHistFeat) + c0;
  const size_t node_words = (size_t)ftiles * nb * 2 * kHistFeat;
  const size_t k = (size_t)(a.mode == 0 ? nd : (nd >> 1)) * node_words + cell;
  // The parent level's histograms (the previous level's split scan) and the built-child
  // flag (the previous leaf-index update) come from grids that have completed: load
  // them while the histogram grid this kernel waits for finishes.
  long long pp[2 * kGainCols], x[2 * kGainCols];
#pragma unroll
  for (int i = 0; i < 2 * (int)kGainCols; i++) pp[i] = x[i] = 0;
  bool built_here = true;
  if (a.mode == 1) {
    if (b < nb) {
      load4(a.hp + k, pp);
      load4(a.hp + k + kHistFeat, pp + kGainCols);
    }
    built_here = (a.built_odd ? a.built_odd[nd >> 1] != 0 : true) == ((nd & 1u) != 0);
  }
  pdl_wait();
  pdl_trigger();
  if (b < nb) {
    load4(a.hb + k, x);
    load4(a.hb + k + kHistFeat, x + kGainCols);
    if (!built_here)
#pragma unroll
      for (int i = 0; i < 2 * (int)kGainCols; i++) x[i] = pp[i] - x[i];
  }
  gain_node(a, nd, x, fq, cell, node_words, wsum, tot);
}

__global__ void __launch_bounds__(kBestThreads) k_best(SplitLaunch a) {
  __shared__ double red_g[kBestThreads / 32];
  __shared__ uint32_t red_i[kBestThreads / 32];
  __shared__ uint32_t s_b;
  const uint32_t f = blockIdx.x;
  const uint32_t nb = a.nb, nsplit = nb - 1, b = threadIdx.x;
  // Before the wait: everything here comes from grids at least two launches back (the
  // previous level's leaf-index update, this round's gradients, the cut table), and the
  // words written are read by no grid before the leaf-index update that follows.
  if (f == 0) {
    // this level's per-node row counts (from the previous level's lists) and the cursors
    // the leaf-index update fills for the next level
    if (a.ncount && a.cursor_prev)
      for (uint32_t c = threadIdx.x; c < a.n_nodes; c += kBestThreads) {
        uint32_t v;
        if (a.subtract) {
          const uint32_t k = c >> 1, built = __ldcg(a.cursor_prev + k);
          v = ((c & 1u) == (uint32_t)__ldcg(a.built_prev + k)) ? built
                                                                 : __ldcg(a.pcount + k) - built;
        } else {
          v = __ldcg(a.cursor_prev + c);
        }
        a.ncount[c] = v;
      }
    if (a.cursor_next)
      for (uint32_t w = threadIdx.x; w < a.cursor_next_words; w += kBestThreads)
        a.cursor_next[w] = 0u;
  }
  const double inv_g = q_inv_scale(__ldcg(a.maxbits)), inv_h = q_inv_scale(__ldcg(a.maxbits + 1));
  const double lambda = a.lambda;
  const float thr_own = b < nsplit ? __ldg(a.cuts + (size_t)f * nsplit + b) : 0.0f;
  const int mono = a.mono ? a.monotone[f] : 0;
  pdl_wait();
  pdl_trigger();
  double key = -RW_INF;
  if (b < nsplit) {
    // the node-order sum (src/cpu.rs adds the nodes' gains in node order)
    double gain = 0.0;
    const double* t = a.term + (size_t)f * a.n_nodes * nsplit + b;
    for (uint32_t nd = 0; nd < a.n_nodes; nd++) gain += __ldcg(t + (size_t)nd * nsplit);
    key = gain;
    // candidate masks (extensions): per-tree column sampling and monotone direction
    const bool dropped = a.colsample < 1.0f &&
                         (float)hash01_bits(f, a.tree_seed ^ 0x5bd1e995u) / 16777215.0f >=
                             a.colsample;
    if (mono) {
      long long* m = a.mono + ((size_t)f * nsplit + b) * 4;
      const double glt = (double)__ldcg(m + 0) * inv_g, hlt = (double)__ldcg(m + 1) * inv_h;
      const double grt = (double)__ldcg(m + 2) * inv_g, hrt = (double)__ldcg(m + 3) * inv_h;
      m[0] = m[1] = m[2] = m[3] = 0;  // ready for the next level
      const double wl = -glt / (hlt + lambda);
      const double wr = -grt / (hrt + lambda);
      if (!dropped && ((mono > 0 && wl > wr) || (mono < 0 && wl < wr))) key = -1e30;
    }
    if (dropped) key = -1e30;
    if (key != key) key = -RW_INF;  // NaN never wins (cpu.rs: `gv > bg`)
  }
  const double key_own = key;
  uint32_t idx = b;
  block_argmax256(key, idx, red_g, red_i);
  if (threadIdx.x == 0) {
    // ties: the lowest bin; an all-infeasible feature reports bin 0
    const uint32_t bb = key == -RW_INF ? 0u : idx;
    s_b = bb;
  }
  __syncthreads();
  if (threadIdx.x == s_b) {
    // the winning bin's thread writes the record (its cut value is in its own reach)
    SplitRec r;
    r.gain = key_own;
    r.bin = s_b;
    r.thr = thr_own;
    a.rec[f] = r;
  }
  __syncthreads();
  const uint32_t bs = s_b;
  // Which child of each node the next level builds if this feature wins: the side with
  // less hessian (ties: the right, odd child); its sibling is derived by subtraction.
  // Any choice gives the same exact histograms; this one reads allreduced sums, so
  // every rank makes the same choice.
  if (!a.last_level && a.choice && a.prefix)
    for (uint32_t nd = threadIdx.x; nd < a.n_nodes; nd += kBestThreads) {
      const long long* pr = a.prefix + ((size_t)f * a.n_nodes + nd) * nb;
      const long long hl = __ldcg(pr + bs), ht = __ldcg(pr + nb - 1);
      a.choice[(size_t)f * a.n_nodes + nd] = (ht - hl) <= hl ? 1 : 0;
    }
}

// --------------------------------------------------------------------------------

// Binning (src/gpu_kernels.rs:496-529 == src/cpu.rs:149-155): bin = #{cut < v}, by binary
// search over the feature's cuts (staged in shared memory); NaN compares false, giving
// bin 0. One CTA bins 256 rows of one 64-feature tile: it writes colbins directly and
// the rows' tile of rowbins through a shared [256][64] staging block (16-byte stores).
constexpr int kBinRows = 256;

__global__ void __launch_bounds__(kBinRows) k_bin(const float* __restrict__ x, uint64_t n,
                                                  uint32_t nf, const float* __restrict__ cuts,
                                                  uint32_t nb1, uint64_t n_pad,
                                                  uint8_t* __restrict__ colbins,
                                                  uint8_t* __restrict__ rowbins) {
  extern __shared__ __align__(16) unsigned char bin_smem[];
  uint8_t* tile = bin_smem;                                        // [kBinRows][kHistFeat]
  float* s_cuts = reinterpret_cast<float*>(bin_smem + kBinRows * kHistFeat);  // [64][nb1]
  const uint32_t t = blockIdx.y, f0 = t * kHistFeat;
  const uint32_t fc = nf - f0 < kHistFeat ? nf - f0 : kHistFeat;
  for (uint32_t i = threadIdx.x; i < fc * nb1; i += kBinRows) s_cuts[i] = cuts[(size_t)f0 * nb1 + i];
  for (uint32_t i = threadIdx.x; i < kBinRows * kHistFeat / 16; i += kBinRows)
    reinterpret_cast<uint4*>(tile)[i] = make_uint4(0u, 0u, 0u, 0u);
  __syncthreads();
  const uint64_t r0 = (uint64_t)blockIdx.x * kBinRows, r = r0 + threadIdx.x;
  if (r < n) {
    for (uint32_t fl = 0; fl < fc; fl++) {
      const float v = __ldg(x + r * nf + f0 + fl);
      const float* c = s_cuts + (size_t)fl * nb1;
      uint32_t lo = 0, hi = nb1;
      while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        if (c[mid] < v) lo = mid + 1;
        else hi = mid;
      }
      colbins[(size_t)(f0 + fl) * n_pad + r] = (uint8_t)lo;
      tile[threadIdx.x * kHistFeat + fl] = (uint8_t)lo;
    }
  }
  __syncthreads();
  // rows r0 .. r0+255 of tile t (rows past n stay zero; n_pad is a multiple of 256)
  for (uint32_t i = threadIdx.x; i < kBinRows * kHistFeat / 16; i += kBinRows) {
    const uint32_t row = i / (kHistFeat / 16), part = i % (kHistFeat / 16);
    if (r0 + row < n_pad)
      *reinterpret_cast<uint4*>(rowbins + ((size_t)t * n_pad + r0 + row) * kHistFeat + part * 16) =
          reinterpret_cast<const uint4*>(tile)[i];
  }
}

// 4-bit packing (src/gpu_kernels.rs:628-643 packs pairs the same way): within each row's
// feature tile, byte k = bin(2k) | bin(2k+1) << 4. One thread per 16 output bytes.
__global__ void k_pack4(const uint8_t* __restrict__ u8, uint64_t n_pad, uint32_t ftiles,
                        uint8_t* __restrict__ packed) {
  const uint64_t items = n_pad * ftiles * 2;  // 2 x 16 output bytes per row tile
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < items;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = i / (ftiles * 2);
    const uint32_t rem = (uint32_t)(i % (ftiles * 2)), t = rem / 2, half = rem % 2;
    const uint8_t* src = u8 + ((size_t)t * n_pad + r) * kHistFeat + half * 32;
    const uint4 a = *reinterpret_cast<const uint4*>(src);
    const uint4 b = *reinterpret_cast<const uint4*>(src + 16);
    const uint32_t in[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    uint32_t out[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint32_t lo = in[2 * k], hi = in[2 * k + 1];
      // bytes (b0 b1 b2 b3) -> nibble pairs (b0|b1<<4, b2|b3<<4)
      const uint32_t plo = (lo & 0xfu) | ((lo >> 4) & 0xf0u) | (((lo >> 16) & 0xfu) << 8) |
                           (((lo >> 24) & 0xfu) << 12);
      const uint32_t phi = (hi & 0xfu) | ((hi >> 4) & 0xf0u) | (((hi >> 16) & 0xfu) << 8) |
                           (((hi >> 24) & 0xfu) << 12);
      out[k] = plo | (phi << 16);
    }
    *reinterpret_cast<uint4*>(packed + ((size_t)t * n_pad + r) * (kHistFeat / 2) + half * 16) =
        make_uint4(out[0], out[1], out[2], out[3]);
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

// A tree's leaf values from its exact wide-fixed-point sums (src/cpu.rs:316-317:
// (-lr * G / (H + lambda)) as f32), one thread per leaf.
__global__ void k_leafval(LeafValues a) {
  pdl_enter();
  const uint32_t mg = __ldcg(a.maxbits);
  const int wg = rw_wscale_exp(mg, a.n_rows);
  const int wh = rw_wscale_exp(__ldcg(a.maxbits + 1), a.n_rows);
  const int wg2 = rw_wscale_exp(rw_sq_maxbits(mg), a.n_rows);
  for (uint32_t l = blockIdx.x * blockDim.x + threadIdx.x; l < a.n_leaves;
       l += gridDim.x * blockDim.x) {
    const double G = rw_wvalue(__ldcg(a.leafsum + l), wg);
    const double H = rw_wvalue(__ldcg(a.leafsum + a.n_leaves + l), wh);
    a.leafval[l] = (float)(-a.lr * G / (H + a.lambda));
    if (a.leafvar)  // PGBM (gpu_kernels.rs:1046-1080), from the exact sums
      a.leafvar[l] = rw_leaf_variance(G, H, rw_wvalue(__ldcg(a.leafsum2 + l), wg2), a.lr);
  }
}

// PGBM: the leaves' g^2 sums (gpu_kernels.rs:1015-1043 adds gi * gi per row), exact in the
// wide fixed point whose scale comes from (max |g|)^2. Per CTA in shared memory (at most
// 4096 leaves), then one global add per nonzero sum. The preceding grid (the tree's last
// leaf-index update) writes the leaf indices, so they are read after the wait.
constexpr int kLeafSqThreads = 256;
__global__ void __launch_bounds__(kLeafSqThreads) k_leafsq(LeafSquares a) {
  __shared__ long long s2[4096];
  for (uint32_t l = threadIdx.x; l < a.n_leaves; l += blockDim.x) s2[l] = 0;
  const int w2 = rw_wscale_exp(rw_sq_maxbits(__ldcg(a.maxbits)), a.n_rows);
  pdl_enter();
  __syncthreads();
  const uint64_t n4 = a.n_pad / 4;
  for (uint64_t qi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; qi < n4;
       qi += (uint64_t)gridDim.x * blockDim.x) {
    const uint2 nd2 = __ldcg(reinterpret_cast<const uint2*>(a.node + qi * 4));
    const float4 g4 = __ldcg(reinterpret_cast<const float4*>(a.g + qi * 4));
    const uint32_t leaf[4] = {nd2.x & 0x7fffu, (nd2.x >> 16) & 0x7fffu, nd2.y & 0x7fffu,
                              (nd2.y >> 16) & 0x7fffu};
    const float gv[4] = {g4.x, g4.y, g4.z, g4.w};
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const long long v = rw_wquantize(gv[k] * gv[k], w2);
      if (v && leaf[k] < a.n_leaves)
        atomicAdd(reinterpret_cast<unsigned long long*>(s2 + leaf[k]), (unsigned long long)v);
    }
  }
  __syncthreads();
  for (uint32_t l = threadIdx.x; l < a.n_leaves; l += blockDim.x)
    if (s2[l]) atomicAdd(reinterpret_cast<unsigned long long*>(a.leafsum2 + l),
                         (unsigned long long)s2[l]);
}

// Gradients (src/cpu.rs:181-193), stride row sampling (src/cpu.rs:172-176, 202-204)
// and the round's maxima over the sampled rows, 4 rows per thread. Unsampled and padded
// rows (n <= i < n_pad) get g = h = 0, which removes them from every histogram and leaf
// sum. With a previous tree, every row first takes its leaf value:
// pred += leafval[leaf] (src/cpu.rs:319-320), in f32 as the reference adds it.
__global__ void k_grad(float* __restrict__ pred, const float* __restrict__ y,
                       float* __restrict__ g, float* __restrict__ h, uint64_t n, uint64_t n_pad,
                       int logistic, uint64_t stride, uint64_t phase, uint64_t row_offset,
                       int compute_max, uint32_t* maxbits, uint32_t* zero_word, PrevTree pt) {
  pdl_enter();
  if (zero_word && blockIdx.x == 0 && threadIdx.x == 0) *zero_word = 0u;
  uint32_t mg = 0, mh = 0;
  const uint64_t n4 = n_pad / 4;
  for (uint64_t qi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; qi < n4;
       qi += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r = qi * 4;
    float4 p4 = make_float4(0.f, 0.f, 0.f, 0.f), y4 = p4;
    if (r < n) {
      p4 = *reinterpret_cast<const float4*>(pred + r);
      y4 = __ldg(reinterpret_cast<const float4*>(y + r));
      if (pt.leafval) {
        const uint2 nd = *reinterpret_cast<const uint2*>(pt.node + r);
        p4.x = p4.x + __ldg(pt.leafval + (nd.x & 0x7fffu));
        p4.y = p4.y + __ldg(pt.leafval + ((nd.x >> 16) & 0x7fffu));
        p4.z = p4.z + __ldg(pt.leafval + (nd.y & 0x7fffu));
        p4.w = p4.w + __ldg(pt.leafval + ((nd.y >> 16) & 0x7fffu));
        *reinterpret_cast<float4*>(pred + r) = p4;  // rows past n are never read
      }
    }
    const float pv[4] = {p4.x, p4.y, p4.z, p4.w}, yv[4] = {y4.x, y4.y, y4.z, y4.w};
    float gv[4], hv[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
      const uint64_t i = r + k;
      gv[k] = 0.0f;
      hv[k] = 0.0f;
      if (i < n) {
        if (logistic) rw_logistic_grad(pv[k], yv[k], &gv[k], &hv[k]);
        else {
          gv[k] = pv[k] - yv[k];
          hv[k] = 1.0f;
        }
      }
      const bool sampled = i < n && (stride <= 1 || ((row_offset + i) % stride) == phase);
      if (!sampled) {
        gv[k] = 0.0f;
        hv[k] = 0.0f;
      }
      mg = max(mg, f32_bits_abs(gv[k]));
      mh = max(mh, f32_bits_abs(hv[k]));
    }
    *reinterpret_cast<float4*>(g + r) = make_float4(gv[0], gv[1], gv[2], gv[3]);
    *reinterpret_cast<float4*>(h + r) = make_float4(hv[0], hv[1], hv[2], hv[3]);
  }
  if (compute_max) block_max2_atomic(mg, mh, maxbits);
}

// Per round: q = round(x * 2^e) for g and h (scales from the final maxima), the row's
// excluded flag (node bit 15; a row whose g and h both quantise to 0 adds nothing to any
// sum) and node reset. Also zeroes the level-0 histogram and counts the rows that are
// not excluded (the root's row count, for the level-0 leaf-index update's list).
constexpr uint16_t kExcluded = 0x8000;

__global__ void k_quant(const float* __restrict__ g, const float* __restrict__ h,
                        const uint32_t* __restrict__ maxbits, uint64_t n_pad,
                        int2* __restrict__ q, uint16_t* __restrict__ node,
                        long long* __restrict__ hb0, uint64_t hb0_words,
                        long long* __restrict__ leafsum, uint32_t leafsum_words,
                        uint32_t* __restrict__ ncount0) {
  pdl_enter();
  __shared__ uint32_t s_rows;
  if (threadIdx.x == 0) s_rows = 0u;
  __syncthreads();
  uint32_t rows = 0;
  const float sg = rw_pow2f(rw_qscale_exp(maxbits[0]));
  const float sh = rw_pow2f(rw_qscale_exp(maxbits[1]));
  const uint64_t tid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t nthr = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t w = tid; w < hb0_words; w += nthr) hb0[w] = 0;
  for (uint64_t w = tid; w < leafsum_words; w += nthr) leafsum[w] = 0;
  for (uint64_t i = tid; i < n_pad; i += nthr) {
    const int32_t a = rw_quantize(g[i], sg), b = rw_quantize(h[i], sh);
    q[i] = make_int2(a, b);
    node[i] = (a | b) == 0 ? kExcluded : 0;
    rows += (a | b) != 0;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) rows += __shfl_down_sync(0xffffffffu, rows, off);
  if ((threadIdx.x & 31) == 0 && rows) atomicAdd(&s_rows, rows);
  __syncthreads();
  if (threadIdx.x == 0 && s_rows && ncount0) atomicAdd(ncount0, s_rows);
}

// Every CTA first picks the level's split from the per-feature records (highest gain,
// ties to the lowest feature: src/cpu.rs:271; no feasible split anywhere gives feature
// 0, bin 0); CTA 0 also writes the model slot and feature importance
// (src/cpu.rs:272-276) and, at the last level, the tree's leaf values.
// Then leaf = 2*leaf + (bin[f*] > t*) (src/cpu.rs:278-281) for 4 rows per thread, keeping
// the excluded flag. Non-final levels also write the next level's row list: node nd owns
// the region [cap[nd], cap[nd+1]) of `entries` (cap = prefix of the nodes' row counts);
// with subtraction it holds the rows of the child k_best chose to build, from its start;
// without, the left child's rows from the start and the right child's from the end.
// Each chunk of rows ranks its rows per group in shared memory (warp-aggregated) and
// reserves space with one global add per nonzero group; the entry carries the row's q.
// The final level adds every row's unquantised g and h, in the wide fixed point
// (rw_wquantize), into its leaf's exact int64 sums (src/cpu.rs:286-318): per CTA in
// shared memory for up to kLeafSmem leaves, then one global add per nonzero sum.
constexpr int kApplyThreads = 256;
constexpr uint32_t kLeafSmem = 1024;

// The level's split from the per-feature records (every CTA), and by CTA 0 the model
// slot and feature importance. Leaves (feature, bin) in s_ft. `r0` is this thread's
// record of feature threadIdx.x (loaded by the caller together with its other reads);
// s_bin holds the bins of the first blockDim.x features.
static_assert(sizeof(SplitRec) == 16, "a record is one 16-byte load (the buffers are allocation-aligned)");
__device__ void choose_split(const ApplyLaunch& a, const SplitRec& r0, uint32_t* s_ft,
                             double* red_g, uint32_t* red_i, uint32_t* s_bin) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double bk = -RW_INF;
  uint32_t bf = 0xffffffffu;
  if (threadIdx.x < a.nf) {
    argmax_merge(bk, bf, r0.gain, threadIdx.x);
    s_bin[threadIdx.x] = r0.bin;
  }
  for (uint32_t ff = threadIdx.x + blockDim.x; ff < a.nf; ff += blockDim.x)
    argmax_merge(bk, bf, __ldcg(&a.rec[ff].gain), ff);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const double g2 = __shfl_down_sync(0xffffffffu, bk, off);
    const uint32_t i2 = __shfl_down_sync(0xffffffffu, bf, off);
    if (lane + off < 32) argmax_merge(bk, bf, g2, i2);
  }
  if (lane == 0) {
    red_g[warp] = bk;
    red_i[warp] = bf;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (uint32_t w = 1; w < blockDim.x / 32; w++) argmax_merge(bk, bf, red_g[w], red_i[w]);
    if (bk == -RW_INF) bf = 0;
    const uint32_t bb = bf < blockDim.x ? s_bin[bf] : __ldcg(&a.rec[bf].bin);
    s_ft[0] = bf;
    s_ft[1] = bb;
    if (blockIdx.x == 0) {
      a.feat[a.slot] = bf;
      a.thr[a.slot] = __ldcg(&a.rec[bf].thr);
      if (a.thr_bin) a.thr_bin[a.slot] = (uint16_t)bb;
      a.fi_gain[bf] += (float)(bk > 0.0 ? bk : 0.0);
      a.fi_count[bf] += 1.0f;
      if (a.split_out) {
        a.split_out[0] = bf;
        a.split_out[1] = bb;
      }
    }
  }
  __syncthreads();
}

// FINAL: the last level of a tree (leaf sums, no list); a separate instantiation keeps
// the listing levels' register count (and so their occupancy) free of the leaf sums.
template <bool FINAL>
__global__ void __launch_bounds__(kApplyThreads, 8) k_apply(ApplyLaunch a) {
  extern __shared__ __align__(16) uint32_t lsm[];
  __shared__ double red_g[kApplyThreads / 32];
  __shared__ uint32_t red_i[kApplyThreads / 32];
  __shared__ uint32_t s_ft[2];
  __shared__ uint32_t warp_sums[33];
  __shared__ uint32_t s_bin[kApplyThreads];
  const uint32_t lane = threadIdx.x & 31;
  const LevelLists& L = a.lists;
  const bool listing = !FINAL && L.entries;
  const uint32_t n_nodes = a.n_children / 2;
  const uint32_t G = L.subtract ? n_nodes : a.n_children;  // next-level groups
  uint32_t* s_cap = lsm;                   // [n_nodes + 1] prefix of the node row counts
  uint32_t* s_cnt = s_cap + n_nodes + 1;   // [G] this chunk's rows per group
  uint32_t* s_base = s_cnt + G;            // [G] their reservation in the group's region
  uint8_t* s_choice = reinterpret_cast<uint8_t*>(s_base + G);  // [n_nodes]
  // final level: the CTA's leaf sums [2][n_leaves] (g, then h) when they fit
  long long* s_ls = reinterpret_cast<long long*>(lsm);
  const bool ls_smem = FINAL && a.n_leaves <= kLeafSmem;
  int wg = 0, wh = 0;
  if (FINAL && ls_smem)
    for (uint32_t l = threadIdx.x; l < 2 * a.n_leaves; l += blockDim.x) s_ls[l] = 0;
  long long* ls = ls_smem ? s_ls : a.leafsum;
  if (listing)
    for (uint32_t g = threadIdx.x; g < G; g += blockDim.x) s_cnt[g] = 0u;
  // Before the wait (the preceding grid is the split scan, which writes neither): the
  // next level's built-histogram buffer is zeroed (the level before last used it and
  // has completed) and the first chunk's leaf indices are loaded (the previous
  // leaf-index update wrote them).
  if (a.hb_next) {
    const uint64_t vec = a.hb_next_words / 2, stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t v = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < vec; v += stride)
      reinterpret_cast<longlong2*>(a.hb_next)[v] = make_longlong2(0, 0);
  }
  const uint64_t n4 = a.n_pad / 4;
  const uint64_t qi0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint2 nd_first = make_uint2(0u, 0u);
  if (qi0 < n4) nd_first = *reinterpret_cast<const uint2*>(a.node + qi0 * 4);
  if (FINAL) {  // this round's scales (the gradient pass, long completed)
    wg = rw_wscale_exp(__ldcg(a.maxbits), a.n_rows);
    wh = rw_wscale_exp(__ldcg(a.maxbits + 1), a.n_rows);
  }
  pdl_wait();
  pdl_trigger();
  // the split records and the node row counts (both from the split scan) in one round
  SplitRec r0 = {};
  if (threadIdx.x < a.nf) {
    const double2 rv = __ldcg(reinterpret_cast<const double2*>(a.rec + threadIdx.x));
    r0.gain = rv.x;
    r0.bin = (uint32_t)__double_as_longlong(rv.y);
  }
  uint32_t nc[4] = {0u, 0u, 0u, 0u};
  const uint32_t nc_per = (n_nodes + blockDim.x - 1) / blockDim.x, nc0 = threadIdx.x * nc_per;
  if (listing)
#pragma unroll
    for (int k = 0; k < 4; k++)
      if (k < (int)nc_per && nc0 + k < n_nodes) nc[k] = __ldcg(L.ncount + nc0 + k);
  choose_split(a, r0, s_ft, red_g, red_i, s_bin);
  const uint32_t f = s_ft[0], t = s_ft[1];
  if (listing) {
    block_exclusive_scan_vals(nc, n_nodes, s_cap, warp_sums);
    if (L.subtract)
      for (uint32_t nd = threadIdx.x; nd < n_nodes; nd += blockDim.x) {
        const uint8_t c = __ldcg(L.choice + (size_t)f * n_nodes + nd);
        s_choice[nd] = c;
        if (blockIdx.x == 0) L.built_odd[nd] = c;
      }
    __syncthreads();
  }
  const uint8_t* col = a.colbins + (size_t)f * a.n_pad;
  // block-uniform chunks of blockDim.x row quads (the list phases synchronise the CTA)
  for (uint64_t c0 = (uint64_t)blockIdx.x * blockDim.x; c0 < n4;
       c0 += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t qi = c0 + threadIdx.x;
    uint32_t nds[4] = {kExcluded, kExcluded, kExcluded, kExcluded}, par[4] = {0, 0, 0, 0};
    if (qi < n4) {
      const uint64_t r = qi * 4;
      const uint32_t b4 = *reinterpret_cast<const uint32_t*>(col + r);
      uint2 nd2 = qi == qi0 ? nd_first : *reinterpret_cast<const uint2*>(a.node + r);
      nds[0] = nd2.x & 0xffffu;
      nds[1] = nd2.x >> 16;
      nds[2] = nd2.y & 0xffffu;
      nds[3] = nd2.y >> 16;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        const uint32_t ex = nds[q] & kExcluded;
        par[q] = nds[q] & 0x7fffu;
        nds[q] = ex | (par[q] * 2u + (((b4 >> (8 * q)) & 0xffu) > t ? 1u : 0u));
      }
      nd2.x = (nds[0] & 0xffffu) | (nds[1] << 16);
      nd2.y = (nds[2] & 0xffffu) | (nds[3] << 16);
      *reinterpret_cast<uint2*>(a.node + r) = nd2;
      if (FINAL) {
        // every sampled row counts, including rows whose 17-bit q are both 0
        const float4 g4 = __ldcg(reinterpret_cast<const float4*>(a.g + r));
        const float4 h4 = __ldcg(reinterpret_cast<const float4*>(a.h + r));
        const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, hv[4] = {h4.x, h4.y, h4.z, h4.w};
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const uint32_t leaf = nds[q] & 0x7fffu;
          const long long qg = rw_wquantize(gv[q], wg), qh = rw_wquantize(hv[q], wh);
          if (qg) atomicAdd(reinterpret_cast<unsigned long long*>(ls + leaf), (unsigned long long)qg);
          if (qh)
            atomicAdd(reinterpret_cast<unsigned long long*>(ls + a.n_leaves + leaf),
                      (unsigned long long)qh);
        }
      }
    }
    if (!listing) continue;
    // the next level's list: group key and the row's rank among this chunk's rows of
    // the group (warp-aggregated shared counters)
    uint32_t key[4], rank[4];
#pragma unroll
    for (int q = 0; q < 4; q++) {
      uint32_t k = 0xffffffffu;
      if (!(nds[q] & kExcluded)) {
        const uint32_t bit = nds[q] & 1u;
        if (!L.subtract) k = nds[q];
        else if (bit == s_choice[par[q]]) k = par[q];
      }
      const uint32_t peers = __match_any_sync(0xffffffffu, k);
      const uint32_t leader = (uint32_t)(__ffs(peers) - 1);
      uint32_t base = 0u;
      if (k != 0xffffffffu && lane == leader) base = atomicAdd(&s_cnt[k], (uint32_t)__popc(peers));
      base = __shfl_sync(0xffffffffu, base, (int)leader);
      key[q] = k;
      rank[q] = base + (uint32_t)__popc(peers & ((1u << lane) - 1u));
    }
    // the listed rows' q go out before the space reservation
    int2 qv[4];
#pragma unroll
    for (int q = 0; q < 4; q++)
      qv[q] = key[q] != 0xffffffffu ? __ldg(L.q + qi * 4 + q) : make_int2(0, 0);
    __syncthreads();
    for (uint32_t g = threadIdx.x; g < G; g += blockDim.x) {
      const uint32_t c = s_cnt[g];
      if (c) {
        s_base[g] = atomicAdd(L.cursor + g, c);
        s_cnt[g] = 0u;
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const uint32_t k = key[q];
      if (k == 0xffffffffu) continue;
      const uint32_t rk = s_base[k] + rank[q];
      uint32_t pos;
      if (L.subtract) {
        pos = s_cap[k] + rk;  // the built child fills its node's region from the start
      } else {
        const uint32_t pn = k >> 1;  // left child from the start, right child from the end
        pos = (k & 1u) ? s_cap[pn + 1] - 1u - rk : s_cap[pn] + rk;
      }
      const uint32_t row = (uint32_t)(qi * 4 + q);
      if (pos < a.n_pad) L.entries[pos] = make_int4((int)row, qv[q].x, qv[q].y, 0);
    }
  }
  if (ls_smem) {
    __syncthreads();
    for (uint32_t l = threadIdx.x; l < 2 * a.n_leaves; l += blockDim.x) {
      const long long v = s_ls[l];
      if (v) atomicAdd(reinterpret_cast<unsigned long long*>(a.leafsum + l), (unsigned long long)v);
    }
  }
}

__global__ void k_fill(float* p, float v, uint64_t n) {
  pdl_enter();
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
       i += (uint64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// ---- GOSS (src/cpu.rs:64-110): exact k-th largest |g| by MSB-first radix select ----

__global__ void k_goss_init(uint32_t* sel, uint64_t k) {
  pdl_enter();
  sel[0] = 0u;  // prefix
  sel[1] = 0u;  // mask of decided bits
  sel[2] = (uint32_t)k;
  sel[3] = 0u;
}

__global__ void k_goss_digit_hist(const float* __restrict__ g, uint64_t n,
                                  unsigned long long* counts, const uint32_t* sel, int pass) {
  pdl_enter();
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
  pdl_enter();
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
  pdl_enter();
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

// Launches a level-loop kernel with programmatic stream serialization (see pdl_enter).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
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

// The dynamic shared-memory limit of a kernel only ever grows (per device), so a launch
// that needs less than an earlier one of the same kernel still fits. Returns the CTAs
// per SM for (kernel, block size, shared bytes), cached.
static int set_smem_and_occupancy(const void* kfn, int threads, size_t smem) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, size_t> limit;
  static std::map<std::pair<std::pair<int, const void*>, size_t>, int> occ;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  const auto kd = std::make_pair(dev, kfn);
  size_t& lim = limit[kd];
  if (smem > lim) {
    if (cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess)
      return 0;
    lim = smem;
  }
  const auto key = std::make_pair(kd, smem);
  auto it = occ.find(key);
  if (it != occ.end()) return it->second;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kfn, threads, smem) != cudaSuccess)
    per_sm = 0;
  occ[key] = per_sm;
  return per_sm;
}

// All training kernels ask for the maximum shared-memory carveout, so consecutive
// launches of the level loop never change the SM's L1/shared split between them.
static void prefer_max_smem(const void* kfn) {
  static std::mutex mu;
  static std::map<std::pair<int, const void*>, bool> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  std::lock_guard<std::mutex> lock(mu);
  bool& d = done[std::make_pair(dev, kfn)];
  if (d) return;
  cudaFuncSetAttribute(kfn, cudaFuncAttributePreferredSharedMemoryCarveout,
                       cudaSharedmemCarveoutMaxShared);
  d = true;
}
#define RW_PREFER_SMEM(k) prefer_max_smem(reinterpret_cast<const void*>(&k))

cudaError_t launch_hist(const HistLaunch& L, cudaStream_t s, int* n_launch) {
  if (L.nb < 2 || L.nb > 256 || (L.packed && L.nb > 16)) return cudaErrorInvalidValue;
  const uint32_t ftiles = (L.nf + kHistFeat - 1) / kHistFeat;
  const uint32_t tb = L.packed ? kHistFeat / 2 : kHistFeat;
  const size_t smem = (size_t)(L.nb + 1) * 2 * kHistFeat * 4 +  // + the dummy bin row
                      (L.entries ? (size_t)kListSlots * kListRows * (tb + 16) +
                                       ((size_t)L.groups * 2 + 2 + L.parents) * 4
                                 : (size_t)kStreamStages * kStreamRows * (tb + 8));
  if (L.entries && (L.groups > 4 * kHistThreads || L.parents > 4 * kHistThreads))
    return cudaErrorInvalidValue;
  if (!L.entries && (L.n_ident % kStreamRows) != 0) return cudaErrorInvalidValue;
  const void* kfn = L.packed ? reinterpret_cast<const void*>(&k_hist<true>)
                             : reinterpret_cast<const void*>(&k_hist<false>);
  const int per_sm = set_smem_and_occupancy(kfn, kHistThreads, smem);
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const int grid = sm_count() * per_sm;
  if (n_launch) (*n_launch)++;
  RW_PREFER_SMEM(k_hist<true>);
  RW_PREFER_SMEM(k_hist<false>);
  return L.packed ? launch_pdl(k_hist<true>, dim3(grid), dim3(kHistThreads), smem, s, L, ftiles)
                  : launch_pdl(k_hist<false>, dim3(grid), dim3(kHistThreads), smem, s, L, ftiles);
}

cudaError_t launch_split(const SplitLaunch& a, cudaStream_t s, int* nl) {
  if (a.nb > (uint32_t)kGainThreads) return cudaErrorInvalidValue;
  RW_PREFER_SMEM(k_gain);
  RW_PREFER_SMEM(k_best);
  const uint32_t ftiles = (a.nf + kHistFeat - 1) / kHistFeat;
  const uint32_t groups = ftiles * (kHistFeat / kGainCols);
  cudaError_t e = launch_pdl(k_gain, dim3(a.n_nodes, groups), dim3(kGainThreads), 0, s, a);
  if (e == cudaSuccess) e = launch_pdl(k_best, dim3(a.nf), dim3(kBestThreads), 0, s, a);
  if (e != cudaSuccess) return e;
  if (nl) (*nl) += 2;
  return cudaGetLastError();
}

cudaError_t launch_bin(const float* x, uint64_t n, uint32_t nf, const float* d_cuts,
                       uint32_t n_bins, uint64_t n_pad, uint8_t* d_colbins, uint8_t* d_rowbins,
                       cudaStream_t s, int* nl) {
  const uint32_t nb1 = n_bins - 1, ftiles = (nf + kHistFeat - 1) / kHistFeat;
  const size_t smem = (size_t)kBinRows * kHistFeat + (size_t)kHistFeat * nb1 * 4;
  if (set_smem_and_occupancy(reinterpret_cast<const void*>(&k_bin), kBinRows, smem) < 1)
    return cudaErrorInvalidConfiguration;
  dim3 grid((unsigned)(n_pad / kBinRows), ftiles);
  k_bin<<<grid, kBinRows, smem, s>>>(x, n, nf, d_cuts, nb1, n_pad, d_colbins, d_rowbins);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_pack4(const uint8_t* d_u8, uint64_t n_pad, uint32_t nf, uint8_t* d_packed,
                         cudaStream_t s, int* nl) {
  const uint32_t ftiles = (nf + kHistFeat - 1) / kHistFeat;
  k_pack4<<<grid_for(n_pad * ftiles * 2, 256), 256, 0, s>>>(d_u8, n_pad, ftiles, d_packed);
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_grad(float* pred, const float* y, float* g, float* h, uint64_t n,
                        uint64_t n_pad, int logistic, uint64_t stride, uint64_t phase,
                        uint64_t row_offset, int compute_max, uint32_t* maxbits,
                        uint32_t* zero_word, const PrevTree& prev, cudaStream_t s, int* nl) {
  if ((n_pad & 3) != 0 || (prev.leafval && !prev.node)) return cudaErrorInvalidValue;
  RW_PREFER_SMEM(k_grad);
  cudaError_t e = launch_pdl(k_grad, dim3(grid_for(n_pad / 4, 256)), dim3(256), 0, s, pred, y, g,
                             h, n, n_pad, logistic, stride, phase, row_offset, compute_max,
                             maxbits, zero_word, prev);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_leafval(const LeafValues& a, cudaStream_t s, int* nl) {
  if (!a.leafsum || !a.leafval || !a.maxbits || a.n_leaves == 0) return cudaErrorInvalidValue;
  const unsigned blocks = (a.n_leaves + 255) / 256;
  cudaError_t e = launch_pdl(k_leafval, dim3(blocks), dim3(256), 0, s, a);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_leafsq(const LeafSquares& a, cudaStream_t s, int* nl) {
  if (!a.node || !a.g || !a.maxbits || !a.leafsum2 || a.n_leaves == 0 || a.n_leaves > 4096 ||
      a.n_pad % 4 != 0)
    return cudaErrorInvalidValue;
  cudaError_t e = launch_pdl(k_leafsq, dim3(grid_for(a.n_pad / 4, kLeafSqThreads)),
                             dim3(kLeafSqThreads), 0, s, a);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_quant(const float* g, const float* h, const uint32_t* maxbits, uint64_t n_pad,
                         int2* q, uint16_t* node, long long* hb0, uint64_t hb0_words,
                         long long* leafsum, uint32_t leafsum_words, uint32_t* ncount0,
                         cudaStream_t s, int* nl) {
  RW_PREFER_SMEM(k_quant);
  cudaError_t e = launch_pdl(k_quant, dim3(grid_for(n_pad, 256)), dim3(256), 0, s, g, h, maxbits,
                             n_pad, q, node, hb0, hb0_words, leafsum, leafsum_words, ncount0);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_apply(const ApplyLaunch& a, cudaStream_t s, int* nl) {
  const uint64_t n4 = a.n_pad / 4;
  const uint32_t n_nodes = a.n_children / 2;
  const uint32_t G = a.lists.subtract ? n_nodes : a.n_children;
  const bool listing = !a.final_level && a.lists.entries;
  if (listing && n_nodes > 4 * kApplyThreads) return cudaErrorInvalidValue;
  if (a.final_level && (!a.leafsum || !a.g || !a.h || !a.maxbits || a.n_leaves != a.n_children))
    return cudaErrorInvalidValue;
  const size_t smem = listing ? ((size_t)n_nodes + 1 + 2 * (size_t)G) * 4 + n_nodes
                      : (a.final_level && a.n_leaves <= kLeafSmem) ? (size_t)a.n_leaves * 16
                                                                   : 0;
  if (smem > 48 * 1024 &&
      set_smem_and_occupancy(a.final_level ? reinterpret_cast<const void*>(&k_apply<true>)
                                           : reinterpret_cast<const void*>(&k_apply<false>),
                             kApplyThreads, smem) < 1)
    return cudaErrorInvalidConfiguration;
  RW_PREFER_SMEM(k_apply<false>);
  RW_PREFER_SMEM(k_apply<true>);
  // The final level ends with every CTA adding its leaf sums into the global ones: two
  // CTAs per SM keep those adds (2 x leaves per CTA onto the same words) few.
  int grid = grid_for(n4, kApplyThreads);
  if (a.final_level) grid = std::min(grid, 2 * sm_count());
  cudaError_t e = a.final_level
                      ? launch_pdl(k_apply<true>, dim3(grid), dim3(kApplyThreads), smem, s, a)
                      : launch_pdl(k_apply<false>, dim3(grid), dim3(kApplyThreads), smem, s, a);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_fill_f32(float* p, float v, uint64_t n, cudaStream_t s, int* nl) {
  cudaError_t e = launch_pdl(k_fill, dim3(grid_for(n, 256)), dim3(256), 0, s, p, v, n);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_goss_init(const GossState& st, uint64_t k, cudaStream_t s, int* nl) {
  cudaError_t e = launch_pdl(k_goss_init, dim3(1), dim3(1), 0, s, st.sel, k);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_goss_digit_hist(const float* g, uint64_t n, const GossState& st, int pass,
                                   cudaStream_t s, int* nl) {
  RW_PREFER_SMEM(k_goss_digit_hist);
  cudaError_t e = launch_pdl(k_goss_digit_hist, dim3(grid_for(n, 256)), dim3(256), 0, s, g, n,
                             st.counts, st.sel, pass);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_goss_digit_select(const GossState& st, int pass, cudaStream_t s, int* nl) {
  cudaError_t e = launch_pdl(k_goss_digit_select, dim3(1), dim3(32), 0, s, st.counts, st.sel, pass);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t launch_goss_apply(float* g, float* h, uint64_t n, uint64_t row_offset,
                              const GossState& st, double keep_prob, float fact, uint64_t seed,
                              uint32_t* maxbits, cudaStream_t s, int* nl) {
  RW_PREFER_SMEM(k_goss_apply);
  cudaError_t e = launch_pdl(k_goss_apply, dim3(grid_for(n, 256)), dim3(256), 0, s, g, h, n,
                             row_offset, st.sel, keep_prob, fact, seed, maxbits);
  if (e != cudaSuccess) return e;
  if (nl) (*nl)++;
  return cudaGetLastError();
}

cudaError_t kernel_binary_version(int* out) {
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, k_fill);
  if (e == cudaSuccess) *out = fa.binaryVersion;
  return e;
}

cudaError_t launch_debug_expf(const float* x, uint64_t n, float* out_rw, float* out_cuda,
                              cudaStream_t s) {
  k_debug_expf<<<grid_for(n, 256), 256, 0, s>>>(x, n, out_rw, out_cuda);
  return cudaGetLastError();
}
