// compute_boundaries (src/data.rs:86-146) on the GPU.
//
// The reference takes every stride-th row (stride = max(n / sample, 1)), sorts each
// feature's sampled values with a stable comparison sort (partial_cmp) and reads the cut
// table off the sorted values: quantile cuts sorted[round((j+1)/B * (m-1))] with a
// monotone fix, or (unique mode) the midpoints of the distinct values, padded with +inf
// or subsampled evenly. Here:
//   k_sample_gather   the sampled rows' values, feature-major [nf][m];
//   k_feature_sort    one CTA per feature: an LSD radix sort of the m values (4 stable
//                     passes of 8 bits over an order-preserving key; -0.0 and +0.0 share a
//                     key, as they compare equal) through two scratch columns;
//   k_feature_cuts    one CTA per feature: the cut table from the sorted column.
// The sort is stable, so the zeros (-0.0 and +0.0 compare equal) stay in sample order as
// in the reference; the cut kernel still reads a zero's sign from the sample order (a
// scan of the sample), which holds for any sort of the keys. Unique mode keeps one zero and only
// uses it in midpoints (0.5 * (x + 0) does not depend on the zero's sign). Samples with
// NaN have no defined order in the reference (partial_cmp gives Equal against
// everything); here NaN sorts after +inf.
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>

#include "rw_internal.cuh"

namespace {

constexpr int kSortThreads = 1024;

__device__ __forceinline__ uint32_t order_key(uint32_t bits) {
  if (bits == 0x80000000u) bits = 0u;  // -0.0 sorts with +0.0
  return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

__global__ void k_sample_gather(const float* __restrict__ x, uint64_t n, uint32_t nf,
                                uint64_t stride, uint64_t m, uint32_t* __restrict__ out) {
  const uint64_t total = m * nf;
  for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
       i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t k = i / nf;
    const uint32_t f = (uint32_t)(i % nf);
    out[(size_t)f * m + k] = __float_as_uint(x[k * stride * nf + f]);
  }
}

// Block-wide exclusive scan of 256 counts held by threads 0..255 (the rest pass 0).
__device__ uint32_t scan256(uint32_t v, uint32_t* s_tmp) {
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, d);
    if (lane >= (uint32_t)d) incl += y;
  }
  if (threadIdx.x < 256 && lane == 31) s_tmp[warp] = incl;
  __syncthreads();
  if (threadIdx.x < 8) {
    uint32_t run = 0;
    for (uint32_t w = 0; w < threadIdx.x; w++) run += s_tmp[w];
    s_tmp[8 + threadIdx.x] = run;
  }
  __syncthreads();
  const uint32_t r = threadIdx.x < 256 ? s_tmp[8 + warp] + incl - v : 0u;
  __syncthreads();
  return r;
}

// One CTA sorts column f: a[f*m .. f*m+m) with b as the second buffer; 4 passes, so the
// sorted values end in a. Each pass is a stable counting sort on one 8-bit digit (LSD
// radix needs stable passes): the column is scattered tile by tile in index order, one
// element per thread; within a tile an element's place is its digit's running offset,
// plus the counts of that digit in the lower warps, plus its rank among the equal digits
// of its own warp.
__global__ void __launch_bounds__(kSortThreads) k_feature_sort(uint32_t* __restrict__ a,
                                                               uint32_t* __restrict__ b,
                                                               uint64_t m) {
  constexpr int kWarps = kSortThreads / 32;
  __shared__ uint32_t s_cnt[256];
  __shared__ uint32_t s_tmp[16];
  __shared__ uint32_t s_wc[kWarps][256];  // per tile: counts, then offsets, per warp and digit
  uint32_t* src = a + (size_t)blockIdx.x * m;
  uint32_t* dst = b + (size_t)blockIdx.x * m;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  for (int pass = 0; pass < 4; pass++) {
    const int shift = 8 * pass;
    if (threadIdx.x < 256) s_cnt[threadIdx.x] = 0u;
    __syncthreads();
    for (uint64_t i = threadIdx.x; i < m; i += kSortThreads)
      atomicAdd(&s_cnt[(order_key(src[i]) >> shift) & 0xffu], 1u);
    __syncthreads();
    const uint32_t c = threadIdx.x < 256 ? s_cnt[threadIdx.x] : 0u;
    const uint32_t base = scan256(c, s_tmp);
    if (threadIdx.x < 256) s_cnt[threadIdx.x] = base;  // the digit's next free slot
    __syncthreads();
    for (uint64_t t0 = 0; t0 < m; t0 += kSortThreads) {
      for (uint32_t w = threadIdx.x; w < kWarps * 256; w += kSortThreads)
        (&s_wc[0][0])[w] = 0u;
      const uint64_t i = t0 + threadIdx.x;
      const bool live = i < m;
      const uint32_t v = live ? src[i] : 0u;
      const uint32_t d = live ? (order_key(v) >> shift) & 0xffu : 256u;  // 256: no element
      const uint32_t peers = __match_any_sync(0xffffffffu, d);
      const uint32_t rank = __popc(peers & lt);
      __syncthreads();  // the counts are zero
      if (live && rank == 0) s_wc[warp][d] = __popc(peers);
      __syncthreads();
      if (threadIdx.x < 256) {  // offsets of each warp's run of this digit, in warp order
        uint32_t off = s_cnt[threadIdx.x];
        for (int w = 0; w < kWarps; w++) {
          const uint32_t k = s_wc[w][threadIdx.x];
          s_wc[w][threadIdx.x] = off;
          off += k;
        }
        s_cnt[threadIdx.x] = off;
      }
      __syncthreads();
      if (live) dst[s_wc[warp][d] + rank] = v;
      __syncthreads();  // s_wc is reused by the next tile
    }
    uint32_t* t = src;
    src = dst;
    dst = t;
  }
}

// The cut table of feature f from its sorted column (sorted) and its sample column in
// sample order (sample, for the signs of zeros); scratch: m words for this feature.
__global__ void __launch_bounds__(kSortThreads) k_feature_cuts(
    const uint32_t* __restrict__ sorted, const uint32_t* __restrict__ sample,
    uint32_t* __restrict__ scratch, uint64_t m, uint32_t n_bins, int unique,
    float* __restrict__ out) {
  __shared__ uint32_t s_warp[kSortThreads / 32 + 1];
  __shared__ uint32_t s_total;
  const uint32_t f = blockIdx.x, nb1 = n_bins - 1;
  const uint32_t* s = sorted + (size_t)f * m;
  const uint32_t* smp = sample + (size_t)f * m;
  uint32_t* scr = scratch + (size_t)f * m;
  float* o = out + (size_t)f * nb1;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  // Ordered compaction (stream compaction in index order): keep[i] -> scr[rank]; used
  // for the zeros' signs (quantile mode) and the distinct values (unique mode).
  auto compact = [&](auto keep, auto value) -> uint32_t {
    uint32_t run = 0;
    for (uint64_t t0 = 0; t0 < m; t0 += kSortThreads) {
      const uint64_t i = t0 + threadIdx.x;
      const bool k = i < m && keep(i);
      const uint32_t bal = __ballot_sync(0xffffffffu, k);
      if (lane == 0) s_warp[warp] = __popc(bal);
      __syncthreads();
      if (threadIdx.x == 0) {
        uint32_t acc = 0;
        for (int w = 0; w < kSortThreads / 32; w++) {
          const uint32_t c = s_warp[w];
          s_warp[w] = acc;
          acc += c;
        }
        s_warp[kSortThreads / 32] = acc;
      }
      __syncthreads();
      if (k) scr[run + s_warp[warp] + __popc(bal & ((1u << lane) - 1u))] = value(i);
      run += s_warp[kSortThreads / 32];
      __syncthreads();
    }
    return run;
  };
  if (!unique) {
    // the run of zeros in the sorted column: [z0, z0 + nz)
    if (threadIdx.x == 0) s_total = 0;
    __syncthreads();
    uint32_t neg = 0;
    for (uint64_t i = threadIdx.x; i < m; i += kSortThreads) {
      const uint32_t k = order_key(s[i]);
      neg += k < 0x80000000u;
    }
    for (int d = 16; d > 0; d >>= 1) neg += __shfl_down_sync(0xffffffffu, neg, d);
    if (lane == 0) atomicAdd(&s_total, neg);
    __syncthreads();
    const uint64_t z0 = s_total;
    // the zeros' sign bits in sample order
    const uint32_t nz = compact([&](uint64_t i) { return (smp[i] & 0x7fffffffu) == 0u; },
                                [&](uint64_t i) { return smp[i]; });
    if (threadIdx.x == 0) {
      float prev = 0.0f;
      for (uint32_t j = 0; j < nb1; j++) {
        const double q = (double)(j + 1) / (double)n_bins;
        uint64_t pos = (uint64_t)round(q * (double)(m - 1));
        if (pos > m - 1) pos = m - 1;
        uint32_t bits = s[pos];
        if (pos >= z0 && pos < z0 + nz) bits = scr[pos - z0];  // the stable sort's zero
        float v = __uint_as_float(bits);
        if (j > 0 && v <= prev) v = prev;  // monotone even with heavy ties
        o[j] = v;
        prev = v;
      }
    }
    return;
  }
  // unique: the distinct values in sorted order (equal by ==, so one of the zeros)
  const uint32_t U = compact(
      [&](uint64_t i) {
        return i == 0 || __uint_as_float(s[i]) != __uint_as_float(s[i - 1]);
      },
      [&](uint64_t i) { return s[i]; });
  __syncthreads();
  const uint32_t nc = U > 0 ? U - 1 : 0;  // midpoint candidates
  for (uint32_t j = threadIdx.x; j < nb1; j += kSortThreads) {
    float v;
    uint32_t c = 0xffffffffu;
    if (nc == 0) c = 0xffffffffu;
    else if (nc <= nb1) c = j < nc ? j : 0xffffffffu;
    else {
      const uint64_t pos = ((uint64_t)(j + 1) * nc) / (nb1 + 1);
      c = (uint32_t)(pos < nc - 1 ? pos : nc - 1);
    }
    if (c == 0xffffffffu) v = INFINITY;
    else v = 0.5f * (__uint_as_float(scr[c]) + __uint_as_float(scr[c + 1]));
    o[j] = v;
  }
}

}  // namespace

cudaError_t launch_boundaries(const float* d_x, uint64_t n, uint32_t nf, uint32_t n_bins,
                              uint64_t sample, int unique, uint32_t* scratch3, float* d_out,
                              cudaStream_t s, uint64_t* m_out) {
  const uint64_t stride = std::max<uint64_t>(n / std::max<uint64_t>(sample, 1), 1);
  const uint64_t m = (n - 1) / stride + 1;
  *m_out = m;
  uint32_t* col = scratch3;                    // sample order
  uint32_t* a = scratch3 + (size_t)nf * m;     // sorted (after 4 passes)
  uint32_t* b = scratch3 + 2 * (size_t)nf * m;
  const uint64_t total = m * nf;
  const int grid = (int)std::min<uint64_t>((total + 255) / 256, 148ull * 16);
  k_sample_gather<<<grid, 256, 0, s>>>(d_x, n, nf, stride, m, col);
  cudaError_t e = cudaMemcpyAsync(a, col, total * 4, cudaMemcpyDeviceToDevice, s);
  if (e != cudaSuccess) return e;
  k_feature_sort<<<nf, kSortThreads, 0, s>>>(a, b, m);
  // b is free again: the cut kernel's compaction scratch
  k_feature_cuts<<<nf, kSortThreads, 0, s>>>(a, col, b, m, n_bins, unique, d_out);
  return cudaGetLastError();
}
