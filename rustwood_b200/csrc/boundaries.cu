// compute_boundaries (src/data.rs:86-146) on the GPU.
//
// The reference takes every stride-th row (stride = max(n / sample, 1)), sorts each
// feature's sampled values with a stable comparison sort (partial_cmp) and reads the cut
// table off the sorted values: quantile cuts sorted[round((j+1)/B * (m-1))] with a
// monotone fix, or (unique mode) the midpoints of the distinct values, padded with +inf
// or subsampled evenly. Here:
//   k_sample_gather   the sampled rows' values, feature-major [nf][m];
//   k_sort_count,     an LSD radix sort of each feature's m values (4 stable passes of 8
//   k_sort_scatter    bits over an order-preserving key; -0.0 and +0.0 share a key, as
//                     they compare equal) through two scratch columns, each column split
//                     over several CTAs;
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

// The sort of column f (m keys) is split over P parts of the column (P CTAs per
// feature, part p = [m*p/P, m*(p+1)/P)), 4 passes of one 8-bit digit each, two kernels per
// pass: k_sort_count counts every part's digits; k_sort_scatter moves each part's keys to
// their places, the digit's start over the whole column plus the same digit's count in
// the lower parts. Within a part the keys are scattered tile by tile in index order, one
// key per thread; within a tile a key's place is its digit's running offset, plus the
// counts of that digit in the lower warps, plus its rank among the equal digits of its own
// warp. So every pass is a stable counting sort, as LSD radix sorting needs.
__global__ void __launch_bounds__(kSortThreads) k_sort_count(const uint32_t* __restrict__ src,
                                                             uint64_t m, uint32_t parts,
                                                             int shift,
                                                             uint32_t* __restrict__ counts) {
  __shared__ uint32_t s_cnt[256];
  const uint32_t f = blockIdx.x, p = blockIdx.y;
  const uint64_t lo = m * p / parts, hi = m * (p + 1) / parts;
  const uint32_t* col = src + (size_t)f * m;
  if (threadIdx.x < 256) s_cnt[threadIdx.x] = 0u;
  __syncthreads();
  for (uint64_t i = lo + threadIdx.x; i < hi; i += kSortThreads)
    atomicAdd(&s_cnt[(order_key(col[i]) >> shift) & 0xffu], 1u);
  __syncthreads();
  if (threadIdx.x < 256) counts[((size_t)f * parts + p) * 256 + threadIdx.x] = s_cnt[threadIdx.x];
}

__global__ void __launch_bounds__(kSortThreads) k_sort_scatter(const uint32_t* __restrict__ src,
                                                               uint32_t* __restrict__ dst,
                                                               uint64_t m, uint32_t parts,
                                                               int shift,
                                                               const uint32_t* __restrict__ counts) {
  constexpr int kWarps = kSortThreads / 32;
  __shared__ uint32_t s_cnt[256];
  __shared__ uint32_t s_tmp[16];
  __shared__ uint32_t s_wc[kWarps][256];  // per tile: counts, then offsets, per warp and digit
  const uint32_t f = blockIdx.x, p = blockIdx.y;
  const uint64_t lo = m * p / parts, hi = m * (p + 1) / parts;
  const uint32_t* col = src + (size_t)f * m;
  uint32_t* out = dst + (size_t)f * m;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  // this part's first place for each digit
  uint32_t total = 0, lower = 0;
  if (threadIdx.x < 256)
    for (uint32_t q = 0; q < parts; q++) {
      const uint32_t c = counts[((size_t)f * parts + q) * 256 + threadIdx.x];
      total += c;
      if (q < p) lower += c;
    }
  const uint32_t base = scan256(threadIdx.x < 256 ? total : 0u, s_tmp);
  if (threadIdx.x < 256) s_cnt[threadIdx.x] = base + lower;  // the digit's next free slot
  __syncthreads();
  for (uint64_t t0 = lo; t0 < hi; t0 += kSortThreads) {
    for (uint32_t w = threadIdx.x; w < kWarps * 256; w += kSortThreads) (&s_wc[0][0])[w] = 0u;
    const uint64_t i = t0 + threadIdx.x;
    const bool live = i < hi;
    const uint32_t v = live ? col[i] : 0u;
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
    if (live) out[s_wc[warp][d] + rank] = v;
    __syncthreads();  // s_wc is reused by the next tile
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
                              uint64_t sample, int unique, uint32_t* scratch, float* d_out,
                              cudaStream_t s, uint64_t* m_out, int* nl) {
  const uint64_t stride = std::max<uint64_t>(n / std::max<uint64_t>(sample, 1), 1);
  const uint64_t m = (n - 1) / stride + 1;
  *m_out = m;
  uint32_t* col = scratch;                    // sample order (kept: the cut kernel reads it)
  uint32_t* a = scratch + (size_t)nf * m;
  uint32_t* b = scratch + 2 * (size_t)nf * m;
  uint32_t* counts = scratch + 3 * (size_t)nf * m;  // [nf][parts][256]
  const uint64_t total = m * nf;
  const int grid = (int)std::min<uint64_t>((total + 255) / 256, 148ull * 16);
  k_sample_gather<<<grid, 256, 0, s>>>(d_x, n, nf, stride, m, col);
  // parts per column: about two sorting CTAs per SM over all features, and at least 4096
  // keys per part
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  uint64_t parts = std::max<uint64_t>(1, (2 * (uint64_t)sms) / nf);
  parts = std::min<uint64_t>(parts, std::max<uint64_t>(1, m / 4096));
  parts = std::min<uint64_t>(parts, kSortMaxParts);
  const dim3 sg(nf, (unsigned)parts);  // features on x: no 65535 limit on their count
  // pass 0 reads the sample column; the passes then alternate a -> b -> a -> b, so the
  // sorted keys end in b
  const uint32_t* src = col;
  uint32_t* dst = a;
  for (int pass = 0; pass < 4; pass++) {
    k_sort_count<<<sg, kSortThreads, 0, s>>>(src, m, (uint32_t)parts, 8 * pass, counts);
    k_sort_scatter<<<sg, kSortThreads, 0, s>>>(src, dst, m, (uint32_t)parts, 8 * pass, counts);
    src = dst;
    dst = dst == a ? b : a;
  }
  // a is free again: the cut kernel's compaction scratch
  k_feature_cuts<<<nf, kSortThreads, 0, s>>>(b, col, a, m, n_bins, unique, d_out);
  if (nl) *nl += 2 + 8;
  return cudaGetLastError();
}
