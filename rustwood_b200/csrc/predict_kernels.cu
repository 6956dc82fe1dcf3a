// Batched oblivious-forest scoring on sm_100a (src/gpu_kernels.rs:1142-1180 is the
// reference's one-thread-per-row global-memory kernel; src/booster.rs:582-601 its CPU
// twin). Both scorers here produce, per row, acc = base; acc += leafval[t][leaf_t]
// for t = 0..T-1 in f32, in tree order, so they are bit-identical to predict_cpu.
//
// The model (split table + leaf values) is staged in shared memory in chunks of trees
// sized to the shared-memory budget; with more than one chunk the running sums go
// through `out` between chunks, which keeps the same sequential f32 order.
//
// u8 scorer: inputs are pre-binned, feature-major [nf][ld] u8. Each thread scores 4
// consecutive rows at once: one 32-bit load fetches the 4 rows' bins of a feature, a
// byte-SIMD compare (__vcmpgtu4) against the broadcast threshold produces the 4 split
// bits, and the 4 leaf indices advance in the bytes of one register
// (leaf4 = 2*leaf4 + bits; depth <= 8 keeps every byte below 256).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "rw_internal.cuh"

namespace {

constexpr int kPredThreads = 256;
constexpr size_t kModelSmem = 200 * 1024;

__device__ __forceinline__ void stage_model(uint32_t t0, uint32_t tc, uint32_t depth,
                                            const uint32_t* __restrict__ g_split,
                                            const float* __restrict__ g_leaf, uint32_t* s_split,
                                            float* s_leaf) {
  const uint32_t nl = 1u << depth;
  for (uint32_t i = threadIdx.x; i < tc * depth; i += blockDim.x)
    s_split[i] = g_split[(size_t)t0 * depth + i];
  for (uint32_t i = threadIdx.x; i < (tc << depth); i += blockDim.x)
    s_leaf[i] = g_leaf[((size_t)t0 << depth) + i];
  (void)nl;
}

__global__ void __launch_bounds__(kPredThreads) k_predict_u8_simd(
    const uint8_t* __restrict__ bins, uint64_t n, uint64_t ld, uint32_t t0, uint32_t tc,
    uint32_t depth, const uint32_t* __restrict__ split8, const float* __restrict__ leafval,
    float base, int first_chunk, float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char pred_raw[];
  float* s_leaf = reinterpret_cast<float*>(pred_raw);
  uint32_t* s_split = reinterpret_cast<uint32_t*>(pred_raw + ((size_t)tc << depth) * 4);
  stage_model(t0, tc, depth, split8, leafval, s_split, s_leaf);
  __syncthreads();
  const uint64_t n4 = (n + 3) / 4;
  for (uint64_t q = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; q < n4;
       q += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t r0 = q * 4;
    float acc[4];
    if (first_chunk) {
      acc[0] = acc[1] = acc[2] = acc[3] = base;
    } else {
#pragma unroll
      for (int s = 0; s < 4; s++) acc[s] = r0 + s < n ? out[r0 + s] : 0.0f;
    }
    const uint8_t* rb = bins + r0;
    for (uint32_t t = 0; t < tc; t++) {
      uint32_t leaf4 = 0;
      const uint32_t* sp = s_split + t * depth;
      for (uint32_t d = 0; d < depth; d++) {
        const uint32_t sv = sp[d];
        const uint32_t b4 = __ldg(reinterpret_cast<const uint32_t*>(rb + (size_t)(sv >> 8) * ld));
        const uint32_t m = __vcmpgtu4(b4, (sv & 0xffu) * 0x01010101u);
        leaf4 = (leaf4 << 1) | (m & 0x01010101u);
      }
      const float* lv = s_leaf + (t << depth);
      acc[0] += lv[leaf4 & 0xffu];
      acc[1] += lv[(leaf4 >> 8) & 0xffu];
      acc[2] += lv[(leaf4 >> 16) & 0xffu];
      acc[3] += lv[leaf4 >> 24];
    }
#pragma unroll
    for (int s = 0; s < 4; s++)
      if (r0 + s < n) out[r0 + s] = acc[s];
  }
}

// Tiled u8 scorer (depth D <= 8 known at compile time): a persistent CTA stages its tree
// chunk in shared memory once, then walks row blocks of kTileRows rows. Per block the
// rows' bins are staged feature-major in shared memory as one 32-bit word per (feature,
// thread) -- the thread's 4 rows -- so every split's bins come from a conflict-free shared
// load; a byte-SIMD compare gives the 4 rows' bits and one LOP3 places them at bit D-1-d of
// each row's byte. Trees are scored in order and each row's sum is sequential f32 (the
// same order as predict_cpu).
constexpr uint32_t kTileRows = kPredThreads * 4;

template <int D>
__global__ void __launch_bounds__(kPredThreads) k_predict_u8_tiled(
    const uint8_t* __restrict__ bins, uint64_t n, uint64_t ld, uint32_t nf, uint32_t t0,
    uint32_t tc, const uint32_t* __restrict__ split8, const float* __restrict__ leafval,
    float base, int first_chunk, float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char pred_raw[];
  float* s_leaf = reinterpret_cast<float*>(pred_raw);
  uint32_t* s_split = reinterpret_cast<uint32_t*>(pred_raw + ((size_t)tc << D) * 4);
  uint32_t* s_rows = s_split + (size_t)tc * D;  // [nf][kPredThreads]
  stage_model(t0, tc, D, split8, leafval, s_split, s_leaf);
  const uint32_t tid = threadIdx.x;
  const uint64_t nblk = (n + kTileRows - 1) / kTileRows;
  for (uint64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const uint64_t r0 = blk * kTileRows + (uint64_t)tid * 4;  // this thread's 4 rows
    __syncthreads();  // the previous block's rows (and the model) are settled
    for (uint32_t f = 0; f < nf; f++)
      s_rows[f * kPredThreads + tid] =
          r0 + 3 < ld ? __ldg(reinterpret_cast<const uint32_t*>(bins + (size_t)f * ld + r0)) : 0u;
    __syncthreads();
    float acc[4];
    if (first_chunk) {
      acc[0] = acc[1] = acc[2] = acc[3] = base;
    } else {
#pragma unroll
      for (int k = 0; k < 4; k++) acc[k] = r0 + k < n ? out[r0 + k] : 0.0f;
    }
    const uint32_t* rows = s_rows + tid;
    for (uint32_t t = 0; t < tc; t++) {
      const uint32_t* sp = s_split + t * D;
      uint32_t leaf4 = 0;
#pragma unroll
      for (int d = 0; d < D; d++) {
        const uint32_t sv = sp[d];
        const uint32_t m = __vcmpgtu4(rows[(sv >> 8) * kPredThreads], (sv & 0xffu) * 0x01010101u);
        leaf4 |= m & (0x01010101u << (D - 1 - d));
      }
      const float* lv = s_leaf + ((size_t)t << D);
      acc[0] += lv[leaf4 & 0xffu];
      acc[1] += lv[(leaf4 >> 8) & 0xffu];
      acc[2] += lv[(leaf4 >> 16) & 0xffu];
      acc[3] += lv[leaf4 >> 24];
    }
#pragma unroll
    for (int k = 0; k < 4; k++)
      if (r0 + k < n) out[r0 + k] = acc[k];
  }
}

template <int D>
const void* tiled_fn() {
  return reinterpret_cast<const void*>(&k_predict_u8_tiled<D>);
}

// One row per thread, any depth and any row stride.
__global__ void __launch_bounds__(kPredThreads) k_predict_u8_scalar(
    const uint8_t* __restrict__ bins, uint64_t n, uint64_t ld, uint32_t t0, uint32_t tc,
    uint32_t depth, const uint32_t* __restrict__ split8, const float* __restrict__ leafval,
    float base, int first_chunk, float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char pred_raw[];
  float* s_leaf = reinterpret_cast<float*>(pred_raw);
  uint32_t* s_split = reinterpret_cast<uint32_t*>(pred_raw + ((size_t)tc << depth) * 4);
  stage_model(t0, tc, depth, split8, leafval, s_split, s_leaf);
  __syncthreads();
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n;
       r += (uint64_t)gridDim.x * blockDim.x) {
    float acc = first_chunk ? base : out[r];
    for (uint32_t t = 0; t < tc; t++) {
      uint32_t leaf = 0;
      for (uint32_t d = 0; d < depth; d++) {
        const uint32_t sv = s_split[t * depth + d];
        const uint32_t b = __ldg(bins + (size_t)(sv >> 8) * ld + r);
        leaf = leaf * 2u + (b > (sv & 0xffu) ? 1u : 0u);
      }
      acc += s_leaf[(t << depth) + leaf];
    }
    out[r] = acc;
  }
}

// Raw f32 row-major features against raw thresholds (Booster::predict semantics).
__global__ void __launch_bounds__(kPredThreads) k_predict_f32(
    const float* __restrict__ x, uint64_t n, uint32_t nf, uint32_t t0, uint32_t tc,
    uint32_t depth, const uint32_t* __restrict__ feat, const float* __restrict__ thr,
    const float* __restrict__ leafval, float base, int first_chunk, float* __restrict__ out) {
  extern __shared__ __align__(16) unsigned char pred_raw[];
  float* s_leaf = reinterpret_cast<float*>(pred_raw);
  uint32_t* s_feat = reinterpret_cast<uint32_t*>(pred_raw + ((size_t)tc << depth) * 4);
  float* s_thr = reinterpret_cast<float*>(s_feat + tc * depth);
  for (uint32_t i = threadIdx.x; i < tc * depth; i += blockDim.x) {
    s_feat[i] = feat[(size_t)t0 * depth + i];
    s_thr[i] = thr[(size_t)t0 * depth + i];
  }
  for (uint32_t i = threadIdx.x; i < (tc << depth); i += blockDim.x)
    s_leaf[i] = leafval[((size_t)t0 << depth) + i];
  __syncthreads();
  for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n;
       r += (uint64_t)gridDim.x * blockDim.x) {
    const float* row = x + r * nf;
    float acc = first_chunk ? base : out[r];
    for (uint32_t t = 0; t < tc; t++) {
      uint32_t leaf = 0;
      for (uint32_t d = 0; d < depth; d++) {
        const uint32_t k = t * depth + d;
        leaf = leaf * 2u + (__ldg(row + s_feat[k]) > s_thr[k] ? 1u : 0u);
      }
      acc += s_leaf[(t << depth) + leaf];
    }
    out[r] = acc;
  }
}

uint32_t trees_per_chunk(uint32_t n_trees, uint32_t depth, size_t per_slot_bytes) {
  const size_t per_tree = ((size_t)4 << depth) + per_slot_bytes * depth;
  size_t tc = kModelSmem / per_tree;
  if (tc < 1) tc = 1;
  if (tc > n_trees) tc = n_trees;
  return (uint32_t)tc;
}

int pred_grid(uint64_t work) {
  uint64_t b = (work + kPredThreads - 1) / kPredThreads;
  const uint64_t cap = 148ull * 8;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

// The tiled scorer for depth 1..8 when the rows' bins fit next to a tree chunk.
static cudaError_t launch_predict_u8_tiled(const uint8_t* bins, uint64_t n, uint64_t ld,
                                           const rw_dmodel& m, float* out, cudaStream_t s,
                                           bool* used) {
  *used = false;
  const size_t rows_bytes = (size_t)m.nf * kPredThreads * 4;
  if (m.depth < 1 || m.depth > 8 || rows_bytes > 96 * 1024) return cudaSuccess;
  const size_t per_tree = ((size_t)4 << m.depth) + 4 * (size_t)m.depth;
  const size_t budget = 220 * 1024 - rows_bytes;
  uint32_t tc = (uint32_t)std::min<size_t>(m.n_trees, budget / per_tree);
  if (tc < 1) return cudaSuccess;
  const void* fns[9] = {nullptr,          tiled_fn<1>(), tiled_fn<2>(), tiled_fn<3>(), tiled_fn<4>(),
                        tiled_fn<5>(),    tiled_fn<6>(), tiled_fn<7>(), tiled_fn<8>()};
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t nblk = (n + kTileRows - 1) / kTileRows;
  for (uint32_t t0 = 0; t0 < m.n_trees; t0 += tc) {
    const uint32_t c = m.n_trees - t0 < tc ? m.n_trees - t0 : tc;
    const size_t smem = ((size_t)c << m.depth) * 4 + (size_t)c * m.depth * 4 + rows_bytes;
    cudaError_t e = cudaFuncSetAttribute(fns[m.depth], cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 1;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fns[m.depth], kPredThreads, smem);
    const uint64_t grid = std::max<uint64_t>(1, std::min<uint64_t>(nblk, (uint64_t)sms * std::max(per_sm, 1)));
    int first = t0 == 0;
    uint64_t nn = n, ll = ld;
    uint32_t nf = m.nf, tt0 = t0, cc = c;
    const uint32_t* sp = m.d_split8;
    const float* lp = m.d_leafval;
    float b = m.base;
    const uint8_t* bp = bins;
    float* op = out;
    void* args[] = {&bp, &nn, &ll, &nf, &tt0, &cc, &sp, &lp, &b, &first, &op};
    e = cudaLaunchKernel(fns[m.depth], dim3((unsigned)grid), dim3(kPredThreads), args, smem, s);
    if (e != cudaSuccess) return e;
  }
  *used = true;
  return cudaSuccess;
}

cudaError_t launch_predict_u8(const uint8_t* bins, uint64_t n, uint64_t ld, const rw_dmodel& m,
                              float* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const bool simd = m.depth <= 8 && (ld % 4) == 0 && ld >= ((n + 3) & ~3ull) &&
                    (reinterpret_cast<uintptr_t>(bins) % 4) == 0;
  if (simd && m.n_trees > 0) {
    bool used = false;
    cudaError_t e = launch_predict_u8_tiled(bins, n, ld, m, out, s, &used);
    if (e != cudaSuccess || used) return e;
  }
  const uint32_t tc = trees_per_chunk(m.n_trees, m.depth, 4);
  for (uint32_t t0 = 0; t0 < m.n_trees; t0 += tc) {
    const uint32_t c = m.n_trees - t0 < tc ? m.n_trees - t0 : tc;
    const size_t smem = ((size_t)c << m.depth) * 4 + (size_t)c * m.depth * 4;
    cudaError_t e;
    if (simd) {
      e = cudaFuncSetAttribute(k_predict_u8_simd, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)smem);
      if (e != cudaSuccess) return e;
      k_predict_u8_simd<<<pred_grid((n + 3) / 4), kPredThreads, smem, s>>>(
          bins, n, ld, t0, c, m.depth, m.d_split8, m.d_leafval, m.base, t0 == 0, out);
    } else {
      e = cudaFuncSetAttribute(k_predict_u8_scalar,
                               cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      k_predict_u8_scalar<<<pred_grid(n), kPredThreads, smem, s>>>(
          bins, n, ld, t0, c, m.depth, m.d_split8, m.d_leafval, m.base, t0 == 0, out);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (m.n_trees == 0) return cudaErrorInvalidValue;
  return cudaSuccess;
}

cudaError_t launch_predict_f32(const float* x, uint64_t n, uint32_t nf, const rw_dmodel& m,
                               float* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  (void)nf;
  const uint32_t tc = trees_per_chunk(m.n_trees, m.depth, 8);
  for (uint32_t t0 = 0; t0 < m.n_trees; t0 += tc) {
    const uint32_t c = m.n_trees - t0 < tc ? m.n_trees - t0 : tc;
    const size_t smem = ((size_t)c << m.depth) * 4 + (size_t)c * m.depth * 8;
    cudaError_t e = cudaFuncSetAttribute(k_predict_f32,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    k_predict_f32<<<pred_grid(n), kPredThreads, smem, s>>>(x, n, m.nf, t0, c, m.depth,
                                                           m.d_feat, m.d_thr, m.d_leafval,
                                                           m.base, t0 == 0, out);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (m.n_trees == 0) return cudaErrorInvalidValue;
  return cudaSuccess;
}
