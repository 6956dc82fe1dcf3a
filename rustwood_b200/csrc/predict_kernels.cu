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
//
// Small batches (a few thousand rows at most) take a different shape: one CTA per row,
// its threads walking different trees at once straight from the model in global memory
// (it stays in L1/L2 across the CTAs), each tree's leaf value into shared memory, then
// one thread adds them in tree order. A row then costs a few dependent memory round
// trips instead of a walk over every tree, and nothing is staged.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>
#include <tuple>
#include <vector>

#include "rw_internal.cuh"

namespace {

constexpr int kPredThreads = 256;
constexpr size_t kModelSmem = 200 * 1024;

__device__ __forceinline__ void stage_model(uint32_t t0, uint32_t tc, uint32_t depth,
                                            const uint32_t* __restrict__ g_split,
                                            const float* __restrict__ g_leaf, uint32_t* s_split,
                                            float* s_leaf) {
  for (uint32_t i = threadIdx.x; i < tc * depth; i += blockDim.x)
    s_split[i] = g_split[(size_t)t0 * depth + i];
  for (uint32_t i = threadIdx.x; i < (tc << depth); i += blockDim.x)
    s_leaf[i] = g_leaf[((size_t)t0 << depth) + i];
}

// Small batches: CTA r scores row r. Thread i walks trees i, i + blockDim.x, ...: the
// tree's D split words and the row's D values are loaded together (independent of each
// other), the leaf index is assembled MSB first, and the tree's leaf value lands in
// s_val[t]; thread 0 then adds base + s_val[0] + s_val[1] + ... in f32, in tree order --
// the same sequence predict_cpu (src/booster.rs:582-601) and the other scorers add.
// U8: feature-major bins [nf][ld], split words (feature << 8) | thr_bin, bit = bin > t.
// F32: row-major x [n][nf], feat/thr, bit = x > thr (NaN gives 0).
constexpr int kRowThreads = 256;
constexpr int kRowMaxDepth = 12;
template <bool U8>
__global__ void __launch_bounds__(kRowThreads) k_predict_rows(
    const void* __restrict__ in, uint64_t ld, uint32_t nf, uint32_t n_trees, uint32_t depth,
    const uint32_t* __restrict__ split8, const uint32_t* __restrict__ feat,
    const float* __restrict__ thr, const float* __restrict__ leafval, float base,
    float* __restrict__ out) {
  extern __shared__ float s_val[];  // [n_trees]
  const uint64_t r = blockIdx.x;
  for (uint32_t t = threadIdx.x; t < n_trees; t += blockDim.x) {
    const size_t k0 = (size_t)t * depth;
    uint32_t bits[kRowMaxDepth];
#pragma unroll
    for (int d = 0; d < kRowMaxDepth; d++) {
      bits[d] = 0u;
      if (d < (int)depth) {
        if (U8) {
          const uint32_t sv = __ldg(split8 + k0 + d);
          const uint32_t f = (sv >> 8) < nf ? (sv >> 8) : 0u;  // the host checks feature < nf
          const uint8_t* bins = static_cast<const uint8_t*>(in);
          bits[d] = (uint32_t)__ldg(bins + (size_t)f * ld + r) > (sv & 0xffu) ? 1u : 0u;
        } else {
          const uint32_t f0 = __ldg(feat + k0 + d), f = f0 < nf ? f0 : 0u;
          const float* x = static_cast<const float*>(in);
          bits[d] = __ldg(x + r * nf + f) > __ldg(thr + k0 + d) ? 1u : 0u;
        }
      }
    }
    uint32_t leaf = 0u;
#pragma unroll
    for (int d = 0; d < kRowMaxDepth; d++)
      if (d < (int)depth) leaf = 2u * leaf + bits[d];
    s_val[t] = __ldg(leafval + ((size_t)t << depth) + leaf);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float acc = base;
    for (uint32_t t = 0; t < n_trees; t++) acc += s_val[t];
    out[r] = acc;
  }
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
// chunk in shared memory once, then walks row blocks of kTileRows rows, 4 rows per
// thread. Per block the rows' bins are staged feature-major as one 32-bit word per
// (feature, thread) -- the thread's 4 rows -- so every split's bins come from one
// conflict-free shared load. The split test runs on the FMA pipe in half precision: two
// byte permutes turn the 4 bins into half values 1024 + bin (exact), and per pair of rows
// c = sat((1024 + bin) - (1024 + t)) is 1.0 exactly when bin > t (the difference is an
// exact integer in [-255, 255]); leaf = 2 * leaf + c is exact too: the leaf starts at
// 2^(10-D), so after D levels it holds 1024 + index < 2048, whose low byte is the index.
// The split table holds two levels per 16-byte entry (feature word offset, -(1024 + t) as
// half2), and two trees are walked together for four independent leaf chains per thread.
// Trees are scored in order and each row's sum is sequential f32 (the same order as
// predict_cpu).
// T threads per CTA (512, or 256 when the rows of 512 threads would not fit)
template <int D, int T>
__global__ void __launch_bounds__(T) k_predict_u8_tiled(
    const uint8_t* __restrict__ bins, uint64_t n, uint64_t ld, uint32_t nf, uint32_t t0,
    uint32_t tc, const uint32_t* __restrict__ split8, const float* __restrict__ leafval,
    float base, int first_chunk, float* __restrict__ out) {
  constexpr int DP = (D + 1) & ~1;  // levels per tree in the table, padded to pairs
  extern __shared__ __align__(16) unsigned char pred_raw[];
  uint2* s_sx = reinterpret_cast<uint2*>(pred_raw);  // [tc][DP]
  float* s_leaf = reinterpret_cast<float*>(pred_raw + (size_t)tc * DP * 8);
  uint32_t* s_rows = reinterpret_cast<uint32_t*>(s_leaf + ((size_t)tc << D));  // [nf][T]
  for (uint32_t i = threadIdx.x; i < tc * DP; i += blockDim.x) {
    const uint32_t tt = i / DP, d = i % DP;
    uint2 e = make_uint2(0u, 0u);
    if (d < (uint32_t)D) {
      const uint32_t sv = split8[((size_t)t0 + tt) * D + d];
      const uint32_t f = (sv >> 8) < nf ? (sv >> 8) : 0u;  // the host checks feature < nf
      const uint32_t nt16 =
          (uint32_t)__half_as_ushort(__float2half_rn(-(1024.0f + (float)(sv & 0xffu))));
      e = make_uint2(f * T * 4, nt16 | (nt16 << 16));
    }
    s_sx[i] = e;
  }
  for (uint32_t i = threadIdx.x; i < (tc << D); i += blockDim.x)
    s_leaf[i] = leafval[((size_t)t0 << D) + i];
  const uint32_t tid = threadIdx.x;
  constexpr uint32_t kTileRows = T * 4;
  const uint64_t nblk = (n + kTileRows - 1) / kTileRows;
  const unsigned char* my_rows = reinterpret_cast<const unsigned char*>(s_rows + tid);
  const __half2 two = __float2half2_rn(2.0f);
  const __half2 leaf0 = __float2half2_rn((float)(1u << (10 - D)));
  for (uint64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const uint64_t r0 = blk * kTileRows + (uint64_t)tid * 4;  // this thread's 4 rows
    __syncthreads();  // the previous block's rows (and the model) are settled
    for (uint32_t f = 0; f < nf; f++)
      s_rows[f * T + tid] =
          r0 + 3 < ld ? __ldg(reinterpret_cast<const uint32_t*>(bins + (size_t)f * ld + r0)) : 0u;
    __syncthreads();
    float acc[4];
    if (first_chunk) {
      acc[0] = acc[1] = acc[2] = acc[3] = base;
    } else {
#pragma unroll
      for (int k = 0; k < 4; k++) acc[k] = r0 + k < n ? out[r0 + k] : 0.0f;
    }
    // two trees per step; the sums still add tree t before tree t + 1
    for (uint32_t t = 0; t < tc; t += 2) {
      const bool second = t + 1 < tc;
      const uint4* sp0 = reinterpret_cast<const uint4*>(s_sx + (size_t)t * DP);
      const uint4* sp1 = reinterpret_cast<const uint4*>(s_sx + (size_t)(second ? t + 1 : t) * DP);
      __half2 la0 = leaf0, lb0 = leaf0, la1 = leaf0, lb1 = leaf0;  // rows (0, 1), (2, 3)
#pragma unroll
      for (int d = 0; d < D; d++) {
        // one 16-byte entry serves levels d and d + 1 (the repeated load folds away)
        const uint4 q0 = sp0[d / 2], q1 = sp1[d / 2];
        const uint32_t off0 = (d & 1) ? q0.z : q0.x, nt0 = (d & 1) ? q0.w : q0.y;
        const uint32_t off1 = (d & 1) ? q1.z : q1.x, nt1 = (d & 1) ? q1.w : q1.y;
        const uint32_t w0 = *reinterpret_cast<const uint32_t*>(my_rows + off0);
        const uint32_t w1 = *reinterpret_cast<const uint32_t*>(my_rows + off1);
        const uint32_t a0 = __byte_perm(w0, 0x64u, 0x4140), b0 = __byte_perm(w0, 0x64u, 0x4342);
        const uint32_t a1 = __byte_perm(w1, 0x64u, 0x4140), b1 = __byte_perm(w1, 0x64u, 0x4342);
        const __half2 n0 = *reinterpret_cast<const __half2*>(&nt0);
        const __half2 n1 = *reinterpret_cast<const __half2*>(&nt1);
        la0 = __hfma2(la0, two, __hadd2_sat(*reinterpret_cast<const __half2*>(&a0), n0));
        lb0 = __hfma2(lb0, two, __hadd2_sat(*reinterpret_cast<const __half2*>(&b0), n0));
        la1 = __hfma2(la1, two, __hadd2_sat(*reinterpret_cast<const __half2*>(&a1), n1));
        lb1 = __hfma2(lb1, two, __hadd2_sat(*reinterpret_cast<const __half2*>(&b1), n1));
      }
      {
        const uint32_t ia = *reinterpret_cast<const uint32_t*>(&la0);
        const uint32_t ib = *reinterpret_cast<const uint32_t*>(&lb0);
        const float* lv = s_leaf + ((size_t)t << D);
        acc[0] += lv[ia & 0xffu];
        acc[1] += lv[(ia >> 16) & 0xffu];
        acc[2] += lv[ib & 0xffu];
        acc[3] += lv[(ib >> 16) & 0xffu];
      }
      if (second) {
        const uint32_t ia = *reinterpret_cast<const uint32_t*>(&la1);
        const uint32_t ib = *reinterpret_cast<const uint32_t*>(&lb1);
        const float* lv = s_leaf + ((size_t)(t + 1) << D);
        acc[0] += lv[ia & 0xffu];
        acc[1] += lv[(ia >> 16) & 0xffu];
        acc[2] += lv[ib & 0xffu];
        acc[3] += lv[(ib >> 16) & 0xffu];
      }
    }
#pragma unroll
    for (int k = 0; k < 4; k++)
      if (r0 + k < n) out[r0 + k] = acc[k];
  }
}

template <int D>
const void* tiled_fn(int threads) {
  return threads == 512 ? reinterpret_cast<const void*>(&k_predict_u8_tiled<D, 512>)
                        : reinterpret_cast<const void*>(&k_predict_u8_tiled<D, 256>);
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

// Batches of at most kRowsMax rows whose model's leaf values fit the default 48 KB of
// shared memory go to k_predict_rows (C5's 500-tree model on B200: 12 us for one row, 19 us
// for 1024, 77 us for 8192, 142 us for 16384, where the tiled scorer's per-thread walk over
// the trees costs about 120 us up to 100k rows).
#ifndef RW_PRED_ROWS_MAX
#define RW_PRED_ROWS_MAX 12288
#endif
constexpr uint64_t kRowsMax = RW_PRED_ROWS_MAX;
bool small_batch(uint64_t n, const rw_dmodel& m) {
  return n <= kRowsMax && m.n_trees > 0 && (size_t)m.n_trees * 4 <= 48 * 1024;
}

int pred_grid(uint64_t work) {
  uint64_t b = (work + kPredThreads - 1) / kPredThreads;
  const uint64_t cap = 148ull * 8;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

// Raises a kernel's dynamic shared-memory limit when a launch needs more than it was last
// set to (per device; the limit only grows, so a smaller launch never lowers it under a
// larger one) and returns the kernel's resident CTAs per SM at that size, queried once per
// (device, kernel, size): the two runtime calls would otherwise sit between the launches
// of every call, which small batches feel.
static cudaError_t tiled_prepare(int dev, const void* fn, int threads, size_t smem, int* per_sm) {
  static std::mutex mu;
  static std::vector<std::tuple<int, const void*, size_t>> limit;       // (dev, fn, bytes)
  static std::vector<std::tuple<int, const void*, size_t, int>> occ;   // (dev, fn, bytes, CTAs)
  std::lock_guard<std::mutex> lock(mu);
  size_t* lim = nullptr;
  for (auto& l : limit)
    if (std::get<0>(l) == dev && std::get<1>(l) == fn) lim = &std::get<2>(l);
  if (!lim || smem > *lim) {
    cudaError_t e =
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (lim) *lim = smem;
    else limit.emplace_back(dev, fn, smem);
  }
  for (const auto& o : occ)
    if (std::get<0>(o) == dev && std::get<1>(o) == fn && std::get<2>(o) == smem) {
      *per_sm = std::get<3>(o);
      return cudaSuccess;
    }
  int k = 1;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&k, fn, threads, smem);
  if (e != cudaSuccess) return e;
  *per_sm = std::max(k, 1);
  if (occ.size() >= 4096) occ.clear();  // many distinct models: keep the table bounded
  occ.emplace_back(dev, fn, smem, *per_sm);
  return cudaSuccess;
}

// The tiled scorer for depth 1..8 when the rows' bins fit next to a tree chunk.
static cudaError_t launch_predict_u8_tiled(const uint8_t* bins, uint64_t n, uint64_t ld,
                                           const rw_dmodel& m, float* out, cudaStream_t s,
                                           bool* used) {
  *used = false;
  // 512 threads when their rows take at most 128 KB of shared memory, else 256
  const int T = (size_t)m.nf * 512 * 4 <= 128 * 1024 ? 512 : 256;
  const size_t rows_bytes = (size_t)m.nf * T * 4;
  if (m.depth < 1 || m.depth > 8 || rows_bytes > 128 * 1024) return cudaSuccess;
  const size_t per_tree = ((size_t)4 << m.depth) + 8 * (size_t)((m.depth + 1) & ~1u);
  const size_t budget = 220 * 1024 - rows_bytes;
  uint32_t tc = (uint32_t)std::min<size_t>(m.n_trees, budget / per_tree);
  if (tc < 1) return cudaSuccess;
  // chunks of equal size (each chunk is one more pass over the rows)
  const uint32_t n_chunks = (m.n_trees + tc - 1) / tc;
  tc = (m.n_trees + n_chunks - 1) / n_chunks;
  const void* fns[9] = {nullptr,         tiled_fn<1>(T), tiled_fn<2>(T), tiled_fn<3>(T),
                        tiled_fn<4>(T),  tiled_fn<5>(T), tiled_fn<6>(T), tiled_fn<7>(T),
                        tiled_fn<8>(T)};
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const uint64_t nblk = (n + (uint64_t)T * 4 - 1) / ((uint64_t)T * 4);
  for (uint32_t t0 = 0; t0 < m.n_trees; t0 += tc) {
    const uint32_t c = m.n_trees - t0 < tc ? m.n_trees - t0 : tc;
    const size_t smem = ((size_t)c << m.depth) * 4 + (size_t)c * ((m.depth + 1) & ~1u) * 8 + rows_bytes;
    int per_sm = 1;
    cudaError_t e = tiled_prepare(dev, fns[m.depth], T, smem, &per_sm);
    if (e != cudaSuccess) return e;
    const uint64_t grid = std::max<uint64_t>(1, std::min<uint64_t>(nblk, (uint64_t)sms * per_sm));
    int first = t0 == 0;
    uint64_t nn = n, ll = ld;
    uint32_t nf = m.nf, tt0 = t0, cc = c;
    const uint32_t* sp = m.d_split8;
    const float* lp = m.d_leafval;
    float b = m.base;
    const uint8_t* bp = bins;
    float* op = out;
    void* args[] = {&bp, &nn, &ll, &nf, &tt0, &cc, &sp, &lp, &b, &first, &op};
    e = cudaLaunchKernel(fns[m.depth], dim3((unsigned)grid), dim3(T), args, smem, s);
    if (e != cudaSuccess) return e;
  }
  *used = true;
  return cudaSuccess;
}

cudaError_t launch_predict_u8(const uint8_t* bins, uint64_t n, uint64_t ld, const rw_dmodel& m,
                              float* out, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (small_batch(n, m)) {
    k_predict_rows<true><<<(unsigned)n, kRowThreads, (size_t)m.n_trees * 4, s>>>(
        bins, ld, m.nf, m.n_trees, m.depth, m.d_split8, nullptr, nullptr, m.d_leafval, m.base,
        out);
    return cudaGetLastError();
  }
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
  if (small_batch(n, m)) {
    k_predict_rows<false><<<(unsigned)n, kRowThreads, (size_t)m.n_trees * 4, s>>>(
        x, 0, m.nf, m.n_trees, m.depth, nullptr, m.d_feat, m.d_thr, m.d_leafval, m.base, out);
    return cudaGetLastError();
  }
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
