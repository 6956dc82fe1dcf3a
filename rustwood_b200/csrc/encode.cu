// Categorical target encoding on the GPU (src/encoding.rs:44-95, fit_transform_train).
//
// Per categorical feature c and row i the reference takes key = key_of(x[i][c]) (the
// category code, optionally folded by the hashing trick), sums y per (key, fold = i % k)
// in f64 in row order, and replaces x[i][c] by the smoothed out-of-fold mean
// (s + a*gm) / (cnt + a) of the other folds (gmean when they are empty); the test-set map
// is the same formula over all folds. Here the keys index dense tables over each feature's
// [min key, max key] range, and the sums are exact int64 sums of y in the wide fixed point
// (rw_wquantize with the scale of max |y| and n): order-free, so they equal the
// reference's sequential f64 sums whenever those are exact -- every label a multiple of
// the fixed point's unit and every partial sum within f64's 53 bits, e.g. 0/1 targets
// or small integer labels. Features whose key range is too wide for dense tables are
// refused (the host encoder handles them).
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <string>
#include <vector>

#include "rw_expf.h"
#include "rw_internal.cuh"

namespace {

constexpr uint64_t kTeHashSalt = 0x0041445650524F50ull;  // src/encoding.rs:27

// key_of (src/encoding.rs:29-40): f32::round (half away from zero), a saturating `as i64`
// (NaN -> 0, out-of-range values clamp to the i64 range), then optionally the hashing trick.
__device__ __forceinline__ long long te_key(float v, unsigned long long buckets) {
  const float r = roundf(v);
  long long c;
  if (!(v == v)) c = 0;
  else if (r >= 9.223372036854775807e18f) c = INT64_MAX;
  else if (r <= -9.223372036854775808e18f) c = INT64_MIN;
  else c = (long long)r;
  if (buckets == 0) return c;
  unsigned long long x = ((unsigned long long)c ^ kTeHashSalt) * 0x9E3779B97F4A7C15ull;
  x ^= x >> 29;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 32;
  return (long long)(x % buckets);
}

struct TeArgs {
  const float* x;   // [n][nf] row-major
  float* x_out;     // the same rows, categorical columns rewritten (may equal x)
  const float* y;
  uint64_t n;
  uint32_t nf, n_cat, k;
  const uint32_t* cat;      // [n_cat] feature indices
  unsigned long long buckets;
  long long* keys;          // [n_cat][n]
  long long* kmin;          // [n_cat]
  long long* kmax;          // [n_cat]
  uint32_t* ymax_bits;      // max |y| as f32 bits
  const uint64_t* off;      // [n_cat] first table entry of each feature (entries = keys * k)
  long long* sums;          // [entries] wide fixed-point y sums per (key, fold)
  uint32_t* cnts;           // [entries] rows per (key, fold)
  long long* gsum;          // the wide sum of all y
  double a;                 // smoothing
  float* full;              // [keys] test-set map values
  uint8_t* present;         // [keys] key seen in training
  const uint64_t* koff;     // [n_cat] first key slot of each feature
};

// Keys of every (row, categorical feature), each feature's key range, and max |y|.
__global__ void k_te_keys(TeArgs a) {
  const uint64_t total = a.n * a.n_cat;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = (uint32_t)(t / a.n);
    const uint64_t i = t % a.n;
    const long long key = te_key(a.x[i * a.nf + a.cat[j]], a.buckets);
    a.keys[t] = key;
    atomicMin(a.kmin + j, key);
    atomicMax(a.kmax + j, key);
    if (j == 0) {
      const float ay = fabsf(a.y[i]);
      if (ay == ay) atomicMax(a.ymax_bits, __float_as_uint(ay));
    }
  }
}

// Per (key, fold) sums and counts, and the global sum (exact integers).
__global__ void k_te_sums(TeArgs a) {
  const int w = rw_wscale_exp(*a.ymax_bits, a.n);
  const uint64_t total = a.n * a.n_cat;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = (uint32_t)(t / a.n);
    const uint64_t i = t % a.n;
    const long long q = rw_wquantize(a.y[i], w);
    const uint64_t e = a.off[j] + (uint64_t)(a.keys[t] - a.kmin[j]) * a.k + i % a.k;
    if (q) atomicAdd(reinterpret_cast<unsigned long long*>(a.sums + e), (unsigned long long)q);
    atomicAdd(a.cnts + e, 1u);
    if (j == 0 && q) atomicAdd(reinterpret_cast<unsigned long long*>(a.gsum), (unsigned long long)q);
  }
}

__device__ __forceinline__ float te_gmean(const TeArgs& a, int w) {
  return (float)(rw_wvalue(*a.gsum, w) / (double)a.n);
}

// The out-of-fold value of every (row, categorical feature) (src/encoding.rs:78-91).
__global__ void k_te_apply(TeArgs a) {
  const int w = rw_wscale_exp(*a.ymax_bits, a.n);
  const float gmean = te_gmean(a, w);
  const double gm = (double)gmean;
  const uint64_t total = a.n * a.n_cat;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = (uint32_t)(t / a.n);
    const uint64_t i = t % a.n;
    const uint64_t e0 = a.off[j] + (uint64_t)(a.keys[t] - a.kmin[j]) * a.k;
    const uint32_t f = (uint32_t)(i % a.k);
    long long s_all = 0;
    unsigned long long c_all = 0;
    for (uint32_t g = 0; g < a.k; g++) {
      s_all += a.sums[e0 + g];
      c_all += a.cnts[e0 + g];
    }
    const double s = rw_wvalue(s_all - a.sums[e0 + f], w);
    const double cnt = (double)(c_all - a.cnts[e0 + f]);
    a.x_out[i * a.nf + a.cat[j]] = cnt > 0.0 ? (float)((s + a.a * gm) / (cnt + a.a)) : gmean;
  }
}

// The test-set map (src/encoding.rs:70-76): every key seen in training.
__global__ void k_te_full(TeArgs a, uint64_t n_keys_total) {
  const int w = rw_wscale_exp(*a.ymax_bits, a.n);
  const double gm = (double)te_gmean(a, w);
  for (uint64_t s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n_keys_total;
       s += (uint64_t)gridDim.x * blockDim.x) {
    uint32_t j = 0;
    while (j + 1 < a.n_cat && a.koff[j + 1] <= s) j++;
    const uint64_t e0 = a.off[j] + (s - a.koff[j]) * a.k;
    long long s_all = 0;
    unsigned long long c_all = 0;
    for (uint32_t g = 0; g < a.k; g++) {
      s_all += a.sums[e0 + g];
      c_all += a.cnts[e0 + g];
    }
    a.present[s] = c_all > 0 ? 1 : 0;
    a.full[s] = c_all > 0 ? (float)((rw_wvalue(s_all, w) + a.a * gm) / ((double)c_all + a.a))
                          : 0.0f;
  }
}

int te_grid(uint64_t work) {
  uint64_t b = (work + 255) / 256;
  if (b > 148ull * 16) b = 148ull * 16;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace

// Host driver (declared in rw_internal.cuh): encodes d_x in place on ctx's stream.
int target_encode_device(rw_ctx* ctx, float* d_x, const float* d_y, uint64_t n, uint32_t nf,
                         const uint32_t* cat, uint32_t n_cat, float smoothing, uint32_t k_folds,
                         uint64_t hash_buckets, float* gmean_out, rw_encoders* enc,
                         std::string* why) {
  cudaStream_t s = ctx->stream;
  const uint32_t k = k_folds < 2 ? 2 : k_folds;
  for (uint32_t j = 0; j < n_cat; j++)
    if (cat[j] >= nf) {
      *why = "categorical feature index out of range";
      return RW_ERR_ARG;
    }
  // phase 1: keys and ranges
  uint32_t* d_cat = nullptr;
  long long *d_keys = nullptr, *d_mm = nullptr;
  uint32_t* d_ymax = nullptr;
  cudaError_t e = cudaMalloc(&d_cat, std::max<size_t>(n_cat, 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&d_keys, std::max<size_t>(n * n_cat, 1) * 8);
  if (e == cudaSuccess) e = cudaMalloc(&d_mm, (size_t)2 * std::max<uint32_t>(n_cat, 1) * 8 + 16);
  if (e == cudaSuccess) e = cudaMalloc(&d_ymax, 4);
  std::vector<long long> mm(2 * (size_t)n_cat);
  for (uint32_t j = 0; j < n_cat; j++) {
    mm[j] = INT64_MAX;
    mm[n_cat + j] = INT64_MIN;
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_cat, cat, (size_t)n_cat * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && n_cat)
    e = cudaMemcpyAsync(d_mm, mm.data(), mm.size() * 8, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(d_ymax, 0, 4, s);
  TeArgs a = {};
  a.x = d_x;
  a.x_out = d_x;
  a.y = d_y;
  a.n = n;
  a.nf = nf;
  a.n_cat = n_cat;
  a.k = k;
  a.cat = d_cat;
  a.buckets = hash_buckets;
  a.keys = d_keys;
  a.kmin = d_mm;
  a.kmax = d_mm + n_cat;
  a.ymax_bits = d_ymax;
  a.a = (double)smoothing;
  if (e == cudaSuccess && n_cat) {
    k_te_keys<<<te_grid(n * n_cat), 256, 0, s>>>(a);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && n_cat)
    e = cudaMemcpyAsync(mm.data(), d_mm, mm.size() * 8, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  // dense tables: one slot per key in [kmin, kmax] per feature
  std::vector<uint64_t> off(n_cat), koff(n_cat);
  uint64_t keys_total = 0;
  const uint64_t kMaxKeys = 1ull << 26;  // all features together
  int rc = RW_OK;
  for (uint32_t j = 0; j < n_cat && e == cudaSuccess && rc == RW_OK; j++) {
    const unsigned long long range =
        (unsigned long long)mm[n_cat + j] - (unsigned long long)mm[j] + 1ull;  // n >= 1
    if (range == 0 || range > kMaxKeys || keys_total + range > kMaxKeys) {
      *why = "category key range too wide for the GPU encoder's dense tables";
      rc = RW_ERR_UNSUPPORTED;
      break;
    }
    koff[j] = keys_total;
    off[j] = keys_total * k;
    keys_total += range;
  }
  long long *d_sums = nullptr, *d_gsum = nullptr;
  uint32_t* d_cnts = nullptr;
  uint64_t *d_off = nullptr, *d_koff = nullptr;
  float* d_full = nullptr;
  uint8_t* d_present = nullptr;
  if (e == cudaSuccess && rc == RW_OK) {
    e = cudaMalloc(&d_sums, std::max<uint64_t>(keys_total * k, 1) * 8);
    if (e == cudaSuccess) e = cudaMalloc(&d_cnts, std::max<uint64_t>(keys_total * k, 1) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&d_gsum, 8);
    if (e == cudaSuccess) e = cudaMalloc(&d_off, std::max<size_t>(n_cat, 1) * 8);
    if (e == cudaSuccess) e = cudaMalloc(&d_koff, std::max<size_t>(n_cat, 1) * 8);
    if (e == cudaSuccess) e = cudaMalloc(&d_full, std::max<uint64_t>(keys_total, 1) * 4);
    if (e == cudaSuccess) e = cudaMalloc(&d_present, std::max<uint64_t>(keys_total, 1));
    if (e == cudaSuccess) e = cudaMemsetAsync(d_sums, 0, std::max<uint64_t>(keys_total * k, 1) * 8, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(d_cnts, 0, std::max<uint64_t>(keys_total * k, 1) * 4, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(d_gsum, 0, 8, s);
    if (e == cudaSuccess && n_cat)
      e = cudaMemcpyAsync(d_off, off.data(), (size_t)n_cat * 8, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess && n_cat)
      e = cudaMemcpyAsync(d_koff, koff.data(), (size_t)n_cat * 8, cudaMemcpyHostToDevice, s);
    a.off = d_off;
    a.koff = d_koff;
    a.sums = d_sums;
    a.cnts = d_cnts;
    a.gsum = d_gsum;
    a.full = d_full;
    a.present = d_present;
    if (e == cudaSuccess && n_cat) {
      k_te_sums<<<te_grid(n * n_cat), 256, 0, s>>>(a);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess && n_cat) {
      k_te_apply<<<te_grid(n * n_cat), 256, 0, s>>>(a);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess && n_cat) {
      k_te_full<<<te_grid(keys_total), 256, 0, s>>>(a, keys_total);
      e = cudaGetLastError();
    }
    // gmean (also when there is no categorical feature: the reference returns it)
    long long gs = 0;
    uint32_t yb = 0;
    if (e == cudaSuccess && n_cat == 0) {
      // no keys pass: the global sum from y directly (k_te_sums needs a feature)
      std::vector<float> hy(n);
      e = cudaMemcpyAsync(hy.data(), d_y, n * 4, cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      if (e == cudaSuccess) {
        double acc = 0.0;
        for (uint64_t i = 0; i < n; i++) acc += (double)hy[i];
        if (gmean_out) *gmean_out = (float)(acc / (double)n);
      }
    } else {
      if (e == cudaSuccess) e = cudaMemcpyAsync(&gs, d_gsum, 8, cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaMemcpyAsync(&yb, d_ymax, 4, cudaMemcpyDeviceToHost, s);
    }
    if (enc && e == cudaSuccess) {
      enc->key_lo.assign(mm.begin(), mm.begin() + n_cat);
      enc->koff = koff;
      enc->n_keys.resize(n_cat);
      for (uint32_t j = 0; j < n_cat; j++)
        enc->n_keys[j] = (j + 1 < n_cat ? koff[j + 1] : keys_total) - koff[j];
      enc->value.resize(keys_total);
      enc->present.resize(keys_total);
      if (keys_total) {
        e = cudaMemcpyAsync(enc->value.data(), d_full, keys_total * 4, cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess)
          e = cudaMemcpyAsync(enc->present.data(), d_present, keys_total, cudaMemcpyDeviceToHost, s);
      }
    }
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && n_cat && gmean_out)
      *gmean_out = (float)(rw_wvalue(gs, rw_wscale_exp(yb, n)) / (double)n);
    if (enc && gmean_out) enc->gmean = *gmean_out;
  }
  cudaFree(d_cat);
  cudaFree(d_keys);
  cudaFree(d_mm);
  cudaFree(d_ymax);
  cudaFree(d_sums);
  cudaFree(d_cnts);
  cudaFree(d_gsum);
  cudaFree(d_off);
  cudaFree(d_koff);
  cudaFree(d_full);
  cudaFree(d_present);
  if (e != cudaSuccess) {
    *why = std::string("target encoding: ") + cudaGetErrorString(e);
    return RW_ERR_CUDA;
  }
  return rc;
}

// =================================================================================
// encoding::transform (src/encoding.rs:96-115) on the GPU: every categorical value of the
// rows becomes its key's test-set value, unseen keys the training mean.

namespace {

struct TeMaps {
  float* x;
  uint64_t n;
  uint32_t nf, n_cat;
  const uint32_t* cat;        // [n_cat]
  const long long* key_lo;    // [n_cat]
  const uint64_t* koff;       // [n_cat]
  const uint64_t* n_keys;     // [n_cat]
  const float* value;         // [slots]
  const uint8_t* present;     // [slots]
  float gmean;
  unsigned long long buckets;
};

__global__ void k_te_transform(TeMaps m) {
  const uint64_t total = m.n * m.n_cat;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t j = (uint32_t)(t / m.n);
    const uint64_t i = t % m.n;
    float* v = m.x + i * m.nf + m.cat[j];
    // the slot of key - key_lo, unsigned so keys below key_lo fall outside too
    const unsigned long long d =
        (unsigned long long)te_key(*v, m.buckets) - (unsigned long long)m.key_lo[j];
    float out = m.gmean;
    if (d < m.n_keys[j] && m.present[m.koff[j] + d]) out = m.value[m.koff[j] + d];
    *v = out;
  }
}

}  // namespace

int target_transform_device(rw_ctx* ctx, float* d_x, uint64_t n, uint32_t nf, const uint32_t* cat,
                            uint32_t n_cat, const rw_encoders& enc, uint64_t hash_buckets,
                            std::string* why) {
  if (enc.key_lo.size() != n_cat) {
    *why = "the encoders hold a different number of categorical features";
    return RW_ERR_ARG;
  }
  for (uint32_t j = 0; j < n_cat; j++)
    if (cat[j] >= nf) {
      *why = "categorical feature index out of range";
      return RW_ERR_ARG;
    }
  if (n == 0 || n_cat == 0) return RW_OK;
  cudaStream_t s = ctx->stream;
  const uint64_t slots = enc.value.size();
  uint32_t* d_cat = nullptr;
  long long* d_lo = nullptr;
  uint64_t *d_koff = nullptr, *d_nk = nullptr;
  float* d_val = nullptr;
  uint8_t* d_pres = nullptr;
  cudaError_t e = cudaMalloc(&d_cat, (size_t)n_cat * 4);
  if (e == cudaSuccess) e = cudaMalloc(&d_lo, (size_t)n_cat * 8);
  if (e == cudaSuccess) e = cudaMalloc(&d_koff, (size_t)n_cat * 8);
  if (e == cudaSuccess) e = cudaMalloc(&d_nk, (size_t)n_cat * 8);
  if (e == cudaSuccess) e = cudaMalloc(&d_val, std::max<uint64_t>(slots, 1) * 4);
  if (e == cudaSuccess) e = cudaMalloc(&d_pres, std::max<uint64_t>(slots, 1));
  if (e == cudaSuccess) e = cudaMemcpyAsync(d_cat, cat, (size_t)n_cat * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_lo, enc.key_lo.data(), (size_t)n_cat * 8, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_koff, enc.koff.data(), (size_t)n_cat * 8, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(d_nk, enc.n_keys.data(), (size_t)n_cat * 8, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && slots)
    e = cudaMemcpyAsync(d_val, enc.value.data(), slots * 4, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess && slots)
    e = cudaMemcpyAsync(d_pres, enc.present.data(), slots, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) {
    TeMaps m;
    m.x = d_x;
    m.n = n;
    m.nf = nf;
    m.n_cat = n_cat;
    m.cat = d_cat;
    m.key_lo = d_lo;
    m.koff = d_koff;
    m.n_keys = d_nk;
    m.value = d_val;
    m.present = d_pres;
    m.gmean = enc.gmean;
    m.buckets = hash_buckets;
    k_te_transform<<<te_grid(n * n_cat), 256, 0, s>>>(m);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  cudaFree(d_cat);
  cudaFree(d_lo);
  cudaFree(d_koff);
  cudaFree(d_nk);
  cudaFree(d_val);
  cudaFree(d_pres);
  if (e != cudaSuccess) {
    *why = std::string("target transform: ") + cudaGetErrorString(e);
    return RW_ERR_CUDA;
  }
  return RW_OK;
}
