// Scoring from host buffers without any device allocation.
//
// rw_predict_f32 stages the model, the input rows and the margins in device buffers it
// allocates per call. Some callers cannot allocate device memory at all: a serving
// process whose device memory is owned by another allocator (a framework's caching
// pool or a fixed pre-reserved budget), or a latency-critical path where the implicit
// device-wide synchronisation of cudaMalloc/cudaFree would stall the other streams.
// rw_predict_f32_noalloc gives them the same scores using only the fixed staging array
// below, which every GPU that loads this library holds until the process exits.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string>

#include "rw_internal.cuh"

namespace {

constexpr size_t kStageBytes = 16u << 20;       // whole staging array: 16 MiB
constexpr size_t kModelMaxBytes = 4u << 20;     // model region limit: 4 MiB
constexpr int kMaxDevices = 64;

// The staging area: [model: feat u32 | thr f32 | leafval f32][rows f32 | margins f32].
static __device__ __align__(256) unsigned char g_stage[kStageBytes];

std::mutex g_stage_mu;
void* g_stage_addr[kMaxDevices] = {};

int fail(rw_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  return code;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

// Device address of this device's copy of g_stage. The host-side name g_stage is only
// a stand-in for the symbol, so the address is looked up once per device (with that
// device current) and cached; the lookup runs on the first call on each device. The
// cache lives as long as the process: a caller that resets a device (cudaDeviceReset)
// and keeps using it must reload the library first.
int stage_address(rw_ctx* ctx, unsigned char** out) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices)
    return fail(ctx, RW_ERR_ARG, "device index beyond the staging table");
  std::lock_guard<std::mutex> lock(g_stage_mu);
  if (!g_stage_addr[ctx->device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_stage);
    if (e != cudaSuccess || !p)
      return fail(ctx, RW_ERR_CUDA,
                  std::string("cudaGetSymbolAddress(g_stage): ") + cudaGetErrorString(e));
    g_stage_addr[ctx->device] = p;
  }
  *out = static_cast<unsigned char*>(g_stage_addr[ctx->device]);
  return RW_OK;
}

}  // namespace

extern "C" int rw_predict_f32_noalloc(rw_ctx* ctx, const rw_model* m, const float* x,
                                      uint64_t n, uint32_t nf, float* out) {
  if (!ctx) return fail(nullptr, RW_ERR_ARG, "ctx is NULL");
  if (!m) return fail(ctx, RW_ERR_ARG, "model is NULL");
  if (m->depth < 1 || m->depth > 12) return fail(ctx, RW_ERR_ARG, "depth must be in 1..=12");
  if (nf != m->n_features) return fail(ctx, RW_ERR_ARG, "nf differs from the model's n_features");
  if (m->n_trees > 0 && (!m->feat || !m->thr || !m->leafval))
    return fail(ctx, RW_ERR_ARG, "NULL model array");
  if (n == 0) return RW_OK;
  if (!x || !out) return fail(ctx, RW_ERR_ARG, "NULL buffer");
  if (!ctx->members.empty()) {
    // a multi-GPU context: contiguous row shards, each GPU through its own staging array
    const uint64_t W = ctx->members.size();
    return for_each_rank(ctx, [&](int i) {
      const uint64_t lo = n * (uint64_t)i / W, hi = n * (uint64_t)(i + 1) / W;
      return rw_predict_f32_noalloc(ctx->members[i], m, x + lo * nf, hi - lo, nf, out + lo);
    });
  }
  const size_t K = (size_t)m->n_trees * m->depth, L = (size_t)m->n_trees << m->depth;
  for (size_t k = 0; k < K; k++)
    if (m->feat[k] >= nf) return fail(ctx, RW_ERR_ARG, "feature index out of range");
  const size_t off_thr = align256(K * 4), off_leaf = off_thr + align256(K * 4);
  const size_t model_bytes = off_leaf + align256(L * 4);
  if (model_bytes > kModelMaxBytes)
    return fail(ctx, RW_ERR_ARG,
                "model needs " + std::to_string(model_bytes) +
                    " staging bytes; rw_predict_f32_noalloc stages at most 4 MiB of model");
  const size_t row_bytes = ((size_t)nf + 1) * 4;
  // 256 bytes of slack cover the alignment of the margins region after the rows.
  const uint64_t batch = (kStageBytes - model_bytes - 256) / row_bytes / 64 * 64;
  if (batch == 0) return fail(ctx, RW_ERR_ARG, "rows too wide for the 16 MiB staging array");

  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return fail(ctx, RW_ERR_CUDA, cudaGetErrorString(e));
  unsigned char* stage = nullptr;
  int rc = stage_address(ctx, &stage);
  if (rc) return rc;
  cudaStream_t s = ctx->stream;

  rw_dmodel dm;
  dm.ctx = ctx;
  dm.n_trees = m->n_trees;
  dm.depth = m->depth;
  dm.nf = nf;
  dm.base = m->base_score;
  dm.d_feat = reinterpret_cast<uint32_t*>(stage);
  dm.d_thr = reinterpret_cast<float*>(stage + off_thr);
  dm.d_leafval = reinterpret_cast<float*>(stage + off_leaf);
  float* d_rows = reinterpret_cast<float*>(stage + model_bytes);
  float* d_out = reinterpret_cast<float*>(stage + model_bytes + align256(batch * nf * 4));
  if (model_bytes + align256(batch * nf * 4) + batch * 4 > kStageBytes)
    return fail(ctx, RW_ERR_ARG, "staging layout overflow");

  if (K) {
    e = cudaMemcpyAsync(dm.d_feat, m->feat, K * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dm.d_thr, m->thr, K * 4, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(dm.d_leafval, m->leafval, L * 4, cudaMemcpyHostToDevice, s);
  }
  for (uint64_t r0 = 0; r0 < n && e == cudaSuccess; r0 += batch) {
    const uint64_t b = n - r0 < batch ? n - r0 : batch;
    e = cudaMemcpyAsync(d_rows, x + r0 * nf, b * nf * 4, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) break;
    if (m->n_trees == 0) {
      int nl = 0;
      e = launch_fill_f32(d_out, m->base_score, b, s, &nl);
    } else {
      e = launch_predict_f32(d_rows, b, nf, dm, d_out, s);
    }
    ctx->launches += 1;
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(out + r0, d_out, b * 4, cudaMemcpyDeviceToHost, s);
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess)
    return fail(ctx, RW_ERR_CUDA, std::string("rw_predict_f32_noalloc: ") + cudaGetErrorString(e));
  return RW_OK;
}
