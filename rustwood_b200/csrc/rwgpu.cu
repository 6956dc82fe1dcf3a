// C-ABI implementation of include/rwgpu.h: contexts, device datasets, the boosting
// loop (the body of rustwood's Booster::fit_inner, src/booster.rs:227-517), scoring
// and the host helpers the reference keeps on the host.
#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>
#include <string.h>

#include <cstdlib>
#include <cstring>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <functional>
#include <string>
#include <thread>
#include <vector>

#include "rw_expf.h"
#include "rw_internal.cuh"

namespace {

thread_local std::string g_tls_error;

int fail(rw_ctx* ctx, int code, const std::string& msg) {
  if (ctx) ctx->last_error = msg;
  g_tls_error = msg;
  return code;
}

int cuda_fail(rw_ctx* ctx, cudaError_t e, const char* what) {
  return fail(ctx, e == cudaErrorMemoryAllocation ? RW_ERR_OOM : RW_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

#define RW_CU(ctx, expr)                                     \
  do {                                                       \
    cudaError_t _e = (expr);                                 \
    if (_e != cudaSuccess) return cuda_fail((ctx), _e, #expr); \
  } while (0)

// The communicator is non-blocking: a call may return ncclInProgress (e.g. while it
// sets up connections on first use) and the communicator takes no further call until
// its state reads ncclSuccess. nccl_settle polls that state, bounded by the context
// timeout (then the communicator is aborted).
ncclResult_t nccl_settle(rw_ctx* ctx, ncclResult_t r);
#define RW_NC(ctx, expr)                                                        \
  do {                                                                          \
    ncclResult_t _r = nccl_settle((ctx), (expr));                               \
    if (_r != ncclSuccess)                                                      \
      return fail((ctx), RW_ERR_NCCL, std::string(#expr) + ": " + ncclGetErrorString(_r)); \
  } while (0)

// Stream-ordered allocation from the context's pool (ordered on the context stream).
cudaError_t pool_alloc(rw_ctx* ctx, void** p, size_t bytes) {
  return cudaMallocFromPoolAsync(p, std::max<size_t>(bytes, 1), ctx->pool, ctx->stream);
}
void pool_free(rw_ctx* ctx, void* p) {
  if (p) cudaFreeAsync(p, ctx->stream);
}

// Device allocation owned by a scope: from the context's pool (alloc(ctx, n), freed in
// stream order) or plain cudaMalloc (alloc(n)).
template <typename T>
struct DBuf {
  T* p = nullptr;
  size_t n = 0;
  rw_ctx* pool_ctx = nullptr;
  DBuf() = default;
  DBuf(const DBuf&) = delete;
  DBuf& operator=(const DBuf&) = delete;
  ~DBuf() {
    if (!p) return;
    if (pool_ctx) pool_free(pool_ctx, p);
    else cudaFree(p);
  }
  cudaError_t alloc(size_t count) {
    n = count;
    return cudaMalloc(reinterpret_cast<void**>(&p), std::max<size_t>(count, 1) * sizeof(T));
  }
  cudaError_t alloc(rw_ctx* ctx, size_t count) {
    n = count;
    pool_ctx = ctx;
    return pool_alloc(ctx, reinterpret_cast<void**>(&p), count * sizeof(T));
  }
  T* release() {
    T* q = p;
    p = nullptr;
    return q;
  }
};

// A view of a named buffer in the dataset's workspace cache (owned by the dataset).
template <typename T>
struct WsBuf {
  T* p = nullptr;
  size_t n = 0;
  cudaError_t get(rw_dataset* ds, const char* name, size_t count) {
    n = count;
    const size_t bytes = std::max<size_t>(count, 1) * sizeof(T);
    auto it = ds->ws.find(name);
    if (it != ds->ws.end() && it->second.second >= bytes) {
      p = static_cast<T*>(it->second.first);
      return cudaSuccess;
    }
    if (it != ds->ws.end()) {
      pool_free(ds->ctx, it->second.first);
      ds->ws.erase(it);
    }
    void* q = nullptr;
    cudaError_t e = pool_alloc(ds->ctx, &q, bytes);
    if (e != cudaSuccess) return e;
    ds->ws[name] = {q, bytes};
    p = static_cast<T*>(q);
    return cudaSuccess;
  }
};

uint64_t round_up(uint64_t v, uint64_t m) { return (v + m - 1) / m * m; }

ncclResult_t nccl_settle(rw_ctx* ctx, ncclResult_t r) {
  if (r != ncclInProgress || !ctx->comm) return r;
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    ncclCommGetAsyncError(ctx->comm, &st);
    if (st != ncclInProgress) return st;
    const double ms = std::chrono::duration<double, std::milli>(
                          std::chrono::steady_clock::now() - t0).count();
    if (ctx->timeout_ms > 0 && ms > (double)ctx->timeout_ms) {
      ncclCommAbort(ctx->comm);
      ctx->comm = nullptr;
      return ncclInternalError;
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

// Wait for the context stream; with a communicator, bound the wait and abort the
// communicator when the limit passes or NCCL reports an asynchronous error.
int wait_stream(rw_ctx* ctx) {
  if (!ctx->comm) {
    RW_CU(ctx, cudaStreamSynchronize(ctx->stream));
    return RW_OK;
  }
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t q = cudaStreamQuery(ctx->stream);
    if (q == cudaSuccess) return RW_OK;
    if (q != cudaErrorNotReady) return cuda_fail(ctx, q, "cudaStreamQuery");
    ncclResult_t as = ncclSuccess;
    ncclCommGetAsyncError(ctx->comm, &as);
    if (as != ncclSuccess && as != ncclInProgress) {
      ncclCommAbort(ctx->comm);
      ctx->comm = nullptr;
      return fail(ctx, RW_ERR_NCCL, std::string("NCCL async error: ") + ncclGetErrorString(as));
    }
    const double ms = std::chrono::duration<double, std::milli>(
                          std::chrono::steady_clock::now() - t0).count();
    if (ctx->timeout_ms > 0 && ms > (double)ctx->timeout_ms) {
      ncclCommAbort(ctx->comm);
      ctx->comm = nullptr;
      return fail(ctx, RW_ERR_TIMEOUT, "collective wait exceeded the context timeout");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// ---- symmetric region for peer exchanges (world > 1) ----------------------------------

void sym_close(rw_ctx* ctx) {
  for (int r = 0; r < kMaxPeers; r++)
    if (ctx->sym_peer[r]) {
      // in-process ranks see each other's regions as plain device pointers (no handle)
      if (ctx->sym_peer_owned) cudaFree(ctx->sym_peer[r]);
      else if (!ctx->group) cudaIpcCloseMemHandle(ctx->sym_peer[r]);
      ctx->sym_peer[r] = nullptr;
    }
  if (ctx->sym) cudaFree(ctx->sym);
  ctx->sym = nullptr;
  ctx->sym_bytes = 0;
}

// ---- in-process ranks (rw_ctx_create with several GPUs) --------------------------------

// A meeting of the group's ranks (host threads): every rank brings `val` and gets the
// minimum over the ranks, or -1 when the meeting broke (a rank failed, or the wait
// passed the context timeout); a broken group fails every later meeting.
int group_meet(rw_ctx* ctx, int val) {
  RankGroup& g = *ctx->group;
  std::unique_lock<std::mutex> lk(g.mu);
  if (g.broken) return -1;
  const uint64_t my = g.gen;
  g.acc = g.arrived == 0 ? val : std::min(g.acc, val);
  if (++g.arrived == g.n) {
    g.result = g.acc;
    g.arrived = 0;
    g.gen++;
    g.cv.notify_all();
    return g.result;
  }
  auto done = [&] { return g.gen != my || g.broken; };
  if (ctx->timeout_ms > 0) {
    if (!g.cv.wait_for(lk, std::chrono::milliseconds(ctx->timeout_ms), done)) {
      g.broken = true;
      g.cv.notify_all();
      return -1;
    }
  } else {
    g.cv.wait(lk, done);
  }
  return g.gen != my ? g.result : -1;
}

void group_break(rw_ctx* ctx) {
  if (!ctx || !ctx->group) return;
  std::lock_guard<std::mutex> lk(ctx->group->mu);
  ctx->group->broken = true;
  ctx->group->cv.notify_all();
}

// sym_ensure for in-process ranks: the same protocol as below, with the regions
// published as device pointers at a host meeting (peer access is enabled between every
// pair of the group's devices when the context is created).
int sym_ensure_group(rw_ctx* ctx, size_t need) {
  RankGroup& g = *ctx->group;
  if (!g.peer_ok) {  // the same answer on every rank
    ctx->peer_mode = 0;
    return RW_OK;
  }
  if (ctx->peer_mode == 1 && ctx->sym_bytes >= need) return RW_OK;
  int rc = wait_stream(ctx);
  if (rc) return rc;
  // nobody still reads or writes the old regions
  if (group_meet(ctx, 1) < 0)
    return fail(ctx, RW_ERR_TIMEOUT, "a rank of this context did not reach the exchange set-up");
  for (int r = 0; r < kMaxPeers; r++) ctx->sym_peer[r] = nullptr;
  if (ctx->sym) cudaFree(ctx->sym);
  ctx->sym = nullptr;
  ctx->sym_bytes = 0;
  const size_t bytes = round_up(need + need / 4, 2u << 20);
  int ok = 1;
  if (cudaMalloc(reinterpret_cast<void**>(&ctx->sym), bytes) != cudaSuccess ||
      cudaMemsetAsync(ctx->sym, 0, bytes, ctx->stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess) {
    cudaGetLastError();
    if (ctx->sym) cudaFree(ctx->sym);
    ctx->sym = nullptr;
    ok = 0;
  }
  {
    std::lock_guard<std::mutex> lk(g.mu);
    g.sym[ctx->rank] = ctx->sym;
  }
  ok = group_meet(ctx, ok);
  if (ok < 0)
    return fail(ctx, RW_ERR_TIMEOUT, "a rank of this context did not reach the exchange set-up");
  if (!ok) {  // some rank has no region: every rank uses NCCL from now on
    if (ctx->sym) cudaFree(ctx->sym);
    ctx->sym = nullptr;
    ctx->peer_mode = 0;
    return RW_OK;
  }
  {
    std::lock_guard<std::mutex> lk(g.mu);
    for (int r = 0; r < ctx->world; r++)
      if (r != ctx->rank) ctx->sym_peer[r] = g.sym[r];
  }
  // every rank has read every pointer before any rank moves on (the next set-up may
  // republish them)
  if (group_meet(ctx, 1) < 0)
    return fail(ctx, RW_ERR_TIMEOUT, "a rank of this context did not reach the exchange set-up");
  ctx->sym_bytes = bytes;
  ctx->peer_epoch = 0;
  ctx->peer_mode = 1;
  return RW_OK;
}

// Runs fn(i) for every rank of a multi-GPU context, one host thread per rank, and
// reports the first failure that is not a timeout (a timeout on one rank is usually the
// consequence of another rank's failure). With break_on_fail, a failed rank breaks the
// group (its peers stop waiting for it at host meetings).
int run_members(rw_ctx* front, const std::function<int(int)>& fn, bool break_on_fail) {
  const int n = (int)front->members.size();
  std::vector<int> rc(n, RW_OK);
  std::vector<std::thread> th;
  bool spawn_failed = false;
  try {
    for (int i = 0; i < n; i++)
      th.emplace_back([&, i] {
        rc[i] = fn(i);
        if (rc[i] && break_on_fail) group_break(front->members[i]);
      });
  } catch (...) {
    spawn_failed = true;
    if (!front->members.empty()) group_break(front->members[0]);
  }
  for (auto& t : th) t.join();
  if (spawn_failed) return fail(front, RW_ERR_OOM, "could not start a thread per GPU");
  int first = -1;
  for (int i = 0; i < n; i++)
    if (rc[i] && (first < 0 || (rc[first] == RW_ERR_TIMEOUT && rc[i] != RW_ERR_TIMEOUT)))
      first = i;
  if (first < 0) return RW_OK;
  return fail(front, rc[first],
              "rank " + std::to_string(first) + " (GPU " +
                  std::to_string(front->members[first]->device) +
                  "): " + front->members[first]->last_error);
}

}  // namespace

int for_each_rank(rw_ctx* front, const std::function<int(int)>& fn) {
  return run_members(front, fn, false);
}

namespace {

// All ranks call this at the same point with the same size (a collective): makes every
// rank's region at least `need` bytes, zeroed, and maps every peer's region. Decides
// once per context between peer memory and NCCL: NCCL when RW_PEER_EXCHANGE=0 is set
// (the same on every rank) or when any rank cannot map a peer's region.
int sym_ensure(rw_ctx* ctx, size_t need) {
  if (ctx->world < 2 || ctx->peer_mode == 0) return RW_OK;
  if (ctx->peer_failed)
    return fail(ctx, RW_ERR_CUDA, "an earlier peer exchange timed out; recreate the context");
  if (ctx->world > kMaxPeers) {
    ctx->peer_mode = 0;
    return RW_OK;
  }
  if (ctx->peer_mode == -1) {
    const char* env = std::getenv("RW_PEER_EXCHANGE");
    if (env && env[0] == '0') {
      ctx->peer_mode = 0;
      return RW_OK;
    }
  }
  if (ctx->group) return sym_ensure_group(ctx, need);
  if (ctx->peer_mode == 1 && ctx->sym_bytes >= need) return RW_OK;
  int rc = wait_stream(ctx);
  if (rc) return rc;
  DBuf<int> flag;
  RW_CU(ctx, flag.alloc(1));
  auto all_ok = [&](int ok) -> int {  // min over ranks of ok, as a barrier
    RW_CU(ctx, cudaMemcpyAsync(flag.p, &ok, 4, cudaMemcpyHostToDevice, ctx->stream));
    RW_NC(ctx, ncclAllReduce(flag.p, flag.p, 1, ncclInt32, ncclMin, ctx->comm, ctx->stream));
    RW_CU(ctx, cudaMemcpyAsync(&ok, flag.p, 4, cudaMemcpyDeviceToHost, ctx->stream));
    int w = wait_stream(ctx);
    if (w) return -1;
    return ok;
  };
  // every rank unmaps the old regions before any rank frees its own
  for (int r = 0; r < kMaxPeers; r++)
    if (ctx->sym_peer[r]) {
      cudaIpcCloseMemHandle(ctx->sym_peer[r]);
      ctx->sym_peer[r] = nullptr;
    }
  if (all_ok(1) < 0) return RW_ERR_NCCL;
  if (ctx->sym) cudaFree(ctx->sym);
  ctx->sym = nullptr;
  ctx->sym_bytes = 0;
  const size_t bytes = round_up(need + need / 4, 2u << 20);
  int ok = 1;
  cudaIpcMemHandle_t mine = {};
  if (cudaMalloc(reinterpret_cast<void**>(&ctx->sym), bytes) != cudaSuccess ||
      cudaMemsetAsync(ctx->sym, 0, bytes, ctx->stream) != cudaSuccess ||
      cudaStreamSynchronize(ctx->stream) != cudaSuccess ||
      cudaIpcGetMemHandle(&mine, ctx->sym) != cudaSuccess) {
    cudaGetLastError();
    ok = 0;
  }
  // exchange the handles (a zeroed handle from a rank that failed is never opened)
  DBuf<char> hbuf;
  RW_CU(ctx, hbuf.alloc((size_t)ctx->world * sizeof(cudaIpcMemHandle_t)));
  RW_CU(ctx, cudaMemcpyAsync(hbuf.p + (size_t)ctx->rank * sizeof mine, &mine, sizeof mine,
                             cudaMemcpyHostToDevice, ctx->stream));
  RW_NC(ctx, ncclAllGather(hbuf.p + (size_t)ctx->rank * sizeof mine, hbuf.p, sizeof mine, ncclChar,
                           ctx->comm, ctx->stream));
  std::vector<cudaIpcMemHandle_t> all(ctx->world);
  RW_CU(ctx, cudaMemcpyAsync(all.data(), hbuf.p, (size_t)ctx->world * sizeof mine,
                             cudaMemcpyDeviceToHost, ctx->stream));
  rc = wait_stream(ctx);
  if (rc) return rc;
  ok = all_ok(ok);
  if (ok < 0) return RW_ERR_NCCL;
  if (ok)
    for (int r = 0; r < ctx->world && ok; r++) {
      if (r == ctx->rank) continue;
      void* p = nullptr;
      if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        ok = 0;
      } else {
        ctx->sym_peer[r] = static_cast<char*>(p);
      }
    }
  ok = all_ok(ok);
  if (ok < 0) return RW_ERR_NCCL;
  if (!ok) {  // some rank cannot use peer memory: every rank uses NCCL from now on
    sym_close(ctx);
    ctx->peer_mode = 0;
    return RW_OK;
  }
  ctx->sym_bytes = bytes;
  ctx->peer_epoch = 0;
  ctx->peer_mode = 1;
  return RW_OK;
}

PeerSet peer_set(const rw_ctx* ctx) {
  PeerSet ps = {};
  for (int r = 0; r < ctx->world; r++) ps.base[r] = r == ctx->rank ? ctx->sym : ctx->sym_peer[r];
  ps.world = ctx->world;
  ps.rank = ctx->rank;
  const int64_t ms = ctx->timeout_ms > 0 ? std::min<int64_t>(ctx->timeout_ms, 10000) : 10000;
  ps.timeout_ns = (uint64_t)ms * 1000000ull;
  return ps;
}

// Phase timing with consecutive CUDA events on the context stream.
struct PhaseTimer {
  bool on = false;
  cudaStream_t s = nullptr;
  std::vector<cudaEvent_t> ev;
  std::vector<int> cat;  // category of the interval ending at ev[i] (i >= 1)
  std::vector<int> hist_idx;
  size_t used = 0;
  int init(bool enable, cudaStream_t stream, size_t cap) {
    on = enable;
    s = stream;
    if (!on) return 0;
    ev.resize(cap);
    cat.assign(cap, -1);
    for (auto& e : ev)
      if (cudaEventCreate(&e) != cudaSuccess) return -1;
    return 0;
  }
  void mark(int category) {
    if (!on || used >= ev.size()) return;
    cat[used] = category;
    cudaEventRecord(ev[used], s);
    if (category == RW_CAT_BUILD_HIST) hist_idx.push_back((int)used);
    used++;
  }
  ~PhaseTimer() {
    for (auto& e : ev) cudaEventDestroy(e);
  }
};

int check_params(rw_ctx* ctx, const rw_train_params* p, uint32_t n_bins) {
  if (!p) return fail(ctx, RW_ERR_ARG, "params is NULL");
  if (p->depth < 1 || p->depth > 12) return fail(ctx, RW_ERR_ARG, "depth must be in 1..=12");
  if (p->n_bins < 2 || p->n_bins > 256) return fail(ctx, RW_ERR_ARG, "n_bins must be in 2..=256");
  if (p->n_bins != n_bins)
    return fail(ctx, RW_ERR_ARG, "params n_bins differs from the dataset's n_bins");
  if (p->objective != RW_OBJ_LOGISTIC && p->objective != RW_OBJ_L2)
    return fail(ctx, RW_ERR_ARG, "unknown objective");
  if (p->clamp_hessian != 0.0f)
    return fail(ctx, RW_ERR_UNSUPPORTED, "clamp_hessian is not supported");
  return RW_OK;
}

}  // namespace

// =================================================================================
// contexts

static void destroy_members(std::vector<rw_ctx*>& m);

extern "C" int rw_ctx_create(const int* gpu_ids, int n_gpus, rw_ctx** out) {
  if (!out) return fail(nullptr, RW_ERR_ARG, "out is NULL");
  *out = nullptr;
  if (n_gpus < 1 || n_gpus > kMaxPeers)
    return fail(nullptr, RW_ERR_ARG, "n_gpus must be in 1..=8");
  if (n_gpus == 1) return rw_ctx_create_rank(gpu_ids ? gpu_ids[0] : 0, 0, 1, nullptr, out);
  if (!gpu_ids) return fail(nullptr, RW_ERR_ARG, "gpu_ids is NULL");
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
  for (int i = 0; i < n_gpus; i++) {
    if (gpu_ids[i] < 0 || gpu_ids[i] >= ndev) return fail(nullptr, RW_ERR_ARG, "gpu id out of range");
    // two ranks on one GPU would wait on each other inside concurrent kernels
    for (int j = 0; j < i; j++)
      if (gpu_ids[j] == gpu_ids[i]) return fail(nullptr, RW_ERR_ARG, "gpu_ids repeat a GPU");
  }
  // One rank per GPU, in this process: NCCL communicators initialised together, one
  // thread per rank.
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess)
    return fail(nullptr, RW_ERR_NCCL, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
  std::vector<rw_ctx*> m(n_gpus, nullptr);
  std::vector<int> rc(n_gpus, RW_OK);
  std::vector<std::string> err(n_gpus);
  {
    std::vector<std::thread> th;
    try {
      for (int i = 0; i < n_gpus; i++)
        th.emplace_back([&, i] {
          rc[i] = rw_ctx_create_rank(gpu_ids[i], i, n_gpus, &id, &m[i]);
          if (rc[i]) err[i] = g_tls_error;
        });
    } catch (...) {
      for (auto& t : th) t.join();
      destroy_members(m);
      return fail(nullptr, RW_ERR_OOM, "could not start a thread per GPU");
    }
    for (auto& t : th) t.join();
  }
  for (int i = 0; i < n_gpus; i++)
    if (rc[i]) {
      destroy_members(m);
      return fail(nullptr, rc[i], "GPU " + std::to_string(gpu_ids[i]) + ": " + err[i]);
    }
  auto grp = std::make_shared<RankGroup>();
  grp->n = n_gpus;
  grp->sym.assign(n_gpus, nullptr);
  // peer access between every pair of the group's devices (kept for the process)
  bool peer_ok = true;
  for (int i = 0; i < n_gpus && peer_ok; i++) {
    cudaSetDevice(gpu_ids[i]);
    for (int j = 0; j < n_gpus && peer_ok; j++) {
      if (i == j) continue;
      int can = 0;
      if (cudaDeviceCanAccessPeer(&can, gpu_ids[i], gpu_ids[j]) != cudaSuccess || !can) {
        peer_ok = false;
        break;
      }
      cudaError_t pe = cudaDeviceEnablePeerAccess(gpu_ids[j], 0);
      if (pe == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
      else if (pe != cudaSuccess) {
        cudaGetLastError();
        peer_ok = false;
      }
    }
  }
  grp->peer_ok = peer_ok;
  auto* front = new rw_ctx();
  front->device = gpu_ids[0];
  front->rank = 0;
  front->world = n_gpus;
  front->members = m;
  for (auto* c : m) c->group = grp;
  *out = front;
  return RW_OK;
}

extern "C" int rw_nccl_unique_id(void* out128) {
  if (!out128) return fail(nullptr, RW_ERR_ARG, "out is NULL");
  ncclUniqueId id;
  ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess)
    return fail(nullptr, RW_ERR_NCCL, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
  static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
  memcpy(out128, &id, sizeof id);
  return RW_OK;
}

extern "C" int rw_ctx_create_rank(int gpu_id, int rank, int world, const void* nccl_id,
                                  rw_ctx** out) {
  if (!out) return fail(nullptr, RW_ERR_ARG, "out is NULL");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world) return fail(nullptr, RW_ERR_ARG, "bad rank/world");
  if (world > 1 && !nccl_id) return fail(nullptr, RW_ERR_ARG, "nccl_id required for world > 1");
  int ndev = 0;
  cudaError_t e = cudaGetDeviceCount(&ndev);
  if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaGetDeviceCount");
  if (gpu_id < 0 || gpu_id >= ndev) return fail(nullptr, RW_ERR_ARG, "gpu id out of range");
  rw_ctx* ctx = new rw_ctx();
  ctx->device = gpu_id;
  ctx->rank = rank;
  ctx->world = world;
  e = cudaSetDevice(gpu_id);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = gpu_id;
    e = cudaMemPoolCreate(&ctx->pool, &props);
    uint64_t keep = UINT64_MAX;
    if (e == cudaSuccess)
      e = cudaMemPoolSetAttribute(ctx->pool, cudaMemPoolAttrReleaseThreshold, &keep);
  }
  if (e != cudaSuccess) {
    int rc = cuda_fail(nullptr, e, "context setup");
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    if (ctx->pool) cudaMemPoolDestroy(ctx->pool);
    delete ctx;
    return rc;
  }
  if (world > 1) {
    ncclUniqueId id;
    memcpy(&id, nccl_id, sizeof id);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&ctx->comm, world, id, rank, &cfg);
    const auto t0 = std::chrono::steady_clock::now();
    while (r == ncclInProgress || r == ncclSuccess) {
      ncclResult_t st = ncclInProgress;
      ncclCommGetAsyncError(ctx->comm, &st);
      if (st == ncclSuccess) {
        r = ncclSuccess;
        break;
      }
      if (st != ncclInProgress) {
        r = st;
        break;
      }
      const double ms = std::chrono::duration<double, std::milli>(
                            std::chrono::steady_clock::now() - t0).count();
      if (ms > (double)ctx->timeout_ms) {
        r = ncclInternalError;
        break;
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    if (r != ncclSuccess) {
      if (ctx->comm) ncclCommAbort(ctx->comm);
      cudaStreamDestroy(ctx->stream);
      cudaMemPoolDestroy(ctx->pool);
      delete ctx;
      return fail(nullptr, RW_ERR_NCCL,
                  std::string("NCCL communicator init failed: ") + ncclGetErrorString(r));
    }
  }
  *out = ctx;
  return RW_OK;
}

// Destroys in-process ranks, one thread each (communicator teardown may involve every
// rank of the communicator).
static void destroy_members(std::vector<rw_ctx*>& m) {
  std::vector<std::thread> th;
  for (auto*& c : m)
    if (c) {
      try {
        th.emplace_back([c] { rw_ctx_destroy(c); });
      } catch (...) {
        rw_ctx_destroy(c);
      }
      c = nullptr;
    }
  for (auto& t : th) t.join();
}

extern "C" void rw_ctx_destroy(rw_ctx* ctx) {
  if (!ctx) return;
  if (!ctx->members.empty()) {
    destroy_members(ctx->members);
    delete ctx;
    return;
  }
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  // In-process ranks have no kernel in flight here (every call waits for all of its
  // ranks' streams before it returns), so they skip the freeing barrier.
  if (ctx->sym && ctx->comm && !ctx->peer_failed && !ctx->group) {
    // no rank frees its region while another may still store into it (bounded wait)
    int* one = nullptr;
    if (cudaMalloc(reinterpret_cast<void**>(&one), 4) == cudaSuccess) {
      if (nccl_settle(ctx, ncclAllReduce(one, one, 1, ncclInt32, ncclSum, ctx->comm,
                                         ctx->stream)) == ncclSuccess)
        wait_stream(ctx);
      cudaFree(one);
    }
  }
  sym_close(ctx);
  for (int i = 0; i < 2 * rw_ctx::kStageWorkers; i++) {
    if (ctx->stage_ev[i]) cudaEventDestroy(ctx->stage_ev[i]);
    if (ctx->stage_host[i]) cudaFreeHost(ctx->stage_host[i]);
  }
  for (int w = 0; w < rw_ctx::kStageWorkers; w++)
    if (ctx->stage_stream[w]) cudaStreamDestroy(ctx->stage_stream[w]);
  if (ctx->comm) ncclCommDestroy(ctx->comm);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  if (ctx->pool) cudaMemPoolDestroy(ctx->pool);
  delete ctx;
}

extern "C" int rw_ctx_peer_failed(const rw_ctx* ctx) {
  if (!ctx) return 0;
  for (auto* c : ctx->members)
    if (c->peer_failed) return 1;
  return ctx->peer_failed ? 1 : 0;
}

extern "C" const char* rw_last_error(const rw_ctx* ctx) {
  return ctx ? ctx->last_error.c_str() : g_tls_error.c_str();
}

extern "C" void* rw_ctx_stream(const rw_ctx* ctx) {
  if (ctx && !ctx->members.empty()) return (void*)ctx->members[0]->stream;
  return ctx ? (void*)ctx->stream : nullptr;
}

extern "C" int rw_ctx_set_timeout(rw_ctx* ctx, int64_t ms) {
  if (!ctx || ms < 0) return fail(ctx, RW_ERR_ARG, "bad timeout");
  ctx->timeout_ms = ms;
  for (auto* c : ctx->members) c->timeout_ms = ms;
  return RW_OK;
}

// =================================================================================
// host-to-device uploads

constexpr size_t kStageSlot = 8u << 20;       // bytes per pinned slot
constexpr size_t kStageMin = 32u << 20;       // smaller pageable copies go to the driver

// Copies `bytes` of host memory at src to the device at dst, ordered on the context
// stream like cudaMemcpyAsync, and like it from pageable memory: src has been read when
// the call returns. Pinned or registered sources (and copies under kStageMin) go straight
// to the copy engine. A large pageable source is split into kStageSlot chunks dealt
// round-robin to kStageWorkers host threads; each worker copies its chunk into one of its
// two pinned slots (after the slot's previous transfer has drained) and queues the
// transfer on its own stream, so host copies by several cores overlap the copy engine.
// The destination's allocation is ordered before the workers' transfers, and the context
// stream waits for all of them.
static cudaError_t upload_h2d(rw_ctx* ctx, void* dst, const void* src, size_t bytes) {
  cudaPointerAttributes at;
  bool pageable = true;
  if (cudaPointerGetAttributes(&at, src) == cudaSuccess) pageable = at.type == cudaMemoryTypeUnregistered;
  else cudaGetLastError();  // clear: plain host pointers are pageable
  if (!pageable || bytes < kStageMin)
    return cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, ctx->stream);
  constexpr int W = rw_ctx::kStageWorkers;
  cudaError_t e = cudaSuccess;
  for (int w = 0; w < W && e == cudaSuccess; w++)
    if (!ctx->stage_stream[w]) e = cudaStreamCreateWithFlags(&ctx->stage_stream[w], cudaStreamNonBlocking);
  for (int i = 0; i < 2 * W && e == cudaSuccess; i++) {
    if (!ctx->stage_host[i]) e = cudaMallocHost(&ctx->stage_host[i], kStageSlot);
    if (e == cudaSuccess && !ctx->stage_ev[i])
      e = cudaEventCreateWithFlags(&ctx->stage_ev[i], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) return e;
  // the destination (a stream-ordered allocation) before any worker transfer
  cudaEvent_t ready = nullptr;
  e = cudaEventCreateWithFlags(&ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventRecord(ready, ctx->stream);
  for (int w = 0; w < W && e == cudaSuccess; w++)
    e = cudaStreamWaitEvent(ctx->stage_stream[w], ready, 0);
  if (e != cudaSuccess) {
    if (ready) cudaEventDestroy(ready);
    return e;
  }
  const size_t chunks = (bytes + kStageSlot - 1) / kStageSlot;
  cudaError_t err[W];
  int last_slot[W];
  auto work = [&](int w) {
    cudaError_t r = cudaSetDevice(ctx->device);
    last_slot[w] = -1;
    int j = 0;
    for (size_t k = (size_t)w; k < chunks && r == cudaSuccess; k += W, j ^= 1) {
      const int slot = 2 * w + j;
      const size_t off = k * kStageSlot, len = std::min(kStageSlot, bytes - off);
      if (ctx->stage_used[slot]) r = cudaEventSynchronize(ctx->stage_ev[slot]);
      if (r != cudaSuccess) break;
      memcpy(ctx->stage_host[slot], static_cast<const char*>(src) + off, len);
      r = cudaMemcpyAsync(static_cast<char*>(dst) + off, ctx->stage_host[slot], len,
                          cudaMemcpyHostToDevice, ctx->stage_stream[w]);
      if (r == cudaSuccess) r = cudaEventRecord(ctx->stage_ev[slot], ctx->stage_stream[w]);
      if (r == cudaSuccess) {
        ctx->stage_used[slot] = true;
        last_slot[w] = slot;
      }
    }
    err[w] = r;
  };
  std::vector<std::thread> th;
  for (int w = 1; w < W; w++) th.emplace_back(work, w);
  work(0);
  for (auto& t : th) t.join();
  cudaSetDevice(ctx->device);
  cudaEventDestroy(ready);
  for (int w = 0; w < W; w++)
    if (err[w] != cudaSuccess) {
      // transfers already queued must not outlive the caller's error path (which frees
      // the destination on the context stream)
      for (int v = 0; v < W; v++) cudaStreamSynchronize(ctx->stage_stream[v]);
      return err[w];
    }
  // the context stream waits for every worker's last transfer (a stream's last event
  // follows all its earlier work)
  for (int w = 0; w < W && e == cudaSuccess; w++)
    if (last_slot[w] >= 0) e = cudaStreamWaitEvent(ctx->stream, ctx->stage_ev[last_slot[w]], 0);
  return e;
}

// =================================================================================
// categorical target encoding (encode.cu)

static rw_ctx* first_rank(rw_ctx* ctx);

extern "C" int rw_target_encode_device(rw_ctx* ctx, float* d_x, const float* d_y, uint64_t n,
                                       uint32_t nf, const uint32_t* categorical, uint32_t n_cat,
                                       float smoothing, uint32_t k_folds, uint64_t hash_buckets,
                                       float* gmean_out, rw_encoders** enc_out) {
  if (!ctx) return fail(nullptr, RW_ERR_ARG, "context is NULL");
  rw_ctx* c = first_rank(ctx);
  if (!d_x || !d_y || (n_cat && !categorical) || n == 0 || nf == 0)
    return fail(ctx, RW_ERR_ARG, "bad target-encoding arguments");
  if (enc_out) *enc_out = nullptr;
  RW_CU(c, cudaSetDevice(c->device));
  auto* enc = enc_out ? new rw_encoders() : nullptr;
  std::string why;
  const int rc = target_encode_device(c, d_x, d_y, n, nf, categorical, n_cat, smoothing, k_folds,
                                      hash_buckets, gmean_out, enc, &why);
  if (rc) {
    delete enc;
    return fail(ctx, rc, why);
  }
  if (enc_out) *enc_out = enc;
  return RW_OK;
}

extern "C" int rw_target_encode(rw_ctx* ctx, float* x, const float* y, uint64_t n, uint32_t nf,
                                const uint32_t* categorical, uint32_t n_cat, float smoothing,
                                uint32_t k_folds, uint64_t hash_buckets, float* gmean_out,
                                rw_encoders** enc_out) {
  if (!ctx) return fail(nullptr, RW_ERR_ARG, "context is NULL");
  if (!x || !y || n == 0 || nf == 0) return fail(ctx, RW_ERR_ARG, "bad target-encoding arguments");
  rw_ctx* c = first_rank(ctx);
  RW_CU(c, cudaSetDevice(c->device));
  DBuf<float> dx, dy;
  RW_CU(c, dx.alloc((size_t)n * nf));
  RW_CU(c, dy.alloc(n));
  RW_CU(c, upload_h2d(c, dx.p, x, (size_t)n * nf * 4));
  RW_CU(c, cudaMemcpyAsync(dy.p, y, n * 4, cudaMemcpyHostToDevice, c->stream));
  int rc = rw_target_encode_device(ctx, dx.p, dy.p, n, nf, categorical, n_cat, smoothing,
                                   k_folds, hash_buckets, gmean_out, enc_out);
  if (rc) return rc;
  RW_CU(c, cudaMemcpyAsync(x, dx.p, (size_t)n * nf * 4, cudaMemcpyDeviceToHost, c->stream));
  RW_CU(c, cudaStreamSynchronize(c->stream));
  return RW_OK;
}

extern "C" int rw_encoders_table(const rw_encoders* enc, uint32_t i, int64_t* key_lo,
                                 uint64_t* n_keys, const float** value, const uint8_t** present) {
  if (!enc || i >= enc->key_lo.size()) return RW_ERR_ARG;
  if (key_lo) *key_lo = enc->key_lo[i];
  if (n_keys) *n_keys = enc->n_keys[i];
  if (value) *value = enc->value.data() + enc->koff[i];
  if (present) *present = enc->present.data() + enc->koff[i];
  return RW_OK;
}

extern "C" void rw_encoders_free(rw_encoders* enc) { delete enc; }

extern "C" int rw_encoders_create(uint32_t n_cat, const int64_t* key_lo, const uint64_t* n_keys,
                                  const float* value, const uint8_t* present, float gmean,
                                  rw_encoders** out) {
  if (!out || (n_cat && (!key_lo || !n_keys))) return RW_ERR_ARG;
  *out = nullptr;
  auto* enc = new rw_encoders();
  uint64_t slots = 0;
  for (uint32_t j = 0; j < n_cat; j++) {
    enc->key_lo.push_back(key_lo[j]);
    enc->koff.push_back(slots);
    enc->n_keys.push_back(n_keys[j]);
    slots += n_keys[j];
  }
  if (slots && (!value || !present)) {
    delete enc;
    return RW_ERR_ARG;
  }
  enc->value.assign(value, value + slots);
  enc->present.assign(present, present + slots);
  enc->gmean = gmean;
  *out = enc;
  return RW_OK;
}

extern "C" int rw_target_transform(rw_ctx* ctx, float* x, uint64_t n, uint32_t nf,
                                   const uint32_t* categorical, uint32_t n_cat,
                                   const rw_encoders* enc, uint64_t hash_buckets) {
  if (!ctx) return fail(nullptr, RW_ERR_ARG, "context is NULL");
  if (!x || !enc || (n_cat && !categorical)) return fail(ctx, RW_ERR_ARG, "bad transform arguments");
  if (n == 0 || n_cat == 0) return RW_OK;
  rw_ctx* c = first_rank(ctx);
  RW_CU(c, cudaSetDevice(c->device));
  DBuf<float> dx;
  RW_CU(c, dx.alloc((size_t)n * nf));
  RW_CU(c, upload_h2d(c, dx.p, x, (size_t)n * nf * 4));
  std::string why;
  const int rc = target_transform_device(c, dx.p, n, nf, categorical, n_cat, *enc, hash_buckets,
                                         &why);
  if (rc) return fail(ctx, rc, why);
  RW_CU(c, cudaMemcpyAsync(x, dx.p, (size_t)n * nf * 4, cudaMemcpyDeviceToHost, c->stream));
  RW_CU(c, cudaStreamSynchronize(c->stream));
  return RW_OK;
}

// =================================================================================
// datasets

static int dataset_build(rw_ctx* ctx, const float* d_x, const float* y, bool y_on_device,
                         uint64_t n, uint32_t nf, const float* cuts, uint32_t n_bins,
                         int32_t pack4, uint64_t n_global, uint64_t row_offset,
                         rw_dataset** out) {
  int nl = 0;
  auto* ds = new rw_dataset();
  ds->ctx = ctx;
  ds->n = n;
  ds->n_pad = round_up(n, kRowAlign);
  ds->n_global = n_global;
  ds->row_offset = row_offset;
  ds->nf = nf;
  ds->n_bins = n_bins;
  ds->packed = (pack4 && n_bins <= 16) ? 1 : 0;
  ds->ftiles = (nf + kHistFeat - 1) / kHistFeat;
  const uint32_t rb_u8 = ds->ftiles * kHistFeat;  // u8 row-bin bytes per row (all tiles)
  ds->cuts.assign(cuts, cuts + (size_t)nf * (n_bins - 1));
  cudaStream_t s = ctx->stream;
  const size_t col_bytes = (size_t)nf * ds->n_pad, row_u8_bytes = (size_t)rb_u8 * ds->n_pad;
  DBuf<uint8_t> colb, rowb;
  DBuf<float> dy, dc;
  cudaError_t e = colb.alloc(ctx, col_bytes);
  if (e == cudaSuccess) e = rowb.alloc(ctx, row_u8_bytes);
  if (e == cudaSuccess) e = dy.alloc(ctx, ds->n_pad);
  if (e == cudaSuccess) e = dc.alloc(ctx, ds->cuts.size());
  if (e == cudaSuccess) e = cudaMemsetAsync(colb.p, 0, col_bytes, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(dy.p, 0, ds->n_pad * sizeof(float), s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dc.p, ds->cuts.data(), ds->cuts.size() * sizeof(float),
                        cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(dy.p, y, n * sizeof(float),
                        y_on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess)
    e = launch_bin(d_x, n, nf, dc.p, n_bins, ds->n_pad, colb.p, rowb.p, s, &nl);
  if (e == cudaSuccess && ds->packed) {
    DBuf<uint8_t> packed;
    e = packed.alloc(ctx, (size_t)(rb_u8 / 2) * ds->n_pad);
    if (e == cudaSuccess) e = launch_pack4(rowb.p, ds->n_pad, nf, packed.p, s, &nl);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);  // before the u8 rows are freed
    if (e == cudaSuccess) ds->d_rowbins = packed.release();
  } else if (e == cudaSuccess) {
    ds->d_rowbins = rowb.release();
  }
  if (e == cudaSuccess) ds->d_colbins = colb.release();
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  ctx->launches += nl;
  if (e != cudaSuccess) {
    int rc = cuda_fail(ctx, e, "dataset upload/binning");
    pool_free(ctx, ds->d_colbins);
    pool_free(ctx, ds->d_rowbins);
    delete ds;
    return rc;
  }
  ds->d_y = dy.release();
  ds->d_cuts = dc.release();
  *out = ds;
  return RW_OK;
}

static int dataset_args_ok(rw_ctx* ctx, const void* x, const void* y, uint64_t n, uint32_t nf,
                           const float* cuts, uint32_t n_bins, uint64_t n_global,
                           uint64_t row_offset, rw_dataset** out) {
  if (!ctx) return fail(nullptr, RW_ERR_ARG, "ctx is NULL");
  if (!out || !x || !y || !cuts) return fail(ctx, RW_ERR_ARG, "NULL buffer");
  if (n == 0 || nf == 0) return fail(ctx, RW_ERR_ARG, "empty dataset");
  if (n_bins < 2 || n_bins > 256) return fail(ctx, RW_ERR_ARG, "n_bins must be in 2..=256");
  if (n_global < n || row_offset + n > n_global)
    return fail(ctx, RW_ERR_ARG, "shard rows exceed n_global");
  if (n_global > 0xffffffffull) return fail(ctx, RW_ERR_ARG, "more than 2^32 rows");
  return RW_OK;
}

// A dataset of a multi-GPU context: the rows split into contiguous shards, one per rank,
// each uploaded and binned by its rank's thread on its own GPU (row ids stay global, so
// hashes and the subsample stride see the same rows as on one GPU).
static int group_dataset_create(rw_ctx* front, const float* x, const float* y, bool on_device,
                                uint64_t n, uint32_t nf, const float* cuts, uint32_t n_bins,
                                int32_t pack4, uint64_t n_global, uint64_t row_offset,
                                rw_dataset** out) {
  const int W = (int)front->members.size();
  if (n_global != n || row_offset != 0)
    return fail(front, RW_ERR_ARG,
                "a multi-GPU context takes the whole dataset (n_global = n, row_offset = 0)");
  if (n < (uint64_t)W) return fail(front, RW_ERR_ARG, "fewer rows than GPUs");
  int src_dev = -1;
  if (on_device) {
    cudaPointerAttributes ax, ay;
    if (cudaPointerGetAttributes(&ax, x) != cudaSuccess ||
        cudaPointerGetAttributes(&ay, y) != cudaSuccess || ax.type != cudaMemoryTypeDevice ||
        ay.type != cudaMemoryTypeDevice || ax.device != ay.device) {
      cudaGetLastError();
      return fail(front, RW_ERR_ARG, "x and y must be device memory of one GPU");
    }
    src_dev = ax.device;
  }
  auto* gd = new rw_dataset();
  gd->ctx = front;
  gd->n = gd->n_pad = gd->n_global = n;
  gd->nf = nf;
  gd->n_bins = n_bins;
  gd->packed = (pack4 && n_bins <= 16) ? 1 : 0;
  gd->ftiles = (nf + kHistFeat - 1) / kHistFeat;
  gd->cuts.assign(cuts, cuts + (size_t)nf * (n_bins - 1));
  gd->shards.assign(W, nullptr);
  gd->shard_lo.resize(W + 1);
  for (int i = 0; i <= W; i++) gd->shard_lo[i] = n * (uint64_t)i / (uint64_t)W;
  int rc = run_members(
      front,
      [&](int i) -> int {
        rw_ctx* c = front->members[i];
        const uint64_t lo = gd->shard_lo[i], rows = gd->shard_lo[i + 1] - lo;
        if (!on_device)
          return rw_dataset_create(c, x + lo * nf, y + lo, rows, nf, cuts, n_bins, pack4, n, lo,
                                   &gd->shards[i]);
        // this rank's slice comes to its own GPU first (peer copy), then it is binned there
        RW_CU(c, cudaSetDevice(c->device));
        DBuf<float> lx, ly;
        RW_CU(c, lx.alloc(c, (size_t)rows * nf));
        RW_CU(c, ly.alloc(c, (size_t)rows));
        RW_CU(c, cudaMemcpyPeerAsync(lx.p, c->device, x + lo * nf, src_dev,
                                     (size_t)rows * nf * sizeof(float), c->stream));
        RW_CU(c, cudaMemcpyPeerAsync(ly.p, c->device, y + lo, src_dev, (size_t)rows * sizeof(float),
                                     c->stream));
        return rw_dataset_create_device(c, lx.p, ly.p, rows, nf, cuts, n_bins, pack4, n, lo,
                                        &gd->shards[i]);
      },
      false);
  if (rc) {
    for (auto* sd : gd->shards) rw_dataset_destroy(sd);
    delete gd;
    return rc;
  }
  *out = gd;
  return RW_OK;
}

extern "C" int rw_dataset_create(rw_ctx* ctx, const float* x, const float* y, uint64_t n,
                                 uint32_t nf, const float* cuts, uint32_t n_bins, int32_t pack4,
                                 uint64_t n_global, uint64_t row_offset, rw_dataset** out) {
  int rc = dataset_args_ok(ctx, x, y, n, nf, cuts, n_bins, n_global, row_offset, out);
  if (rc) return rc;
  *out = nullptr;
  if (!ctx->members.empty())
    return group_dataset_create(ctx, x, y, false, n, nf, cuts, n_bins, pack4, n_global,
                                row_offset, out);
  RW_CU(ctx, cudaSetDevice(ctx->device));
  DBuf<float> dx;
  RW_CU(ctx, dx.alloc(ctx, (size_t)n * nf));
  RW_CU(ctx, upload_h2d(ctx, dx.p, x, (size_t)n * nf * sizeof(float)));
  return dataset_build(ctx, dx.p, y, false, n, nf, cuts, n_bins, pack4, n_global, row_offset,
                       out);
}

extern "C" int rw_dataset_create_device(rw_ctx* ctx, const float* d_x, const float* d_y,
                                        uint64_t n, uint32_t nf, const float* cuts,
                                        uint32_t n_bins, int32_t pack4, uint64_t n_global,
                                        uint64_t row_offset, rw_dataset** out) {
  int rc = dataset_args_ok(ctx, d_x, d_y, n, nf, cuts, n_bins, n_global, row_offset, out);
  if (rc) return rc;
  *out = nullptr;
  if (!ctx->members.empty())
    return group_dataset_create(ctx, d_x, d_y, true, n, nf, cuts, n_bins, pack4, n_global,
                                row_offset, out);
  RW_CU(ctx, cudaSetDevice(ctx->device));
  return dataset_build(ctx, d_x, d_y, true, n, nf, cuts, n_bins, pack4, n_global, row_offset,
                       out);
}

extern "C" void rw_dataset_destroy(rw_dataset* ds) {
  if (!ds) return;
  if (!ds->shards.empty()) {
    for (auto* sd : ds->shards) rw_dataset_destroy(sd);
    delete ds;
    return;
  }
  cudaSetDevice(ds->ctx->device);
  rw_ctx* ctx = ds->ctx;
  pool_free(ctx, ds->d_colbins);
  pool_free(ctx, ds->d_rowbins);
  pool_free(ctx, ds->d_y);
  pool_free(ctx, ds->d_cuts);
  for (auto& kv : ds->ws) pool_free(ctx, kv.second.first);
  delete ds;
}

extern "C" int rw_dataset_bins(const rw_dataset* ds, uint8_t* out) {
  if (!ds || !out) return fail(nullptr, RW_ERR_ARG, "NULL argument");
  if (!ds->shards.empty()) {
    // shard i holds columns [lo_i, lo_{i+1}) of every feature row of the [nf][n] matrix
    for (size_t i = 0; i < ds->shards.size(); i++) {
      const rw_dataset* sd = ds->shards[i];
      rw_ctx* c = sd->ctx;
      RW_CU(c, cudaSetDevice(c->device));
      RW_CU(c, cudaMemcpy2DAsync(out + ds->shard_lo[i], ds->n, sd->d_colbins, sd->n_pad, sd->n,
                                 sd->nf, cudaMemcpyDeviceToHost, c->stream));
      RW_CU(c, cudaStreamSynchronize(c->stream));
    }
    return RW_OK;
  }
  rw_ctx* ctx = ds->ctx;
  RW_CU(ctx, cudaSetDevice(ctx->device));
  RW_CU(ctx, cudaMemcpy2DAsync(out, ds->n, ds->d_colbins, ds->n_pad, ds->n, ds->nf,
                               cudaMemcpyDeviceToHost, ctx->stream));
  RW_CU(ctx, cudaStreamSynchronize(ctx->stream));
  return RW_OK;
}

// =================================================================================
// training loop

static int group_fit(rw_dataset* gd, const rw_train_params* p, float base_score, uint32_t* feat,
                     float* thr, uint16_t* thr_bin, float* leafval, float* leafvar,
                     float* fi_gain, float* fi_count, rw_profile* prof);

extern "C" int rw_fit_dataset(rw_dataset* ds, const rw_train_params* p, float base_score,
                              uint32_t* feat, float* thr, uint16_t* thr_bin, float* leafval,
                              float* leafvar, float* fi_gain, float* fi_count, rw_profile* prof) {
  if (!ds) return fail(nullptr, RW_ERR_ARG, "dataset is NULL");
  if (!ds->shards.empty())
    return group_fit(ds, p, base_score, feat, thr, thr_bin, leafval, leafvar, fi_gain, fi_count,
                     prof);
  rw_ctx* ctx = ds->ctx;
  int rc = check_params(ctx, p, ds->n_bins);
  if (rc) return rc;
  if (p->n_trees > 0 && (!feat || !thr || !leafval))
    return fail(ctx, RW_ERR_ARG, "NULL model output");
  if (!fi_gain || !fi_count) return fail(ctx, RW_ERR_ARG, "NULL feature-importance output");
  RW_CU(ctx, cudaSetDevice(ctx->device));
  cudaStream_t s = ctx->stream;

  const uint32_t T = p->n_trees, D = p->depth, NL = 1u << D, nf = ds->nf, nb = ds->n_bins;
  const uint64_t n = ds->n, n_pad = ds->n_pad;
  // PGBM (gpu_kernels.rs:1015-1080): with a leafvar output the last level also sums g^2
  // per leaf (a third row of the leaf sums) and the leaf pass writes the variances
  const bool want_var = leafvar != nullptr;
  const uint32_t LS = (want_var ? 3u : 2u) * NL;  // leaf-sum words
  const bool subtract = p->subtract != 0;
  const bool logistic = p->objective == RW_OBJ_LOGISTIC;
  const bool goss = p->goss_top > 0.0f;
  uint64_t stride = 1;
  if (!goss && p->subsample < 0.999f) {
    double sd = std::round(1.0 / (double)p->subsample);
    if (sd < 1.0) sd = 1.0;
    stride = sd >= 1.8446744073709552e19 ? UINT64_MAX : (uint64_t)sd;
  }

  // int64 words per histogram node: [tile][bin][g|h][kHistFeat columns]
  const uint64_t cell = (uint64_t)ds->ftiles * nb * 2 * kHistFeat;
  const uint64_t hb_groups = subtract ? std::max<uint64_t>(1, D >= 2 ? (1ull << (D - 2)) : 1)
                                      : (1ull << (D - 1));
  const uint64_t hf_nodes = 1ull << (D - 1);

  // Working buffers live in the dataset's cache: repeated fits allocate nothing.
  WsBuf<float> pred, g, h, d_leafval, d_thr, d_fi_gain, d_fi_count;
  WsBuf<uint16_t> node, d_thr_bin;
  WsBuf<int2> q;
  WsBuf<uint32_t> rl_counts;  // [ncount: 2][NL], [cursor: 2][NL] (alternating levels)
  WsBuf<int4> rl_entries;
  WsBuf<uint8_t> rl_built, rl_choice;
  WsBuf<long long> hb0, hb1, hf0, hf1;
  WsBuf<uint32_t> d_feat, maxbits;
  WsBuf<SplitRec> rec;
  WsBuf<long long> leafsum;  // [2 or 3][NL] per-leaf wide-fixed-point sums of g, h (, g^2)
  WsBuf<double> term;
  WsBuf<long long> mono_sums;
  WsBuf<int32_t> d_mono;
  WsBuf<unsigned long long> goss_counts;
  WsBuf<uint32_t> goss_sel;
  RW_CU(ctx, pred.get(ds, "pred", n_pad));
  RW_CU(ctx, g.get(ds, "g", n_pad));
  RW_CU(ctx, h.get(ds, "h", n_pad));
  RW_CU(ctx, node.get(ds, "node", n_pad));
  RW_CU(ctx, q.get(ds, "q", n_pad));
  RW_CU(ctx, rl_entries.get(ds, "rl_entries", n_pad));
  RW_CU(ctx, rl_counts.get(ds, "rl_counts", 4 * (size_t)NL));
  RW_CU(ctx, rl_built.get(ds, "rl_built", (size_t)NL / 2));
  RW_CU(ctx, rl_choice.get(ds, "rl_choice", (size_t)nf * NL / 2));
  uint32_t* const ncount[2] = {rl_counts.p, rl_counts.p + NL};
  uint32_t* const cursor[2] = {rl_counts.p + 2 * (size_t)NL, rl_counts.p + 3 * (size_t)NL};
  // Built histograms (alternating levels). With several ranks exchanging over peer
  // memory they, and their all-rank sum, live in the symmetric region instead.
  const uint64_t hb_bytes = round_up(hb_groups * cell * 8, 256);
  // receive area of the peer all-reduce: 2 parities x W copies of a 1/W slice
  const uint64_t recv_bytes =
      ctx->world > 1 ? round_up(peer_recv_bytes(ctx->world, hb_groups * cell), 256) : 0;
  if (ctx->world > 1) {
    rc = sym_ensure(ctx, kPeerDataOff + 3 * hb_bytes + recv_bytes);
    if (rc) return rc;
  }
  const bool peer = ctx->world > 1 && ctx->peer_mode == 1;
  const PeerSet ps = peer ? peer_set(ctx) : PeerSet{};
  const uint64_t off_hb[2] = {kPeerDataOff, kPeerDataOff + hb_bytes};
  const uint64_t off_hsum = kPeerDataOff + 2 * hb_bytes;
  const uint64_t off_recv = kPeerDataOff + 3 * hb_bytes;
  // one parity half of the receive area, in 16-byte vectors, sized by the fit's largest
  // exchange and the same for all of them
  const uint64_t recv_half =
      ctx->world > 1 ? peer_recv_bytes(ctx->world, hb_groups * cell) / 32 : 0;
  long long* hbp[2];
  long long* hsum = nullptr;
  if (peer) {
    hbp[0] = reinterpret_cast<long long*>(ctx->sym + off_hb[0]);
    hbp[1] = reinterpret_cast<long long*>(ctx->sym + off_hb[1]);
    hsum = reinterpret_cast<long long*>(ctx->sym + off_hsum);
  } else {
    RW_CU(ctx, hb0.get(ds, "hb0", hb_groups * cell));
    RW_CU(ctx, hb1.get(ds, "hb1", hb_groups * cell));
    hbp[0] = hb0.p;
    hbp[1] = hb1.p;
  }
  RW_CU(ctx, hf0.get(ds, "hf0", hf_nodes * cell));
  RW_CU(ctx, hf1.get(ds, "hf1", hf_nodes * cell));
  RW_CU(ctx, d_feat.get(ds, "feat", (size_t)T * D));
  RW_CU(ctx, d_thr.get(ds, "thr", (size_t)T * D));
  RW_CU(ctx, d_thr_bin.get(ds, "thr_bin", (size_t)T * D));
  RW_CU(ctx, d_leafval.get(ds, "leafval", (size_t)T * NL));
  WsBuf<float> d_leafvar;
  if (want_var) RW_CU(ctx, d_leafvar.get(ds, "leafvar", (size_t)T * NL));
  RW_CU(ctx, d_fi_gain.get(ds, "fi_gain", nf));
  RW_CU(ctx, d_fi_count.get(ds, "fi_count", nf));
  RW_CU(ctx, maxbits.get(ds, "maxbits", (size_t)std::max<uint32_t>(T, 1) * 2));
  WsBuf<int> kerr;
  RW_CU(ctx, kerr.get(ds, "kernel_err", 1));
  RW_CU(ctx, cudaMemsetAsync(kerr.p, 0, sizeof(int), s));
  RW_CU(ctx, rec.get(ds, "split_rec", nf));
  RW_CU(ctx, leafsum.get(ds, "leaf_sums", (size_t)LS));
  RW_CU(ctx, term.get(ds, "gain_terms", (size_t)nf * (NL / 2) * (nb - 1)));
  WsBuf<long long> prefix;
  RW_CU(ctx, prefix.get(ds, "leaf_prefix", (size_t)nf * (NL / 2) * nb * 2));
  RW_CU(ctx, cudaMemsetAsync(g.p, 0, n_pad * 4, s));
  RW_CU(ctx, cudaMemsetAsync(h.p, 0, n_pad * 4, s));
  RW_CU(ctx, cudaMemsetAsync(node.p, 0, n_pad * 2, s));
  RW_CU(ctx, cudaMemsetAsync(d_fi_gain.p, 0, nf * 4, s));
  RW_CU(ctx, cudaMemsetAsync(d_fi_count.p, 0, nf * 4, s));
  RW_CU(ctx, cudaMemsetAsync(maxbits.p, 0, maxbits.n * 4, s));
  RW_CU(ctx, cudaMemsetAsync(d_leafval.p, 0, std::max<size_t>(d_leafval.n, 1) * 4, s));
  bool any_mono = false;
  std::vector<int32_t> mono(nf, 0);
  for (uint32_t i = 0; i < std::min<uint32_t>(nf, p->monotone ? p->n_monotone : 0); i++) {
    mono[i] = p->monotone[i];
    any_mono |= mono[i] != 0;
  }
  if (any_mono) {
    RW_CU(ctx, d_mono.get(ds, "mono", nf));
    RW_CU(ctx, cudaMemcpyAsync(d_mono.p, mono.data(), nf * 4, cudaMemcpyHostToDevice, s));
    RW_CU(ctx, mono_sums.get(ds, "mono_sums", (size_t)nf * (nb - 1) * 4));
    RW_CU(ctx, cudaMemsetAsync(mono_sums.p, 0, mono_sums.n * sizeof(long long), s));
  }
  GossState gst{nullptr, nullptr};
  if (goss) {
    RW_CU(ctx, goss_counts.get(ds, "goss_counts", 256));
    RW_CU(ctx, goss_sel.get(ds, "goss_sel", 4));
    RW_CU(ctx, cudaMemsetAsync(goss_counts.p, 0, 256 * 8, s));
    gst.counts = goss_counts.p;
    gst.sel = goss_sel.p;
  }
  int nl = 0;
  RW_CU(ctx, launch_fill_f32(pred.p, base_score, n_pad, s, &nl));

  PhaseTimer pt;
  const bool profiling = prof && prof->enable;
  if (pt.init(profiling, s, (size_t)T * (5 * D + 8) + 4) != 0)
    return fail(ctx, RW_ERR_CUDA, "event creation failed");
  cudaEvent_t ev0, ev1;
  RW_CU(ctx, cudaEventCreate(&ev0));
  RW_CU(ctx, cudaEventCreate(&ev1));
  RW_CU(ctx, cudaEventRecord(ev0, s));
  pt.mark(-1);

  // GOSS constants (src/cpu.rs:72-78), over the global row count.
  const uint64_t ng = ds->n_global;
  const double top = (double)p->goss_top, other = (double)p->goss_other;
  double tn = top * (double)ng;
  uint64_t topn = tn <= 0.0 ? 0 : (uint64_t)tn;
  topn = std::min<uint64_t>(std::max<uint64_t>(topn, 1), ng);
  const uint64_t goss_k = std::min<uint64_t>(topn - 1, ng - 1);
  double keep_prob = other / std::max(1.0 - top, 1e-9);
  keep_prob = std::min(std::max(keep_prob, 0.0), 1.0);
  const float goss_fact = (float)((1.0 - top) / std::max(other, 1e-9));

  double alg_bytes = 0.0;
  uint64_t hist_launches = 0;
  const double bin_bytes = ds->packed ? 0.5 : 1.0;
  const uint64_t dsz = n_pad * 4;
  (void)dsz;

  for (uint32_t t = 0; t < T; t++) {
    uint32_t* mb = maxbits.p + 2 * (size_t)t;
    // the previous tree's pred update runs in this round's gradient kernel
    PrevTree prev = {};
    if (t > 0) {
      prev.leafval = d_leafval.p + (size_t)(t - 1) * NL;
      prev.node = node.p;
    }
    if (goss) {
      RW_CU(ctx, launch_grad(pred.p, ds->d_y, g.p, h.p, n, n_pad, logistic, 1, 0, ds->row_offset,
                             0, mb, ncount[0], prev, s, &nl));
      RW_CU(ctx, launch_goss_init(gst, goss_k, s, &nl));
      for (int pass = 0; pass < 4; pass++) {
        RW_CU(ctx, launch_goss_digit_hist(g.p, n, gst, pass, s, &nl));
        if (peer)
          RW_CU(ctx, launch_peer_small(ps, gst.counts, 256, 0, ++ctx->peer_epoch, kerr.p, s, &nl));
        else if (ctx->comm)
          RW_NC(ctx, ncclAllReduce(gst.counts, gst.counts, 256, ncclUint64, ncclSum, ctx->comm, s));
        RW_CU(ctx, launch_goss_digit_select(gst, pass, s, &nl));
      }
      RW_CU(ctx, launch_goss_apply(g.p, h.p, n, ds->row_offset, gst, keep_prob, goss_fact,
                                   (uint64_t)t, mb, s, &nl));
    } else {
      RW_CU(ctx, launch_grad(pred.p, ds->d_y, g.p, h.p, n, n_pad, logistic, stride,
                             stride > 1 ? (uint64_t)t % stride : 0, ds->row_offset, 1, mb,
                             ncount[0], prev, s, &nl));
    }
    if (peer)
      RW_CU(ctx, launch_peer_small(ps, mb, 2, 1, ++ctx->peer_epoch, kerr.p, s, &nl));
    else if (ctx->comm)
      RW_NC(ctx, ncclAllReduce(mb, mb, 2, ncclUint32, ncclMax, ctx->comm, s));
    RW_CU(ctx, launch_quant(g.p, h.p, mb, n_pad, q.p, node.p, hbp[0], cell, leafsum.p, LS,
                            ncount[0], s, &nl));
    pt.mark(RW_CAT_GRADIENTS);

    const uint32_t tree_seed = t * 2654435761u + 0x455A4B41u;  // src/booster.rs:351
    for (uint32_t d = 0; d < D; d++) {
      const uint32_t n_nodes = 1u << d;
      const int mode = (d == 0 || !subtract) ? 0 : 1;
      const uint32_t groups = mode == 0 ? n_nodes : n_nodes / 2;
      long long* hb = hbp[d & 1];
      long long* hb_next = hbp[(d + 1) & 1];
      const uint32_t groups_next =
          d + 1 < D ? (subtract ? (1u << d) : (1u << (d + 1))) : 0u;
      HistLaunch hl;
      hl.rowbins = ds->d_rowbins;
      hl.n_pad = n_pad;
      hl.packed = ds->packed;
      hl.q = q.p;
      // level 0: every row; deeper: the list k_apply wrote (one group per built node)
      hl.entries = d == 0 ? nullptr : rl_entries.p;
      hl.pcount = d == 0 ? nullptr : ncount[(d - 1) & 1];
      hl.glen = d == 0 ? nullptr : cursor[(d - 1) & 1];
      hl.parents = n_nodes / 2;
      hl.pairs = mode;
      hl.n_ident = (uint32_t)round_up(n, 512);  // rows past n carry q = 0
      hl.err = kerr.p;
      hl.groups = groups;
      hl.nf = nf;
      hl.nb = nb;
      hl.out = hb;
      RW_CU(ctx, launch_hist(hl, s, &nl));
      hist_launches++;
      alg_bytes += (double)n * nf * bin_bytes + 12.0 * (double)n + 8.0 * nf * nb * groups;
      pt.mark(RW_CAT_BUILD_HIST);
      if (peer) {
        RW_CU(ctx, launch_peer_sum_i64(ps, off_hb[d & 1], off_hsum, off_recv, recv_half,
                                       (uint64_t)groups * cell, ++ctx->peer_epoch, kerr.p, s,
                                       &nl));
        pt.mark(RW_CAT_ALLREDUCE);
      } else if (ctx->comm) {
        RW_NC(ctx, ncclAllReduce(hb, hb, (size_t)groups * cell, ncclInt64, ncclSum, ctx->comm, s));
        pt.mark(RW_CAT_ALLREDUCE);
      }
      SplitLaunch sl;
      sl.hb = peer ? hsum : hb;
      sl.hp = (d & 1) ? hf0.p : hf1.p;
      sl.hf = (d & 1) ? hf1.p : hf0.p;
      sl.n_nodes = n_nodes;
      sl.nf = nf;
      sl.nb = nb;
      sl.mode = mode;
      sl.built_odd = mode == 1 ? rl_built.p : nullptr;
      sl.choice = subtract && d + 1 < D ? rl_choice.p : nullptr;
      sl.pcount = d == 0 ? nullptr : ncount[(d - 1) & 1];
      sl.cursor_prev = d == 0 ? nullptr : cursor[(d - 1) & 1];
      sl.built_prev = rl_built.p;
      sl.ncount = ncount[d & 1];
      sl.cursor_next = d + 1 < D ? cursor[d & 1] : nullptr;
      sl.cursor_next_words = subtract ? n_nodes : 2 * n_nodes;
      sl.subtract = subtract ? 1 : 0;
      sl.maxbits = mb;
      sl.lambda = (double)p->lambda;
      sl.min_child = (double)p->min_child_h;
      sl.lr = (double)p->learning_rate;
      sl.monotone = any_mono ? d_mono.p : nullptr;
      sl.mono = any_mono ? mono_sums.p : nullptr;
      sl.term = term.p;
      // prefixes only feed the next level's built-child choice
      sl.prefix = subtract && d + 1 < D ? prefix.p : nullptr;
      sl.colsample = p->colsample;
      sl.tree_seed = tree_seed;
      sl.cuts = ds->d_cuts;
      sl.rec = rec.p;
      sl.last_level = d == D - 1;
      RW_CU(ctx, launch_split(sl, s, &nl));
      pt.mark(RW_CAT_SPLIT);
      const uint32_t n_children = 2u << d;
      ApplyLaunch al;
      al.colbins = ds->d_colbins;
      al.n_pad = n_pad;
      al.node = node.p;
      al.rec = rec.p;
      al.nf = nf;
      al.n_children = n_children;
      al.lists.entries = d + 1 < D ? rl_entries.p : nullptr;
      al.lists.q = q.p;
      al.lists.ncount = ncount[d & 1];
      al.lists.cursor = cursor[d & 1];
      al.lists.choice = rl_choice.p;
      al.lists.built_odd = rl_built.p;
      al.lists.subtract = subtract ? 1 : 0;
      al.final_level = d == D - 1;
      al.n_leaves = NL;
      al.g = g.p;
      al.h = h.p;
      al.maxbits = mb;
      al.n_rows = ds->n_global;
      al.leafsum = leafsum.p;
      al.feat = d_feat.p;
      al.thr = d_thr.p;
      al.thr_bin = d_thr_bin.p;
      al.fi_gain = d_fi_gain.p;
      al.fi_count = d_fi_count.p;
      al.slot = t * D + d;
      al.split_out = nullptr;
      al.hb_next = groups_next ? hb_next : nullptr;
      al.hb_next_words = (uint64_t)groups_next * cell;
      RW_CU(ctx, launch_apply(al, s, &nl));
      if (want_var && d == D - 1) {
        LeafSquares sq;
        sq.node = node.p;
        sq.g = g.p;
        sq.n_pad = n_pad;
        sq.maxbits = mb;
        sq.n_rows = ds->n_global;
        sq.n_leaves = NL;
        sq.leafsum2 = leafsum.p + 2 * (size_t)NL;
        RW_CU(ctx, launch_leafsq(sq, s, &nl));
      }
      pt.mark(d == D - 1 ? RW_CAT_UPDATE_PRED : RW_CAT_APPLY);
    }
    // every rank's leaf sums (exact integers: any order gives the same totals)
    if (peer) {
      RW_CU(ctx, launch_peer_small(ps, leafsum.p, 2 * NL, 0, ++ctx->peer_epoch, kerr.p, s, &nl));
      if (want_var)  // the g^2 sums in a second exchange (the small slots hold 2 * 4096)
        RW_CU(ctx, launch_peer_small(ps, leafsum.p + 2 * (size_t)NL, NL, 0, ++ctx->peer_epoch,
                                     kerr.p, s, &nl));
      pt.mark(RW_CAT_ALLREDUCE);
    } else if (ctx->comm) {
      RW_NC(ctx, ncclAllReduce(leafsum.p, leafsum.p, (size_t)LS, ncclInt64, ncclSum, ctx->comm,
                               s));
      pt.mark(RW_CAT_ALLREDUCE);
    }
    LeafValues lv;
    lv.leafsum = leafsum.p;
    lv.maxbits = mb;
    lv.n_leaves = NL;
    lv.n_rows = ds->n_global;
    lv.lr = (double)p->learning_rate;
    lv.lambda = (double)p->lambda;
    lv.leafval = d_leafval.p + (size_t)t * NL;
    lv.leafsum2 = want_var ? leafsum.p + 2 * (size_t)NL : nullptr;
    lv.leafvar = want_var ? d_leafvar.p + (size_t)t * NL : nullptr;
    RW_CU(ctx, launch_leafval(lv, s, &nl));
    pt.mark(RW_CAT_UPDATE_PRED);
  }
  RW_CU(ctx, cudaEventRecord(ev1, s));
  rc = wait_stream(ctx);
  if (rc) return rc;
  ctx->launches += nl;

  if (T > 0) {
    RW_CU(ctx, cudaMemcpy(feat, d_feat.p, (size_t)T * D * 4, cudaMemcpyDeviceToHost));
    RW_CU(ctx, cudaMemcpy(thr, d_thr.p, (size_t)T * D * 4, cudaMemcpyDeviceToHost));
    if (thr_bin)
      RW_CU(ctx, cudaMemcpy(thr_bin, d_thr_bin.p, (size_t)T * D * 2, cudaMemcpyDeviceToHost));
    RW_CU(ctx, cudaMemcpy(leafval, d_leafval.p, (size_t)T * NL * 4, cudaMemcpyDeviceToHost));
    if (want_var)
      RW_CU(ctx, cudaMemcpy(leafvar, d_leafvar.p, (size_t)T * NL * 4, cudaMemcpyDeviceToHost));
  }
  int kerr_h = 0;
  RW_CU(ctx, cudaMemcpy(&kerr_h, kerr.p, sizeof(int), cudaMemcpyDeviceToHost));
  if (kerr_h) {
    cudaEventDestroy(ev0);
    cudaEventDestroy(ev1);
    if (kerr_h == 2) ctx->peer_failed = true;
    return fail(ctx, RW_ERR_TIMEOUT,
                kerr_h == 1   ? "a histogram bulk-copy wait gave up (bounded wait expired)"
                : kerr_h == 2 ? "a wait on a peer rank expired (peer exchange)"
                              : "a peer rank reported a failed wait");
  }
  RW_CU(ctx, cudaMemcpy(fi_gain, d_fi_gain.p, nf * 4, cudaMemcpyDeviceToHost));
  RW_CU(ctx, cudaMemcpy(fi_count, d_fi_count.p, nf * 4, cudaMemcpyDeviceToHost));

  if (prof) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ev0, ev1);
    prof->total_ms = ms;
    for (int c = 0; c < RW_N_CATEGORIES; c++) prof->category_ms[c] = 0.0;
    if (profiling) {
      for (size_t i = 1; i < pt.used; i++) {
        float dt = 0.f;
        cudaEventElapsedTime(&dt, pt.ev[i - 1], pt.ev[i]);
        if (pt.cat[i] >= 0) prof->category_ms[pt.cat[i]] += dt;
      }
    }
    prof->hist_alg_bytes = alg_bytes;
    prof->hist_launches = hist_launches;
    prof->kernel_launches = (uint64_t)nl;
  }
  cudaEventDestroy(ev0);
  cudaEventDestroy(ev1);
  return RW_OK;
}

// The tree loop on every rank of a multi-GPU context at once (one host thread per GPU):
// each rank fits its shard and exchanges the per-level histograms with the others, so
// every rank ends with the same model, which rank 0 writes to the caller's buffers.
static int group_fit(rw_dataset* gd, const rw_train_params* p, float base_score, uint32_t* feat,
                     float* thr, uint16_t* thr_bin, float* leafval, float* leafvar,
                     float* fi_gain, float* fi_count, rw_profile* prof) {
  rw_ctx* front = gd->ctx;
  int rc = check_params(front, p, gd->n_bins);
  if (rc) return rc;
  if (p->n_trees > 0 && (!feat || !thr || !leafval))
    return fail(front, RW_ERR_ARG, "NULL model output");
  if (!fi_gain || !fi_count) return fail(front, RW_ERR_ARG, "NULL feature-importance output");
  const int W = (int)gd->shards.size();
  const size_t K = (size_t)p->n_trees * p->depth, L = (size_t)p->n_trees << p->depth;
  const size_t nf = gd->nf;
  struct Out {
    std::vector<uint32_t> feat;
    std::vector<float> thr, leafval, leafvar, fig, fic;
    std::vector<uint16_t> tb;
    rw_profile prof;
  };
  std::vector<Out> o(W);
  for (auto& q : o) {
    q.feat.resize(std::max<size_t>(K, 1));
    q.thr.resize(std::max<size_t>(K, 1));
    q.tb.resize(std::max<size_t>(K, 1));
    q.leafval.resize(std::max<size_t>(L, 1));
    if (leafvar) q.leafvar.resize(std::max<size_t>(L, 1));  // every rank runs the same exchanges
    q.fig.resize(nf);
    q.fic.resize(nf);
    memset(&q.prof, 0, sizeof q.prof);
    q.prof.enable = prof ? prof->enable : 0;
  }
  rc = run_members(
      front,
      [&](int i) {
        Out& q = o[i];
        return rw_fit_dataset(gd->shards[i], p, base_score, q.feat.data(), q.thr.data(),
                              q.tb.data(), q.leafval.data(), leafvar ? q.leafvar.data() : nullptr,
                              q.fig.data(), q.fic.data(), &q.prof);
      },
      true);
  if (rc) return rc;
  // every split decision reads all-rank sums, so every rank holds the same model
  for (int i = 1; i < W; i++)
    if (memcmp(o[i].feat.data(), o[0].feat.data(), K * 4) ||
        memcmp(o[i].thr.data(), o[0].thr.data(), K * 4) ||
        memcmp(o[i].tb.data(), o[0].tb.data(), K * 2) ||
        memcmp(o[i].leafval.data(), o[0].leafval.data(), L * 4) ||
        (leafvar && memcmp(o[i].leafvar.data(), o[0].leafvar.data(), L * 4)) ||
        memcmp(o[i].fig.data(), o[0].fig.data(), nf * 4) ||
        memcmp(o[i].fic.data(), o[0].fic.data(), nf * 4))
      return fail(front, RW_ERR_CUDA, "ranks produced different models");
  if (K) {
    memcpy(feat, o[0].feat.data(), K * 4);
    memcpy(thr, o[0].thr.data(), K * 4);
    if (thr_bin) memcpy(thr_bin, o[0].tb.data(), K * 2);
    memcpy(leafval, o[0].leafval.data(), L * 4);
    if (leafvar) memcpy(leafvar, o[0].leafvar.data(), L * 4);
  }
  memcpy(fi_gain, o[0].fig.data(), nf * 4);
  memcpy(fi_count, o[0].fic.data(), nf * 4);
  if (prof) {
    const int32_t en = prof->enable;
    *prof = o[0].prof;
    prof->enable = en;
    for (int i = 1; i < W; i++) prof->total_ms = std::max(prof->total_ms, o[i].prof.total_ms);
  }
  return RW_OK;
}

extern "C" int rw_fit(rw_ctx* ctx, const rw_train_params* p, const float* x, const float* y,
                      uint64_t n, uint32_t nf, const float* cuts, float base_score,
                      uint32_t* feat, float* thr, uint16_t* thr_bin, float* leafval,
                      float* leafvar, float* fi_gain, float* fi_count, rw_profile* prof) {
  if (!p) return fail(ctx, RW_ERR_ARG, "params is NULL");
  rw_dataset* ds = nullptr;
  int rc = rw_dataset_create(ctx, x, y, n, nf, cuts, p->n_bins, p->pack4, n, 0, &ds);
  if (rc) return rc;
  rc = rw_fit_dataset(ds, p, base_score, feat, thr, thr_bin, leafval, leafvar, fi_gain, fi_count,
                      prof);
  rw_dataset_destroy(ds);
  return rc;
}

// =================================================================================
// scoring

static int model_check(rw_ctx* ctx, const rw_model* m, bool need_bins) {
  if (!ctx) return fail(nullptr, RW_ERR_ARG, "ctx is NULL");
  if (!m) return fail(ctx, RW_ERR_ARG, "model is NULL");
  if (m->depth < 1 || m->depth > 12) return fail(ctx, RW_ERR_ARG, "depth must be in 1..=12");
  if (m->n_trees > 0 && (!m->feat || !m->leafval)) return fail(ctx, RW_ERR_ARG, "NULL model array");
  if (m->n_trees > 0 && !need_bins && !m->thr) return fail(ctx, RW_ERR_ARG, "NULL thr");
  if (m->n_trees > 0 && need_bins && !m->thr_bin)
    return fail(ctx, RW_ERR_ARG, "u8 scoring needs thr_bin");
  for (size_t k = 0; k < (size_t)m->n_trees * m->depth; k++) {
    if (m->feat[k] >= m->n_features) return fail(ctx, RW_ERR_ARG, "feature index out of range");
    if (need_bins && m->thr_bin[k] > 255) return fail(ctx, RW_ERR_ARG, "thr_bin above 255");
  }
  return RW_OK;
}

// Entry points that take device pointers or a device-resident model run on the first
// GPU of a multi-GPU context.
static rw_ctx* first_rank(rw_ctx* ctx) {
  return ctx && !ctx->members.empty() ? ctx->members[0] : ctx;
}

extern "C" int rw_model_upload(rw_ctx* ctx, const rw_model* m, rw_dmodel** out) {
  ctx = first_rank(ctx);
  if (!out) return fail(ctx, RW_ERR_ARG, "out is NULL");
  *out = nullptr;
  int rc = model_check(ctx, m, false);
  if (rc) return rc;
  RW_CU(ctx, cudaSetDevice(ctx->device));
  const size_t K = (size_t)m->n_trees * m->depth, L = (size_t)m->n_trees << m->depth;
  DBuf<uint32_t> df, ds8;
  DBuf<float> dt, dl;
  RW_CU(ctx, df.alloc(K));
  RW_CU(ctx, dt.alloc(K));
  RW_CU(ctx, dl.alloc(L));
  RW_CU(ctx, ds8.alloc(K));
  std::vector<uint32_t> s8(K, 0);
  for (size_t k = 0; k < K; k++)
    s8[k] = (m->feat[k] << 8) | (m->thr_bin ? (uint32_t)(m->thr_bin[k] & 0xff) : 0u);
  if (K) {
    RW_CU(ctx, cudaMemcpy(df.p, m->feat, K * 4, cudaMemcpyHostToDevice));
    if (m->thr) RW_CU(ctx, cudaMemcpy(dt.p, m->thr, K * 4, cudaMemcpyHostToDevice));
    RW_CU(ctx, cudaMemcpy(ds8.p, s8.data(), K * 4, cudaMemcpyHostToDevice));
    RW_CU(ctx, cudaMemcpy(dl.p, m->leafval, L * 4, cudaMemcpyHostToDevice));
  }
  auto* dm = new rw_dmodel();
  dm->ctx = ctx;
  dm->n_trees = m->n_trees;
  dm->depth = m->depth;
  dm->nf = m->n_features;
  dm->base = m->base_score;
  dm->has_bins = m->thr_bin != nullptr;
  dm->d_feat = df.release();
  dm->d_thr = dt.release();
  dm->d_split8 = ds8.release();
  dm->d_leafval = dl.release();
  *out = dm;
  return RW_OK;
}

extern "C" void rw_model_free(rw_dmodel* dm) {
  if (!dm) return;
  cudaSetDevice(dm->ctx->device);
  cudaFree(dm->d_feat);
  cudaFree(dm->d_thr);
  cudaFree(dm->d_split8);
  cudaFree(dm->d_leafval);
  delete dm;
}

static int predict_device_common(rw_ctx* ctx, const rw_dmodel* dm, float* d_out, uint64_t n,
                                 float* kernel_ms, bool u8, const void* in, uint64_t ld) {
  ctx = first_rank(ctx);
  if (!ctx || !dm || (n > 0 && (!in || !d_out))) return fail(ctx, RW_ERR_ARG, "NULL argument");
  if (dm->ctx != ctx) return fail(ctx, RW_ERR_ARG, "the model was uploaded on another context");
  if (u8 && !dm->has_bins) return fail(ctx, RW_ERR_ARG, "model uploaded without thr_bin");
  if (u8 && ld < n) return fail(ctx, RW_ERR_ARG, "ld < n");
  RW_CU(ctx, cudaSetDevice(ctx->device));
  cudaEvent_t a = nullptr, b = nullptr;
  if (kernel_ms) {
    RW_CU(ctx, cudaEventCreate(&a));
    RW_CU(ctx, cudaEventCreate(&b));
    RW_CU(ctx, cudaEventRecord(a, ctx->stream));
  }
  cudaError_t e = cudaSuccess;
  int nl = 0;
  if (n > 0) {
    if (dm->n_trees == 0) e = launch_fill_f32(d_out, dm->base, n, ctx->stream, &nl);
    else if (u8) e = launch_predict_u8((const uint8_t*)in, n, ld, *dm, d_out, ctx->stream);
    else e = launch_predict_f32((const float*)in, n, dm->nf, *dm, d_out, ctx->stream);
    nl += 1;
  }
  if (e != cudaSuccess) return cuda_fail(ctx, e, "predict launch");
  ctx->launches += nl;
  if (kernel_ms) {
    RW_CU(ctx, cudaEventRecord(b, ctx->stream));
    RW_CU(ctx, cudaEventSynchronize(b));
    cudaEventElapsedTime(kernel_ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
  }
  return RW_OK;
}

extern "C" int rw_predict_u8_device(rw_ctx* ctx, const rw_dmodel* dm, const uint8_t* d_bins,
                                    uint64_t n, uint64_t ld, float* d_out, float* kernel_ms) {
  return predict_device_common(ctx, dm, d_out, n, kernel_ms, true, d_bins, ld);
}

extern "C" int rw_predict_f32_device(rw_ctx* ctx, const rw_dmodel* dm, const float* d_x,
                                     uint64_t n, float* d_out, float* kernel_ms) {
  return predict_device_common(ctx, dm, d_out, n, kernel_ms, false, d_x, 0);
}

// Row ranges of a multi-GPU context's ranks for n rows (contiguous, in rank order).
static uint64_t rank_lo(uint64_t n, int i, int W) { return n * (uint64_t)i / (uint64_t)W; }

// PGBM predict_var (gpu_kernels.rs:1084-1120): the same traversal as the margins, summing
// the leaves' variances in tree order in f32 from 0 -- exactly rw_predict_f32 over a model
// whose leaf table is leafvar and whose base score is 0.
extern "C" int rw_predict_var_f32(rw_ctx* ctx, const rw_model* m, const float* leafvar,
                                  const float* x, uint64_t n, uint32_t nf, float* out) {
  if (!m) return fail(ctx, RW_ERR_ARG, "model is NULL");
  if (!leafvar && m->n_trees > 0) return fail(ctx, RW_ERR_ARG, "leafvar is NULL");
  rw_model mv = *m;
  mv.leafval = leafvar;
  mv.base_score = 0.0f;
  return rw_predict_f32(ctx, &mv, x, n, nf, out);
}

extern "C" int rw_predict_f32(rw_ctx* ctx, const rw_model* m, const float* x, uint64_t n,
                              uint32_t nf, float* out) {
  int rc = model_check(ctx, m, false);
  if (rc) return rc;
  if (nf != m->n_features) return fail(ctx, RW_ERR_ARG, "nf differs from the model's n_features");
  if (n == 0) return RW_OK;
  if (!x || !out) return fail(ctx, RW_ERR_ARG, "NULL buffer");
  if (!ctx->members.empty()) {  // row shards, one per GPU, no communication
    const int W = (int)ctx->members.size();
    return run_members(
        ctx,
        [&](int i) {
          const uint64_t lo = rank_lo(n, i, W), rows = rank_lo(n, i + 1, W) - lo;
          return rw_predict_f32(ctx->members[i], m, x + lo * nf, rows, nf, out + lo);
        },
        false);
  }
  rw_dmodel* dm = nullptr;
  rc = rw_model_upload(ctx, m, &dm);
  if (rc) return rc;
  DBuf<float> dx, dout;
  cudaError_t e = dx.alloc((size_t)n * nf);
  if (e == cudaSuccess) e = dout.alloc(n);
  if (e == cudaSuccess)
    e = upload_h2d(ctx, dx.p, x, (size_t)n * nf * 4);
  if (e != cudaSuccess) {
    rw_model_free(dm);
    return cuda_fail(ctx, e, "predict upload");
  }
  rc = rw_predict_f32_device(ctx, dm, dx.p, n, dout.p, nullptr);
  if (!rc) {
    e = cudaMemcpyAsync(out, dout.p, n * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) rc = cuda_fail(ctx, e, "predict download");
  }
  rw_model_free(dm);
  return rc;
}

// n rows of feature-major u8 bins whose feature rows are `pitch` bytes apart.
static int predict_u8_host(rw_ctx* ctx, const rw_model* m, const uint8_t* bins, uint64_t n,
                           uint64_t pitch, uint32_t nf, float* out) {
  if (n == 0) return RW_OK;
  rw_dmodel* dm = nullptr;
  int rc = rw_model_upload(ctx, m, &dm);
  if (rc) return rc;
  const uint64_t ld = round_up(n, 16);
  DBuf<uint8_t> db;
  DBuf<float> dout;
  cudaError_t e = db.alloc((size_t)nf * ld);
  if (e == cudaSuccess) e = dout.alloc(n);
  if (e == cudaSuccess) e = cudaMemsetAsync(db.p, 0, (size_t)nf * ld, ctx->stream);
  if (e == cudaSuccess)
    e = cudaMemcpy2DAsync(db.p, ld, bins, pitch, n, nf, cudaMemcpyHostToDevice, ctx->stream);
  if (e != cudaSuccess) {
    rw_model_free(dm);
    return cuda_fail(ctx, e, "predict upload");
  }
  rc = rw_predict_u8_device(ctx, dm, db.p, n, ld, dout.p, nullptr);
  if (!rc) {
    e = cudaMemcpyAsync(out, dout.p, n * 4, cudaMemcpyDeviceToHost, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) rc = cuda_fail(ctx, e, "predict download");
  }
  rw_model_free(dm);
  return rc;
}

extern "C" int rw_predict_u8(rw_ctx* ctx, const rw_model* m, const uint8_t* bins, uint64_t n,
                             uint32_t nf, float* out) {
  int rc = model_check(ctx, m, true);
  if (rc) return rc;
  if (nf != m->n_features) return fail(ctx, RW_ERR_ARG, "nf differs from the model's n_features");
  if (n == 0) return RW_OK;
  if (!bins || !out) return fail(ctx, RW_ERR_ARG, "NULL buffer");
  if (!ctx->members.empty()) {  // row shards, one per GPU, no communication
    const int W = (int)ctx->members.size();
    return run_members(
        ctx,
        [&](int i) {
          const uint64_t lo = rank_lo(n, i, W), rows = rank_lo(n, i + 1, W) - lo;
          return predict_u8_host(ctx->members[i], m, bins + lo, rows, n, nf, out + lo);
        },
        false);
  }
  return predict_u8_host(ctx, m, bins, n, n, nf, out);
}

// =================================================================================
// host helpers (reference host code, restated natively)

extern "C" void rw_compute_boundaries(const float* x, uint64_t n, uint32_t nf, uint32_t n_bins,
                                      uint64_t sample, int32_t unique, float* out) {
  // src/data.rs:86-146: strided sample, stable sort, quantile (or unique-midpoint) cuts.
  if (!x || !out || n_bins < 2 || n == 0) return;
  const uint32_t nbound = n_bins - 1;
  const uint64_t stride = std::max<uint64_t>(n / std::max<uint64_t>(sample, 1), 1);
  // features are independent: host threads take them in turn (feature f on thread
  // f % workers), each writing only its features' cuts
  const uint32_t workers =
      std::max<uint32_t>(1, std::min<uint32_t>(nf, std::thread::hardware_concurrency()));
  auto run = [&](uint32_t w) {
    std::vector<float> s;
    s.reserve(n / stride + 1);
    for (uint32_t f = w; f < nf; f += workers) {
      s.clear();
      for (uint64_t i = 0; i < n; i += stride) s.push_back(x[i * nf + f]);
      std::stable_sort(s.begin(), s.end(), [](float a, float b) { return a < b; });
      float* b = out + (size_t)f * nbound;
      if (unique) {
        std::vector<float> u;
        for (float v : s)
          if (u.empty() || u.back() != v) u.push_back(v);
        std::vector<float> cand;
        for (size_t i = 0; i + 1 < u.size(); i++) cand.push_back(0.5f * (u[i] + u[i + 1]));
        for (uint32_t j = 0; j < nbound; j++) {
          if (cand.empty()) b[j] = INFINITY;
          else if (cand.size() <= nbound) b[j] = j < cand.size() ? cand[j] : INFINITY;
          else {
            size_t pos = ((size_t)(j + 1) * cand.size()) / (nbound + 1);
            b[j] = cand[std::min(pos, cand.size() - 1)];
          }
        }
      } else {
        const size_t m = s.size();
        for (uint32_t j = 0; j < nbound; j++) {
          const double q = (double)(j + 1) / (double)n_bins;
          const size_t pos = (size_t)std::round(q * (double)(m - 1));
          b[j] = s[std::min(pos, m - 1)];
        }
        for (uint32_t j = 1; j < nbound; j++)
          if (b[j] <= b[j - 1]) b[j] = b[j - 1];
      }
    }
  };
  std::vector<std::thread> th;
  for (uint32_t w = 1; w < workers; w++) th.emplace_back(run, w);
  run(0);
  for (auto& t : th) t.join();
}

extern "C" int rw_compute_boundaries_device(rw_ctx* ctx, const float* d_x, uint64_t n,
                                            uint32_t nf, uint32_t n_bins, uint64_t sample,
                                            int32_t unique, float* out) {
  ctx = first_rank(ctx);
  if (!ctx) return fail(nullptr, RW_ERR_ARG, "ctx is NULL");
  if (!d_x || !out || n == 0 || nf == 0 || n_bins < 2 || n_bins > 256)
    return fail(ctx, RW_ERR_ARG, "bad argument");
  RW_CU(ctx, cudaSetDevice(ctx->device));
  const uint64_t m = boundary_sample_rows(n, sample);
  DBuf<uint32_t> scratch;
  DBuf<float> dout;
  RW_CU(ctx, scratch.alloc(ctx, boundary_scratch_words(nf, m)));
  RW_CU(ctx, dout.alloc(ctx, (size_t)nf * (n_bins - 1)));
  uint64_t mm = 0;
  int nl = 0;
  RW_CU(ctx, launch_boundaries(d_x, n, nf, n_bins, sample, unique, scratch.p, dout.p,
                               ctx->stream, &mm, &nl));
  ctx->launches += nl;
  RW_CU(ctx, cudaMemcpyAsync(out, dout.p, (size_t)nf * (n_bins - 1) * 4, cudaMemcpyDeviceToHost,
                             ctx->stream));
  RW_CU(ctx, cudaStreamSynchronize(ctx->stream));
  return RW_OK;
}

extern "C" int rw_fit_with_boundaries(rw_ctx* ctx, const rw_train_params* p, const float* x,
                                      const float* y, uint64_t n, uint32_t nf, uint64_t sample,
                                      int32_t unique, float base_score, float* cuts_out,
                                      uint32_t* feat, float* thr, uint16_t* thr_bin,
                                      float* leafval, float* leafvar, float* fi_gain,
                                      float* fi_count, rw_profile* prof) {
  if (!ctx) return fail(nullptr, RW_ERR_ARG, "ctx is NULL");
  if (!p) return fail(ctx, RW_ERR_ARG, "params is NULL");
  if (!x || !y || n == 0 || nf == 0) return fail(ctx, RW_ERR_ARG, "empty or NULL dataset");
  if (p->n_bins < 2 || p->n_bins > 256) return fail(ctx, RW_ERR_ARG, "n_bins must be in 2..=256");
  std::vector<float> cuts((size_t)nf * (p->n_bins - 1));
  rw_ctx* c0 = first_rank(ctx);
  RW_CU(c0, cudaSetDevice(c0->device));
  if (ctx->members.empty()) {
    // one upload of x serves the sample and the binning
    DBuf<float> dx;
    RW_CU(ctx, dx.alloc(ctx, (size_t)n * nf));
    RW_CU(ctx, upload_h2d(ctx, dx.p, x, (size_t)n * nf * 4));
    int rc = rw_compute_boundaries_device(ctx, dx.p, n, nf, p->n_bins, sample, unique,
                                          cuts.data());
    if (rc) return rc;
    rw_dataset* ds = nullptr;
    rc = dataset_build(ctx, dx.p, y, false, n, nf, cuts.data(), p->n_bins, p->pack4, n, 0, &ds);
    if (rc) return rc;
    rc = rw_fit_dataset(ds, p, base_score, feat, thr, thr_bin, leafval, leafvar, fi_gain,
                        fi_count, prof);
    rw_dataset_destroy(ds);
    if (!rc && cuts_out) memcpy(cuts_out, cuts.data(), cuts.size() * 4);
    return rc;
  }
  // several GPUs: the sampled rows go to the first GPU for the cut table, then every
  // rank uploads and bins its own shard against it
  const uint64_t m = boundary_sample_rows(n, sample);
  const uint64_t stride = std::max<uint64_t>(n / std::max<uint64_t>(sample, 1), 1);
  std::vector<float> smp((size_t)m * nf);
  for (uint64_t k = 0; k < m; k++) memcpy(&smp[k * nf], x + k * stride * nf, (size_t)nf * 4);
  DBuf<float> ds_smp;
  RW_CU(c0, ds_smp.alloc(c0, smp.size()));
  RW_CU(c0, cudaMemcpyAsync(ds_smp.p, smp.data(), smp.size() * 4, cudaMemcpyHostToDevice,
                            c0->stream));
  int rc = rw_compute_boundaries_device(c0, ds_smp.p, m, nf, p->n_bins, m, unique, cuts.data());
  if (rc) return fail(ctx, rc, c0->last_error);
  rc = rw_fit(ctx, p, x, y, n, nf, cuts.data(), base_score, feat, thr, thr_bin, leafval, leafvar,
              fi_gain, fi_count, prof);
  if (!rc && cuts_out) memcpy(cuts_out, cuts.data(), cuts.size() * 4);
  return rc;
}

extern "C" int rw_model_thr_bins(const rw_model* m, const float* cuts, uint32_t n_bins,
                                 uint16_t* thr_bin) {
  // A split tests x > thr with thr = cuts[f][b] (the trainer writes cut values,
  // src/gpu_kernels.rs:966-967); with bin = #{cut < x}, bin > b <=> x > cuts[f][b] for
  // every b holding that value, so the first such b serves the u8 scorer.
  if (!m || !cuts || !thr_bin || n_bins < 2 || n_bins > 256)
    return fail(nullptr, RW_ERR_ARG, "bad argument");
  const size_t K = (size_t)m->n_trees * m->depth;
  if (K && (!m->feat || !m->thr)) return fail(nullptr, RW_ERR_ARG, "NULL model array");
  const uint32_t nb1 = n_bins - 1;
  for (size_t k = 0; k < K; k++) {
    if (m->feat[k] >= m->n_features) return fail(nullptr, RW_ERR_ARG, "feature index out of range");
    const float* c = cuts + (size_t)m->feat[k] * nb1;
    const float* it = std::lower_bound(c, c + nb1, m->thr[k]);
    if (it == c + nb1 || !(*it == m->thr[k]))
      return fail(nullptr, RW_ERR_ARG,
                  "split " + std::to_string(k) + ": threshold is not a cut of feature " +
                      std::to_string(m->feat[k]) + " in this table");
    thr_bin[k] = (uint16_t)(it - c);
  }
  return RW_OK;
}

extern "C" float rw_base_score(const float* y, uint64_t n, int32_t objective) {
  // src/booster.rs:201-205: f32 sequential mean, clamped, logit for logistic.
  float s = 0.0f;
  for (uint64_t i = 0; i < n; i++) s += y[i];
  float mean = s / (float)n;
  mean = std::min(std::max(mean, 1e-6f), 1.0f - 1e-6f);
  return objective == RW_OBJ_LOGISTIC ? std::log(mean / (1.0f - mean)) : mean;
}

// =================================================================================
// test hooks

extern "C" int rw_debug_level_hist(rw_dataset* ds, const int32_t* node, const float* g,
                                   const float* h, int32_t e_g, int32_t e_h, uint32_t groups,
                                   int32_t odd_only, int64_t* out) {
  if (!ds || !node || !g || !h || !out || groups == 0) return fail(nullptr, RW_ERR_ARG, "NULL argument");
  if (!ds->shards.empty())
    return fail(ds->ctx, RW_ERR_UNSUPPORTED, "a multi-GPU dataset has no single histogram hook");
  rw_ctx* ctx = ds->ctx;
  RW_CU(ctx, cudaSetDevice(ctx->device));
  const uint64_t n = ds->n, n_pad = ds->n_pad;
  // The level's row list, grouped by histogram group (counting sort), and q per row.
  std::vector<int2> qv(n_pad, make_int2(0, 0));
  std::vector<int32_t> grp(n, -1);
  std::vector<uint32_t> seg(groups + 1, 0);
  const float sg = rw_pow2f(e_g), sh = rw_pow2f(e_h);
  for (uint64_t i = 0; i < n; i++) {
    if (node[i] < 0) continue;
    if (node[i] > 0x7fff) return fail(ctx, RW_ERR_ARG, "node index above 32767");
    const int32_t a = rw_quantize(g[i], sg), b = rw_quantize(h[i], sh);
    // the histogram kernel's exact 32-bit partial sums rely on |q| <= 2^RW_QBITS
    if (std::abs(a) > (1 << RW_QBITS) || std::abs(b) > (1 << RW_QBITS))
      return fail(ctx, RW_ERR_ARG, "e_g/e_h put |q| above 2^RW_QBITS");
    if ((a | b) == 0) continue;
    qv[i] = make_int2(a, b);
    const int32_t gi = odd_only ? ((node[i] & 1) ? (node[i] >> 1) : -1) : node[i];
    if (gi < 0) continue;
    if ((uint32_t)gi >= groups) return fail(ctx, RW_ERR_ARG, "node beyond the groups");
    grp[i] = gi;
    seg[gi + 1]++;
  }
  for (uint32_t k = 0; k < groups; k++) seg[k + 1] += seg[k];
  std::vector<int4> rows(std::max<uint32_t>(seg[groups], 1), make_int4(0, 0, 0, 0));
  {
    std::vector<uint32_t> cur(seg.begin(), seg.end() - 1);
    for (uint64_t i = 0; i < n; i++)
      if (grp[i] >= 0) rows[cur[grp[i]]++] = make_int4((int)i, qv[i].x, qv[i].y, 0);
  }
  // device cells: [group][tile][bin][g|h][kHistFeat columns]; out: [group][nf][nb][2]
  const size_t words = (size_t)groups * ds->ftiles * ds->n_bins * 2 * kHistFeat;
  DBuf<int2> dq;
  DBuf<int4> drows;
  DBuf<uint32_t> dlen;  // group lengths (each group is its own region: pcount = glen)
  DBuf<long long> dout;
  RW_CU(ctx, dq.alloc(n_pad));
  RW_CU(ctx, drows.alloc(rows.size()));
  std::vector<uint32_t> len(groups);
  for (uint32_t k = 0; k < groups; k++) len[k] = seg[k + 1] - seg[k];
  RW_CU(ctx, dlen.alloc(groups));
  RW_CU(ctx, dout.alloc(words));
  RW_CU(ctx, cudaMemcpy(dq.p, qv.data(), n_pad * sizeof(int2), cudaMemcpyHostToDevice));
  RW_CU(ctx, cudaMemcpy(drows.p, rows.data(), rows.size() * sizeof(int4), cudaMemcpyHostToDevice));
  RW_CU(ctx, cudaMemcpy(dlen.p, len.data(), groups * 4, cudaMemcpyHostToDevice));
  RW_CU(ctx, cudaMemset(dout.p, 0, words * 8));
  HistLaunch hl;
  hl.rowbins = ds->d_rowbins;
  hl.n_pad = ds->n_pad;
  hl.packed = ds->packed;
  hl.err = nullptr;
  hl.q = dq.p;
  hl.entries = drows.p;
  hl.pcount = dlen.p;
  hl.glen = dlen.p;
  hl.parents = groups;
  hl.pairs = 1;
  hl.n_ident = 0;
  hl.groups = groups;
  hl.nf = ds->nf;
  hl.nb = ds->n_bins;
  hl.out = dout.p;
  int nl = 0;
  RW_CU(ctx, launch_hist(hl, ctx->stream, &nl));
  RW_CU(ctx, cudaStreamSynchronize(ctx->stream));
  ctx->launches += nl;
  std::vector<int64_t> cells(words);
  RW_CU(ctx, cudaMemcpy(cells.data(), dout.p, words * 8, cudaMemcpyDeviceToHost));
  const uint32_t nf = ds->nf, nb = ds->n_bins;
  for (uint32_t gi = 0; gi < groups; gi++)
    for (uint32_t f = 0; f < nf; f++) {
      const uint32_t t = f / kHistFeat, j = f % kHistFeat, col = (j >> 1) + 32u * (j & 1u);
      for (uint32_t b = 0; b < nb; b++) {
        const size_t k = (((size_t)gi * ds->ftiles + t) * nb + b) * 2 * kHistFeat + col;
        int64_t* o = out + (((size_t)gi * nf + f) * nb + b) * 2;
        o[0] = cells[k];
        o[1] = cells[k + kHistFeat];
      }
    }
  return RW_OK;
}

extern "C" int rw_debug_level_step(rw_dataset* ds, const rw_train_params* p,
                                   const int32_t* node, const float* g, const float* h,
                                   uint32_t n_nodes, uint32_t tree, double* gain_out,
                                   uint32_t* bin_out, uint32_t* chosen) {
  if (!ds || !node || !g || !h || !gain_out || !bin_out || !chosen)
    return fail(nullptr, RW_ERR_ARG, "NULL argument");
  if (!ds->shards.empty())
    return fail(ds->ctx, RW_ERR_UNSUPPORTED, "a multi-GPU dataset has no single level hook");
  rw_ctx* ctx = ds->ctx;
  int rc = check_params(ctx, p, ds->n_bins);
  if (rc) return rc;
  if (n_nodes == 0 || (n_nodes & (n_nodes - 1)) || n_nodes > 2048)
    return fail(ctx, RW_ERR_ARG, "n_nodes must be a power of two up to 2048");
  RW_CU(ctx, cudaSetDevice(ctx->device));
  const uint64_t n = ds->n, n_pad = ds->n_pad;
  const uint32_t nf = ds->nf, nb = ds->n_bins;
  // the round's maxima over the level's rows and their fixed-point scales (k_grad, k_quant)
  uint32_t mbits[2] = {0u, 0u};
  for (uint64_t i = 0; i < n; i++) {
    if (node[i] < 0) continue;
    if ((uint32_t)node[i] >= n_nodes) return fail(ctx, RW_ERR_ARG, "node beyond n_nodes");
    uint32_t bg, bh;
    const float ag = std::fabs(g[i]);
    memcpy(&bg, &ag, 4);
    memcpy(&bh, &h[i], 4);
    mbits[0] = std::max(mbits[0], bg & 0x7fffffffu);
    mbits[1] = std::max(mbits[1], bh & 0x7fffffffu);
  }
  const float sg = rw_pow2f(rw_qscale_exp(mbits[0])), sh = rw_pow2f(rw_qscale_exp(mbits[1]));
  // the level's row list, grouped by node (a counting sort), entries (row, q(g), q(h), 0)
  std::vector<int2> qv(n_pad, make_int2(0, 0));
  std::vector<uint32_t> seg(n_nodes + 1, 0);
  for (uint64_t i = 0; i < n; i++) {
    if (node[i] < 0) continue;
    const int32_t a = rw_quantize(g[i], sg), b = rw_quantize(h[i], sh);
    if ((a | b) == 0) continue;
    qv[i] = make_int2(a, b);
    seg[node[i] + 1]++;
  }
  for (uint32_t k = 0; k < n_nodes; k++) seg[k + 1] += seg[k];
  std::vector<int4> rows(std::max<uint32_t>(seg[n_nodes], 1), make_int4(0, 0, 0, 0));
  {
    std::vector<uint32_t> cur(seg.begin(), seg.end() - 1);
    for (uint64_t i = 0; i < n; i++)
      if (node[i] >= 0 && (qv[i].x | qv[i].y) != 0)
        rows[cur[node[i]]++] = make_int4((int)i, qv[i].x, qv[i].y, 0);
  }
  std::vector<uint32_t> len(n_nodes);
  for (uint32_t k = 0; k < n_nodes; k++) len[k] = seg[k + 1] - seg[k];
  const size_t cell = (size_t)ds->ftiles * nb * 2 * kHistFeat;
  std::vector<int32_t> mono(nf, 0);
  bool any_mono = false;
  for (uint32_t i = 0; i < std::min<uint32_t>(nf, p->monotone ? p->n_monotone : 0); i++) {
    mono[i] = p->monotone[i];
    any_mono |= mono[i] != 0;
  }
  DBuf<int2> dq;
  DBuf<int4> drows;
  DBuf<uint32_t> dlen, dmb;
  DBuf<long long> dhb, dhf, dmono_sums;
  DBuf<double> dterm;
  DBuf<SplitRec> drec;
  DBuf<int32_t> dmono;
  RW_CU(ctx, dq.alloc(n_pad));
  RW_CU(ctx, drows.alloc(rows.size()));
  RW_CU(ctx, dlen.alloc(n_nodes));
  RW_CU(ctx, dmb.alloc(2));
  RW_CU(ctx, dhb.alloc((size_t)n_nodes * cell));
  RW_CU(ctx, dhf.alloc((size_t)n_nodes * cell));
  RW_CU(ctx, dterm.alloc((size_t)nf * n_nodes * (nb - 1)));
  RW_CU(ctx, drec.alloc(nf));
  RW_CU(ctx, cudaMemcpy(dq.p, qv.data(), n_pad * sizeof(int2), cudaMemcpyHostToDevice));
  RW_CU(ctx, cudaMemcpy(drows.p, rows.data(), rows.size() * sizeof(int4), cudaMemcpyHostToDevice));
  RW_CU(ctx, cudaMemcpy(dlen.p, len.data(), n_nodes * 4, cudaMemcpyHostToDevice));
  RW_CU(ctx, cudaMemcpy(dmb.p, mbits, 8, cudaMemcpyHostToDevice));
  RW_CU(ctx, cudaMemset(dhb.p, 0, (size_t)n_nodes * cell * 8));
  if (any_mono) {
    RW_CU(ctx, dmono.alloc(nf));
    RW_CU(ctx, dmono_sums.alloc((size_t)nf * (nb - 1) * 4));
    RW_CU(ctx, cudaMemcpy(dmono.p, mono.data(), nf * 4, cudaMemcpyHostToDevice));
    RW_CU(ctx, cudaMemset(dmono_sums.p, 0, (size_t)nf * (nb - 1) * 4 * 8));
  }
  HistLaunch hl;
  hl.rowbins = ds->d_rowbins;
  hl.n_pad = n_pad;
  hl.packed = ds->packed;
  hl.err = nullptr;
  hl.q = dq.p;
  hl.entries = drows.p;
  hl.pcount = dlen.p;
  hl.glen = dlen.p;
  hl.parents = n_nodes;
  hl.pairs = 1;
  hl.n_ident = 0;
  hl.groups = n_nodes;
  hl.nf = nf;
  hl.nb = nb;
  hl.out = dhb.p;
  int nl = 0;
  RW_CU(ctx, launch_hist(hl, ctx->stream, &nl));
  SplitLaunch sl = {};
  sl.hb = dhb.p;
  sl.hp = nullptr;
  sl.hf = dhf.p;
  sl.n_nodes = n_nodes;
  sl.nf = nf;
  sl.nb = nb;
  sl.mode = 0;
  sl.maxbits = dmb.p;
  sl.lambda = (double)p->lambda;
  sl.min_child = (double)p->min_child_h;
  sl.lr = (double)p->learning_rate;
  sl.monotone = any_mono ? dmono.p : nullptr;
  sl.mono = any_mono ? dmono_sums.p : nullptr;
  sl.term = dterm.p;
  sl.prefix = nullptr;
  sl.colsample = p->colsample;
  sl.tree_seed = tree * 2654435761u + 0x455A4B41u;  // src/booster.rs:351
  sl.cuts = ds->d_cuts;
  sl.rec = drec.p;
  sl.last_level = 1;
  RW_CU(ctx, launch_split(sl, ctx->stream, &nl));
  RW_CU(ctx, cudaStreamSynchronize(ctx->stream));
  ctx->launches += nl;
  std::vector<SplitRec> rec(nf);
  RW_CU(ctx, cudaMemcpy(rec.data(), drec.p, nf * sizeof(SplitRec), cudaMemcpyDeviceToHost));
  // the cross-feature choice k_apply makes: highest gain, ties to the lowest feature,
  // feature 0 bin 0 when no split is feasible
  double best = -INFINITY;
  uint32_t bf = 0xffffffffu;
  for (uint32_t f = 0; f < nf; f++) {
    gain_out[f] = rec[f].gain;
    bin_out[f] = rec[f].bin;
    if (rec[f].gain > best) {
      best = rec[f].gain;
      bf = f;
    }
  }
  if (bf == 0xffffffffu) bf = 0;
  chosen[0] = bf;
  chosen[1] = best == -INFINITY ? 0u : rec[bf].bin;
  return RW_OK;
}

// ---- failure detection on one GPU: a peer that never signals -----------------------

// Two regions of the symmetric-region layout on this context's device: [0] plays this
// rank (0), [1] a rank 1 that never runs.
static int fake_peer_regions(rw_ctx* ctx, size_t bytes, char** r0, char** r1) {
  *r0 = *r1 = nullptr;
  RW_CU(ctx, cudaMalloc(reinterpret_cast<void**>(r0), bytes));
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(r1), bytes);
  if (e != cudaSuccess) {
    cudaFree(*r0);
    *r0 = nullptr;
    return cuda_fail(ctx, e, "cudaMalloc");
  }
  RW_CU(ctx, cudaMemset(*r0, 0, bytes));
  RW_CU(ctx, cudaMemset(*r1, 0, bytes));
  return RW_OK;
}

extern "C" int rw_debug_peer_wait(rw_ctx* ctx, int32_t mode, int64_t timeout_ms,
                                  int32_t* err_out, float* kernel_ms) {
  ctx = first_rank(ctx);
  if (!ctx || !err_out || !kernel_ms || mode < 0 || mode > 3 || timeout_ms < 1 ||
      timeout_ms > 10000)
    return fail(ctx, RW_ERR_ARG, "bad argument");
  RW_CU(ctx, cudaSetDevice(ctx->device));
  char *r0 = nullptr, *r1 = nullptr;
  int rc = fake_peer_regions(ctx, kPeerDataOff + (1u << 20), &r0, &r1);
  if (rc) return rc;
  PeerSet ps = {};
  ps.base[0] = r0;
  ps.base[1] = r1;
  ps.world = 2;
  ps.rank = 0;
  ps.timeout_ns = (uint64_t)timeout_ms * 1000000ull;
  const uint64_t epoch = 1;
  DBuf<int> err;
  DBuf<unsigned long long> data;
  cudaEvent_t a = nullptr, b = nullptr;
  cudaError_t e = err.alloc(1);
  if (e == cudaSuccess) e = data.alloc(16);
  if (e == cudaSuccess) e = cudaMemset(data.p, 0, 16 * 8);
  // mode 2: an earlier wait already expired on this rank
  const int err0 = mode == 2 ? 2 : 0;
  if (e == cudaSuccess) e = cudaMemcpy(err.p, &err0, 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess && (mode == 1 || mode == 3)) {
    // rank 1's signal in this rank's small word: the epoch, with its error bit (mode 1)
    const uint64_t v = 2 * epoch + (mode == 1 ? 1u : 0u);
    e = cudaMemcpy(r0 + sizeof(uint64_t), &v, 8, cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) e = cudaEventCreate(&a);
  if (e == cudaSuccess) e = cudaEventCreate(&b);
  int nl = 0;
  if (e == cudaSuccess) e = cudaEventRecord(a, ctx->stream);
  if (e == cudaSuccess) e = launch_peer_small(ps, data.p, 16, 0, epoch, err.p, ctx->stream, &nl);
  if (e == cudaSuccess) e = cudaEventRecord(b, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e == cudaSuccess) e = cudaEventElapsedTime(kernel_ms, a, b);
  if (e == cudaSuccess) e = cudaMemcpy(err_out, err.p, 4, cudaMemcpyDeviceToHost);
  if (a) cudaEventDestroy(a);
  if (b) cudaEventDestroy(b);
  cudaFree(r0);
  cudaFree(r1);
  ctx->launches += nl;
  if (e != cudaSuccess) return cuda_fail(ctx, e, "peer wait test");
  return RW_OK;
}

extern "C" int rw_debug_lonely_rank_ctx(int gpu_id, int64_t timeout_ms, rw_ctx** out) {
  if (!out || timeout_ms < 1 || timeout_ms > 10000) return fail(nullptr, RW_ERR_ARG, "bad argument");
  *out = nullptr;
  rw_ctx* ctx = nullptr;
  int rc = rw_ctx_create_rank(gpu_id, 0, 1, nullptr, &ctx);
  if (rc) return rc;
  // rank 0 of 2 with peer exchanges on; rank 1's region is a local buffer nobody signals
  const size_t bytes = 64u << 20;
  char *r0 = nullptr, *r1 = nullptr;
  rc = fake_peer_regions(ctx, bytes, &r0, &r1);
  if (rc) {
    std::string msg = ctx->last_error;
    rw_ctx_destroy(ctx);
    return fail(nullptr, rc, msg);
  }
  ctx->world = 2;
  ctx->sym = r0;
  ctx->sym_bytes = bytes;
  ctx->sym_peer[1] = r1;
  ctx->sym_peer_owned = true;
  ctx->peer_mode = 1;
  ctx->timeout_ms = timeout_ms;
  *out = ctx;
  return RW_OK;
}

extern "C" int rw_debug_binary_version(rw_ctx* ctx, int32_t* out) {
  ctx = first_rank(ctx);
  if (!ctx || !out) return fail(ctx, RW_ERR_ARG, "NULL argument");
  RW_CU(ctx, cudaSetDevice(ctx->device));
  int v = 0;
  RW_CU(ctx, kernel_binary_version(&v));
  *out = v;
  return RW_OK;
}

extern "C" int rw_debug_expf(rw_ctx* ctx, const float* x, uint64_t n, float* out_rw,
                             float* out_cuda) {
  ctx = first_rank(ctx);
  if (!ctx || !x || !out_rw || !out_cuda) return fail(ctx, RW_ERR_ARG, "NULL argument");
  RW_CU(ctx, cudaSetDevice(ctx->device));
  DBuf<float> dx, dr, dc;
  RW_CU(ctx, dx.alloc(n));
  RW_CU(ctx, dr.alloc(n));
  RW_CU(ctx, dc.alloc(n));
  RW_CU(ctx, cudaMemcpy(dx.p, x, n * 4, cudaMemcpyHostToDevice));
  RW_CU(ctx, launch_debug_expf(dx.p, n, dr.p, dc.p, ctx->stream));
  RW_CU(ctx, cudaStreamSynchronize(ctx->stream));
  RW_CU(ctx, cudaMemcpy(out_rw, dr.p, n * 4, cudaMemcpyDeviceToHost));
  RW_CU(ctx, cudaMemcpy(out_cuda, dc.p, n * 4, cudaMemcpyDeviceToHost));
  ctx->launches += 1;
  return RW_OK;
}
