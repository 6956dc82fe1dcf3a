// Cross-rank exchanges over NVLink peer memory (one process per GPU, world > 1).
//
// Every rank owns one "symmetric" device region of the same size and layout, mapped
// into every other rank by CUDA IPC (rwgpu.cu sets it up). It holds the per-level
// built histograms, the reduced copy, small exchange slots and the signal words:
//
//   [0, kPeerHdr)    signal words (u64 epochs written by the peers): small[kMaxPeers],
//                    arrive[kPeerMaxCtas][kMaxPeers], depart[kPeerMaxCtas][kMaxPeers]
//   [kPeerHdr, ...)  small slots [2 parities][kMaxPeers][kPeerSmallWords] u64
//   then             the buffers the caller places (built histograms, the sum)
//
// Each exchange carries an epoch, one higher than the last exchange on the context,
// identical on every rank because every rank issues the same exchanges in order. A rank
// signals a peer by storing 2*epoch + e into the peer's word for this rank (after a
// release fence at system scope; e = 1 when this rank's error word is set, so an error
// on one rank reaches every rank), and waits by polling its own words with relaxed loads
// until all reach the epoch, then an acquire fence. (On B200 a relaxed poll plus one
// fence costs about 0.6 us over an empty launch; acquire loads in the poll loop and a
// counter shared by all CTAs cost several microseconds more.) Waits are bounded by a
// %globaltimer limit; on expiry the kernel sets the error word to 2 and returns (the
// host reports RW_ERR_TIMEOUT), and later exchanges skip their waits. Error word: 1 a
// histogram copy wait expired, 2 a peer wait expired, 3 a peer reported an error.
//
//   k_peer_sum_i64   two-shot all-reduce (sum) of int64 words, src -> dst on every rank,
//                    by stores only: rank q pushes its copy of slice r into rank r's
//                    receive area, rank r adds the W copies of slice r and pushes the
//                    sums into every rank's dst; (W-1)/W of the bytes cross NVLink in
//                    each direction, as in a ring all-reduce, in one launch. CTA b of
//                    every rank meets CTA b of every other rank only: after the scatter
//                    (every rank's part b of the copies has landed here) and after the
//                    gather (every rank's part b of the sums has landed here), so no CTA
//                    waits for another CTA of its own grid. The receive area is doubled
//                    by epoch parity, so a rank that runs one exchange ahead never
//                    overwrites copies a slower rank is still adding.
//   k_peer_sum1_i64  one-shot all-reduce for 2 ranks: every rank
//                    pushes its whole src into every rank's receive area, CTA b of every
//                    rank meets CTA b of every other rank once, and every rank adds the
//                    W copies into its own dst (one barrier instead of two).
//   k_peer_small     one-shot all-reduce of up to kPeerSmallWords words (u64 sum or u32
//                    max): each rank stores its words into slot [rank] of every rank,
//                    then reduces the W slots in rank order. The round's fixed-point
//                    maxima and the GOSS digit counts.
//
// Integer sums are exact in any order, so the result equals the NCCL all-reduce.
#include <cuda_runtime.h>
#include <stdint.h>

#include "rw_internal.cuh"

namespace {

constexpr int kPeerThreads = 256;

// signal words: kind 0 small (one per rank), 1 arrive and 2 depart (per CTA and rank)
__device__ __forceinline__ uint64_t* sig(char* base, int kind, uint32_t cta) {
  uint64_t* w = reinterpret_cast<uint64_t*>(base);
  return kind == 0 ? w : w + kMaxPeers * (1 + (size_t)(kind - 1) * kPeerMaxCtas + cta);
}

__device__ __forceinline__ void st_relaxed_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Tell every rank that this rank has reached `epoch`: a release fence (this thread's
// prior writes, and those ordered before them by the CTA barrier), then the stores.
__device__ void signal_all(const PeerSet& ps, int kind, uint32_t cta, uint64_t epoch,
                           const int* err) {
  fence_acq_rel_sys();
  const uint64_t v = 2 * epoch + (*reinterpret_cast<const volatile int*>(err) != 0 ? 1u : 0u);
  for (int r = 0; r < ps.world; r++) st_relaxed_sys(sig(ps.base[r], kind, cta) + ps.rank, v);
}

// Wait until every rank has signalled `epoch` into this rank's words (then an acquire
// fence); false when the wait expires (error word 2) or an earlier one did.
__device__ bool wait_all(const PeerSet& ps, int kind, uint32_t cta, uint64_t epoch, int* err) {
  if (*reinterpret_cast<volatile int*>(err) == 2) return false;
  const uint64_t* w = sig(ps.base[ps.rank], kind, cta);
  const uint64_t t0 = globaltimer_ns();
  bool peer_err = false;
  for (int r = 0; r < ps.world; r++) {
    uint64_t v;
    while (((v = ld_relaxed_sys(w + r)) >> 1) < epoch) {
      if (globaltimer_ns() - t0 > ps.timeout_ns) {
        atomicExch(err, 2);
        return false;
      }
    }
    peer_err |= (v & 1u) != 0;
  }
  fence_acq_rel_sys();
  if (peer_err) atomicCAS(err, 0, 3);
  return true;
}

__device__ __forceinline__ void pdl_wait_only() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// W ranks known at compile time. Push-only two-shot: rank q stores its src slice r into
// rank r's receive area [parity][q] (remote stores, posted), CTA b of every rank meets
// CTA b of every other rank, then rank r adds its own slice r to the W - 1 received
// copies (local loads) and stores the sums into every rank's dst; a second meeting of
// the CTAs b ends it. No NVLink loads: every byte crosses as a store. Each thread moves
// U = 16 / W vectors per step.
template <int W>
__global__ void __launch_bounds__(kPeerThreads) k_peer_sum_i64(PeerSet ps, uint64_t src_off,
                                                               uint64_t dst_off, uint64_t recv_off,
                                                               uint64_t recv_half, uint64_t words,
                                                               uint64_t epoch, int* err) {
  constexpr int U = 16 / W;
  pdl_wait_only();  // this rank's src is complete
  __shared__ int s_ok;
  const uint64_t nvec = words / 2;
  const uint64_t per = (nvec + W - 1) / W;  // vectors of one slice
  const uint32_t me = (uint32_t)ps.rank;
  const uint64_t parity = epoch & 1u;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t j0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const longlong2* src = reinterpret_cast<const longlong2*>(ps.base[me] + src_off);
  // rank r's receive area for the copy from rank q
  auto recv = [&](uint32_t q, uint32_t r) {
    return reinterpret_cast<longlong2*>(ps.base[r] + recv_off) + parity * recv_half + q * per;
  };
  // phase 1: scatter the other ranks' slices
  for (uint64_t j = j0; j < per; j += U * stride) {
    longlong2 x[U][W];
#pragma unroll
    for (int u = 0; u < U; u++)
#pragma unroll
      for (int r = 0; r < W; r++) {
        const uint64_t ju = j + u * stride, v = (uint64_t)r * per + ju;
        x[u][r] = (r != (int)me && ju < per && v < nvec) ? __ldcg(src + v) : make_longlong2(0, 0);
      }
#pragma unroll
    for (int u = 0; u < U; u++)
#pragma unroll
      for (int r = 0; r < W; r++) {
        const uint64_t ju = j + u * stride, v = (uint64_t)r * per + ju;
        if (r != (int)me && ju < per && v < nvec) recv(me, r)[ju] = x[u][r];
      }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    signal_all(ps, 1, blockIdx.x, epoch, err);
    s_ok = wait_all(ps, 1, blockIdx.x, epoch, err);
  }
  __syncthreads();
  if (s_ok) {
    // phase 2: this rank's slice, its own copy plus the received ones, to every rank
    longlong2* dst[W];
#pragma unroll
    for (int r = 0; r < W; r++) dst[r] = reinterpret_cast<longlong2*>(ps.base[r] + dst_off);
    for (uint64_t j = j0; j < per; j += U * stride) {
      longlong2 x[U][W];
#pragma unroll
      for (int u = 0; u < U; u++)
#pragma unroll
        for (int q = 0; q < W; q++) {
          const uint64_t ju = j + u * stride, v = (uint64_t)me * per + ju;
          x[u][q] = (ju < per && v < nvec)
                        ? (q == (int)me ? __ldcg(src + v) : __ldcv(recv(q, me) + ju))
                        : make_longlong2(0, 0);
        }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const uint64_t ju = j + u * stride, v = (uint64_t)me * per + ju;
        if (ju >= per || v >= nvec) break;
        longlong2 sum = make_longlong2(0, 0);
#pragma unroll
        for (int q = 0; q < W; q++) {
          sum.x += x[u][q].x;
          sum.y += x[u][q].y;
        }
#pragma unroll
        for (int r = 0; r < W; r++) dst[r][v] = sum;
      }
    }
  }
  // The next kernel may launch now; it waits for this grid to complete before it reads.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // The CTA's stores are ordered before thread 0's release by the barrier; CTA b then
  // tells every rank that its part b has landed and waits for every rank's part b.
  __syncthreads();
  if (threadIdx.x == 0 && s_ok) {
    signal_all(ps, 2, blockIdx.x, epoch, err);
    wait_all(ps, 2, blockIdx.x, epoch, err);
  }
}

// One-shot variant for 2 ranks: rank q pushes its whole src into every rank's receive
// area [parity][q], CTA b of every rank meets CTA b of every other rank once, and every
// rank adds the W copies itself (local loads, local dst). One barrier instead of two;
// (W-1) x the bytes leave each rank, the same as the two-shot's 2 (W-1)/W x at W = 2.
template <int W>
__global__ void __launch_bounds__(kPeerThreads) k_peer_sum1_i64(PeerSet ps, uint64_t src_off,
                                                                uint64_t dst_off, uint64_t recv_off,
                                                                uint64_t recv_half, uint64_t words,
                                                                uint64_t epoch, int* err) {
  constexpr int U = 16 / W;
  pdl_wait_only();  // this rank's src is complete
  __shared__ int s_ok;
  const uint64_t nvec = words / 2;
  const uint32_t me = (uint32_t)ps.rank;
  const uint64_t parity = epoch & 1u;
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t j0 = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const longlong2* src = reinterpret_cast<const longlong2*>(ps.base[me] + src_off);
  auto recv = [&](uint32_t q, uint32_t r) {
    return reinterpret_cast<longlong2*>(ps.base[r] + recv_off) + parity * recv_half + q * nvec;
  };
  for (uint64_t j = j0; j < nvec; j += U * stride) {
    longlong2 x[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint64_t ju = j + u * stride;
      x[u] = ju < nvec ? __ldcg(src + ju) : make_longlong2(0, 0);
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint64_t ju = j + u * stride;
      if (ju >= nvec) break;
#pragma unroll
      for (int r = 0; r < W; r++)
        if (r != (int)me) recv(me, r)[ju] = x[u];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    signal_all(ps, 1, blockIdx.x, epoch, err);
    s_ok = wait_all(ps, 1, blockIdx.x, epoch, err);
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (!s_ok) return;
  longlong2* dst = reinterpret_cast<longlong2*>(ps.base[me] + dst_off);
  for (uint64_t j = j0; j < nvec; j += U * stride) {
    longlong2 x[U][W];
#pragma unroll
    for (int u = 0; u < U; u++)
#pragma unroll
      for (int q = 0; q < W; q++) {
        const uint64_t ju = j + u * stride;
        x[u][q] = ju < nvec ? (q == (int)me ? __ldcg(src + ju) : __ldcv(recv(q, me) + ju))
                            : make_longlong2(0, 0);
      }
#pragma unroll
    for (int u = 0; u < U; u++) {
      const uint64_t ju = j + u * stride;
      if (ju >= nvec) break;
      longlong2 sum = make_longlong2(0, 0);
#pragma unroll
      for (int q = 0; q < W; q++) {
        sum.x += x[u][q].x;
        sum.y += x[u][q].y;
      }
      dst[ju] = sum;
    }
  }
}

__global__ void __launch_bounds__(kPeerThreads) k_peer_small(PeerSet ps, void* data, uint32_t n,
                                                             int max_u32, uint64_t epoch,
                                                             int* err) {
  pdl_wait_only();
  __shared__ int s_ok;
  const int parity = (int)(epoch & 1u);
  auto slot = [&](int owner, int from) {
    return reinterpret_cast<uint64_t*>(ps.base[owner] + kPeerHdr) +
           ((size_t)parity * kMaxPeers + from) * kPeerSmallWords;
  };
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    const uint64_t v = max_u32 ? (uint64_t) reinterpret_cast<const uint32_t*>(data)[i]
                               : reinterpret_cast<const uint64_t*>(data)[i];
    for (int r = 0; r < ps.world; r++) slot(r, ps.rank)[i] = v;
  }
  __syncthreads();  // the slot stores precede thread 0's release (signal_all fences)
  if (threadIdx.x == 0) {
    signal_all(ps, 0, 0, epoch, err);
    s_ok = wait_all(ps, 0, 0, epoch, err);
  }
  __syncthreads();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (!s_ok) return;
  for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
    uint64_t acc = 0;
    for (int r = 0; r < ps.world; r++) {
      const uint64_t v = __ldcv(reinterpret_cast<const unsigned long long*>(slot(ps.rank, r)) + i);
      acc = max_u32 ? (v > acc ? v : acc) : acc + v;
    }
    if (max_u32) reinterpret_cast<uint32_t*>(data)[i] = (uint32_t)acc;
    else reinterpret_cast<uint64_t*>(data)[i] = acc;
  }
}

template <typename... KArgs, typename... Args>
cudaError_t launch_after(void (*k)(KArgs...), dim3 grid, dim3 block, cudaStream_t s,
                         Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, args...);
}

}  // namespace

cudaError_t launch_peer_sum_i64(const PeerSet& ps, uint64_t src_off, uint64_t dst_off,
                                uint64_t recv_off, uint64_t recv_half, uint64_t words,
                                uint64_t epoch, int* err, cudaStream_t s, int* nl) {
  if (ps.world < 2 || ps.world > kMaxPeers || (words & 1u) || (src_off | dst_off | recv_off) % 16)
    return cudaErrorInvalidValue;
  // One-shot for 2 ranks (the same bytes as two-shot, one barrier), two-shot for more.
  // A context keeps one kind: the two lay out the receive area differently, and the
  // one-shot ends without a second barrier, so mixing them would let a fast rank's next
  // copies land where a slow rank is still adding.
  const bool one_shot = ps.world == 2;
  const uint64_t per = one_shot ? words / 2 : (words / 2 + ps.world - 1) / ps.world;
  // the W copies of this exchange fit in one parity half of the receive area
  if ((uint64_t)ps.world * per > recv_half) return cudaErrorInvalidValue;
  // 16 / W vectors per thread per step; at most kPeerMaxCtas CTAs (each with its signal
  // words), fewer for small exchanges
  const uint64_t per_cta = (uint64_t)kPeerThreads * (16 / ps.world);
  uint64_t blocks = (per + per_cta - 1) / per_cta;
  blocks = blocks < 1 ? 1 : (blocks > (uint64_t)kPeerMaxCtas ? (uint64_t)kPeerMaxCtas : blocks);
  const dim3 g((unsigned)blocks), b(kPeerThreads);
  cudaError_t e;
  if (one_shot) {
    e = launch_after(k_peer_sum1_i64<2>, g, b, s, ps, src_off, dst_off, recv_off, recv_half,
                     words, epoch, err);
  } else {
#define RW_PEER_CASE(w)                                                                   \
  case w:                                                                               \
    e = launch_after(k_peer_sum_i64<w>, g, b, s, ps, src_off, dst_off, recv_off, recv_half, \
                     words, epoch, err);                                                \
    break;
    switch (ps.world) {
      RW_PEER_CASE(3)
      RW_PEER_CASE(4)
      RW_PEER_CASE(5)
      RW_PEER_CASE(6)
      RW_PEER_CASE(7)
      default:
        e = launch_after(k_peer_sum_i64<8>, g, b, s, ps, src_off, dst_off, recv_off, recv_half,
                         words, epoch, err);
        break;
    }
#undef RW_PEER_CASE
  }
  if (e == cudaSuccess && nl) (*nl)++;
  return e;
}

cudaError_t launch_peer_small(const PeerSet& ps, void* data, uint32_t n, int max_u32,
                              uint64_t epoch, int* err, cudaStream_t s, int* nl) {
  if (ps.world < 2 || ps.world > kMaxPeers || n > (uint32_t)kPeerSmallWords)
    return cudaErrorInvalidValue;
  cudaError_t e = launch_after(k_peer_small, dim3(1), dim3(kPeerThreads), s, ps, data, n, max_u32,
                               epoch, err);
  if (e == cudaSuccess && nl) (*nl)++;
  return e;
}
