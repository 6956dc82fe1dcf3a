// Cross-rank exchanges over NVLink peer memory (one process per GPU, world > 1).
//
// Every rank owns one "symmetric" device region of the same size and layout, mapped
// into every other rank by CUDA IPC (rwgpu.cu sets it up). It holds the per-level
// built histograms, the reduced copy, small exchange slots and the signal words:
//
//   [0, kPeerHdr)    signal words: arrive[kMaxPeers], depart[kMaxPeers], small[kMaxPeers]
//                    (u64 epochs written by the peers), done counter (u32, local)
//   [kPeerHdr, ...)  small slots [2 parities][kMaxPeers][kPeerSmallWords] u64
//   then             the buffers the caller places (built histograms, the sum)
//
// Each exchange carries an epoch, one higher than the last exchange on the context,
// identical on every rank because every rank issues the same exchanges in order. A
// rank signals a peer by storing 2*epoch + e into the peer's word for this rank (release
// at system scope; e = 1 when this rank's error word is set, so an error on one rank
// reaches every rank) and waits until all its words have reached the epoch (acquire).
// Waits are bounded by a %globaltimer limit; on expiry the kernel sets the error word
// to 2 and returns (the host reports RW_ERR_TIMEOUT), and later exchanges skip their
// waits. Error word: 1 a histogram copy wait expired, 2 a peer wait expired, 3 a peer
// reported an error.
//
//   k_peer_sum_i64   two-shot all-reduce (sum) of int64 words, src -> dst on every rank:
//                    rank r reduces slice r of the words over all ranks (its own copy
//                    and W-1 peer loads) and stores the sums into every rank's dst.
//                    The per-level histograms: (W-1)/W of the bytes cross NVLink in
//                    each direction, as in a ring all-reduce, in one launch.
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

__device__ __forceinline__ uint64_t* sig(char* base, int kind) {
  return reinterpret_cast<uint64_t*>(base) + kind * kMaxPeers;
}
__device__ __forceinline__ unsigned int* done_counter(char* base) {
  return reinterpret_cast<unsigned int*>(base + 3 * kMaxPeers * sizeof(uint64_t));
}

__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Tell every rank that this rank has reached `epoch` (kind: which signal words).
__device__ void signal_all(const PeerSet& ps, int kind, uint64_t epoch, const int* err) {
  __threadfence_system();
  const uint64_t v = 2 * epoch + (*reinterpret_cast<const volatile int*>(err) != 0 ? 1u : 0u);
  for (int r = 0; r < ps.world; r++) st_release_sys(sig(ps.base[r], kind) + ps.rank, v);
}

// Wait until every rank has signalled `epoch` into this rank's words; false when the
// wait expires (error word 2) or an earlier one did.
__device__ bool wait_all(const PeerSet& ps, int kind, uint64_t epoch, int* err) {
  if (*reinterpret_cast<volatile int*>(err) == 2) return false;
  const uint64_t* w = sig(ps.base[ps.rank], kind);
  const uint64_t t0 = globaltimer_ns();
  bool peer_err = false;
  for (int r = 0; r < ps.world; r++) {
    uint64_t v;
    while (((v = ld_acquire_sys(w + r)) >> 1) < epoch) {
      if (globaltimer_ns() - t0 > ps.timeout_ns) {
        atomicExch(err, 2);
        return false;
      }
      __nanosleep(64);
    }
    peer_err |= (v & 1u) != 0;
  }
  if (peer_err) atomicCAS(err, 0, 3);
  return true;
}

__device__ __forceinline__ void pdl_wait_only() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// W ranks known at compile time: each thread sums U = 16 / W vectors per step with all
// W * U loads in flight before the adds.
template <int W>
__global__ void __launch_bounds__(kPeerThreads) k_peer_sum_i64(PeerSet ps, uint64_t src_off,
                                                               uint64_t dst_off, uint64_t words,
                                                               uint64_t epoch, int* err) {
  constexpr int U = 16 / W;
  // Waits for the producing kernel; does not let the next kernel start early, so every
  // CTA of this grid is resident before a dependent grid can take SM resources.
  pdl_wait_only();
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) signal_all(ps, kPeerArrive, epoch, err);  // this rank's src is complete
    s_ok = wait_all(ps, kPeerArrive, epoch, err);
  }
  __syncthreads();
  if (s_ok) {
    // slice of 2-word vectors owned by this rank
    const uint64_t nvec = words / 2;
    const uint64_t per = (nvec + W - 1) / W;
    const uint64_t v0 = per * ps.rank, v1 = min(nvec, v0 + per);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const longlong2* src[W];
    longlong2* dst[W];
#pragma unroll
    for (int r = 0; r < W; r++) {
      src[r] = reinterpret_cast<const longlong2*>(ps.base[r] + src_off);
      dst[r] = reinterpret_cast<longlong2*>(ps.base[r] + dst_off);
    }
    for (uint64_t v = v0 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; v < v1;
         v += U * stride) {
      longlong2 x[U][W];
#pragma unroll
      for (int u = 0; u < U; u++)
#pragma unroll
        for (int r = 0; r < W; r++) {
          const uint64_t vu = v + u * stride;
          x[u][r] = vu < v1 ? (r == ps.rank ? __ldcg(src[r] + vu) : __ldcv(src[r] + vu))
                            : make_longlong2(0, 0);
        }
#pragma unroll
      for (int u = 0; u < U; u++) {
        const uint64_t vu = v + u * stride;
        if (vu >= v1) break;
        longlong2 sum = make_longlong2(0, 0);
#pragma unroll
        for (int r = 0; r < W; r++) {
          sum.x += x[u][r].x;
          sum.y += x[u][r].y;
        }
#pragma unroll
        for (int r = 0; r < W; r++) dst[r][vu] = sum;
      }
    }
  }
  // The next kernel may launch now; it waits for this grid to complete before it reads.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // The CTA's stores are ordered before its count by the barrier and one system-scope
  // fence (cumulative); the last CTA of this rank tells every rank that its slice has
  // landed, then waits for all ranks' slices.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    unsigned int* done = done_counter(ps.base[ps.rank]);
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      atomicExch(done, 0u);
      if (s_ok) {
        signal_all(ps, kPeerDepart, epoch, err);
        wait_all(ps, kPeerDepart, epoch, err);
      }
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
    signal_all(ps, kPeerSmall, epoch, err);
    s_ok = wait_all(ps, kPeerSmall, epoch, err);
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
                                uint64_t words, uint64_t epoch, int* err, cudaStream_t s,
                                int* nl) {
  if (ps.world < 2 || ps.world > kMaxPeers || (words & 1u) || (src_off | dst_off) % 16)
    return cudaErrorInvalidValue;
  const uint64_t per = (words / 2 + ps.world - 1) / ps.world;
  uint64_t blocks = (per + kPeerThreads - 1) / kPeerThreads;
  // one wave (two CTAs per SM at most): every CTA is resident while CTA 0 signals
  blocks = blocks < 1 ? 1 : (blocks > 296 ? 296 : blocks);
  const dim3 g((unsigned)blocks), b(kPeerThreads);
  cudaError_t e;
  switch (ps.world) {
    case 2: e = launch_after(k_peer_sum_i64<2>, g, b, s, ps, src_off, dst_off, words, epoch, err); break;
    case 3: e = launch_after(k_peer_sum_i64<3>, g, b, s, ps, src_off, dst_off, words, epoch, err); break;
    case 4: e = launch_after(k_peer_sum_i64<4>, g, b, s, ps, src_off, dst_off, words, epoch, err); break;
    case 5: e = launch_after(k_peer_sum_i64<5>, g, b, s, ps, src_off, dst_off, words, epoch, err); break;
    case 6: e = launch_after(k_peer_sum_i64<6>, g, b, s, ps, src_off, dst_off, words, epoch, err); break;
    case 7: e = launch_after(k_peer_sum_i64<7>, g, b, s, ps, src_off, dst_off, words, epoch, err); break;
    default: e = launch_after(k_peer_sum_i64<8>, g, b, s, ps, src_off, dst_off, words, epoch, err); break;
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
