// Internal declarations shared by the rwgpu translation units.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

#include <algorithm>
#include <condition_variable>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/rwgpu.h"

// Cross-rank exchange over NVLink peer memory (peer_kernels.cu): every rank's symmetric
// region, mapped into every rank. Layout: signal words, then the small-exchange slots,
// then caller-placed buffers from kPeerDataOff.
constexpr int kMaxPeers = 8;
constexpr int kPeerMaxCtas = 148;  // CTAs of one all-reduce (each has its own signal words)
// signal words: small[kMaxPeers], then arrive and depart [kPeerMaxCtas][kMaxPeers] (u64)
constexpr size_t kPeerHdr = 64 * 1024;
static_assert((1 + 2 * (size_t)kPeerMaxCtas) * kMaxPeers * 8 <= kPeerHdr, "signal words fit");
// one-shot exchange slots: the round maxima, GOSS digit counts and the per-tree leaf
// sums ([2][2^depth] int64, up to 8192 words at depth 12)
constexpr int kPeerSmallWords = 8192;
constexpr size_t kPeerDataOff = kPeerHdr + 2 * (size_t)kMaxPeers * kPeerSmallWords * 8;
struct PeerSet {
  char* base[kMaxPeers];  // each rank's region as mapped in this process (own at [rank])
  int world, rank;
  uint64_t timeout_ns;    // bound of every wait on a peer
};

// The ranks of one multi-GPU context created in-process (rw_ctx_create with n_gpus > 1):
// a host rendezvous with a bounded wait, and each rank's symmetric region as a plain
// device pointer (peer access is enabled between the ranks' devices, no IPC).
struct RankGroup {
  int n = 0;
  std::mutex mu;
  std::condition_variable cv;
  int arrived = 0;
  uint64_t gen = 0;
  int acc = 0, result = 0;     // min over the ranks of the values they bring
  bool broken = false;         // a rank gave up waiting (or failed): every later meeting fails
  bool peer_ok = false;        // every pair of devices has peer access
  std::vector<char*> sym;      // each rank's region, published at the meeting
};

struct rw_ctx {
  int device = 0;
  int rank = 0;
  int world = 1;
  cudaStream_t stream = nullptr;
  // Stream-ordered pool for datasets and working buffers; it keeps freed memory, so
  // repeated fits (rw_fit, a serving loop) allocate without device synchronisation.
  cudaMemPool_t pool = nullptr;
  ncclComm_t comm = nullptr;
  int64_t timeout_ms = 60000;
  std::string last_error;
  uint64_t launches = 0;  // kernels launched on this context (all time)
  // world > 1: the symmetric region (cudaMalloc, exported by IPC) and its peer mappings
  char* sym = nullptr;
  size_t sym_bytes = 0;
  char* sym_peer[kMaxPeers] = {};
  uint64_t peer_epoch = 0;   // exchanges issued on the region (identical on every rank)
  int peer_mode = -1;        // -1 undecided, 0 NCCL, 1 peer memory
  bool peer_failed = false;  // a bounded wait expired: the region's epochs are unusable
  bool sym_peer_owned = false;  // test contexts: the peer regions are local allocations
  // in-process ranks: the shared group (each rank), or the ranks this context drives
  // (the context rw_ctx_create returned for several GPUs; it owns no stream itself)
  std::shared_ptr<RankGroup> group;
  std::vector<rw_ctx*> members;
  // Large pageable host inputs are copied through pinned slots (two per worker thread,
  // created on first use): the workers' memcpy into one slot overlaps the copy engine's
  // drain of the other. See upload_h2d.
  static constexpr int kStageWorkers = 4;
  void* stage_host[2 * kStageWorkers] = {};
  cudaEvent_t stage_ev[2 * kStageWorkers] = {};
  bool stage_used[2 * kStageWorkers] = {};
  cudaStream_t stage_stream[kStageWorkers] = {};
};

// Bins are stored twice in HBM:
//   colbins  feature-major u8 [nf][n_pad]: the split feature's column read by the leaf-index
//            update, and the host-visible copy;
//   rowbins  tile-major [ftiles][n_pad][tile bytes]: features in tiles of kHistFeat, each
//            row's tile t is one contiguous run of kHistFeat bytes (u8) or kHistFeat/2 bytes
//            (4-bit pairs, the even feature in the low nibble), so the histogram build
//            gathers a row's tile in one access and streams a tile's rows sequentially.
constexpr uint32_t kHistFeat = 64;

struct rw_dataset {
  rw_ctx* ctx = nullptr;
  uint64_t n = 0;         // local rows
  uint64_t n_pad = 0;     // rows rounded up (padded rows carry g = h = 0)
  uint64_t n_global = 0;  // rows across all ranks
  uint64_t row_offset = 0;
  uint32_t nf = 0, n_bins = 0;
  int packed = 0;
  uint32_t ftiles = 0;           // ceil(nf / kHistFeat)
  uint8_t* d_colbins = nullptr;  // u8 [nf][n_pad]
  uint8_t* d_rowbins = nullptr;  // [ftiles][n_pad][tile bytes], u8 or 4-bit pairs
  float* d_y = nullptr;          // [n_pad]
  float* d_cuts = nullptr;       // [nf][n_bins-1]
  std::vector<float> cuts;
  // Working buffers of the boosting loop, kept across fits (named, grown on demand).
  std::map<std::string, std::pair<void*, size_t>> ws;
  // A dataset of a multi-GPU context: one contiguous row shard per rank (shard i on
  // ctx->members[i]); the fields above describe the whole dataset.
  std::vector<rw_dataset*> shards;
  std::vector<uint64_t> shard_lo;
};

struct rw_dmodel {
  rw_ctx* ctx = nullptr;
  uint32_t n_trees = 0, depth = 0, nf = 0;
  float base = 0.f;
  uint32_t* d_feat = nullptr;
  float* d_thr = nullptr;
  uint32_t* d_split8 = nullptr;  // (feat << 8) | thr_bin per slot, for the u8 scorer
  float* d_leafval = nullptr;
  int has_bins = 0;
};

// Runs fn(i) for every rank of a multi-GPU context (ctx->members), one host thread per
// rank, and returns the first failure (its message on the front context).
int for_each_rank(rw_ctx* front, const std::function<int(int)>& fn);

// ---- kernel launchers (train_kernels.cu) ------------------------------------------

// One level's histogram build. Without a list, every row in [0, n_ident) belongs to
// group 0 (q from `q`). With a list, the entries (row id, q(g), q(h), 0) of the previous
// level's node k occupy the region [cap(k), cap(k) + pcount[k]) of `entries`, cap = the
// exclusive prefix of pcount (rows per node). With pairs != 0 group k is node k's built
// child: its glen[k] entries start the region. With pairs == 0 group c is child c of node
// c/2: the left child's glen[c] entries start the region, the right child's end it.
struct HistLaunch {
  const uint8_t* rowbins;
  uint64_t n_pad;         // rows per tile in rowbins
  int packed;
  const int2* q;          // per row: (fixed-point g, fixed-point h), rw_quantize
  const int4* entries;    // the list, or nullptr for every row
  const uint32_t* pcount; // [parents] non-excluded rows per previous-level node
  const uint32_t* glen;   // [groups] entries per group
  uint32_t parents;       // previous-level nodes
  int pairs;              // 1: group k = node k's built child; 0: group c = child c
  uint32_t n_ident;       // identity list length, a multiple of 512 (rows past n have q = 0)
  uint32_t groups;        // histogram groups written (out has `groups` slots)
  uint32_t nf, nb;
  long long* out;         // int64 [groups][tile][nb][2][64], zeroed by the caller
  int* err;               // nullable: set to 1 if a bounded wait on a bulk copy gave up
};
cudaError_t launch_hist(const HistLaunch& a, cudaStream_t s, int* n_launch);

// Per-level row lists. At level d the leaf-index update writes, for the next level, the
// entries of the rows to build into per-node regions sized by the node's row count
// (ncount, known before the rows move), so no pass over all rows is needed to size them.
struct LevelLists {
  int4* entries;          // [n_pad] (row, q(g), q(h), 0)
  const int2* q;          // per row q, copied into the entries
  const uint32_t* ncount; // [n_nodes] non-excluded rows per node of this level
  uint32_t* cursor;       // [groups] entries written per next-level group (zeroed before)
  const uint8_t* choice;  // [nf][n_nodes] per feature: 1 = build the right (odd) child
  uint8_t* built_odd;     // [n_nodes] out: the winning feature's choice row
  int subtract;           // 1: list the built child of each pair; 0: list every child
};

// A feature's best split at one level: gain (-inf when no bin is feasible), threshold
// bin and its cut value.
struct SplitRec {
  double gain;
  uint32_t bin;
  float thr;
};

struct SplitLaunch {
  const long long* hb;  // built histogram
  const long long* hp;  // parent level full histogram (mode 1)
  long long* hf;        // this level's full histogram (out)
  uint32_t n_nodes, nf, nb;
  int mode;             // 0: hb holds every node; 1: hb holds one child per pair, keyed by parent
  const uint8_t* built_odd;  // mode 1: per pair, 1 if the odd child was built (else the even)
  const uint32_t* maxbits;
  double lambda, min_child, lr;
  const int32_t* monotone;  // device [nf] or null
  long long* mono;      // with monotone: [nf][nb-1][4] exact left/right sums, zero on entry
  double* term;         // [nf][n_nodes][nb-1] per-node gain terms
  long long* prefix;    // non-last levels with subtraction: [nf][n_nodes][nb] exact
                        // per-node hessian prefixes over bins, for the built-child choice;
                        // or null
  float colsample;
  uint32_t tree_seed;
  const float* cuts;
  SplitRec* rec;        // [nf] out
  int last_level;
  uint8_t* choice;      // non-last levels, with subtraction: [nf][n_nodes] out, 1 = build
                        // the right (odd) child of the node (the side with less hessian)
  // per-node row counts of this level from the previous level's lists (level > 0):
  // ncount[c] = cursor_prev[c/2] for the built child, pcount[c/2] - that for its sibling
  // (with subtraction), or cursor_prev[c] (without); cursor_next is zeroed.
  const uint32_t* pcount;
  const uint32_t* cursor_prev;
  const uint8_t* built_prev;
  uint32_t* ncount;
  uint32_t* cursor_next;
  uint32_t cursor_next_words;
  int subtract;
};
cudaError_t launch_split(const SplitLaunch& a, cudaStream_t s, int* nl);

// Rows are padded to a multiple of kRowAlign (whole 4-row steps for every kernel).
constexpr uint64_t kRowAlign = 4096;

// Bins both layouts (colbins u8; rowbins u8, packed to 4-bit pairs by launch_pack4).
cudaError_t launch_bin(const float* x_rowmajor, uint64_t n, uint32_t nf, const float* d_cuts,
                       uint32_t n_bins, uint64_t n_pad, uint8_t* d_colbins, uint8_t* d_rowbins,
                       cudaStream_t s, int* nl);
// rowbins u8 -> 4-bit pairs (separate buffers).
cudaError_t launch_pack4(const uint8_t* d_u8, uint64_t n_pad, uint32_t nf, uint8_t* d_packed,
                         cudaStream_t s, int* nl);
// A tree's leaf values from its per-leaf exact sums of the unquantised g and h in the
// wide fixed point (rw_wquantize, [2][n_leaves] int64, all ranks' rows) and that round's
// maxima: leafval[l] = (float)(-lr * G / (H + lambda)) (src/cpu.rs:316-317).
struct LeafValues {
  const long long* leafsum;
  const uint32_t* maxbits;
  uint32_t n_leaves;
  uint64_t n_rows;  // global row count (the wide scale's row bound)
  double lr, lambda;
  float* leafval;   // out: the tree's slot of the model's leaf values
  const long long* leafsum2 = nullptr;  // PGBM: per-leaf wide sums of g^2, or null
  float* leafvar = nullptr;  // PGBM out: the tree's slot of the leaf variances (with leafsum2)
};
cudaError_t launch_leafval(const LeafValues& a, cudaStream_t s, int* nl);
// Target encoding on the GPU (encode.cu): the test-set maps of the categorical features,
// as dense tables over each feature's key range.
struct rw_encoders {
  std::vector<long long> key_lo;   // [n_cat] first key of each feature's table
  std::vector<uint64_t> koff;      // [n_cat] first slot of each feature in value/present
  std::vector<uint64_t> n_keys;    // [n_cat] slots per feature
  std::vector<float> value;        // smoothed full-train mean per key
  std::vector<uint8_t> present;    // key seen in training
  float gmean = 0.0f;
};
int target_encode_device(rw_ctx* ctx, float* d_x, const float* d_y, uint64_t n, uint32_t nf,
                         const uint32_t* cat, uint32_t n_cat, float smoothing, uint32_t k_folds,
                         uint64_t hash_buckets, float* gmean_out, rw_encoders* enc,
                         std::string* why);
int target_transform_device(rw_ctx* ctx, float* d_x, uint64_t n, uint32_t nf, const uint32_t* cat,
                            uint32_t n_cat, const rw_encoders& enc, uint64_t hash_buckets,
                            std::string* why);

// PGBM: every row's g^2 (f32) in the wide fixed point into its leaf's exact int64 sum
// (the leaf_g2 sums of gpu_kernels.rs:1015-1043); run after the tree's last level.
struct LeafSquares {
  const uint16_t* node;  // the rows' leaf indices (low 15 bits)
  const float* g;        // 0 for unsampled and padded rows
  uint64_t n_pad;
  const uint32_t* maxbits;
  uint64_t n_rows;  // global row count (the wide scale's row bound)
  uint32_t n_leaves;
  long long* leafsum2;  // [n_leaves], zeroed with the other leaf sums
};
cudaError_t launch_leafsq(const LeafSquares& a, cudaStream_t s, int* nl);
// The previous tree's pred update, done by the next round's gradient kernel:
// pred += leafval[node & 0x7fff] for every row (src/cpu.rs:319-320).
struct PrevTree {
  const float* leafval;  // null: no previous tree
  const uint16_t* node;
};
// Gradients of one round, after the previous tree's pred update (prev.leafval != null).
// Also zeroes *zero_word (the level-0 row count k_quant accumulates), when non-null.
cudaError_t launch_grad(float* pred, const float* y, float* g, float* h, uint64_t n,
                        uint64_t n_pad, int logistic, uint64_t stride, uint64_t phase,
                        uint64_t row_offset, int compute_max, uint32_t* maxbits,
                        uint32_t* zero_word, const PrevTree& prev, cudaStream_t s, int* nl);
// Per round: fixed-point q = (qg, qh), the excluded flag (bit 15 of node) and node reset;
// also zeroes the level-0 built histogram (hb0_words int64) and the round's leaf sums
// (leafsum_words int64).
cudaError_t launch_quant(const float* g, const float* h, const uint32_t* maxbits, uint64_t n_pad,
                         int2* q, uint16_t* node, long long* hb0, uint64_t hb0_words,
                         long long* leafsum, uint32_t leafsum_words, uint32_t* ncount0,
                         cudaStream_t s, int* nl);
// The level's split (argmax over the per-feature records) and model slot, then
// leaf = 2*leaf + (bin > t) keeping the excluded flag; at non-final levels it writes the
// next level's row list (`lists`) and zeroes the next level's built histogram, at the
// final level it adds every row's unquantised g and h (wide fixed point) into its leaf's
// sums (src/cpu.rs:286-318); launch_leafval turns them into leaf values and the next
// round's gradient kernel adds them to pred.
struct ApplyLaunch {
  const uint8_t* colbins;
  uint64_t n_pad;
  uint16_t* node;
  const SplitRec* rec;
  uint32_t nf;
  uint32_t n_children;
  LevelLists lists;     // non-final levels: the next level's row list
  int final_level;
  uint32_t n_leaves;
  const float* g;       // final level: per-row unquantised g, h
  const float* h;
  const uint32_t* maxbits;  // the round's maxima (the wide scales)
  uint64_t n_rows;      // global row count
  long long* leafsum;   // final level: [2][n_leaves] int64 out (zeroed by k_quant)
  uint32_t* feat;
  float* thr;
  uint16_t* thr_bin;
  float* fi_gain;
  float* fi_count;
  uint32_t slot;
  uint32_t* split_out;  // nullable: (feature, bin) of the chosen split
  long long* hb_next;   // built-histogram buffer of the next level, zeroed here (nullable)
  uint64_t hb_next_words;  // even
};
cudaError_t launch_apply(const ApplyLaunch& a, cudaStream_t s, int* nl);
cudaError_t launch_fill_f32(float* p, float v, uint64_t n, cudaStream_t s, int* nl);

// ---- peer exchanges (peer_kernels.cu) ---------------------------------------------
// Sum of `words` int64 (even) at src_off of every rank's region into dst_off of every
// rank's region (16-byte aligned offsets). recv_off: a receive area in two halves of
// recv_half 16-byte vectors each (one per epoch parity), recv_half fixed for the context's
// exchanges and at least peer_recv_bytes(W, words) / 32 for the largest of them: with
// halves that do not move, an exchange never writes where the previous one (the other
// parity) may still be read, and the one before that is ordered by the previous
// exchange's barrier.
cudaError_t launch_peer_sum_i64(const PeerSet& ps, uint64_t src_off, uint64_t dst_off,
                                uint64_t recv_off, uint64_t recv_half, uint64_t words,
                                uint64_t epoch, int* err, cudaStream_t s, int* nl);
inline uint64_t peer_recv_bytes(int world, uint64_t words) {
  // two parities x W copies: whole (one-shot, 2 ranks) or of a 1/W slice (two-shot,
  // more ranks); the larger, so either fits
  const uint64_t whole = 2ull * world * (words / 2) * 16;
  const uint64_t slice = 2ull * world * ((words / 2 + world - 1) / world) * 16;
  return whole > slice ? whole : slice;
}
// In place over `data` (local device memory): n u64 summed, or n u32 maxed (max_u32).
cudaError_t launch_peer_small(const PeerSet& ps, void* data, uint32_t n, int max_u32,
                              uint64_t epoch, int* err, cudaStream_t s, int* nl);

// GOSS: exact k-th largest |g| by radix selection (4 passes of 8-bit digits).
struct GossState {
  unsigned long long* counts;  // [256]
  uint32_t* sel;               // [4]: prefix, mask, rank k, threshold bits
};
cudaError_t launch_goss_digit_hist(const float* g, uint64_t n, const GossState& st, int pass,
                                   cudaStream_t s, int* nl);
cudaError_t launch_goss_digit_select(const GossState& st, int pass, cudaStream_t s, int* nl);
cudaError_t launch_goss_init(const GossState& st, uint64_t k, cudaStream_t s, int* nl);
cudaError_t launch_goss_apply(float* g, float* h, uint64_t n, uint64_t row_offset,
                              const GossState& st, double keep_prob, float fact, uint64_t seed,
                              uint32_t* maxbits, cudaStream_t s, int* nl);

// ---- scoring (predict_kernels.cu) -------------------------------------------------
cudaError_t launch_predict_f32(const float* x, uint64_t n, uint32_t nf, const rw_dmodel& m,
                               float* out, cudaStream_t s);
cudaError_t launch_predict_u8(const uint8_t* bins, uint64_t n, uint64_t ld, const rw_dmodel& m,
                              float* out, cudaStream_t s);

// ---- compute_boundaries on the GPU (boundaries.cu) ---------------------------------
// The sample of n row-major rows (stride max(n / sample, 1)) and its cut table
// d_out[nf][n_bins-1]; scratch3 holds 3 * nf * m words, m = the sampled row count
// (returned in m_out; ceil(n / stride)).
// scratch: boundary_scratch_words(nf, m) words (three [nf][m] columns and the sort's
// per-part digit counts); *nl counts the launches.
cudaError_t launch_boundaries(const float* d_x, uint64_t n, uint32_t nf, uint32_t n_bins,
                              uint64_t sample, int unique, uint32_t* scratch, float* d_out,
                              cudaStream_t s, uint64_t* m_out, int* nl);
inline uint64_t boundary_sample_rows(uint64_t n, uint64_t sample) {
  const uint64_t st = std::max<uint64_t>(n / std::max<uint64_t>(sample, 1), 1);
  return (n - 1) / st + 1;
}
constexpr uint32_t kSortMaxParts = 16;
inline size_t boundary_scratch_words(uint32_t nf, uint64_t m) {
  return 3 * (size_t)nf * m + (size_t)nf * kSortMaxParts * 256;
}

// ---- test hooks ------------------------------------------------------------------
cudaError_t launch_debug_expf(const float* x, uint64_t n, float* out_rw, float* out_cuda,
                              cudaStream_t s);
// The SASS architecture the loaded kernels run as (cudaFuncAttributes::binaryVersion,
// major * 10 + minor), on the current device.
cudaError_t kernel_binary_version(int* out);
