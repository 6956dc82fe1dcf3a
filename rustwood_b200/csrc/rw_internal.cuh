// Internal declarations shared by the rwgpu translation units.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

#include "../../include/rwgpu.h"

struct rw_ctx {
  int device = 0;
  int rank = 0;
  int world = 1;
  cudaStream_t stream = nullptr;
  ncclComm_t comm = nullptr;
  int64_t timeout_ms = 60000;
  std::string last_error;
  uint64_t launches = 0;  // kernels launched on this context (all time)
};

// Bins in HBM are stored column-major in tiles of kBinTile rows: tile t holds rows
// [t*kBinTile, +kBinTile) and, inside it, feature f's bins form one row of `rs` bytes
// (kBinTile u8, or kBinTile/2 bytes of 4-bit pairs, plus 16 bytes of padding). A feature
// slice of a tile is therefore one contiguous block (one TMA bulk copy), and the padding
// (an odd number of 16-byte units) keeps 16-byte shared-memory reads of consecutive
// features on distinct banks.
constexpr uint32_t kBinTile = 512;

struct BinLayout {
  uint32_t nf = 0;
  uint32_t rs = 0;          // bytes per feature row within a tile
  uint64_t tile_bytes = 0;  // nf * rs
  int packed = 0;
  __host__ __device__ uint64_t offset(uint32_t f, uint64_t r) const {
    const uint64_t in = r % kBinTile;
    return (r / kBinTile) * tile_bytes + (uint64_t)f * rs + (packed ? in / 2 : in);
  }
  static BinLayout make(uint32_t nf, int packed) {
    BinLayout L;
    L.nf = nf;
    L.packed = packed;
    L.rs = (packed ? kBinTile / 2 : kBinTile) + 16;
    L.tile_bytes = (uint64_t)nf * L.rs;
    return L;
  }
};

struct rw_dataset {
  rw_ctx* ctx = nullptr;
  uint64_t n = 0;         // local rows
  uint64_t n_pad = 0;     // rows rounded up (padded rows carry g = h = 0)
  uint64_t n_global = 0;  // rows across all ranks
  uint64_t row_offset = 0;
  uint32_t nf = 0, n_bins = 0;
  int packed = 0;
  BinLayout lay;                // layout of d_bins
  uint8_t* d_bins = nullptr;    // row-tiled column-major (u8 or 4-bit packed), see BinLayout
  uint8_t* d_bins_u8 = nullptr; // u8 copy (row-tiled) kept only when packed
  float* d_y = nullptr;         // [n_pad]
  float* d_cuts = nullptr;      // [nf][n_bins-1]
  std::vector<float> cuts;
  // Working buffers of the boosting loop, kept across fits (named, grown on demand).
  std::map<std::string, std::pair<void*, size_t>> ws;
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

// ---- kernel launchers (train_kernels.cu) ------------------------------------------

struct HistLaunch {
  const uint8_t* bins;
  BinLayout lay;
  const int16_t* slot;   // per row: histogram group this level builds into, or -1
  const int32_t* qg;     // per row: fixed-point g (rw_quantize)
  const int32_t* qh;     // per row: fixed-point h
  uint64_t n_pad;        // multiple of kRowAlign
  uint32_t nf, nb;
  uint32_t groups;       // histogram groups written (out has `groups` slots)
  long long* out;        // int64 [groups][nf][nb][2], zeroed by the caller
  int* err;              // set to a nonzero code if a bounded wait gave up
};
cudaError_t launch_hist(const HistLaunch& a, cudaStream_t s, int* n_launch);

struct SplitLaunch {
  const long long* hb;  // built histogram
  const long long* hp;  // parent level full histogram (mode 1)
  long long* hf;        // this level's full histogram (out)
  long long* hb_next;   // built-histogram buffer of the next level, zeroed here (nullable)
  uint64_t hb_next_words;
  uint32_t n_nodes, nf, nb;
  int mode;             // 0: hb holds every node; 1: hb holds odd nodes keyed by parent
  const uint32_t* maxbits;
  double lambda, min_child, lr;
  const int32_t* monotone;  // device [nf] or null
  float colsample;
  uint32_t tree_seed;
  double* best_gain;
  uint32_t* best_bin;
  uint32_t* counter;
  const float* cuts;
  uint32_t* feat;
  float* thr;
  uint16_t* thr_bin;
  uint32_t* split_ft;
  float* fi_gain;
  float* fi_count;
  uint32_t slot;
  int last_level;
  float* leafval;
  uint32_t leaf_base;
};
cudaError_t launch_split(const SplitLaunch& a, cudaStream_t s);

// Rows are padded to a multiple of kRowAlign so every histogram CTA's row range is a
// whole number of steps for every lane.
constexpr uint64_t kRowAlign = 4096;

cudaError_t launch_bin(const float* x_rowmajor, uint64_t n, uint32_t nf, const float* d_cuts,
                       uint32_t n_bins, uint8_t* d_bins, const BinLayout& lay, cudaStream_t s,
                       int* nl);
cudaError_t launch_pack4(const uint8_t* d_bins, const BinLayout& lay_u8, uint64_t n_pad,
                         uint8_t* d_packed, const BinLayout& lay_p, cudaStream_t s, int* nl);
cudaError_t launch_grad(const float* pred, const float* y, float* g, float* h, uint64_t n,
                        uint64_t n_pad, int logistic, uint64_t stride, uint64_t phase,
                        uint64_t row_offset, int compute_max, uint32_t* maxbits,
                        cudaStream_t s, int* nl);
// Per round: fixed-point q, the excluded flag (bit 15 of node) and level-0 slots; also
// zeroes the level-0 built histogram (hb0_words int64).
cudaError_t launch_quant(const float* g, const float* h, const uint32_t* maxbits, uint64_t n_pad,
                         int32_t* qg, int32_t* qh, uint16_t* node, int16_t* slot,
                         long long* hb0, uint64_t hb0_words, cudaStream_t s, int* nl);
// leaf = 2*leaf + (bin > t) keeping the excluded flag; writes the next level's build
// slot (next_odd_only: odd children keyed by parent), or at the final level updates pred.
cudaError_t launch_apply(const uint8_t* bins, const BinLayout& lay, uint16_t* node,
                         int16_t* slot, const uint32_t* split_ft, uint64_t n_pad,
                         int next_odd_only, int final_level, const float* leafval,
                         uint32_t leaf_base, float* pred, cudaStream_t s, int* nl);
cudaError_t launch_fill_f32(float* p, float v, uint64_t n, cudaStream_t s, int* nl);

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

// ---- test hooks ------------------------------------------------------------------
cudaError_t launch_debug_expf(const float* x, uint64_t n, float* out_rw, float* out_cuda,
                              cudaStream_t s);
