/* CPU oracle for the rustwood oblivious-tree hot path -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm
 * may load this library, and only as the checker or the timed CPU baseline. The
 * product (rustwood_b200/ and librwgpu.so) never links or calls it.
 *
 * It restates, in plain C, the reference's CPU trainer and host helpers:
 *   src/cpu.rs:17-325        histogram GBDT trainer (oracle for the whole fit)
 *   src/data.rs:86-146       compute_boundaries (quantile / unique-midpoint cuts)
 *   src/booster.rs:201-205   base_score
 *   src/booster.rs:582-601   predict_cpu (sequential f32 scoring)
 *   src/metrics.rs:4-94      auc / logloss / rmse / mae / r2 / accuracy
 *   src/encoding.rs:25-115   out-of-fold target encoding
 *
 * Two training modes:
 *   exact = 0 ("oracle_ref"): faithful cpu.rs. f32 per-chunk private histograms over
 *     chunks of ceil(m/nt) sampled rows, combined by rayon's reduce tree (midpoint
 *     split down to single chunks), f64 gains, f64 leaf sums, glibc expf.
 *   exact = 1 ("oracle_exact"): the same algorithm with the GPU library's
 *     deterministic arithmetic: per-round 17-bit fixed-point quantisation of g/h for
 *     the histograms (rw_qscale_exp / rw_quantize), exact int64 histogram sums, leaf
 *     sums of the unquantised f32 g/h as exact int64 sums in a wide fixed point
 *     (rw_wscale_exp / rw_wquantize, <= 2^-43 of the round's maximum per value at 1M
 *     rows), and the library's rw_expf. The CUDA path must match this mode
 *     bit-for-bit.
 *
 * Parity pinning: the reference ships no tests, fixtures or golden vectors, and
 * its Rust sources cannot be built in this environment (no cargo/rustc). This
 * restatement is therefore "parity unpinned" against the reference binary; it is
 * pinned by the reference's own runtime self-checks restated as known-answer
 * tests, and by an independent pure-Python restatement on small cases.
 */
#ifndef RW_ORACLE_H
#define RW_ORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_params {
  uint32_t n_trees, depth, n_bins;
  float learning_rate, lambda, min_child_h;
  float subsample, colsample, goss_top, goss_other;
  int32_t objective; /* 0 = logistic, 1 = squared error */
  int32_t subtract;  /* histogram subtraction (cpu.rs:213) */
  const int32_t* monotone; /* nullable; extension (gpu_kernels.rs:888-896) */
  uint32_t n_monotone;
  int32_t exact;     /* 0 = oracle_ref, 1 = oracle_exact */
  int32_t n_threads; /* rayon pool size nt (cpu.rs:138-143); <= 0 -> the reference rule */
  /* nullable, exact mode only: PGBM per-leaf variances [n_trees][2^depth]
   * (gpu_kernels.rs:1046-1080: lr^2 * max(S2/H - (G/H)^2, 0) when H > 1, else 0, with
   * S2 the leaf's sum of g^2), from exact wide-fixed-point sums evaluated in f64 */
  float* leafvar;
} orc_params;

/* Optional per-level trace of the FIRST tree (exact mode only): the full level
 * histograms [2^d][nf][n_bins][2] (int64 q-sums) for levels 0..depth-1, the q-scale
 * exponents and per-level (feature, bin). Any pointer may be NULL. */
typedef struct orc_trace {
  int64_t* level_hist[16];
  int32_t e_g, e_h;
  uint32_t split_f[16], split_b[16];
  double loop_seconds; /* out: wall time of the tree loop (after binning) */
  /* Optional record of the first trace_trees trees (either mode), for teacher-forced
   * checks of one level at a time: each tree's g and h as its histograms use them
   * ([trace_trees][n]; 0 for rows outside the tree's sample) and every row's final leaf
   * index ([trace_trees][n]; the node at level d is leaf >> (depth - d)). */
  uint32_t trace_trees;
  float* tree_g;
  float* tree_h;
  uint16_t* tree_leaf;
} orc_trace;

int orc_default_threads(void);

void orc_compute_boundaries(const float* x, uint64_t n, uint32_t nf, uint32_t n_bins,
                            uint64_t sample, int unique, float* out);
void orc_bin_rowmajor(const float* x, uint64_t n, uint32_t nf, const float* cuts,
                      uint32_t n_bins, uint8_t* bins_rowmajor);
float orc_base_score(const float* y, uint64_t n, int objective);

int orc_train(const orc_params* p, const float* x, const float* y, uint64_t n, uint32_t nf,
              const float* cuts, float base_score, uint32_t* feat, float* thr,
              uint32_t* thr_bin, float* leafval, float* fi_gain, float* fi_count,
              orc_trace* trace);

void orc_predict(const float* x, uint64_t n, uint32_t nf, uint32_t n_trees, uint32_t depth,
                 const uint32_t* feat, const float* thr, const float* leafval, float base,
                 float* out);

/* Exact-mode level histogram over a given node assignment (for kernel-level tests).
 * bins are row-major [n][nf]; rows with node < 0 are excluded. When odd_only, only
 * rows with odd node contribute, keyed by node>>1. out: [groups][nf][n_bins][2]. */
void orc_level_hist_exact(const uint8_t* bins_rowmajor, uint64_t n, uint32_t nf,
                          uint32_t n_bins, const int32_t* node, const float* g,
                          const float* h, int e_g, int e_h, uint32_t groups, int odd_only,
                          int64_t* out);

double orc_auc(const float* s, const float* y, uint64_t n);
double orc_logloss(const float* s, const float* y, uint64_t n);
double orc_rmse(const float* s, const float* y, uint64_t n);
double orc_mae(const float* s, const float* y, uint64_t n);
double orc_r2(const float* s, const float* y, uint64_t n);
double orc_accuracy(const float* s, const float* y, uint64_t n);

/* Out-of-fold target encoding (encoding.rs:44-95) in place on row-major x.
 * Returns the number of distinct keys per categorical column in n_keys_out (len n_cat)
 * and fills keys_out/vals_out (flattened, per column, ascending key order) with the
 * full-train maps when non-NULL (capacity cap per column). gmean_out: global mean. */
int orc_target_encode(float* x, uint64_t n, uint32_t nf, const float* y,
                      const uint32_t* cat, uint32_t n_cat, float smoothing, uint32_t k_folds,
                      uint64_t hash_buckets, float* gmean_out);

float orc_rw_expf(float x); /* the shared exponential (exact mode), for tests */

#ifdef __cplusplus
}
#endif
#endif
