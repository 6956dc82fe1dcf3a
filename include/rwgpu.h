/* rwgpu -- B200 (sm_100a) oblivious-tree boosting hot path behind a C ABI.
 *
 * This is the drop-in boundary for rustwood's `--device gpu` path. Every entry point
 * takes plain pointers and sizes; no C++ or torch types cross it. The Rust host (or
 * any FFI: ctypes, cgo, JNI) binds these symbols in place of the cuda-oxide kernel
 * launches that rustwood's `Booster` issues today.
 *
 * Conventions (mirroring src/booster.rs's single-stream design):
 *  - Every call returns RW_OK (0) or a negative RW_ERR_* code; the message for the
 *    last failure on a context is available from rw_last_error(). No exception or
 *    abort crosses the ABI.
 *  - The caller owns every host buffer; outputs are written in full before return;
 *    no caller pointer is retained after a call returns.
 *  - A context (and the datasets/models created from it) is used by one host thread
 *    at a time. All device work of a context runs on one CUDA stream it owns.
 *  - Model semantics are rustwood's: for tree t and level d, slot k = t*depth + d holds
 *    feat[k] (feature index) and thr[k] (raw cut value); a row's leaf index is built
 *    MSB-first as leaf = 2*leaf + (x[feat[k]] > thr[k]) (src/gpu_kernels.rs:1009),
 *    and leafval is [n_trees][2^depth] (src/booster.rs:54-69).
 */
#ifndef RWGPU_H
#define RWGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define RW_OK 0
#define RW_ERR_ARG (-1)         /* invalid argument */
#define RW_ERR_OOM (-2)         /* device or host allocation failed */
#define RW_ERR_CUDA (-3)        /* CUDA runtime error */
#define RW_ERR_NCCL (-4)        /* NCCL error */
#define RW_ERR_UNSUPPORTED (-5) /* option not implemented on this path */
#define RW_ERR_TIMEOUT (-6)     /* collective or device wait exceeded its limit */

typedef struct rw_ctx rw_ctx;         /* device, stream, optional NCCL communicator */
typedef struct rw_dataset rw_dataset; /* device-resident binned training shard */
typedef struct rw_dmodel rw_dmodel;   /* device-resident model for scoring */

enum { RW_OBJ_LOGISTIC = 0, RW_OBJ_L2 = 1 };

/* Hyperparameters on the hot path: the fields of rustwood's Config
 * (src/config.rs:19-88) that fit_inner reads. replicas/smem_hist/f16_hist/int_hist/
 * int_scale only select among the reference's atomic strategies; they are accepted
 * and ignored (this library always uses exact fixed-point histograms). */
typedef struct rw_train_params {
  uint32_t n_trees;
  uint32_t depth;         /* 1..12 */
  uint32_t n_bins;        /* 2..256 */
  float learning_rate;
  float lambda;
  float min_child_h;
  float subsample;        /* < 0.999: every round(1/subsample)-th row (src/cpu.rs:172-176) */
  float colsample;        /* < 1: per-tree feature drop (src/gpu_kernels.rs:837) */
  const int32_t* monotone; /* nullable, n_monotone entries of -1/0/+1 */
  uint32_t n_monotone;
  int32_t subtract;       /* histogram subtraction (src/cpu.rs:213) */
  float goss_top;         /* > 0 enables GOSS (src/cpu.rs:64-110) */
  float goss_other;
  float clamp_hessian;    /* experimental in the reference; must be 0 here */
  int32_t pack4;          /* 4-bit bins when n_bins <= 16 */
  int32_t pgbm;           /* Config::pgbm; the variances are computed when leafvar != NULL */
  int32_t objective;      /* RW_OBJ_LOGISTIC or RW_OBJ_L2 */
  uint32_t replicas;      /* accepted, ignored */
  int32_t smem_hist, f16_hist, int_hist; /* accepted, ignored */
  float int_scale;        /* accepted, ignored */
} rw_train_params;

/* Per-phase device time of one fit, from CUDA events on the context stream
 * (the reference's profile categories, src/booster.rs:42-52, plus the collective). */
enum {
  RW_CAT_GRADIENTS = 0,
  RW_CAT_ZERO_HIST,
  RW_CAT_BUILD_HIST,
  RW_CAT_ALLREDUCE,
  RW_CAT_SPLIT,
  RW_CAT_APPLY,
  RW_CAT_UPDATE_PRED,
  RW_N_CATEGORIES
};

typedef struct rw_profile {
  int32_t enable;                      /* in: record per-phase events (adds no syncs) */
  double total_ms;                     /* out: tree loop, first launch to last (events) */
  double category_ms[RW_N_CATEGORIES]; /* out: per-phase sums */
  double hist_alg_bytes;               /* out: sum over levels of n*F*s + 12n + 8*F*B*G */
  uint64_t hist_launches;              /* out: histogram kernel launches */
  uint64_t kernel_launches;            /* out: all kernels this library launched */
} rw_profile;

/* A host-side model view (rustwood's Booster fields feat/thr/leafval/base_score).
 * thr_bin (bin-space thresholds, bin > thr_bin <=> x > thr) is needed only by the
 * u8 scorer. */
typedef struct rw_model {
  uint32_t n_trees, depth, n_features;
  float base_score;
  const uint32_t* feat;     /* [n_trees*depth] */
  const float* thr;         /* [n_trees*depth] */
  const uint16_t* thr_bin;  /* [n_trees*depth], nullable for f32 scoring */
  const float* leafval;     /* [n_trees << depth] */
} rw_model;

/* ---- contexts --------------------------------------------------------------- */

/* Replaces CudaContext::new(cfg.gpu) (src/booster.rs:137) and, for --serve, the
 * resident shared context (Booster::with_ctx, src/booster.rs:159). With n_gpus > 1 the
 * one context drives every listed GPU from this process (one rank per GPU inside the
 * library, one host thread each per call): datasets shard rows over them, fits run all
 * ranks, host-buffer scoring shards rows, device-pointer entry points use the first
 * GPU. */
int rw_ctx_create(const int* gpu_ids, int n_gpus, rw_ctx** out);

/* No counterpart in the reference (rustwood runs one process on one GPU): one process
 * per GPU, rank `rank` of `world` on device gpu_id, joined by an NCCL communicator built
 * from the 128-byte id that rank 0 obtained with rw_nccl_unique_id and broadcast out of
 * band. With world == 1, id may be NULL. */
int rw_ctx_create_rank(int gpu_id, int rank, int world, const void* nccl_id, rw_ctx** out);
int rw_nccl_unique_id(void* out128);
/* Destroys the context; its datasets and uploaded models must be destroyed first (they
 * live in the context's memory pool). */
void rw_ctx_destroy(rw_ctx* ctx);
/* The message behind the last failing call on ctx (what rustwood's Box<dyn Error>
 * carries, src/booster.rs:32); with ctx == NULL, the last failure on this thread of a
 * call that had no context to record it on. */
const char* rw_last_error(const rw_ctx* ctx);
/* The context's CUDA stream (a cudaStream_t), for callers that order their own work
 * or CUDA events with the library's. */
void* rw_ctx_stream(const rw_ctx* ctx);
/* Multi-GPU only (no counterpart in the reference): bound (milliseconds) on each
 * collective wait; 0 = wait forever. Default 60000. */
int rw_ctx_set_timeout(rw_ctx* ctx, int64_t ms);
/* 1 when a wait on a peer rank expired on this context (its exchanges can no longer be
 * trusted: later fits return an error; recreate the context), else 0. */
int rw_ctx_peer_failed(const rw_ctx* ctx);

/* ---- training ---------------------------------------------------------------- */

/* Host prep of fit_inner (src/booster.rs:255-277): upload row-major x and y, bin on
 * the GPU against the cut table cuts[nf*(n_bins-1)] (bin = #{cut < v}), optionally
 * pack 4-bit. For a row shard, n is the local row count, n_global the total and
 * row_offset this shard's first global row (row-index hashes and the subsample stride
 * use global indices). Single process: n_global = n, row_offset = 0. */
int rw_dataset_create(rw_ctx* ctx, const float* x_rowmajor, const float* y, uint64_t n,
                      uint32_t nf, const float* cuts, uint32_t n_bins, int32_t pack4,
                      uint64_t n_global, uint64_t row_offset, rw_dataset** out);
/* Same, from device pointers (row-major x, y) that stay owned by the caller. */
int rw_dataset_create_device(rw_ctx* ctx, const float* d_x_rowmajor, const float* d_y,
                             uint64_t n, uint32_t nf, const float* cuts, uint32_t n_bins,
                             int32_t pack4, uint64_t n_global, uint64_t row_offset,
                             rw_dataset** out);
void rw_dataset_destroy(rw_dataset* ds);
/* Copy out the binned matrix fit_inner builds (bin_features, src/booster.rs:255-277),
 * feature-major [nf][n] u8 (unpacked). */
int rw_dataset_bins(const rw_dataset* ds, uint8_t* out);

/* compute_boundaries (src/data.rs:86-146) on the GPU for row-major x already in device
 * memory (d_x [n][nf]): every max(n / sample, 1)-th row, per-feature sort, quantile cuts
 * with the monotone fix or (unique != 0) distinct-value midpoints padded with +inf.
 * out: host [nf*(n_bins-1)], bit-identical to rw_compute_boundaries on samples without
 * NaN (whose order the reference leaves undefined). */
int rw_compute_boundaries_device(rw_ctx* ctx, const float* d_x, uint64_t n, uint32_t nf,
                                 uint32_t n_bins, uint64_t sample, int32_t unique, float* out);

/* rw_fit with fit_inner's cut table computed on the GPU too (src/booster.rs:246-277:
 * compute_boundaries then binning): x is uploaded once and serves both. sample/unique
 * are Config's bin_sample and unique_bins; cuts_out (nullable) receives the table. */
int rw_fit_with_boundaries(rw_ctx* ctx, const rw_train_params* p, const float* x_rowmajor,
                           const float* y, uint64_t n, uint32_t nf, uint64_t sample,
                           int32_t unique, float base_score, float* cuts_out, uint32_t* feat,
                           float* thr, uint16_t* thr_bin, float* leafval, float* leafvar,
                           float* fi_gain, float* fi_count, rw_profile* prof);

/* The tree loop of fit_inner (src/booster.rs:349-513). Outputs (caller-allocated):
 * feat/thr/thr_bin [n_trees*depth], leafval [n_trees<<depth], fi_gain/fi_count [nf].
 * thr_bin, leafvar and prof may be NULL. leafvar [n_trees<<depth], when not NULL,
 * receives the PGBM leaf variances (src/gpu_kernels.rs:1015-1080): lr^2 * max(S2/H -
 * (G/H)^2, 0) for leaves with H > 1, else 0, where G, H and S2 are the leaf's sums of g,
 * h and g*g over the tree's sampled rows -- here exact wide-fixed-point sums evaluated in
 * f64 and rounded once to f32 (the reference sums in f32 atomics). */
int rw_fit_dataset(rw_dataset* ds, const rw_train_params* p, float base_score,
                   uint32_t* feat, float* thr, uint16_t* thr_bin, float* leafval,
                   float* leafvar, float* fi_gain, float* fi_count, rw_profile* prof);

/* Whole Booster::fit_inner replacement (src/booster.rs:227-517): dataset creation
 * from host buffers, the tree loop and the model download in one call. */
int rw_fit(rw_ctx* ctx, const rw_train_params* p, const float* x_rowmajor, const float* y,
           uint64_t n, uint32_t nf, const float* cuts, float base_score, uint32_t* feat,
           float* thr, uint16_t* thr_bin, float* leafval, float* leafvar, float* fi_gain,
           float* fi_count, rw_profile* prof);

/* ---- scoring ----------------------------------------------------------------- */

/* Booster::predict (src/booster.rs:531-555): raw margins of n row-major f32 rows,
 * accumulated per row in tree order in f32 (bit-identical to predict_cpu,
 * src/booster.rs:582-601). */
int rw_predict_f32(rw_ctx* ctx, const rw_model* m, const float* x_rowmajor, uint64_t n,
                   uint32_t nf, float* out);
/* PGBM predict_var (src/gpu_kernels.rs:1084-1120, Booster::predict_std before its
 * square root, src/booster.rs:559-577): per row the sum over trees, in tree order in f32
 * from 0, of the variance leafvar[t << depth | leaf] of the leaf the row reaches; m's
 * leafval and base_score are not used. leafvar is rw_fit's PGBM output. */
int rw_predict_var_f32(rw_ctx* ctx, const rw_model* m, const float* leafvar,
                       const float* x_rowmajor, uint64_t n, uint32_t nf, float* out);
/* Same margins from pre-binned feature-major u8 rows bins[nf][n] and thr_bin (the
 * reference scores binned rows in bench_throughput, src/booster.rs:654-698). */
int rw_predict_u8(rw_ctx* ctx, const rw_model* m, const uint8_t* bins_featmajor, uint64_t n,
                  uint32_t nf, float* out);

/* Device-resident model and scoring of device-resident inputs (the model is uploaded
 * once, as bench_latency/bench_throughput do, src/booster.rs:608-698). ld is the row
 * stride of d_bins in bytes (>= n). kernel_ms (nullable) receives the kernel time. */
int rw_model_upload(rw_ctx* ctx, const rw_model* m, rw_dmodel** out);
void rw_model_free(rw_dmodel* dm);
int rw_predict_u8_device(rw_ctx* ctx, const rw_dmodel* dm, const uint8_t* d_bins, uint64_t n,
                         uint64_t ld, float* d_out, float* kernel_ms);
int rw_predict_f32_device(rw_ctx* ctx, const rw_dmodel* dm, const float* d_x, uint64_t n,
                          float* d_out, float* kernel_ms);

/* Booster::predict from host buffers WITHOUT ANY DEVICE ALLOCATION. No counterpart in
 * the reference: this entry point exists for callers that cannot call cudaMalloc --
 * e.g. a serving process whose device memory belongs to another allocator (a
 * framework's caching pool or a fixed reserved budget), or a latency-critical path
 * where cudaMalloc/cudaFree's implicit device synchronisation would stall other work.
 * Same margins as rw_predict_f32 (bit-identical). The model, a batch of rows and their
 * margins are staged through one 16 MiB device array compiled into the library, which
 * every GPU that loads the library holds until the process exits; rows are processed
 * in batches that fit beside the model. Limits: the staged model (feat, thr and leafval,
 * each rounded up to 256 bytes) must fit in 4 MiB, otherwise RW_ERR_ARG is returned
 * with the size in the message. The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress, with that device current), so make the first
 * call on a device before any CUDA stream capture; the address is kept for the life of
 * the process, so a caller that resets a device (cudaDeviceReset) must reload the
 * library before scoring on it again. Every call on a device shares the array: calls
 * that overlap on the GPU (from other threads or contexts on the same device) race and
 * must be serialised by the caller. Nothing in the array has to start at zero: each
 * call overwrites the regions it reads before reading them. */
int rw_predict_f32_noalloc(rw_ctx* ctx, const rw_model* m, const float* x_rowmajor,
                           uint64_t n, uint32_t nf, float* out);

/* ---- categorical target encoding on the GPU ----------------------------------- */

/* encoding.rs fit_transform_train (src/encoding.rs:44-95): every categorical column of the
 * row-major rows becomes its smoothed out-of-fold target mean (folds = row index mod
 * max(k_folds, 2)); gmean_out receives the global label mean and enc_out (nullable) the
 * test-set maps (free with rw_encoders_free). The sums are exact fixed-point integers, so
 * the values equal the reference's sequential f64 sums wherever those are exact (0/1 or
 * small integer labels: no partial sum rounds). RW_ERR_UNSUPPORTED when a feature's key range is too
 * wide for dense tables (more than 2^26 keys over all features): encode on the host.
 * rw_target_encode_device works on device rows and labels in place; rw_target_encode
 * takes host buffers and writes the encoded rows back into x_rowmajor. */
typedef struct rw_encoders rw_encoders;
int rw_target_encode_device(rw_ctx* ctx, float* d_x, const float* d_y, uint64_t n, uint32_t nf,
                            const uint32_t* categorical, uint32_t n_cat, float smoothing,
                            uint32_t k_folds, uint64_t hash_buckets, float* gmean_out,
                            rw_encoders** enc_out);
int rw_target_encode(rw_ctx* ctx, float* x_rowmajor, const float* y, uint64_t n, uint32_t nf,
                     const uint32_t* categorical, uint32_t n_cat, float smoothing,
                     uint32_t k_folds, uint64_t hash_buckets, float* gmean_out,
                     rw_encoders** enc_out);
/* Feature i's map: keys key_lo .. key_lo + n_keys - 1; value[j] holds key_lo + j's encoded
 * value where present[j] != 0 (unseen keys take gmean, src/encoding.rs:99-115). The
 * pointers stay valid until rw_encoders_free. */
int rw_encoders_table(const rw_encoders* enc, uint32_t i, int64_t* key_lo, uint64_t* n_keys,
                      const float** value, const uint8_t** present);
void rw_encoders_free(rw_encoders* enc);
/* The reference's Encoders (src/encoding.rs:16, one key -> value map per categorical
 * feature) built from maps held elsewhere (the caller's own fit, a loaded model): n_cat
 * dense tables concatenated in value/present, table i covering keys key_lo[i] ..
 * key_lo[i] + n_keys[i] - 1; gmean is the value of unseen keys. */
int rw_encoders_create(uint32_t n_cat, const int64_t* key_lo, const uint64_t* n_keys,
                       const float* value, const uint8_t* present, float gmean,
                       rw_encoders** out);
/* encoding::transform (src/encoding.rs:96-115) on the GPU: the categorical values of host
 * rows x_rowmajor [n][nf] become their keys' values in enc (unseen keys: enc's gmean), in
 * place. */
int rw_target_transform(rw_ctx* ctx, float* x_rowmajor, uint64_t n, uint32_t nf,
                        const uint32_t* categorical, uint32_t n_cat, const rw_encoders* enc,
                        uint64_t hash_buckets);

/* ---- host helpers kept from the reference host code --------------------------- */

/* compute_boundaries (src/data.rs:86-146): out[nf*(n_bins-1)]. */
void rw_compute_boundaries(const float* x_rowmajor, uint64_t n, uint32_t nf, uint32_t n_bins,
                           uint64_t sample, int32_t unique, float* out);
/* The u8 scorer's bin-space thresholds of a model that carries only raw thresholds (a
 * .rwood v1 file stores feat/thr/leafval, src/booster.rs:797-824): thr_bin[k] = the
 * first b with cuts[feat[k]][b] == thr[k], given the cut table cuts[nf*(n_bins-1)] the
 * model was trained with (bin > b <=> x > cuts[b] for every b holding that value).
 * RW_ERR_ARG when a threshold is not a cut of its feature in this table. */
int rw_model_thr_bins(const rw_model* m, const float* cuts, uint32_t n_bins, uint16_t* thr_bin);
/* base_score (src/booster.rs:201-205 / 280-284). */
float rw_base_score(const float* y, uint64_t n, int32_t objective);

/* ---- test hooks (no counterpart in the reference) ------------------------------ */

/* Runs the production histogram kernel once on caller data: node[n] (>= 0 in-sample,
 * < 0 excluded), g/h[n], scales 2^e_g / 2^e_h; odd_only keys odd nodes by node>>1.
 * out: int64 [groups][nf][n_bins][2] fixed-point (g, h) sums. */
int rw_debug_level_hist(rw_dataset* ds, const int32_t* node, const float* g, const float* h,
                        int32_t e_g, int32_t e_h, uint32_t groups, int32_t odd_only,
                        int64_t* out);
/* Runs the production split search for one level on caller data (teacher forcing):
 * node[n] in [0, n_nodes) (< 0 excluded), g/h[n] f32, quantised with the scales the
 * trainer takes from their maxima; every node's histogram is built (k_hist over a row
 * list) and scanned (k_gain, k_best) with p's lambda/min_child_h/colsample/monotone and
 * tree index `tree` (the colsample seed). Out: each feature's best gain and bin
 * (gain_out/bin_out [nf]) and the level's choice chosen[2] = (feature, bin), picked as
 * the trainer picks it (highest gain, ties to the lowest feature). */
int rw_debug_level_step(rw_dataset* ds, const rw_train_params* p, const int32_t* node,
                        const float* g, const float* h, uint32_t n_nodes, uint32_t tree,
                        double* gain_out, uint32_t* bin_out, uint32_t* chosen);
/* Failure detection without a fault: one one-shot peer exchange on this device whose
 * rank 1 is a local region that nothing runs for, with each wait bounded by timeout_ms
 * (1..10000). mode 0: rank 1 never signals (the wait expires: error word 2); 1: rank 1's
 * signal carries its error bit (error word 3); 2: this rank's error word is already 2
 * (the wait is skipped); 3: rank 1 signalled normally (error word 0). Out: the error
 * word and the exchange kernel's time. */
int rw_debug_peer_wait(rw_ctx* ctx, int32_t mode, int64_t timeout_ms, int32_t* err_out,
                       float* kernel_ms);
/* A context on gpu_id that is rank 0 of 2 with peer exchanges on, whose rank 1 never
 * runs (its region is a local buffer), and whose waits expire after timeout_ms: every
 * fit on it must return RW_ERR_TIMEOUT instead of waiting. */
int rw_debug_lonely_rank_ctx(int gpu_id, int64_t timeout_ms, rw_ctx** out);
/* The architecture the library's kernels run as on the context's device
 * (cudaFuncAttributes::binaryVersion: 100 for sm_100a code). */
int rw_debug_binary_version(rw_ctx* ctx, int32_t* out);
/* Evaluates the device exponential on n inputs (tests compare it with the host). */
int rw_debug_expf(rw_ctx* ctx, const float* x, uint64_t n, float* out_rw, float* out_cuda);

#ifdef __cplusplus
}
#endif
#endif /* RWGPU_H */
