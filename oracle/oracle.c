/* CPU oracle for the rustwood oblivious-tree hot path -- TEST INFRASTRUCTURE ONLY.
 * See oracle.h for the scope, the two modes and the parity-pinning status.
 * Compile with -ffp-contract=off (the Makefile does): the exact mode must evaluate
 * the shared exponential with the same IEEE operations as the GPU.
 */
#define _GNU_SOURCE
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <unistd.h>

#include "../rustwood_b200/csrc/rw_expf.h"

float orc_rw_expf(float x) { return rw_expf(x); }

/* ------------------------------------------------------------------------- */
/* threads                                                                    */

/* cpu.rs:134-143: RUSTWOOD_THREADS, else all cores if <= 16, else min(cores/2, 32). */
int orc_default_threads(void) {
  const char* env = getenv("RUSTWOOD_THREADS");
  if (env) {
    long v = strtol(env, NULL, 10);
    if (v > 0) return (int)v;
  }
  long avail = sysconf(_SC_NPROCESSORS_ONLN);
  if (avail <= 0) avail = 4;
  long nt = avail <= 16 ? avail : (avail / 2 < 32 ? avail / 2 : 32);
  return nt < 1 ? 1 : (int)nt;
}

typedef void (*par_fn)(int ti, void* arg);
typedef struct {
  par_fn fn;
  void* arg;
  int ti;
} par_slot;

static void* par_tramp(void* p) {
  par_slot* s = (par_slot*)p;
  s->fn(s->ti, s->arg);
  return NULL;
}

/* Run fn(ti, arg) for ti in [0, nt) concurrently. Results never depend on timing:
 * every task writes only its own slot. */
static void par_run(int nt, par_fn fn, void* arg) {
  if (nt <= 1) {
    for (int i = 0; i < (nt < 1 ? 1 : nt); i++) fn(i, arg);
    return;
  }
  pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nt);
  par_slot* sl = (par_slot*)malloc(sizeof(par_slot) * nt);
  for (int i = 0; i < nt; i++) {
    sl[i].fn = fn;
    sl[i].arg = arg;
    sl[i].ti = i;
    if (i > 0) pthread_create(&th[i], NULL, par_tramp, &sl[i]);
  }
  fn(0, arg);
  for (int i = 1; i < nt; i++) pthread_join(th[i], NULL);
  free(th);
  free(sl);
}

/* rayon's reduce over (0..nt).into_par_iter(): bridge_producer_consumer splits the
 * index range at len/2 until single items (the splitter budget starts at nt, which
 * always suffices), each leaf folds (identity op item) and joins combine (left op
 * right). For f32/f64 vector addition this fixes the summation tree. */
static float* rayon_tree_f32(float** loc, int lo, int hi, size_t len) {
  if (hi - lo == 1) {
    float* v = loc[lo];
    for (size_t i = 0; i < len; i++) v[i] = 0.0f + v[i];
    return v;
  }
  int mid = (hi - lo) / 2;
  float* a = rayon_tree_f32(loc, lo, lo + mid, len);
  float* b = rayon_tree_f32(loc, lo + mid, hi, len);
  for (size_t i = 0; i < len; i++) a[i] += b[i];
  free(b);
  return a;
}

static double* rayon_tree_f64(double** loc, int lo, int hi, size_t len) {
  if (hi - lo == 1) {
    double* v = loc[lo];
    for (size_t i = 0; i < len; i++) v[i] = 0.0 + v[i];
    return v;
  }
  int mid = (hi - lo) / 2;
  double* a = rayon_tree_f64(loc, lo, lo + mid, len);
  double* b = rayon_tree_f64(loc, lo + mid, hi, len);
  for (size_t i = 0; i < len; i++) a[i] += b[i];
  free(b);
  return a;
}

/* ------------------------------------------------------------------------- */
/* data.rs:86-146 compute_boundaries                                          */

static void merge_sort_f32(float* a, float* tmp, size_t n) {
  /* stable bottom-up merge sort with the partial order "a < b"; equal (or
   * unordered) elements keep their input order like Rust's stable sort_by. */
  for (size_t w = 1; w < n; w *= 2) {
    for (size_t lo = 0; lo < n; lo += 2 * w) {
      size_t mid = lo + w < n ? lo + w : n;
      size_t hi = lo + 2 * w < n ? lo + 2 * w : n;
      size_t i = lo, j = mid, k = lo;
      while (i < mid && j < hi) {
        if (a[j] < a[i]) tmp[k++] = a[j++];
        else tmp[k++] = a[i++];
      }
      while (i < mid) tmp[k++] = a[i++];
      while (j < hi) tmp[k++] = a[j++];
    }
    memcpy(a, tmp, n * sizeof(float));
  }
}

void orc_compute_boundaries(const float* x, uint64_t n, uint32_t nf, uint32_t n_bins,
                            uint64_t sample, int unique, float* out) {
  uint32_t n_bound = n_bins - 1;
  uint64_t stride = n / (sample > 1 ? sample : 1);
  if (stride < 1) stride = 1;
  size_t cap = (size_t)(n / stride + 1);
  float* s = (float*)malloc(cap * sizeof(float));
  float* tmp = (float*)malloc(cap * sizeof(float));
  float* uniq = (float*)malloc(cap * sizeof(float));
  float* cand = (float*)malloc(cap * sizeof(float));
  for (uint32_t f = 0; f < nf; f++) {
    size_t m = 0;
    for (uint64_t i = 0; i < n; i += stride) s[m++] = x[i * nf + f];
    merge_sort_f32(s, tmp, m);
    float* b = out + (size_t)f * n_bound;
    if (unique) {
      size_t nu = 0;
      for (size_t i = 0; i < m; i++)
        if (nu == 0 || uniq[nu - 1] != s[i]) uniq[nu++] = s[i];
      size_t nc = nu > 0 ? nu - 1 : 0;
      for (size_t i = 0; i < nc; i++) cand[i] = 0.5f * (uniq[i] + uniq[i + 1]);
      for (uint32_t j = 0; j < n_bound; j++) {
        if (nc == 0) b[j] = INFINITY;
        else if (nc <= n_bound) b[j] = j < nc ? cand[j] : INFINITY;
        else {
          size_t pos = ((size_t)(j + 1) * nc) / (n_bound + 1);
          b[j] = cand[pos < nc - 1 ? pos : nc - 1];
        }
      }
    } else {
      for (uint32_t j = 0; j < n_bound; j++) {
        double q = (double)(j + 1) / (double)n_bins;
        double posd = round(q * (double)(m - 1));
        size_t pos = (size_t)posd;
        b[j] = s[pos < m - 1 ? pos : m - 1];
      }
      for (uint32_t j = 1; j < n_bound; j++)
        if (b[j] <= b[j - 1]) b[j] = b[j - 1];
    }
  }
  free(s);
  free(tmp);
  free(uniq);
  free(cand);
}

/* cpu.rs:149-155: bin = partition_point(|c| c < v).min(nb1). */
static inline uint8_t bin_of(const float* cuts, uint32_t nb1, float v) {
  uint32_t lo = 0, hi = nb1;
  while (lo < hi) {
    uint32_t mid = (lo + hi) / 2;
    if (cuts[mid] < v) lo = mid + 1;
    else hi = mid;
  }
  return (uint8_t)(lo < nb1 ? lo : nb1);
}

void orc_bin_rowmajor(const float* x, uint64_t n, uint32_t nf, const float* cuts,
                      uint32_t n_bins, uint8_t* bins) {
  uint32_t nb1 = n_bins - 1;
  for (uint64_t r = 0; r < n; r++)
    for (uint32_t f = 0; f < nf; f++)
      bins[r * nf + f] = bin_of(cuts + (size_t)f * nb1, nb1, x[r * nf + f]);
}

typedef struct {
  const float* x;
  uint64_t n;
  uint32_t nf;
  const float* cuts;
  uint32_t nbins;
  uint8_t* bins;
  uint8_t* bins_col;
  int nt;
} bin_job;

static void bin_rows_worker(int ti, void* arg) {
  bin_job* J = (bin_job*)arg;
  uint64_t chunk = (J->n + (uint64_t)J->nt - 1) / (uint64_t)J->nt;
  uint64_t lo = (uint64_t)ti * chunk, hi = lo + chunk < J->n ? lo + chunk : J->n;
  uint32_t nb1 = J->nbins - 1;
  for (uint64_t r = lo; r < hi; r++)
    for (uint32_t f = 0; f < J->nf; f++)
      J->bins[r * J->nf + f] = bin_of(J->cuts + (size_t)f * nb1, nb1, J->x[r * J->nf + f]);
}

static void bin_cols_worker(int ti, void* arg) {
  bin_job* J = (bin_job*)arg;
  for (uint32_t f = (uint32_t)ti; f < J->nf; f += (uint32_t)J->nt)
    for (uint64_t r = 0; r < J->n; r++) J->bins_col[(size_t)f * J->n + r] = J->bins[r * J->nf + f];
}

/* booster.rs:201-205 */
float orc_base_score(const float* y, uint64_t n, int objective) {
  float s = 0.0f;
  for (uint64_t i = 0; i < n; i++) s += y[i];
  float mean = s / (float)n;
  if (mean < 1e-6f) mean = 1e-6f;
  if (mean > 1.0f - 1e-6f) mean = 1.0f - 1e-6f;
  return objective == 0 ? logf(mean / (1.0f - mean)) : mean;
}

/* ------------------------------------------------------------------------- */
/* sampling helpers                                                           */

/* cpu.rs:68 */
static const uint64_t kGossSalt = 0x00424552455A4B41ull;
/* gpu_kernels.rs (hash01 salts) and booster.rs:36 (per-tree seed salt) */
static const uint32_t kSampleSalt = 0x455A4B41u;
static const uint32_t kSeedSalt = 0x455A4B41u;

static inline float hash01(uint32_t id, uint32_t seed) {
  uint32_t x = id * 2654435761u + (seed ^ kSampleSalt);
  x ^= x >> 15;
  x *= 2246822519u;
  x ^= x >> 13;
  return (float)(x & 0x00FFFFFFu) / 16777215.0f;
}

static inline uint32_t tree_seed_of(uint32_t tree) { return tree * 2654435761u + kSeedSalt; }

static int cmp_desc_f32(const void* a, const void* b) {
  float x = *(const float*)a, y = *(const float*)b;
  return (x < y) - (x > y);
}

/* value of the k-th element (0-based) of |g| sorted descending (cpu.rs:73-76);
 * three-way quickselect, any selection algorithm yields the same value. */
static float kth_largest_abs(const float* g, uint64_t n, uint64_t k) {
  float* a = (float*)malloc(n * sizeof(float));
  for (uint64_t i = 0; i < n; i++) a[i] = fabsf(g[i]);
  uint64_t lo = 0, hi = n;
  float result;
  for (;;) {
    if (hi - lo <= 16) {
      qsort(a + lo, hi - lo, sizeof(float), cmp_desc_f32);
      result = a[k];
      break;
    }
    float x0 = a[lo], x1 = a[lo + (hi - lo) / 2], x2 = a[hi - 1];
    float pv = x0 > x1 ? (x1 > x2 ? x1 : (x0 > x2 ? x2 : x0)) : (x0 > x2 ? x0 : (x1 > x2 ? x2 : x1));
    uint64_t lt = lo, i = lo, gt = hi;
    while (i < gt) {
      float v = a[i];
      if (v > pv) {
        a[i] = a[lt];
        a[lt] = v;
        lt++;
        i++;
      } else if (v < pv) {
        gt--;
        a[i] = a[gt];
        a[gt] = v;
      } else {
        i++;
      }
    }
    if (k < lt) hi = lt;
    else if (k < gt) {
      result = pv;
      break;
    } else lo = gt;
  }
  free(a);
  return result;
}

/* cpu.rs:70-110. Fills sel with the sampled rows (ascending), returns count. */
static uint64_t goss_sample(float* g, float* h, uint64_t n, double top, double other,
                            uint64_t seed, uint32_t* sel) {
  double tn = top * (double)n;
  uint64_t topn = tn <= 0.0 ? 0 : (uint64_t)tn;
  if (topn < 1) topn = 1;
  if (topn > n) topn = n;
  uint64_t k = topn - 1 < n - 1 ? topn - 1 : n - 1;
  float thresh = kth_largest_abs(g, n, k);
  double d1 = 1.0 - top > 1e-9 ? 1.0 - top : 1e-9;
  double keep_prob = other / d1;
  if (keep_prob < 0.0) keep_prob = 0.0;
  if (keep_prob > 1.0) keep_prob = 1.0;
  float fact = (float)((1.0 - top) / (other > 1e-9 ? other : 1e-9));
  uint64_t m = 0;
  for (uint64_t r = 0; r < n; r++) {
    h[r] = 1.0f;
    if (fabsf(g[r]) >= thresh) {
      sel[m++] = (uint32_t)r;
    } else {
      uint64_t hh = (r ^ (seed * 0x9E3779B97F4A7C15ull) ^ kGossSalt) * 0xD6E8FEB86659FD93ull;
      hh ^= hh >> 32;
      if ((double)(hh >> 11) / (double)(1ull << 53) < keep_prob) {
        g[r] *= fact;
        h[r] = fact;
        sel[m++] = (uint32_t)r;
      }
    }
  }
  return m;
}

/* ------------------------------------------------------------------------- */
/* histogram builds (cpu.rs:17-62)                                            */

typedef struct {
  const uint32_t* rows;
  uint64_t m, chunk;
  uint32_t index_nodes, nf, nb;
  const uint32_t* node;
  const float* g;
  const float* h;
  const int32_t* qg;
  const int32_t* qh;
  const uint8_t* bins;
  int odd_only;
  size_t hsz;
  float** locf;
  int64_t** loci;
} hist_job;

static void hist_ref_worker(int ti, void* arg) {
  hist_job* J = (hist_job*)arg;
  float* loc = (float*)calloc(J->hsz * 2, sizeof(float));
  J->locf[ti] = loc;
  uint64_t lo = (uint64_t)ti * J->chunk, hi = (uint64_t)(ti + 1) * J->chunk;
  if (hi > J->m) hi = J->m;
  const size_t fb = (size_t)J->nf * J->nb;
  for (uint64_t q = lo; q < hi; q++) {
    uint32_t r = J->rows[q];
    uint32_t nv = J->node[r];
    size_t idx_node;
    if (J->odd_only) {
      if ((nv & 1u) == 0) continue;
      idx_node = nv >> 1;
    } else {
      idx_node = nv;
    }
    float gr = J->g[r], hr = J->h[r];
    size_t off = idx_node * fb;
    const uint8_t* rb = J->bins + (size_t)r * J->nf;
    for (uint32_t f = 0; f < J->nf; f++) {
      size_t idx = (off + (size_t)f * J->nb + rb[f]) * 2;
      loc[idx] += gr;
      loc[idx + 1] += hr;
    }
  }
}

static void hist_exact_worker(int ti, void* arg) {
  hist_job* J = (hist_job*)arg;
  int64_t* loc = (int64_t*)calloc(J->hsz * 2, sizeof(int64_t));
  J->loci[ti] = loc;
  uint64_t lo = (uint64_t)ti * J->chunk, hi = (uint64_t)(ti + 1) * J->chunk;
  if (hi > J->m) hi = J->m;
  const size_t fb = (size_t)J->nf * J->nb;
  for (uint64_t q = lo; q < hi; q++) {
    uint32_t r = J->rows[q];
    uint32_t nv = J->node[r];
    size_t idx_node;
    if (J->odd_only) {
      if ((nv & 1u) == 0) continue;
      idx_node = nv >> 1;
    } else {
      idx_node = nv;
    }
    int64_t gr = J->qg[r], hr = J->qh[r];
    size_t off = idx_node * fb;
    const uint8_t* rb = J->bins + (size_t)r * J->nf;
    for (uint32_t f = 0; f < J->nf; f++) {
      size_t idx = (off + (size_t)f * J->nb + rb[f]) * 2;
      loc[idx] += gr;
      loc[idx + 1] += hr;
    }
  }
}

static float* build_hist_ref(hist_job* J, int nt) {
  J->chunk = (J->m + (uint64_t)nt - 1) / (uint64_t)nt;
  J->locf = (float**)calloc((size_t)nt, sizeof(float*));
  par_run(nt, hist_ref_worker, J);
  float* out = rayon_tree_f32(J->locf, 0, nt, J->hsz * 2);
  free(J->locf);
  return out;
}

static int64_t* build_hist_exact(hist_job* J, int nt) {
  J->chunk = (J->m + (uint64_t)nt - 1) / (uint64_t)nt;
  J->loci = (int64_t**)calloc((size_t)nt, sizeof(int64_t*));
  par_run(nt, hist_exact_worker, J);
  int64_t* out = J->loci[0];
  for (int t = 1; t < nt; t++) {
    for (size_t i = 0; i < J->hsz * 2; i++) out[i] += J->loci[t][i];
    free(J->loci[t]);
  }
  free(J->loci);
  return out;
}

void orc_level_hist_exact(const uint8_t* bins, uint64_t n, uint32_t nf, uint32_t n_bins,
                          const int32_t* node, const float* g, const float* h, int e_g,
                          int e_h, uint32_t groups, int odd_only, int64_t* out) {
  float sg = rw_pow2f(e_g), sh = rw_pow2f(e_h);
  size_t fb = (size_t)nf * n_bins;
  memset(out, 0, sizeof(int64_t) * groups * fb * 2);
  for (uint64_t r = 0; r < n; r++) {
    if (node[r] < 0) continue;
    uint32_t nv = (uint32_t)node[r];
    if (odd_only && (nv & 1u) == 0) continue;
    size_t gi = odd_only ? (nv >> 1) : nv;
    int64_t qg = rw_quantize(g[r], sg), qh = rw_quantize(h[r], sh);
    for (uint32_t f = 0; f < nf; f++) {
      size_t idx = (gi * fb + (size_t)f * n_bins + bins[r * nf + f]) * 2;
      out[idx] += qg;
      out[idx + 1] += qh;
    }
  }
}

/* ------------------------------------------------------------------------- */
/* split search (cpu.rs:234-276) + monotone/colsample extensions              */

typedef struct {
  uint32_t n_nodes, nf, nb;
  const float* histf;   /* ref mode */
  const int64_t* histi; /* exact mode */
  double inv_g, inv_h;
  double lambda, min_child;
  const int32_t* monotone;
  uint32_t n_monotone;
  float colsample;
  uint32_t tree_seed;
  double* best_g;
  uint32_t* best_b;
} split_job;

/* Monotone extension (gpu_kernels.rs:888-896): the child weights use the left/right
 * (g, h) totals over all nodes. In exact mode the totals are exact integer sums of the
 * nodes' fixed-point prefixes, converted once; in ref mode f64 sums in node order. */
static void split_feature(uint32_t f, split_job* J, double* gain, double* pg, double* ph,
                          double* glt, double* hlt, double* grt, double* hrt) {
  uint32_t nb = J->nb, nsplit = nb - 1;
  int mono = (J->monotone && f < J->n_monotone) ? J->monotone[f] : 0;
  int64_t* mi = mono && J->histi ? (int64_t*)calloc((size_t)nsplit * 4, sizeof(int64_t)) : NULL;
  for (uint32_t b = 0; b < nsplit; b++) {
    gain[b] = 0.0;
    glt[b] = hlt[b] = grt[b] = hrt[b] = 0.0;
  }
  for (uint32_t nd = 0; nd < J->n_nodes; nd++) {
    size_t hb = ((size_t)nd * J->nf + f) * nb;
    double gl = 0.0, hl = 0.0;
    if (J->histf) {
      for (uint32_t b = 0; b < nb; b++) {
        gl += (double)J->histf[(hb + b) * 2];
        hl += (double)J->histf[(hb + b) * 2 + 1];
        pg[b] = gl;
        ph[b] = hl;
      }
    } else {
      int64_t sg = 0, sh = 0, tg = 0, th = 0;
      for (uint32_t b = 0; b < nb; b++) {
        tg += J->histi[(hb + b) * 2];
        th += J->histi[(hb + b) * 2 + 1];
      }
      for (uint32_t b = 0; b < nb; b++) {
        sg += J->histi[(hb + b) * 2];
        sh += J->histi[(hb + b) * 2 + 1];
        pg[b] = (double)sg * J->inv_g;
        ph[b] = (double)sh * J->inv_h;
        if (mi && b < nsplit) {
          mi[4 * b] += sg;
          mi[4 * b + 1] += sh;
          mi[4 * b + 2] += tg - sg;
          mi[4 * b + 3] += th - sh;
        }
      }
      gl = pg[nb - 1];
      hl = ph[nb - 1];
    }
    double gt = gl, ht = hl;
    double parent = gt * gt / (ht + J->lambda);
    for (uint32_t b = 0; b < nsplit; b++) {
      double gl2 = pg[b], hl2 = ph[b];
      double gr = gt - gl2, hr = ht - hl2;
      double valid = (double)((hl2 >= J->min_child) & (hr >= J->min_child));
      gain[b] += valid * (gl2 * gl2 / (hl2 + J->lambda) + gr * gr / (hr + J->lambda) - parent);
      if (mono && !mi) {
        glt[b] += gl2;
        hlt[b] += hl2;
        grt[b] += gr;
        hrt[b] += hr;
      }
    }
  }
  if (mi) {
    for (uint32_t b = 0; b < nsplit; b++) {
      glt[b] = (double)mi[4 * b] * J->inv_g;
      hlt[b] = (double)mi[4 * b + 1] * J->inv_h;
      grt[b] = (double)mi[4 * b + 2] * J->inv_g;
      hrt[b] = (double)mi[4 * b + 3] * J->inv_h;
    }
    free(mi);
  }
  int dropped = J->colsample < 1.0f && hash01(f, J->tree_seed ^ 0x5bd1e995u) >= J->colsample;
  for (uint32_t b = 0; b < nsplit; b++) {
    if (dropped) {
      gain[b] = -1e30;
      continue;
    }
    if (mono) {
      double wl = -glt[b] / (hlt[b] + J->lambda);
      double wr = -grt[b] / (hrt[b] + J->lambda);
      if ((mono > 0 && wl > wr) || (mono < 0 && wl < wr)) gain[b] = -1e30;
    }
  }
  double bg = -INFINITY;
  uint32_t bb = 0;
  for (uint32_t b = 0; b < nsplit; b++)
    if (gain[b] > bg) {
      bg = gain[b];
      bb = b;
    }
  J->best_g[f] = bg;
  J->best_b[f] = bb;
}

typedef struct {
  split_job* J;
  int nt;
} split_par;

static void split_worker(int ti, void* arg) {
  split_par* P = (split_par*)arg;
  split_job* J = P->J;
  uint32_t nb = J->nb;
  double* buf = (double*)malloc(sizeof(double) * nb * 7);
  for (uint32_t f = (uint32_t)ti; f < J->nf; f += (uint32_t)P->nt)
    split_feature(f, J, buf, buf + nb, buf + 2 * nb, buf + 3 * nb, buf + 4 * nb, buf + 5 * nb,
                  buf + 6 * nb);
  free(buf);
}

/* ------------------------------------------------------------------------- */
/* trainer (cpu.rs:123-325)                                                   */

typedef struct {
  const float* pred;
  const float* y;
  float* g;
  float* h;
  uint64_t n;
  int logistic, exact, nt;
} grad_job;

static void grad_worker(int ti, void* arg) {
  grad_job* J = (grad_job*)arg;
  uint64_t chunk = (J->n + (uint64_t)J->nt - 1) / (uint64_t)J->nt;
  uint64_t lo = (uint64_t)ti * chunk, hi = lo + chunk < J->n ? lo + chunk : J->n;
  for (uint64_t i = lo; i < hi; i++) {
    if (J->logistic) {
      if (J->exact) {
        rw_logistic_grad(J->pred[i], J->y[i], &J->g[i], &J->h[i]);
      } else {
        float pr = 1.0f / (1.0f + expf(-J->pred[i]));
        J->g[i] = pr - J->y[i];
        float hv = pr * (1.0f - pr);
        J->h[i] = hv > 1e-6f ? hv : 1e-6f;
      }
    } else {
      J->g[i] = J->pred[i] - J->y[i];
      J->h[i] = 1.0f;
    }
  }
}

int orc_train(const orc_params* p, const float* x, const float* y, uint64_t n, uint32_t nf,
              const float* cuts, float base_score, uint32_t* feat, float* thr,
              uint32_t* thr_bin, float* leafval, float* fi_gain, float* fi_count,
              orc_trace* trace) {
  const uint32_t nbins = p->n_bins, nb1 = nbins - 1, depth = p->depth;
  const uint32_t leaves = 1u << depth;
  const double lambda = (double)p->lambda, lr = (double)p->learning_rate;
  const double min_child = (double)p->min_child_h;
  const int nt = p->n_threads > 0 ? p->n_threads : orc_default_threads();
  const int exact = p->exact != 0;
  const int logistic = p->objective == 0;
  if (nbins < 2 || nbins > 256 || depth < 1 || depth > 12 || n == 0 || nf == 0) return -1;

  /* cpu.rs:148-161: bin once row-major, then a column-major copy (both in parallel) */
  uint8_t* bins = (uint8_t*)malloc(n * nf);
  uint8_t* bins_col = (uint8_t*)malloc(n * nf);
  bin_job bj = {x, n, nf, cuts, nbins, bins, bins_col, nt};
  par_run(nt, bin_rows_worker, &bj);
  par_run(nt, bin_cols_worker, &bj);
  struct timespec ts0;
  clock_gettime(CLOCK_MONOTONIC, &ts0);

  float* pred = (float*)malloc(n * sizeof(float));
  for (uint64_t i = 0; i < n; i++) pred[i] = base_score;
  uint32_t* node = (uint32_t*)calloc(n, sizeof(uint32_t));
  float* hess = (float*)malloc(n * sizeof(float));
  for (uint64_t i = 0; i < n; i++) hess[i] = 1.0f;
  float* g = (float*)malloc(n * sizeof(float));
  int32_t* qg = exact ? (int32_t*)calloc(n, sizeof(int32_t)) : NULL;
  int32_t* qh = exact ? (int32_t*)calloc(n, sizeof(int32_t)) : NULL;
  uint32_t* all_rows = (uint32_t*)malloc(n * sizeof(uint32_t));
  for (uint64_t i = 0; i < n; i++) all_rows[i] = (uint32_t)i;
  uint32_t* samp_buf = (uint32_t*)malloc(n * sizeof(uint32_t));
  memset(fi_gain, 0, nf * sizeof(float));
  memset(fi_count, 0, nf * sizeof(float));

  uint64_t stride = 1;
  if (p->subsample < 0.999f) {
    double sd = round(1.0 / (double)p->subsample);
    if (sd < 1.0) sd = 1.0;
    stride = sd >= 1.8446744073709552e19 ? UINT64_MAX : (uint64_t)sd;
  }
  double* best_g = (double*)malloc(nf * sizeof(double));
  uint32_t* best_b = (uint32_t*)malloc(nf * sizeof(uint32_t));
  const size_t strideh = (size_t)nf * nbins;

  for (uint32_t t = 0; t < p->n_trees; t++) {
    grad_job gj = {pred, y, g, hess, n, logistic, exact, nt};
    par_run(nt, grad_worker, &gj);
    memset(node, 0, n * sizeof(uint32_t));

    const uint32_t* samp;
    uint64_t m;
    if (p->goss_top > 0.0f) {
      m = goss_sample(g, hess, n, (double)p->goss_top, (double)p->goss_other, (uint64_t)t,
                      samp_buf);
      samp = samp_buf;
    } else if (stride > 1) {
      m = 0;
      for (uint64_t r = t % stride; r < n; r += stride) {
        samp_buf[m++] = (uint32_t)r;
        if (r > UINT64_MAX - stride) break;
      }
      samp = samp_buf;
    } else {
      samp = all_rows;
      m = n;
    }

    if (trace && t < trace->trace_trees && trace->tree_g && trace->tree_h) {
      float* tg = trace->tree_g + (size_t)t * n;
      float* th = trace->tree_h + (size_t)t * n;
      memset(tg, 0, n * sizeof(float));
      memset(th, 0, n * sizeof(float));
      for (uint64_t q = 0; q < m; q++) {
        tg[samp[q]] = g[samp[q]];
        th[samp[q]] = hess[samp[q]];
      }
    }
    int e_g = 0, e_h = 0, w_g = 0, w_h = 0;
    uint32_t bits_g = 0; /* IEEE bits of the round's max |g| (exact mode) */
    if (exact) {
      /* per-round fixed-point scales from the maxima over the sampled rows */
      float mg = 0.0f, mh = 0.0f;
      for (uint64_t q = 0; q < m; q++) {
        uint32_t r = samp[q];
        float ag = fabsf(g[r]);
        if (ag > mg) mg = ag;
        if (hess[r] > mh) mh = hess[r];
      }
      uint32_t bg, bh;
      memcpy(&bg, &mg, 4);
      memcpy(&bh, &mh, 4);
      bits_g = bg;
      e_g = rw_qscale_exp(bg);
      e_h = rw_qscale_exp(bh);
      w_g = rw_wscale_exp(bg, n);
      w_h = rw_wscale_exp(bh, n);
      float sg = rw_pow2f(e_g), sh = rw_pow2f(e_h);
      memset(qg, 0, n * sizeof(int32_t));
      memset(qh, 0, n * sizeof(int32_t));
      for (uint64_t q = 0; q < m; q++) {
        uint32_t r = samp[q];
        qg[r] = rw_quantize(g[r], sg);
        qh[r] = rw_quantize(hess[r], sh);
      }
      if (trace && t == 0) {
        trace->e_g = e_g;
        trace->e_h = e_h;
      }
    }
    const double inv_g = exact ? 1.0 / (double)rw_pow2f(e_g) : 1.0;
    const double inv_h = exact ? 1.0 / (double)rw_pow2f(e_h) : 1.0;

    float* prev_f = NULL;
    int64_t* prev_i = NULL;
    for (uint32_t level = 0; level < depth; level++) {
      uint32_t n_nodes = 1u << level;
      float* histf = NULL;
      int64_t* histi = NULL;
      hist_job hj;
      memset(&hj, 0, sizeof hj);
      hj.rows = samp;
      hj.m = m;
      hj.nf = nf;
      hj.nb = nbins;
      hj.node = node;
      hj.g = g;
      hj.h = hess;
      hj.qg = qg;
      hj.qh = qh;
      hj.bins = bins;
      if (level == 0 || !p->subtract) {
        hj.index_nodes = n_nodes;
        hj.hsz = (size_t)n_nodes * strideh;
        hj.odd_only = 0;
        if (exact) histi = build_hist_exact(&hj, nt);
        else histf = build_hist_ref(&hj, nt);
      } else {
        uint32_t prev_nodes = n_nodes / 2;
        hj.index_nodes = prev_nodes;
        hj.hsz = (size_t)prev_nodes * strideh;
        hj.odd_only = 1;
        size_t sl = strideh * 2;
        if (exact) {
          int64_t* odd = build_hist_exact(&hj, nt);
          histi = (int64_t*)malloc(sizeof(int64_t) * n_nodes * sl);
          for (uint32_t i = 0; i < prev_nodes; i++)
            for (size_t xx = 0; xx < sl; xx++) {
              histi[(2 * i + 1) * sl + xx] = odd[i * sl + xx];
              histi[(2 * i) * sl + xx] = prev_i[i * sl + xx] - odd[i * sl + xx];
            }
          free(odd);
        } else {
          float* odd = build_hist_ref(&hj, nt);
          histf = (float*)malloc(sizeof(float) * n_nodes * sl);
          for (uint32_t i = 0; i < prev_nodes; i++)
            for (size_t xx = 0; xx < sl; xx++) {
              histf[(2 * i + 1) * sl + xx] = odd[i * sl + xx];
              histf[(2 * i) * sl + xx] = prev_f[i * sl + xx] - odd[i * sl + xx];
            }
          free(odd);
        }
      }
      if (trace && t == 0 && exact && level < 16 && trace->level_hist[level])
        memcpy(trace->level_hist[level], histi, sizeof(int64_t) * n_nodes * strideh * 2);

      split_job sj;
      memset(&sj, 0, sizeof sj);
      sj.n_nodes = n_nodes;
      sj.nf = nf;
      sj.nb = nbins;
      sj.histf = histf;
      sj.histi = histi;
      sj.inv_g = inv_g;
      sj.inv_h = inv_h;
      sj.lambda = lambda;
      sj.min_child = min_child;
      sj.monotone = p->monotone;
      sj.n_monotone = p->n_monotone;
      sj.colsample = p->colsample;
      sj.tree_seed = tree_seed_of(t);
      sj.best_g = best_g;
      sj.best_b = best_b;
      split_par sp = {&sj, nt};
      par_run(nt, split_worker, &sp);
      double bgain = -INFINITY;
      uint32_t bf = 0, bb = 0;
      for (uint32_t f = 0; f < nf; f++)
        if (best_g[f] > bgain) {
          bgain = best_g[f];
          bf = f;
          bb = best_b[f];
        }

      size_t k = (size_t)t * depth + level;
      feat[k] = bf;
      thr[k] = cuts[(size_t)bf * nb1 + bb];
      if (thr_bin) thr_bin[k] = bb;
      fi_gain[bf] += (float)(bgain > 0.0 ? bgain : 0.0);
      fi_count[bf] += 1.0f;
      if (trace && t == 0 && level < 16) {
        trace->split_f[level] = bf;
        trace->split_b[level] = bb;
      }
      const uint8_t* col = bins_col + (size_t)bf * n;
      for (uint64_t r = 0; r < n; r++) node[r] = node[r] * 2 + (col[r] > bb ? 1u : 0u);
      free(prev_f);
      free(prev_i);
      prev_f = histf;
      prev_i = histi;
    }
    free(prev_f);
    free(prev_i);

    if (trace && t < trace->trace_trees && trace->tree_leaf)
      for (uint64_t r = 0; r < n; r++) trace->tree_leaf[(size_t)t * n + r] = (uint16_t)node[r];
    /* leaf values (cpu.rs:286-318) */
    double* lg;
    double* lc;
    if (exact) {
      /* exact int64 sums of the unquantised f32 g/h in the wide fixed point
       * (rw_wquantize), so the leaf values do not depend on the histogram's 17-bit q */
      int64_t* sg = (int64_t*)calloc(leaves, sizeof(int64_t));
      int64_t* sh = (int64_t*)calloc(leaves, sizeof(int64_t));
      int64_t* s2 = p->leafvar ? (int64_t*)calloc(leaves, sizeof(int64_t)) : NULL;
      /* the g^2 scale: (max |g|)^2 in f32 bounds every g*g (f32 rounding is monotone) */
      const int w_g2 = p->leafvar ? rw_wscale_exp(rw_sq_maxbits(bits_g), n) : 0;
      for (uint64_t q = 0; q < m; q++) {
        uint32_t r = samp[q];
        sg[node[r]] += rw_wquantize(g[r], w_g);
        sh[node[r]] += rw_wquantize(hess[r], w_h);
        if (s2) s2[node[r]] += rw_wquantize(g[r] * g[r], w_g2);
      }
      lg = (double*)malloc(leaves * sizeof(double));
      lc = (double*)malloc(leaves * sizeof(double));
      for (uint32_t l = 0; l < leaves; l++) {
        lg[l] = rw_wvalue(sg[l], w_g);
        lc[l] = rw_wvalue(sh[l], w_h);
      }
      if (s2)
        for (uint32_t l = 0; l < leaves; l++)
          p->leafvar[(size_t)t * leaves + l] =
              rw_leaf_variance(lg[l], lc[l], rw_wvalue(s2[l], w_g2), lr);
      free(s2);
      free(sg);
      free(sh);
    } else {
      uint64_t lchunk = (m + (uint64_t)nt - 1) / (uint64_t)nt;
      double** lgs = (double**)malloc(sizeof(double*) * nt);
      double** lcs = (double**)malloc(sizeof(double*) * nt);
      for (int ti = 0; ti < nt; ti++) {
        lgs[ti] = (double*)calloc(leaves, sizeof(double));
        lcs[ti] = (double*)calloc(leaves, sizeof(double));
        uint64_t lo = (uint64_t)ti * lchunk, hi = lo + lchunk < m ? lo + lchunk : m;
        for (uint64_t q = lo; q < hi; q++) {
          uint32_t r = samp[q];
          lgs[ti][node[r]] += (double)g[r];
          lcs[ti][node[r]] += (double)hess[r];
        }
      }
      /* cpu.rs reduces the (lg, lc) pairs with one tree; both vectors follow it. */
      lg = rayon_tree_f64(lgs, 0, nt, leaves);
      lc = rayon_tree_f64(lcs, 0, nt, leaves);
      free(lgs);
      free(lcs);
    }
    for (uint32_t l = 0; l < leaves; l++)
      leafval[(size_t)t * leaves + l] = (float)(-lr * lg[l] / (lc[l] + lambda));
    free(lg);
    free(lc);
    const float* lv = leafval + (size_t)t * leaves;
    for (uint64_t r = 0; r < n; r++) pred[r] += lv[node[r]];
  }

  if (trace) {
    struct timespec ts1;
    clock_gettime(CLOCK_MONOTONIC, &ts1);
    trace->loop_seconds = (double)(ts1.tv_sec - ts0.tv_sec) + 1e-9 * (double)(ts1.tv_nsec - ts0.tv_nsec);
  }
  free(bins);
  free(bins_col);
  free(pred);
  free(node);
  free(hess);
  free(g);
  free(qg);
  free(qh);
  free(all_rows);
  free(samp_buf);
  free(best_g);
  free(best_b);
  return 0;
}

/* ------------------------------------------------------------------------- */
/* booster.rs:582-601 predict_cpu                                             */

void orc_predict(const float* x, uint64_t n, uint32_t nf, uint32_t n_trees, uint32_t depth,
                 const uint32_t* feat, const float* thr, const float* leafval, float base,
                 float* out) {
  uint32_t nl = 1u << depth;
  for (uint64_t i = 0; i < n; i++) {
    const float* row = x + i * nf;
    float acc = base;
    for (uint32_t t = 0; t < n_trees; t++) {
      uint32_t leaf = 0;
      for (uint32_t d = 0; d < depth; d++) {
        size_t k = (size_t)t * depth + d;
        leaf = leaf * 2 + (row[feat[k]] > thr[k] ? 1u : 0u);
      }
      acc += leafval[(size_t)t * nl + leaf];
    }
    out[i] = acc;
  }
}

/* ------------------------------------------------------------------------- */
/* metrics.rs                                                                 */

static const float* g_auc_scores;
static int cmp_idx_score(const void* a, const void* b) {
  uint64_t i = *(const uint64_t*)a, j = *(const uint64_t*)b;
  float x = g_auc_scores[i], y = g_auc_scores[j];
  if (x < y) return -1;
  if (x > y) return 1;
  return (i > j) - (i < j); /* stable */
}

double orc_auc(const float* s, const float* y, uint64_t n) {
  uint64_t* order = (uint64_t*)malloc(n * sizeof(uint64_t));
  for (uint64_t i = 0; i < n; i++) order[i] = i;
  g_auc_scores = s;
  qsort(order, n, sizeof(uint64_t), cmp_idx_score);
  double* ranks = (double*)malloc(n * sizeof(double));
  uint64_t i = 0;
  while (i < n) {
    uint64_t j = i + 1;
    while (j < n && s[order[j]] == s[order[i]]) j++;
    double avg = (double)((i + 1) + j) / 2.0;
    for (uint64_t k = i; k < j; k++) ranks[order[k]] = avg;
    i = j;
  }
  double sum_pos = 0.0, n_pos = 0.0;
  for (uint64_t k = 0; k < n; k++)
    if (y[k] > 0.5f) {
      sum_pos += ranks[k];
      n_pos += 1.0;
    }
  double n_neg = (double)n - n_pos;
  free(order);
  free(ranks);
  if (n_pos == 0.0 || n_neg == 0.0) return NAN;
  return (sum_pos - n_pos * (n_pos + 1.0) / 2.0) / (n_pos * n_neg);
}

double orc_logloss(const float* s, const float* y, uint64_t n) {
  const double eps = 1e-7;
  double acc = 0.0;
  for (uint64_t i = 0; i < n; i++) {
    double p = 1.0 / (1.0 + exp(-(double)s[i]));
    if (p < eps) p = eps;
    if (p > 1.0 - eps) p = 1.0 - eps;
    acc += -((double)y[i] * log(p) + (1.0 - (double)y[i]) * log(1.0 - p));
  }
  return acc / (double)n;
}

double orc_rmse(const float* s, const float* y, uint64_t n) {
  double acc = 0.0;
  for (uint64_t i = 0; i < n; i++) {
    double d = (double)s[i] - (double)y[i];
    acc += d * d;
  }
  return sqrt(acc / (double)n);
}

double orc_mae(const float* s, const float* y, uint64_t n) {
  double acc = 0.0;
  for (uint64_t i = 0; i < n; i++) acc += fabs((double)s[i] - (double)y[i]);
  return acc / (double)n;
}

double orc_r2(const float* s, const float* y, uint64_t n) {
  double mean = 0.0;
  for (uint64_t i = 0; i < n; i++) mean += (double)y[i];
  mean /= (double)n;
  double sse = 0.0, sst = 0.0;
  for (uint64_t i = 0; i < n; i++) {
    double yd = (double)y[i];
    sse += pow((double)s[i] - yd, 2.0);
    sst += pow(yd - mean, 2.0);
  }
  return sst == 0.0 ? NAN : 1.0 - sse / sst;
}

double orc_accuracy(const float* s, const float* y, uint64_t n) {
  uint64_t correct = 0;
  for (uint64_t i = 0; i < n; i++) {
    float pred = s[i] > 0.0f ? 1.0f : 0.0f;
    if (fabsf(pred - y[i]) < 0.5f) correct++;
  }
  return (double)correct / (double)n;
}

/* ------------------------------------------------------------------------- */
/* encoding.rs:18-95 out-of-fold target encoding                              */

static const uint64_t kHashSalt = 0x0041445650524F50ull; /* encoding.rs:27 */

static int64_t code_of(float v) {
  /* f32::round (half away from zero) then a saturating `as i64` cast */
  if (v != v) return 0;
  float r = roundf(v);
  if (r >= 9.223372036854775807e18f) return INT64_MAX;
  if (r <= -9.223372036854775808e18f) return INT64_MIN;
  return (int64_t)r;
}

static int64_t key_of(float v, uint64_t hb) {
  int64_t c = code_of(v);
  if (hb == 0) return c;
  uint64_t x = ((uint64_t)c ^ kHashSalt) * 0x9E3779B97F4A7C15ull;
  x ^= x >> 29;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 32;
  return (int64_t)(x % hb);
}

typedef struct {
  int64_t key;
  int used;
  double* sum;
  uint64_t* cnt;
} te_slot;

typedef struct {
  te_slot* s;
  size_t cap;
} te_map;

static te_slot* te_get(te_map* m, int64_t key, uint32_t k) {
  size_t h = (size_t)(((uint64_t)key * 0x9E3779B97F4A7C15ull) >> 17) & (m->cap - 1);
  while (m->s[h].used && m->s[h].key != key) h = (h + 1) & (m->cap - 1);
  if (!m->s[h].used) {
    m->s[h].used = 1;
    m->s[h].key = key;
    m->s[h].sum = (double*)calloc(k, sizeof(double));
    m->s[h].cnt = (uint64_t*)calloc(k, sizeof(uint64_t));
  }
  return &m->s[h];
}

int orc_target_encode(float* x, uint64_t n, uint32_t nf, const float* y, const uint32_t* cat,
                      uint32_t n_cat, float smoothing, uint32_t k_folds, uint64_t hash_buckets,
                      float* gmean_out) {
  uint32_t k = k_folds < 2 ? 2 : k_folds;
  double a = (double)smoothing;
  double ys = 0.0;
  for (uint64_t i = 0; i < n; i++) ys += (double)y[i];
  float gmean = (float)(ys / (double)n);
  double gm = (double)gmean;
  for (uint32_t ci = 0; ci < n_cat; ci++) {
    uint32_t c = cat[ci];
    te_map mp;
    mp.cap = 1;
    while (mp.cap < 2 * n + 16) mp.cap <<= 1;
    mp.s = (te_slot*)calloc(mp.cap, sizeof(te_slot));
    for (uint64_t i = 0; i < n; i++) {
      te_slot* sl = te_get(&mp, key_of(x[i * nf + c], hash_buckets), k);
      uint32_t f = (uint32_t)(i % k);
      sl->sum[f] += (double)y[i];
      sl->cnt[f] += 1;
    }
    for (uint64_t i = 0; i < n; i++) {
      te_slot* sl = te_get(&mp, key_of(x[i * nf + c], hash_buckets), k);
      uint32_t f = (uint32_t)(i % k);
      double s = 0.0;
      uint64_t ct = 0;
      for (uint32_t j = 0; j < k; j++) s += sl->sum[j];
      for (uint32_t j = 0; j < k; j++) ct += sl->cnt[j];
      s -= sl->sum[f];
      double cnt = (double)ct - (double)sl->cnt[f];
      x[i * nf + c] = cnt > 0.0 ? (float)((s + a * gm) / (cnt + a)) : gmean;
    }
    for (size_t h = 0; h < mp.cap; h++)
      if (mp.s[h].used) {
        free(mp.s[h].sum);
        free(mp.s[h].cnt);
      }
    free(mp.s);
  }
  if (gmean_out) *gmean_out = gmean;
  return 0;
}
