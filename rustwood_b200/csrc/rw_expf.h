/* Deterministic single-precision exponential shared by the GPU kernels and the
 * exact-mode CPU restatement.
 *
 * rustwood's CPU trainer computes the logistic link with Rust's `f32::exp`
 * (src/cpu.rs:185), which on linux-gnu is glibc `expf`; the reference GPU kernel
 * uses whatever its compiler lowers `exp` to (src/gpu_kernels.rs:680). Neither
 * is reproducible bit-for-bit on both a CPU and a GPU, so this library defines
 * its own routine and uses the SAME code on both sides.
 *
 * Method (published): Cody & Waite additive range reduction (W. J. Cody and
 * W. Waite, "Software Manual for the Elementary Functions", Prentice-Hall, 1980):
 *   x = k*ln2 + r,  k = nearest integer to x/ln2,  |r| <= ln2/2,
 * with ln2 split into a 32-bit head (so k*LN2_HI is exact) and a tail.
 * e^r is the Taylor series sum_{i=0..12} r^i / i!, evaluated by Horner's rule
 * in double precision (truncation error < 2e-16 for |r| <= 0.347), then scaled
 * by 2^k and rounded once to float. The double-precision evaluation makes the
 * float result the correctly rounded e^x except when e^x lies within ~1e-15
 * relative of a rounding midpoint.
 *
 * Bit-reproducibility: every operation is an IEEE-754 double add/multiply with
 * round-to-nearest. On the device they are written as __dadd_rn/__dmul_rn,
 * which the compiler never contracts into FMAs; host code that includes this
 * header must be compiled with -ffp-contract=off. The constants below are the
 * mathematical values 1/i! and ln2 (head truncated to 32 bits, tail = ln2 - head),
 * computed for this file.
 */
#ifndef RW_EXPF_H
#define RW_EXPF_H

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define RW_HD __host__ __device__ __forceinline__
#else
#define RW_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define RW_DADD(a, b) __dadd_rn((a), (b))
#define RW_DMUL(a, b) __dmul_rn((a), (b))
#define RW_RINT(a) rint(a)
#else
#include <math.h>
#define RW_DADD(a, b) ((a) + (b))
#define RW_DMUL(a, b) ((a) * (b))
#define RW_RINT(a) nearbyint(a)
#endif

#define RW_LN2_HI 0x1.62e42fee00000p-1
#define RW_LN2_LO 0x1.a39ef35793c76p-33
#define RW_LOG2E 1.4426950408889634

RW_HD double rw_pow2i(int k) {
  /* 2^k for -1022 <= k <= 1023, built from its IEEE-754 bit pattern. */
  uint64_t bits = (uint64_t)(int64_t)(k + 1023) << 52;
  double d;
  memcpy(&d, &bits, sizeof d);
  return d;
}

RW_HD float rw_expf(float xf) {
  if (xf != xf) return xf;                  /* NaN propagates */
  if (xf > 89.0f) return (float)1e300;      /* rounds to +inf */
  if (xf < -104.0f) return 0.0f;            /* below the smallest subnormal */
  double x = (double)xf;
  double kd = RW_RINT(RW_DMUL(x, RW_LOG2E));
  double r = RW_DADD(RW_DADD(x, -RW_DMUL(kd, RW_LN2_HI)), -RW_DMUL(kd, RW_LN2_LO));
  double p = 1.0 / 479001600.0; /* 1/12! */
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 39916800.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 3628800.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 362880.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 40320.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 5040.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 720.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 120.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 24.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0 / 6.0);
  p = RW_DADD(RW_DMUL(p, r), 0.5);
  p = RW_DADD(RW_DMUL(p, r), 1.0);
  p = RW_DADD(RW_DMUL(p, r), 1.0);
  double y = RW_DMUL(p, rw_pow2i((int)kd));
  return (float)y;
}

/* Logistic link and hessian exactly as src/cpu.rs:185-187 writes them, with the
 * exponential above: pr = 1/(1+e^-p), g = pr - y, h = max(pr*(1-pr), 1e-6). The
 * float operations are single IEEE ops (no contraction possible). */
RW_HD void rw_logistic_grad(float p, float y, float* g, float* h) {
  float e = rw_expf(-p);
  float pr = 1.0f / (1.0f + e);
  *g = pr - y;
  float hv = pr * (1.0f - pr);
  *h = hv > 1e-6f ? hv : 1e-6f; /* f32::max(hv, 1e-6) for non-NaN hv */
}

/* Fixed-point quantisation of gradients and hessians.
 *
 * Histogram sums are accumulated exactly in 64-bit integers so that they do not
 * depend on summation order (thread scheduling, GPU count). Per boosting round,
 * each of g and h gets a power-of-two scale 2^e chosen from the round's maximum
 * magnitude M so that |q| = |round(x * 2^e)| <= 2^RW_QBITS:
 *     e = RW_QBITS - E,  where 2^(E-1) <= M < 2^E (frexp exponent of M),
 * clamped to [-126, 100] so 2^e is a normal float. M == 0 gives e = 0.
 * The quantisation error per value is <= 2^-(e+1) <= M * 2^-(RW_QBITS+1).
 *
 * RW_QBITS = 17 lets a 32-bit partial sum hold up to 2^13 rows exactly (|sum| <= 2^30),
 * which is what the GPU histogram kernel accumulates per CTA in shared memory before
 * adding into the int64 cells. The per-value error (2^-18 of the round's maximum) is
 * below the rounding error that f32 accumulation of a few thousand rows already has;
 * on the C1/C2 workloads every split of a 100-200 tree fit matches the f32 reference
 * trainer and test AUC/logloss agree to 6 decimals.
 */
#ifndef RW_QBITS
#define RW_QBITS 17
#endif

RW_HD int rw_qscale_exp(uint32_t max_bits) {
  /* max_bits: IEEE bit pattern of a non-negative float M. */
  if ((max_bits & 0x7fffffffu) == 0u) return 0;
  int biased = (int)((max_bits >> 23) & 0xffu);
  int E = (biased == 0 ? 1 : biased) - 126; /* frexp exponent (subnormals: -125) */
  int e = RW_QBITS - E;
  if (e > 100) e = 100;
  if (e < -126) e = -126;
  return e;
}

RW_HD float rw_pow2f(int e) {
  /* 2^e as float for -126 <= e <= 127. */
  uint32_t bits = (uint32_t)(e + 127) << 23;
  float f;
  memcpy(&f, &bits, sizeof f);
  return f;
}

RW_HD int32_t rw_quantize(float x, float scale) {
  /* round-half-even of x*scale; x*scale is exact (power-of-two scale). */
  if (x != x) return 0;
#if defined(__CUDA_ARCH__)
  return __float2int_rn(__fmul_rn(x, scale));
#else
  return (int32_t)lrintf(x * scale);
#endif
}

/* Wide fixed point for the leaf sums.
 *
 * src/cpu.rs:286-318 sums the sampled rows' unquantised f32 g and h per leaf in f64.
 * Here each row's g and h are scaled by a per-round power of two 2^w chosen from the
 * same maxima M as the histogram scale and from the global row count n:
 *     w = (62 - bitlen(n)) - E,  where 2^(E-1) <= M < 2^E,
 * so every |round(x * 2^w)| <= 2^(62 - bitlen(n)) and the int64 sum over n rows stays
 * within 2^62: the per-leaf sums are exact integers, identical in any summation order
 * and at any GPU count. The rounding error per value is at most M * 2^-(63 - bitlen(n))
 * (2^-43 of M at one million rows); values down to M * 2^-(39 - bitlen(n)) convert
 * exactly. The sum goes back to double as (double)S * 2^-w (one rounding, like the
 * reference's f64 accumulator). */
RW_HD int rw_bitlen64(uint64_t v) {
  int b = 0;
  while (v) {
    b++;
    v >>= 1;
  }
  return b;
}

RW_HD int rw_wscale_exp(uint32_t max_bits, uint64_t n_rows) {
  /* max_bits: IEEE bit pattern of a non-negative finite float M. */
  if ((max_bits & 0x7fffffffu) == 0u) return 0;
  int biased = (int)((max_bits >> 23) & 0xffu);
  if (biased == 0xff) return 0; /* not finite: no meaningful scale */
  int E = (biased == 0 ? 1 : biased) - 126;
  int nb = rw_bitlen64(n_rows);
  if (nb < 1) nb = 1;
  return (62 - nb) - E; /* within [-98, 209]: rw_pow2i covers it */
}

RW_HD int64_t rw_wquantize(float x, int w) {
  /* round-half-even of x * 2^w; the product is exact in double. */
  if (!(x - x == 0.0f)) return 0; /* NaN or infinity */
  double v = RW_DMUL((double)x, rw_pow2i(w));
#if defined(__CUDA_ARCH__)
  return (int64_t)__double2ll_rn(v);
#else
  return (int64_t)llrint(v);
#endif
}

RW_HD double rw_wvalue(int64_t s, int w) {
  /* (double)s * 2^-w: one round-to-nearest conversion, then an exact scaling. */
  return RW_DMUL((double)s, rw_pow2i(-w));
}

/* PGBM (gpu_kernels.rs:1046-1080): IEEE bits of M*M in f32 for the bits of a
 * non-negative M, clamped to the largest finite float; since f32 rounding is monotone,
 * every g*g with |g| <= M is at most this value, so it sets the g^2 sums' wide scale. */
RW_HD uint32_t rw_sq_maxbits(uint32_t max_bits) {
  float m;
  memcpy(&m, &max_bits, 4);
  float m2 = m * m;
  if (!(m2 <= 3.4028234663852886e38f)) m2 = 3.4028234663852886e38f; /* inf or NaN */
  uint32_t b;
  memcpy(&b, &m2, 4);
  return b;
}

/* A leaf's PGBM variance from its exact sums (G, H, S2 = sum of g^2), evaluated in f64:
 * lr^2 * max(S2/H - (G/H)^2, 0) when H > 1, else 0; rounded once to f32. */
RW_HD float rw_leaf_variance(double G, double H, double S2, double lr) {
  if (!(H > 1.0)) return 0.0f;
  const double m = G / H;
  const double v = RW_DADD(S2 / H, -RW_DMUL(m, m));
  return (float)RW_DMUL(RW_DMUL(lr, lr), v > 0.0 ? v : 0.0);
}

#endif /* RW_EXPF_H */
