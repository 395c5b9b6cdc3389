/*
 * CPU oracle for the preemptible persistent-GEMM runtime.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker: only tests/, the
 * smoke() entry of __graft_entry__.py and the cpu_baseline / reference arm of
 * bench.py may load it.  The product path (apk_b200/, libapk.so) never links,
 * loads or calls anything here.
 *
 * What it restates (reference = AyaanFaisal21/APK, paths relative to it):
 *
 *  - oracle_gen_uniform_glibc:  the reference's input generator,
 *      srand(21); for A then B: v = (float)(rand() / (double)RAND_MAX * 2 - 1)
 *    src/persistent.cu:132-135 (identical in src/yield.cu:367-370,
 *    src/urgent_baseline.cu:187-190, src/midyield.cu, src/tcyield.cu:461-472).
 *    It calls the C library's own srand/rand, so on glibc it IS the
 *    reference's generator, not a re-implementation.
 *
 *  - oracle_gemm_f64:  the reference's float64 host GEMM, an i-k-j loop that
 *    widens each A element to double once per (i,k) and accumulates
 *    a * B[k][j] into a double C row, src/persistent.cu:221-227.
 *
 *  - oracle_check_f32:  the reference's error metric err / max(1, |ref|)
 *    (src/persistent.cu:230-234) with the north-star tolerance supplied by
 *    the caller (fp32: 1e-5*sqrt(K); bf16: 1e-2).
 *
 *  - oracle_round_bf16 / oracle_gemm_f64_bf16:  the quantise-then-reference
 *    rule of src/tcyield.cu:459-483 (the float64 reference is computed from
 *    the already-rounded 16-bit inputs, so quantisation is not part of the
 *    error), applied to bf16 with round-to-nearest-even.
 *
 *  - oracle_gen_normal_bf16:  an independent restatement of the runtime's
 *    seeded N(0,1) generator (counter-based SplitMix64 + Box-Muller, rounded
 *    to bf16) used for the bf16 configurations; the reference has no bf16
 *    generator, so this one is defined by this project and written twice
 *    (here and in apk_b200/csrc/datagen.cpp) so each checks the other.
 *
 * Parity pin: for M=N=K=1024 and seed 21 the reference's loop gives
 * ref[0] = 12.687869863082142 (known-answer value derived from the
 * reference's own loop); tests/test_oracle.py asserts it.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* src/persistent.cu:132-135 — A first (M*K values), then B (K*N values),
 * from one srand(seed) stream. */
void oracle_gen_uniform_glibc(unsigned seed, float *A, size_t nA, float *B,
                              size_t nB) {
  srand(seed);
  for (size_t i = 0; i < nA; ++i)
    A[i] = (float)(rand() / (double)RAND_MAX * 2.0 - 1.0);
  for (size_t i = 0; i < nB; ++i)
    B[i] = (float)(rand() / (double)RAND_MAX * 2.0 - 1.0);
}

/* src/persistent.cu:221-227 — float64 reference, single thread, i-k-j. */
void oracle_gemm_f64(const float *A, const float *B, double *C, int M, int N,
                     int K) {
  memset(C, 0, (size_t)M * N * sizeof(double));
  for (int i = 0; i < M; ++i)
    for (int k = 0; k < K; ++k) {
      const double a = A[(size_t)i * K + k];
      const size_t crow = (size_t)i * N, brow = (size_t)k * N;
      for (int j = 0; j < N; ++j) C[crow + j] += a * B[brow + j];
    }
}

/* Same loop restricted to rows [row0, row0+nrows): used to check a sampled
 * row band of a large product.  C holds nrows*N doubles. */
void oracle_gemm_f64_rows(const float *A, const float *B, double *C, int N,
                          int K, int row0, int nrows) {
  memset(C, 0, (size_t)nrows * N * sizeof(double));
  for (int r = 0; r < nrows; ++r) {
    const int i = row0 + r;
    for (int k = 0; k < K; ++k) {
      const double a = A[(size_t)i * K + k];
      const size_t crow = (size_t)r * N, brow = (size_t)k * N;
      for (int j = 0; j < N; ++j) C[crow + j] += a * B[brow + j];
    }
  }
}

/* Row-parallel restatement of the same loop on all host cores (OpenMP).
 * Each output row is still accumulated by one thread in k order, so the
 * result is bit-identical to oracle_gemm_f64.  Used as the labelled
 * multi-core CPU baseline beside the single-threaded one. */
void oracle_gemm_f64_omp(const float *A, const float *B, double *C, int M,
                         int N, int K, int nthreads) {
  memset(C, 0, (size_t)M * N * sizeof(double));
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
  for (int i = 0; i < M; ++i)
    for (int k = 0; k < K; ++k) {
      const double a = A[(size_t)i * K + k];
      const size_t crow = (size_t)i * N, brow = (size_t)k * N;
      for (int j = 0; j < N; ++j) C[crow + j] += a * B[brow + j];
    }
}

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Error metric of src/persistent.cu:230-234: rel = |got-ref| / max(1,|ref|).
 * Counts NaNs (never-written elements under a NaN pre-fill) and elements
 * whose rel exceeds tol.  Returns the max rel over non-NaN elements. */
double oracle_check_f32(const float *got, const double *ref, size_t n,
                        double tol, long long *n_bad, long long *n_nan) {
  long long bad = 0, nans = 0;
  double max_rel = 0.0;
  for (size_t i = 0; i < n; ++i) {
    const float g = got[i];
    if (isnan(g)) {
      ++nans;
      continue;
    }
    const double err = fabs((double)g - ref[i]);
    const double rel = err / fmax(1.0, fabs(ref[i]));
    if (rel > max_rel) max_rel = rel;
    if (!(rel <= tol)) ++bad;
  }
  if (n_bad) *n_bad = bad;
  if (n_nan) *n_nan = nans;
  return max_rel;
}

/* ---- bf16 helpers ------------------------------------------------------ */

static inline uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu))
    return (uint16_t)((u >> 16) | 0x40); /* quiet NaN */
  const uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

static inline float bf16_to_f32(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

void oracle_round_bf16(const float *in, uint16_t *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = f32_to_bf16_rne(in[i]);
}

void oracle_bf16_to_f32(const uint16_t *in, float *out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = bf16_to_f32(in[i]);
}

/* float64 reference over bf16 inputs (quantise-then-reference,
 * src/tcyield.cu:459-483), rows [row0, row0+nrows), row-parallel. */
void oracle_gemm_f64_bf16_rows(const uint16_t *A, const uint16_t *B,
                               double *C, int N, int K, int row0, int nrows,
                               int nthreads) {
  memset(C, 0, (size_t)nrows * N * sizeof(double));
#ifdef _OPENMP
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
#endif
  for (int r = 0; r < nrows; ++r) {
    const int i = row0 + r;
    for (int k = 0; k < K; ++k) {
      const double a = bf16_to_f32(A[(size_t)i * K + k]);
      const size_t crow = (size_t)r * N, brow = (size_t)k * N;
      for (int j = 0; j < N; ++j) C[crow + j] += a * bf16_to_f32(B[brow + j]);
    }
  }
}

/* ---- seeded N(0,1) -> bf16 --------------------------------------------
 * Element pair p (elements 2p, 2p+1) draws two 64-bit words
 * w0 = splitmix64(seed*2^32 + 2p), w1 = splitmix64(seed*2^32 + 2p + 1);
 * u1 = ((w0 >> 11) + 1) * 2^-53 in (0,1], u2 = (w1 >> 11) * 2^-53 in [0,1);
 * r = sqrt(-2 ln u1); z0 = r cos(2 pi u2), z1 = r sin(2 pi u2);
 * each rounded double -> float -> bf16 (RNE).  SplitMix64 is Steele, Lea
 * and Flood's published mixer (constants 0x9E3779B97F4A7C15,
 * 0xBF58476D1CE4E5B9, 0x94D049BB133111EB). */
static inline uint64_t splitmix64_at(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

void oracle_gen_normal_bf16(uint64_t seed, uint16_t *out, size_t n) {
  const double two_pi = 6.283185307179586476925286766559;
  const uint64_t base = seed << 32;
  for (size_t i = 0; i < n; i += 2) {
    const uint64_t p = i >> 1;
    const uint64_t w0 = splitmix64_at(base + 2 * p);
    const uint64_t w1 = splitmix64_at(base + 2 * p + 1);
    const double u1 = (double)((w0 >> 11) + 1) * 0x1.0p-53;
    const double u2 = (double)(w1 >> 11) * 0x1.0p-53;
    const double r = sqrt(-2.0 * log(u1));
    const double z0 = r * cos(two_pi * u2);
    const double z1 = r * sin(two_pi * u2);
    out[i] = f32_to_bf16_rne((float)z0);
    if (i + 1 < n) out[i + 1] = f32_to_bf16_rne((float)z1);
  }
}

/* uniform[-1,1) through the glibc stream, rounded to bf16: the bf16 inputs
 * of the scaling-surface cells (same generator as fp32, then RNE). */
void oracle_gen_uniform_glibc_bf16(unsigned seed, uint16_t *A, size_t nA,
                                   uint16_t *B, size_t nB) {
  srand(seed);
  for (size_t i = 0; i < nA; ++i)
    A[i] = f32_to_bf16_rne((float)(rand() / (double)RAND_MAX * 2.0 - 1.0));
  for (size_t i = 0; i < nB; ++i)
    B[i] = f32_to_bf16_rne((float)(rand() / (double)RAND_MAX * 2.0 - 1.0));
}
