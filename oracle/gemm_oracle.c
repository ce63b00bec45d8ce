/* gemm_oracle.c - TEST INFRASTRUCTURE: the CPU restatement of the reference's GEMM path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this file's library
 * (oracle/liboracle.so). Nothing in the product links or calls it.
 *
 * What it restates, each against the reference file:line it follows (paths inside Davinchy/macuda):
 *   orc_gemm            C = alpha * op(A) op(B) + beta * C in fp64, column-major, both transposes,
 *                       lda/ldb/ldc, strided batches, inputs f32/f16/bf16 - the arithmetic every
 *                       reference kernel implements (cuda-shim/libtinycublas/gemm.cu:7-35 scalar
 *                       kernel; :241-388 tc2 template), evaluated exactly instead of in fp32, plus the
 *                       normalisation scale |alpha| * |op(A)_i| * |op(B)_j| + |beta| * |C0_ij| used by
 *                       the error gate.
 *   orc_ref_splitk_plan the reference's split-K plan (cuda-shim/libtinycublas/cublas.c:69-78), with the
 *                       SM count as a parameter (the reference hard-codes 170).
 *   orc_ref_contract    the reference's type contract (cublas.c:118-134).
 *   orc_half_bits_to_float, orc_float_to_half_bits, orc_float_to_bf16_bits: IEEE conversions
 *                       (cublas.c:110-116 restates the first), round to nearest even.
 *   orc_cpu_gemm_f16_tn a multithreaded fp16 GEMM on the host (F16C conversion, AVX2 FMA, OpenMP) that
 *                       stands in for ggml-cpu's fp16 matmul, which the reference fetches at build time
 *                       and which is not in this tree: the timed CPU baseline.
 */
#include <immintrin.h>
#include <math.h>
#include <omp.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ---- conversions -------------------------------------------------------------------------------- */

float orc_half_bits_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1fu, f = h & 0x3ffu, bits;
  if (e == 0x1f) bits = sign | 0x7f800000u | (f << 13);
  else if (e == 0) {
    if (f == 0) bits = sign;
    else {
      int shift = 0;
      while (!(f & 0x400u)) { f <<= 1; shift++; }
      f &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 + 1 - shift) << 23) | (f << 13);
    }
  } else bits = sign | ((e + 127 - 15) << 23) | (f << 13);
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

/* float -> binary16, round to nearest even, overflow to inf, NaN kept quiet */
uint16_t orc_float_to_half_bits(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  uint32_t sign = (u >> 16) & 0x8000u;
  uint32_t ax = u & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* rounds to >= 65520: inf */
  if (ax < 0x38800000u) {                                    /* below the smallest normal half */
    if (ax < 0x33000000u) return (uint16_t)sign;             /* below half the smallest subnormal */
    /* value = mant * 2^(e-150); in units of the half subnormal 2^-24 that is mant * 2^(e-126) */
    const uint32_t mant = (ax & 0x7fffffu) | 0x800000u;
    const int e = (int)(ax >> 23);
    const int shift = 126 - e; /* 14..24 here */
    uint32_t q = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (ax >> 23) - 127 + 15;
  uint32_t mant = ax & 0x7fffffu;
  uint32_t q = (e << 10) | (mant >> 13);
  uint32_t rem = mant & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) q++;
  return (uint16_t)(sign | q);
}

float orc_bf16_bits_to_float(uint16_t h) {
  uint32_t bits = (uint32_t)h << 16;
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

uint16_t orc_float_to_bf16_bits(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return (uint16_t)(u >> 16);
}

void orc_f32_to_f16(const float *x, uint16_t *y, long long n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; i++) y[i] = orc_float_to_half_bits(x[i]);
}
void orc_f32_to_bf16(const float *x, uint16_t *y, long long n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; i++) y[i] = orc_float_to_bf16_bits(x[i]);
}
void orc_f16_to_f32(const uint16_t *x, float *y, long long n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; i++) y[i] = orc_half_bits_to_float(x[i]);
}
void orc_bf16_to_f32(const uint16_t *x, float *y, long long n) {
#pragma omp parallel for schedule(static)
  for (long long i = 0; i < n; i++) y[i] = orc_bf16_bits_to_float(x[i]);
}

/* type codes as the reference's dtype_code (cublas.c:107): 0 f32, 1 f16, 2 bf16 */
static inline double elem(const void *p, long long i, int t) {
  if (t == 0) return (double)((const float *)p)[i];
  if (t == 1) return (double)orc_half_bits_to_float(((const uint16_t *)p)[i]);
  return (double)orc_bf16_bits_to_float(((const uint16_t *)p)[i]);
}

/* ---- the fp64 GEMM ---------------------------------------------------------------------------- */

/* R[b][jj][ii] = alpha * sum_k op(A)[rows[ii], k] * op(B)[k, cols[jj]] + beta * C0[rows[ii], cols[jj]]
 * S[b][jj][ii] = |alpha| * ||op(A) row|| * ||op(B) col|| + |beta| * |C0|   (S may be NULL)
 * rows/cols NULL = all of them (nrows = m, ncols = n). C0 may be NULL when beta == 0.
 * Pointer tables (Ap/Bp/Cp, length batch) override base + stride when non-NULL. */
void orc_gemm(int opA, int opB, int m, int n, int k, double alpha, const void *A, const void *const *Ap, int Atype,
              int lda, long long sA, const void *B, const void *const *Bp, int Btype, int ldb, long long sB, double beta,
              const void *C0, const void *const *Cp, int Ctype, int ldc, long long sC, int batch, const int *rows,
              int nrows, const int *cols, int ncols, double *R, double *S) {
  if (!rows) nrows = m;
  if (!cols) ncols = n;
  const long long per = (long long)nrows * ncols;
  const int esA = Atype == 0 ? 4 : 2, esB = Btype == 0 ? 4 : 2, esC = Ctype == 0 ? 4 : 2;
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int b = 0; b < batch; b++) {
    for (int jj = 0; jj < ncols; jj++) {
      const char *Ab = Ap ? (const char *)Ap[b] : (const char *)A + (long long)b * sA * esA;
      const char *Bb = Bp ? (const char *)Bp[b] : (const char *)B + (long long)b * sB * esB;
      const char *Cb = Cp ? (const char *)Cp[b] : (C0 ? (const char *)C0 + (long long)b * sC * esC : NULL);
      const int j = cols ? cols[jj] : jj;
      double *bcol = (double *)malloc(sizeof(double) * (k > 0 ? k : 1));
      double bn2 = 0;
      for (int kk = 0; kk < k; kk++) {
        long long bi = opB == 0 ? kk + (long long)j * ldb : j + (long long)kk * ldb;
        bcol[kk] = elem(Bb, bi, Btype);
        bn2 += bcol[kk] * bcol[kk];
      }
      for (int ii = 0; ii < nrows; ii++) {
        const int i = rows ? rows[ii] : ii;
        double acc = 0, an2 = 0;
        if (opA == 1) {
          const long long base = (long long)i * lda;
          for (int kk = 0; kk < k; kk++) {
            double a = elem(Ab, base + kk, Atype);
            acc += a * bcol[kk];
            an2 += a * a;
          }
        } else {
          for (int kk = 0; kk < k; kk++) {
            double a = elem(Ab, i + (long long)kk * lda, Atype);
            acc += a * bcol[kk];
            an2 += a * a;
          }
        }
        double c0 = 0;
        if (beta != 0 && Cb) c0 = elem(Cb, i + (long long)j * ldc, Ctype);
        R[b * per + (long long)jj * nrows + ii] = alpha * acc + beta * c0;
        if (S) S[b * per + (long long)jj * nrows + ii] = fabs(alpha) * sqrt(an2) * sqrt(bn2) + fabs(beta) * fabs(c0);
      }
      free(bcol);
    }
  }
}

/* X * A = alpha * B for one batch element, A upper-triangular non-unit (n x n, lda), B rows x n
 * (ldb), fp64, result into X (rows x n, ld = rows): the operation of gemm.cu:41-49. */
void orc_trsm_rupn(const float *A, const float *B, int rows, int n, int lda, int ldb, double alpha, double *X) {
  for (int i = 0; i < rows; i++)
    for (int j = 0; j < n; j++) {
      double acc = alpha * B[i + (long long)j * ldb];
      for (int l = 0; l < j; l++) acc -= X[i + (long long)l * rows] * A[l + (long long)j * lda];
      X[i + (long long)j * rows] = acc / A[j + (long long)j * lda];
    }
}

/* ---- the reference's host decisions, restated ------------------------------------------------- */

/* cublas.c:69-78 (SPLITK_WS_BYTES 8 MiB and SPLITK_CNT_N 16384 from cublas.c:66-67) */
int orc_ref_splitk_plan(int m, int n, int k, int batch, int num_sms) {
  if (m <= 0 || n <= 0 || k <= 0 || batch <= 0) return 1;
  long long gx = (m + 63) / 64, gy = (n + 63) / 64;
  if (gy != 1) return 1;
  int S = 1;
  while (gx * S < num_sms && S < 16) S *= 2;
  while (S > 1 && k < 128 * S) S /= 2;
  if (S == 1) return 1;
  if ((long long)batch * S * gx * gy * 64 * 64 * 4 > (8ll << 20) || batch * gx * gy > 16384 || (long long)batch * S > 65535)
    return 1;
  return S;
}

/* cublas.c:118-134. Type codes are CUDA's cudaDataType values (0 = R_32F, 2 = R_16F, 14 = R_16BF),
 * compute types cuBLAS's. Returns 0 (served) or -1 (NOT_SUPPORTED). */
int orc_ref_contract(int At, int Bt, int Ct, int ct) {
  int in = At == 0 ? 0 : At == 2 ? 1 : At == 14 ? 2 : -1;
  int out = Ct == 0 ? 0 : Ct == 2 ? 1 : Ct == 14 ? 2 : -1;
  int bin = Bt == 0 ? 0 : Bt == 2 ? 1 : Bt == 14 ? 2 : -1;
  if (in < 0 || out < 0 || bin != in) return -1;
  int c32 = ct == 68 || ct == 69;
  int c16 = ct == 64 || ct == 65;
  if (in == 0) return (c32 || ct == 77 || ct == 74 || ct == 75) ? 0 : -1;
  if (in == 1) return (c32 || (c16 && out == 1)) ? 0 : -1;
  return c32 ? 0 : -1;
}

/* ---- CPU baseline: fp16 GEMM, C (f32, m x n, ldc) = A^T B, A k x m (lda), B k x n (ldb) --------- */

__attribute__((target("avx2,fma,f16c"))) static inline float hsum256(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v), hi = _mm256_extractf128_ps(v, 1);
  lo = _mm_add_ps(lo, hi);
  lo = _mm_hadd_ps(lo, lo);
  lo = _mm_hadd_ps(lo, lo);
  return _mm_cvtss_f32(lo);
}

__attribute__((target("avx2,fma,f16c"))) void orc_cpu_gemm_f16_tn(int m, int n, int k, const uint16_t *A, int lda,
                                                                    const uint16_t *B, int ldb, float *C, int ldc,
                                                                    int nthreads) {
  if (nthreads > 0) omp_set_num_threads(nthreads);
  const int k8 = k & ~7;
  /* activations converted once to f32, column by column */
  const size_t kp = ((size_t)k + 15) & ~(size_t)15; /* row pitch in floats: 64-byte aligned rows */
  float *Bf = (float *)aligned_alloc(64, sizeof(float) * kp * (size_t)n);
#pragma omp parallel for schedule(static)
  for (int j = 0; j < n; j++)
    for (int kk = 0; kk < k; kk++) Bf[(size_t)j * kp + kk] = orc_half_bits_to_float(B[kk + (size_t)j * ldb]);
  const int MB = 4, NB = 4;
#pragma omp parallel
  {
    float *Af = (float *)aligned_alloc(64, sizeof(float) * (size_t)MB * kp);
#pragma omp for schedule(dynamic, 1)
    for (int i0 = 0; i0 < m; i0 += MB) {
      const int mi = m - i0 < MB ? m - i0 : MB;
      for (int r = 0; r < MB; r++) {
        const uint16_t *src = A + (size_t)(i0 + (r < mi ? r : 0)) * lda;
        for (int kk = 0; kk < k8; kk += 8)
          _mm256_store_ps(Af + (size_t)r * kp + kk, _mm256_cvtph_ps(_mm_loadu_si128((const __m128i *)(src + kk))));
        for (int kk = k8; kk < k; kk++) Af[(size_t)r * kp + kk] = orc_half_bits_to_float(src[kk]);
      }
      for (int j0 = 0; j0 < n; j0 += NB) {
        const int nj = n - j0 < NB ? n - j0 : NB;
        __m256 acc[MB][NB];
        for (int r = 0; r < MB; r++)
          for (int c = 0; c < NB; c++) acc[r][c] = _mm256_setzero_ps();
        const float *bcol[NB];
        for (int c = 0; c < NB; c++) bcol[c] = Bf + (size_t)(j0 + (c < nj ? c : 0)) * kp;
        for (int kk = 0; kk < k8; kk += 8) {
          __m256 bv[NB];
          for (int c = 0; c < NB; c++) bv[c] = _mm256_load_ps(bcol[c] + kk);
          for (int r = 0; r < MB; r++) {
            __m256 av = _mm256_load_ps(Af + (size_t)r * kp + kk);
            for (int c = 0; c < NB; c++) acc[r][c] = _mm256_fmadd_ps(av, bv[c], acc[r][c]);
          }
        }
        for (int r = 0; r < mi; r++)
          for (int c = 0; c < nj; c++) {
            float s = hsum256(acc[r][c]);
            for (int kk = k8; kk < k; kk++) s += Af[(size_t)r * kp + kk] * bcol[c][kk];
            C[(size_t)(i0 + r) + (size_t)(j0 + c) * ldc] = s;
          }
      }
    }
    free(Af);
  }
  free(Bf);
}

int orc_max_threads(void) { return omp_get_max_threads(); }
