/* ggml_calls.c - a C caller of libtinycublas_b200.so that makes the calls ggml-cuda makes, through CUDA's
 * own cublas_v2.h declarations, linked with -ltinycublas_b200 in place of -lcublas. Integer-valued data
 * small enough that every product and sum is exact in fp32, so each output element is compared for
 * equality against a host computation. Exit status 0 when every check passes. */
#include <cublas_v2.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define CK(x)                                                                          \
  do {                                                                                 \
    cudaError_t e_ = (x);                                                              \
    if (e_ != cudaSuccess) {                                                           \
      fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
      exit(2);                                                                         \
    }                                                                                  \
  } while (0)
#define CB(x)                                                                          \
  do {                                                                                 \
    cublasStatus_t s_ = (x);                                                           \
    if (s_ != CUBLAS_STATUS_SUCCESS) {                                                 \
      fprintf(stderr, "%s:%d %s: status %d\n", __FILE__, __LINE__, #x, (int)s_);        \
      exit(3);                                                                         \
    }                                                                                  \
  } while (0)

static int failures = 0;

static float val(long long i, int salt) { return (float)((int)((i * 7 + salt * 13) % 9) - 4); } /* -4..4 */

/* op T weights (k x m, lda = k) times op N activations (k x n, ldb = k) into column-major m x n */
static void ref_tn(const float *A, const float *B, int m, int n, int k, double *R) {
  for (int j = 0; j < n; j++)
    for (int i = 0; i < m; i++) {
      double s = 0;
      for (int p = 0; p < k; p++) s += (double)A[(long long)i * k + p] * B[(long long)j * k + p];
      R[(long long)j * m + i] = s;
    }
}

static void check(const char *what, const float *got, const double *want, long long count) {
  long long bad = 0;
  for (long long i = 0; i < count; i++)
    if ((double)got[i] != want[i]) {
      if (bad < 3) fprintf(stderr, "%s: element %lld got %g want %g\n", what, i, got[i], want[i]);
      bad++;
    }
  printf("%-44s %s (%lld elements)\n", what, bad ? "FAIL" : "ok", count);
  failures += bad != 0;
}

/* IEEE binary16 bits of a float that binary16 represents exactly (the small integers used here), and back */
static uint16_t half_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) == 0) return (uint16_t)(u >> 16);
  return (uint16_t)(((u >> 16) & 0x8000u) | ((((u >> 23) & 0xffu) - 127 + 15) << 10) | ((u >> 13) & 0x3ffu));
}
static float half_value(uint16_t hb) {
  uint32_t u = ((uint32_t)(hb & 0x8000u) << 16);
  if (hb & 0x7fffu) u |= ((uint32_t)(((hb >> 10) & 0x1fu) - 15 + 127) << 23) | ((uint32_t)(hb & 0x3ffu) << 13);
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static uint16_t *dev_half(const float *h, long long count) {
  uint16_t *tmp = (uint16_t *)malloc(count * sizeof(uint16_t)), *d;
  for (long long i = 0; i < count; i++) tmp[i] = half_bits(h[i]);
  CK(cudaMalloc((void **)&d, count * sizeof(uint16_t)));
  CK(cudaMemcpy(d, tmp, count * sizeof(uint16_t), cudaMemcpyHostToDevice));
  free(tmp);
  return d;
}

int main(void) {
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
    fprintf(stderr, "no CUDA device\n");
    return 4;
  }
  cublasHandle_t h;
  cudaStream_t st;
  CB(cublasCreate(&h));
  CK(cudaStreamCreate(&st));
  CB(cublasSetStream(h, st));
  CB(cublasSetMathMode(h, CUBLAS_DEFAULT_MATH));

  /* 1. ggml's prefill projection: cublasGemmEx(T, N), f16 in, f32 out, COMPUTE_32F */
  const int m = 1000, n = 72, k = 512, batch = 3;
  float *A = malloc(sizeof(float) * m * k * batch), *B = malloc(sizeof(float) * k * n * batch);
  for (long long i = 0; i < (long long)m * k * batch; i++) A[i] = val(i, 1);
  for (long long i = 0; i < (long long)k * n * batch; i++) B[i] = val(i, 2);
  uint16_t *dA = dev_half(A, (long long)m * k * batch), *dB = dev_half(B, (long long)k * n * batch);
  float *dC, *C = malloc(sizeof(float) * m * n * batch);
  double *R = malloc(sizeof(double) * m * n * batch);
  CK(cudaMalloc((void **)&dC, sizeof(float) * m * n * batch));
  const float one = 1.f, zero = 0.f;
  CB(cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, m, n, k, &one, dA, CUDA_R_16F, k, dB, CUDA_R_16F, k, &zero, dC,
                  CUDA_R_32F, m, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT));
  CK(cudaStreamSynchronize(st));
  CK(cudaMemcpy(C, dC, sizeof(float) * m * n, cudaMemcpyDeviceToHost));
  ref_tn(A, B, m, n, k, R);
  check("cublasGemmEx T,N f16 -> f32", C, R, (long long)m * n);

  /* 2. attention-style strided batch */
  CB(cublasGemmStridedBatchedEx(h, CUBLAS_OP_T, CUBLAS_OP_N, m, n, k, &one, dA, CUDA_R_16F, k, (long long)m * k, dB,
                                CUDA_R_16F, k, (long long)k * n, &zero, dC, CUDA_R_32F, m, (long long)m * n, batch,
                                CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT));
  CK(cudaStreamSynchronize(st));
  CK(cudaMemcpy(C, dC, sizeof(float) * m * n * batch, cudaMemcpyDeviceToHost));
  for (int b = 0; b < batch; b++) ref_tn(A + (long long)b * m * k, B + (long long)b * k * n, m, n, k, R + (long long)b * m * n);
  check("cublasGemmStridedBatchedEx (batch 3)", C, R, (long long)m * n * batch);

  /* 3. pointer arrays in device memory, the first weight broadcast to every element (GQA-style) */
  const void *hA[3], *hB[3];
  void *hC[3];
  for (int b = 0; b < batch; b++) {
    hA[b] = dA;
    hB[b] = dB + (long long)b * k * n;
    hC[b] = dC + (long long)b * m * n;
  }
  void **dArr;
  CK(cudaMalloc((void **)&dArr, sizeof(void *) * 9));
  CK(cudaMemcpy(dArr, hA, sizeof(hA), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dArr + 3, hB, sizeof(hB), cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dArr + 6, hC, sizeof(hC), cudaMemcpyHostToDevice));
  CK(cudaMemset(dC, 0xff, sizeof(float) * m * n * batch));
  CB(cublasGemmBatchedEx(h, CUBLAS_OP_T, CUBLAS_OP_N, m, n, k, &one, (const void *const *)dArr, CUDA_R_16F, k,
                         (const void *const *)(dArr + 3), CUDA_R_16F, k, &zero, dArr + 6, CUDA_R_32F, m, batch,
                         CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT));
  CK(cudaStreamSynchronize(st));
  CK(cudaMemcpy(C, dC, sizeof(float) * m * n * batch, cudaMemcpyDeviceToHost));
  for (int b = 0; b < batch; b++) ref_tn(A, B + (long long)b * k * n, m, n, k, R + (long long)b * m * n);
  check("cublasGemmBatchedEx (device pointer arrays)", C, R, (long long)m * n * batch);

  /* 4. decode: n = 1 */
  CB(cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, m, 1, k, &one, dA, CUDA_R_16F, k, dB, CUDA_R_16F, k, &zero, dC,
                  CUDA_R_32F, m, CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT));
  CK(cudaStreamSynchronize(st));
  CK(cudaMemcpy(C, dC, sizeof(float) * m, cudaMemcpyDeviceToHost));
  ref_tn(A, B, m, 1, k, R);
  check("cublasGemmEx decode n = 1", C, R, m);

  /* 5. cublasSgemm (exact fp32 in the default math mode), N,N */
  const int sm = 48;
  float *SA = malloc(sizeof(float) * sm * sm), *SB = malloc(sizeof(float) * sm * sm);
  for (int i = 0; i < sm * sm; i++) {
    SA[i] = val(i, 3);
    SB[i] = val(i, 4);
  }
  float *dSA, *dSB, *dSC;
  CK(cudaMalloc((void **)&dSA, sizeof(float) * sm * sm));
  CK(cudaMalloc((void **)&dSB, sizeof(float) * sm * sm));
  CK(cudaMalloc((void **)&dSC, sizeof(float) * sm * sm));
  CK(cudaMemcpy(dSA, SA, sizeof(float) * sm * sm, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(dSB, SB, sizeof(float) * sm * sm, cudaMemcpyHostToDevice));
  CB(cublasSgemm(h, CUBLAS_OP_N, CUBLAS_OP_N, sm, sm, sm, &one, dSA, sm, dSB, sm, &zero, dSC, sm));
  CK(cudaStreamSynchronize(st));
  CK(cudaMemcpy(C, dSC, sizeof(float) * sm * sm, cudaMemcpyDeviceToHost));
  for (int j = 0; j < sm; j++)
    for (int i = 0; i < sm; i++) {
      double s = 0;
      for (int p = 0; p < sm; p++) s += (double)SA[p * sm + i] * SB[j * sm + p];
      R[j * sm + i] = s;
    }
  check("cublasSgemm N,N 48^3", C, R, sm * sm);

  /* 6. COMPUTE_16F with f16 C and half alpha/beta (ggml's f16 path) */
  const uint16_t h1 = half_bits(1.f), h0 = half_bits(0.f);
  uint16_t *dH, *H = malloc(sizeof(uint16_t) * m * 8);
  CK(cudaMalloc((void **)&dH, sizeof(uint16_t) * m * 8));
  CB(cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, m, 8, 64, &h1, dA, CUDA_R_16F, k, dB, CUDA_R_16F, k, &h0, dH, CUDA_R_16F,
                  m, CUBLAS_COMPUTE_16F, CUBLAS_GEMM_DEFAULT));
  CK(cudaStreamSynchronize(st));
  CK(cudaMemcpy(H, dH, sizeof(uint16_t) * m * 8, cudaMemcpyDeviceToHost));
  for (int j = 0; j < 8; j++)
    for (int i = 0; i < m; i++) {
      double s = 0;
      for (int p = 0; p < 64; p++) s += (double)A[(long long)i * k + p] * B[(long long)j * k + p];
      R[(long long)j * m + i] = s;  /* |s| <= 64 * 16: exact in f16 */
      C[(long long)j * m + i] = half_value(H[(long long)j * m + i]);
    }
  check("cublasGemmEx COMPUTE_16F, f16 C", C, R, (long long)m * 8);

  CB(cublasDestroy(h));
  CK(cudaStreamDestroy(st));
  printf("%s\n", failures ? "FAILED" : "ALL OK");
  return failures ? 1 : 0;
}
