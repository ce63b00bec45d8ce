// aux_kernels.cu - the small kernels beside the GEMMs: batched triangular solve, the row-block
// gather used after an N-sharded GEMM's all-gather, HBM bandwidth probes, and device queries.
#include <cuda_runtime.h>
#include <stdio.h>
#include <string.h>
#include "tb200_internal.h"
#include "tinycublas_b200.h"

namespace {

// X * A = alpha * B, in place in B (X overwrites B), A n x n upper-triangular non-unit (lda),
// B rows x n (ldb), column-major; one thread per row of X, forward substitution over the columns.
// The case ggml's solve_tri issues through cublasStrsmBatched (reference gemm.cu:41-49); here one
// launch covers the whole batch and the pointer arrays are read on the device.
__global__ void tb200_trsm_rupn_kernel(const float *const *Aarr, float *const *Barr, int rows, int n, int lda, int ldb,
                                       float alpha, int z0) {
  const int b = blockIdx.y + z0;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  const float *A = Aarr[b];
  float *X = Barr[b];
  for (int j = 0; j < n; ++j) {
    float acc = alpha * X[i + (long long)j * ldb];
    for (int l = 0; l < j; ++l) acc = fmaf(-X[i + (long long)l * ldb], A[l + (long long)j * lda], acc);
    X[i + (long long)j * ldb] = acc / A[j + (long long)j * lda];
  }
}

// parts: P blocks of rows x n, each column-major with ld = rows, back to back; block r goes to rows
// [r*rows, (r+1)*rows) of C, rows >= m_total dropped. Consecutive threads walk rows, so reads and writes
// coalesce.
template <typename E>
__global__ void tb200_gather_rows_kernel(const E *parts, int P, int rows, int n, E *C, int ldc, int m_total) {
  const long long per = (long long)rows * n;
  const long long total = (long long)P * per;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (long long)gridDim.x * blockDim.x) {
    const int r = (int)(e / per);
    const long long w = e - (long long)r * per;
    const int col = (int)(w / rows), i = (int)(w - (long long)col * rows);
    const long long row = (long long)r * rows + i;
    if (row < m_total) C[row + (long long)col * ldc] = parts[e];
  }
}

__global__ void tb200_bw_write_kernel(float4 *p, long long n4, float v) {
  const float4 val = make_float4(v, v, v, v);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x)
    p[i] = val;
}

__global__ void tb200_bw_read_kernel(const float4 *p, long long n4, float *sink) {
  float acc = 0.f;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    const float4 x = __ldcs(p + i);
    acc += x.x + x.y + x.z + x.w;
  }
  if (acc == 1.234567e30f) *sink = acc;  // keeps the loads; practically never true
}

}  // namespace

extern "C" int tb200_num_sms(void) {
  static int cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    cache[dev] = v;
  }
  return cache[dev];
}

extern "C" int tb200_launch_trsm_rupn(const float *const *A, float *const *B, int rows, int n, int lda, int ldb,
                                      float alpha, int batch, cudaStream_t s) {
  const unsigned gx = (unsigned)((rows + 127) / 128);
  for (int z0 = 0; z0 < batch; z0 += 65535) {
    const unsigned gy = (unsigned)(batch - z0 < 65535 ? batch - z0 : 65535);
    tb200_trsm_rupn_kernel<<<dim3(gx, gy, 1), 128, 0, s>>>(A, B, rows, n, lda, ldb, alpha, z0);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}

static unsigned grid_for(long long work, int threads) {
  long long g = (work + threads - 1) / threads;
  const long long cap = (long long)tb200_num_sms() * 8;
  if (g > cap) g = cap;
  return (unsigned)(g < 1 ? 1 : g);
}

extern "C" __attribute__((visibility("default"))) cublasStatus_t tb200_gather_row_blocks(
    const void *parts, int P, int rows, int n, int elem_bytes, void *C, int ldc, int m_total, cudaStream_t stream) {
  if (P <= 0 || rows < 0 || n < 0 || m_total < 0 || (long long)m_total > (long long)P * rows || ldc < m_total ||
      ldc < 1 || (elem_bytes != 2 && elem_bytes != 4))
    return CUBLAS_STATUS_INVALID_VALUE;
  if (rows == 0 || n == 0 || m_total == 0) return CUBLAS_STATUS_SUCCESS;
  const long long total = (long long)P * rows * n;
  const unsigned g = grid_for(total, 256);
  if (elem_bytes == 4)
    tb200_gather_rows_kernel<float><<<g, 256, 0, stream>>>((const float *)parts, P, rows, n, (float *)C, ldc, m_total);
  else
    tb200_gather_rows_kernel<unsigned short>
        <<<g, 256, 0, stream>>>((const unsigned short *)parts, P, rows, n, (unsigned short *)C, ldc, m_total);
  return cudaGetLastError() == cudaSuccess ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

// ---- mixture of experts: tokens into expert order, and expert outputs back to tokens ----------------
// Xp column p = X column ids[p] (row_bytes bytes each; ld in bytes): one warp per column, 16-byte copies
// when every address and stride allows, else bytes. An id outside [0, n_src) gives a zero column.
__global__ void tb200_moe_gather_kernel(const char *X, long long ldx, int n_src, const int *ids, int n_total,
                                        int row_bytes, char *Xp, long long ldp, int vec) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long p = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); p < n_total; p += warps) {
    const int t = ids[p];
    const bool ok = t >= 0 && t < n_src;
    char *dst = Xp + p * ldp;
    const char *src = X + (ok ? (long long)t * ldx : 0);
    if (vec) {
      for (int o = lane * 16; o < row_bytes; o += 32 * 16)
        *(uint4 *)(dst + o) = ok ? __ldg((const uint4 *)(src + o)) : make_uint4(0, 0, 0, 0);
    } else {
      for (int o = lane; o < row_bytes; o += 32) dst[o] = ok ? src[o] : 0;
    }
  }
}

// Y column t = sum over j < topk, in j order, of w[t * topk + j] * Cp column pos[t * topk + j] (m f32 rows);
// a position outside [0, n_total) contributes nothing. Deterministic: no atomics.
__global__ void tb200_moe_combine_kernel(const float *Cp, int m, long long ldc, int n_total, const int *pos,
                                         const float *w, int topk, int n_tokens, float *Y, long long ldy) {
  const long long rows_blocks = (m + blockDim.x - 1) / blockDim.x;
  for (long long bt = blockIdx.x; bt < rows_blocks * n_tokens; bt += gridDim.x) {
    const int t = (int)(bt / rows_blocks);
    const int row = (int)(bt % rows_blocks) * blockDim.x + threadIdx.x;
    if (row >= m) continue;
    float acc = 0.f;
    for (int j = 0; j < topk; ++j) {
      const int p = pos[(long long)t * topk + j];
      if (p >= 0 && p < n_total) acc = fmaf(w[(long long)t * topk + j], Cp[row + (long long)p * ldc], acc);
    }
    Y[row + (long long)t * ldy] = acc;
  }
}

extern "C" int tb200_launch_moe_gather(const void *X, long long ldx_bytes, int n_src, const int *ids, int n_total,
                                       int row_bytes, void *Xp, long long ldp_bytes, cudaStream_t s) {
  if (n_total <= 0 || row_bytes <= 0) return 0;
  const int vec = ((((uintptr_t)X) | ((uintptr_t)Xp)) & 15) == 0 && ldx_bytes % 16 == 0 && ldp_bytes % 16 == 0 &&
                  row_bytes % 16 == 0;
  const unsigned blocks = (unsigned)((n_total + 7) / 8 < 4096 ? (n_total + 7) / 8 : 4096);  // 8 warps per block
  tb200_moe_gather_kernel<<<blocks, 256, 0, s>>>((const char *)X, ldx_bytes, n_src, ids, n_total, row_bytes,
                                                 (char *)Xp, ldp_bytes, vec);
  return (int)cudaGetLastError();
}

extern "C" int tb200_launch_moe_combine(const float *Cp, int m, long long ldc, int n_total, const int *pos,
                                        const float *w, int topk, int n_tokens, float *Y, long long ldy,
                                        cudaStream_t s) {
  if (m <= 0 || n_tokens <= 0) return 0;
  const long long work = (long long)((m + 255) / 256) * n_tokens;
  const unsigned blocks = (unsigned)(work < 8192 ? work : 8192);
  tb200_moe_combine_kernel<<<blocks, 256, 0, s>>>(Cp, m, ldc, n_total, pos, w, topk, n_tokens, Y, ldy);
  return (int)cudaGetLastError();
}

// ---- the sharded GEMM's exchange on the copy engines: this rank's block of C into every peer's replica ----
extern "C" __attribute__((visibility("default"))) cublasStatus_t tb200_push_block(
    void *const *replicas, int P, int self, long long row0, long long rows, long long col0, long long ncols,
    long long ldc, int elem_bytes, const cudaStream_t *streams, int nstreams) {
  if (!replicas || P < 1 || self < 0 || self >= P || row0 < 0 || rows < 0 || col0 < 0 || ncols < 0 ||
      ldc < row0 + rows || ldc < 1 || (elem_bytes != 2 && elem_bytes != 4) || !streams || nstreams < 1)
    return CUBLAS_STATUS_INVALID_VALUE;
  if (rows == 0 || ncols == 0 || P == 1) return CUBLAS_STATUS_SUCCESS;
  const size_t pitch = (size_t)ldc * elem_bytes;
  const size_t off = (size_t)(row0 + col0 * ldc) * elem_bytes;
  const char *src = (const char *)replicas[self] + off;
  // peers in ring order from self + 1: with one stream every rank sends to a different peer at each moment
  // (no peer receives from all the others at once)
  for (int s = 1; s < P; ++s) {
    const int q = (self + s) % P;
    if (!replicas[q]) return CUBLAS_STATUS_INVALID_VALUE;
    cudaError_t e = cudaMemcpy2DAsync((char *)replicas[q] + off, pitch, src, pitch, (size_t)rows * elem_bytes,
                                      (size_t)ncols, cudaMemcpyDefault, streams[q % nstreams]);
    if (e != cudaSuccess) {
      fprintf(stderr, "[tinycublas_b200] tb200_push_block to rank %d: %s\n", q, cudaGetErrorString(e));
      return CUBLAS_STATUS_EXECUTION_FAILED;
    }
  }
  return CUBLAS_STATUS_SUCCESS;
}

extern "C" __attribute__((visibility("default"))) cublasStatus_t tb200_bw_write(void *p, long long n4, float v, cudaStream_t stream) {
  if (n4 <= 0) return CUBLAS_STATUS_SUCCESS;
  tb200_bw_write_kernel<<<grid_for(n4, 256), 256, 0, stream>>>((float4 *)p, n4, v);
  return cudaGetLastError() == cudaSuccess ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

extern "C" __attribute__((visibility("default"))) cublasStatus_t tb200_bw_read(const void *p, long long n4, float *sink, cudaStream_t stream) {
  if (n4 <= 0) return CUBLAS_STATUS_SUCCESS;
  tb200_bw_read_kernel<<<grid_for(n4, 256), 256, 0, stream>>>((const float4 *)p, n4, sink);
  return cudaGetLastError() == cudaSuccess ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

// ---- device memory that other processes of the node can map (the N-sharded GEMM's C replicas) ----
// Set-up calls, never on the GEMM path. `handle` is the 64-byte cudaIpcMemHandle_t.
extern "C" __attribute__((visibility("default"))) cublasStatus_t tb200_ipc_alloc(size_t bytes, void **ptr,
                                                                                  void *handle) {
  if (!ptr || !handle || bytes == 0) return CUBLAS_STATUS_INVALID_VALUE;
  *ptr = nullptr;
  if (cudaMalloc(ptr, bytes) != cudaSuccess) return CUBLAS_STATUS_ALLOC_FAILED;
  cudaIpcMemHandle_t hd;
  if (cudaIpcGetMemHandle(&hd, *ptr) != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return CUBLAS_STATUS_EXECUTION_FAILED;
  }
  memcpy(handle, &hd, sizeof hd);
  return CUBLAS_STATUS_SUCCESS;
}

extern "C" __attribute__((visibility("default"))) cublasStatus_t tb200_ipc_open(const void *handle, void **ptr) {
  if (!ptr || !handle) return CUBLAS_STATUS_INVALID_VALUE;
  cudaIpcMemHandle_t hd;
  memcpy(&hd, handle, sizeof hd);
  *ptr = nullptr;
  return cudaIpcOpenMemHandle(ptr, hd, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? CUBLAS_STATUS_SUCCESS
                                                                                      : CUBLAS_STATUS_EXECUTION_FAILED;
}

extern "C" __attribute__((visibility("default"))) cublasStatus_t tb200_ipc_close(void *ptr) {
  return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

extern "C" __attribute__((visibility("default"))) cublasStatus_t tb200_ipc_free(void *ptr) {
  return cudaFree(ptr) == cudaSuccess ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}
