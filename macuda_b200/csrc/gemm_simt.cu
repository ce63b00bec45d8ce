// gemm_simt.cu - the general GEMM kernel: any operand alignment, any transpose, f32/f16/bf16 in and
// out, strided or pointer-array batches (pointers read on the device), fp32 FMA accumulation.
//
// It serves what the tensor-core and skinny kernels do not take: unaligned or odd leading
// dimensions, k == 0 (C = beta * C), pointer-array batches with n > 8, and fp32 GEMMs outside TF32
// math mode (where fp32 FMA is the exact cuBLAS "pedantic"/default behaviour). It replaces the
// reference's scalar tinyblas_gemm_f32 (cuda-shim/libtinycublas/gemm.cu:7-35), which ran one thread
// per output and one launch per batch element, with a shared-memory-tiled kernel over the whole
// batch in one launch.
//
// Tile 64 x 64 x 16, 256 threads, each thread 4 x 4 outputs strided by 16 so that consecutive
// threads own consecutive rows: every load and store instruction of a warp walks the contiguous
// dimension of its operand.
#include <cuda_runtime.h>
#include <stdio.h>
#include "tb200_internal.h"
#include "tb200_device.cuh"

using namespace tb200;

namespace {

constexpr int SB_M = 64, SB_N = 64, SB_K = 16, SB_T = 256;

template <typename TI>
__device__ __forceinline__ void simt_tile(const tb200_gemm_t &g, int b, int m0, int n0, float (&As)[SB_K][SB_M + 4],
                                          float (&Bs)[SB_K][SB_N + 4]) {
  const TI *A = g.Aarr ? (const TI *)g.Aarr[b] : (const TI *)g.A + (long long)b * g.sA;
  const TI *B = g.Barr ? (const TI *)g.Barr[b] : (const TI *)g.B + (long long)b * g.sB;
  const int osz = g.out_type == 0 ? 4 : 2;
  char *C = g.Carr ? (char *)g.Carr[b] : (char *)g.C + (long long)b * g.sC * osz;
  const int tid = threadIdx.x, ty = tid & 15, tx = tid >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int k0 = 0; k0 < g.k; k0 += SB_K) {
#pragma unroll
    for (int r = 0; r < (SB_M * SB_K) / SB_T; ++r) {
      const int idx = tid + r * SB_T;
      int i, kk;
      long long off;
      if (g.opA == 0) { i = idx % SB_M; kk = idx / SB_M; off = (long long)(m0 + i) + (long long)(k0 + kk) * g.lda; }
      else            { kk = idx % SB_K; i = idx / SB_K; off = (long long)(k0 + kk) + (long long)(m0 + i) * g.lda; }
      As[kk][i] = (m0 + i < g.m && k0 + kk < g.k) ? to_f32(A[off]) : 0.f;
    }
#pragma unroll
    for (int r = 0; r < (SB_N * SB_K) / SB_T; ++r) {
      const int idx = tid + r * SB_T;
      int j, kk;
      long long off;
      if (g.opB == 0) { kk = idx % SB_K; j = idx / SB_K; off = (long long)(k0 + kk) + (long long)(n0 + j) * g.ldb; }
      else            { j = idx % SB_N; kk = idx / SB_N; off = (long long)(n0 + j) + (long long)(k0 + kk) * g.ldb; }
      Bs[kk][j] = (n0 + j < g.n && k0 + kk < g.k) ? to_f32(B[off]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SB_K; ++kk) {
      float a[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty + 16 * i];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], bv[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int col = n0 + tx + 16 * j;
    if (col >= g.n) continue;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = m0 + ty + 16 * i;
      if (row >= g.m) continue;
      const long long ci = row + (long long)col * g.ldc;
      float v = g.alpha * acc[i][j];
      if (g.beta != 0.f) v += g.beta * load_out(C, ci, g.out_type);
      store_out(C, ci, v, g.out_type);
    }
  }
}

// Grid-stride over the 64 x 64 output tiles of every batch element (a grid of a few CTAs per SM), so that
// a launch that has nothing to do (run_if not raised for this call) costs a few microseconds whatever the
// problem size.
template <typename TI>
__global__ void __launch_bounds__(SB_T) tb200_gemm_simt_kernel(const tb200_gemm_t g, int gx, int gy) {
  __shared__ float As[SB_K][SB_M + 4];
  __shared__ float Bs[SB_K][SB_N + 4];
  // launched with programmatic stream serialization behind the kernels of this library: wait for the kernel
  // before this one to complete before touching memory, then let the next one be scheduled
  griddep_wait();
  griddep_launch_dependents();
  if (g.run_if && *(volatile const int *)g.run_if != g.run_if_gen) return;  // the tensor-core launch did the work
  const long long tiles_xy = (long long)gx * gy, total = tiles_xy * g.batch;
  for (long long t = blockIdx.x; t < total; t += gridDim.x) {
    const int b = (int)(t / tiles_xy);
    const long long r = t - (long long)b * tiles_xy;
    simt_tile<TI>(g, b, (int)(r % gx) * SB_M, (int)(r / gx) * SB_N, As, Bs);
  }
}

}  // namespace

extern "C" int tb200_launch_simt(const tb200_gemm_t *g, cudaStream_t s) {
  const long long gx = (g->m + SB_M - 1) / SB_M, gy = (g->n + SB_N - 1) / SB_N;
  if (gx > 0x7fffffffLL || gy > 0x7fffffffLL) return (int)cudaErrorInvalidConfiguration;
  const long long total = gx * gy * g->batch;
  // 8 resident CTAs of 256 threads per SM; a stand-by launch (run_if) usually has nothing to do, so one per SM
  const long long cap = (g->run_if ? 1LL : 8LL) * tb200_num_sms();
  const unsigned grid = (unsigned)(total < cap ? total : cap);
  if (grid == 0) return 0;
  if (tb200_trace())
    fprintf(stderr, "[trace] launch tb200_gemm_simt grid=(%u,1,1) block=(%d,1,1) tiles=%lld m=%d n=%d k=%d in=%d out=%d\n",
            grid, SB_T, total, g->m, g->n, g->k, g->in_type, g->out_type);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(SB_T, 1, 1);
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = tb200_pdl() ? 1 : 0;
  cudaError_t e;
  if (g->in_type == TB200_F32) e = cudaLaunchKernelEx(&cfg, tb200_gemm_simt_kernel<float>, *g, (int)gx, (int)gy);
  else if (g->in_type == TB200_F16) e = cudaLaunchKernelEx(&cfg, tb200_gemm_simt_kernel<__half>, *g, (int)gx, (int)gy);
  else e = cudaLaunchKernelEx(&cfg, tb200_gemm_simt_kernel<__nv_bfloat16>, *g, (int)gx, (int)gy);
  return (int)e;
}
