// gemm_skinny.cu - decode-shaped GEMMs (n <= 8) with the weight under op T: a bandwidth-bound path.
//
// C (m x n, n <= 8) = alpha * A^T B + beta * C with A stored k x m (each output row's k weights are
// contiguous) and B stored k x n. Every byte of A is read exactly once, so the kernel is bound by
// HBM bandwidth; its job is to keep enough 128-bit loads in flight and to keep the arithmetic off
// the critical path. Replaces the reference's split-K tc2k kernels (cuda-shim/libtinycublas/
// gemm.cu:317-348, :408-415) and their plan (cublas.c:69-78) for these shapes.
//
// Decomposition: one CTA per 16 output rows (and batch element), W warps splitting k in 32-wide
// chunks (warp w takes chunks w, w+W, ...; W = 4, 8 or 16 by the GEMM's shape, below). Per chunk a lane (g = lane/4, c = lane%4) issues two
// 16-byte loads of A (rows g and g+8, k = 8c..8c+7) and one 16-byte load of B (column g), and the
// warp multiplies them on the tensor cores with two mma.m16n8k16 (fp32 accumulate). The k order
// inside a chunk is permuted identically for A and B, which leaves every dot product unchanged and
// lets the fragments come straight from 128-bit loads. The warps' partial tiles are summed in
// shared memory in warp order, so the result is deterministic, needs no global workspace, no
// counters and no second launch (the reference's split-K needed all three, and its per-handle
// workspace raced across streams: splitk-20260923/burst-3090.out).
//
// k split across a cluster: with S > 1 the S CTAs of a cluster share one 16-row block, CTA rank r taking
// the r-th of S contiguous ranges of 32-wide chunks (the last also takes the k % 32 tail). Each CTA sums
// its warps as above into shared memory; after a cluster barrier rank 0 adds the S partial tiles in rank
// order over distributed shared memory (deterministic) and stores C, and a second barrier keeps the other
// CTAs resident until it has read them. The host picks S so that the units of work (16-row blocks x S)
// spread evenly over the SMs: one CTA per block leaves 4096-row weights on 256 CTAs over 148 SMs.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include "tb200_internal.h"
#include "tb200_device.cuh"

using namespace tb200;

namespace {

constexpr int SK_ROWS = 16;

__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {  // read once: no L1 allocation
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ld_cached_v4(const void *p) { return __ldg((const uint4 *)p); }

template <typename T>
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1);
template <>
__device__ __forceinline__ void mma16816<__half>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<__nv_bfloat16>(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                                        uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// SK_WARPS warps per CTA split the block's k; each keeps SK_UNROLL 32-wide chunks of loads in flight
template <typename T, int SK_WARPS, int SK_UNROLL>
__global__ void __launch_bounds__(SK_WARPS * 32) tb200_gemm_skinny_kernel(const tb200_gemm_t g, int z0, int S) {
  __shared__ float red[SK_WARPS][SK_ROWS][8];
  __shared__ float part[SK_ROWS * 8];  // this CTA's k-slice sums, read by cluster rank 0 (S > 1)
  // launched with programmatic stream serialization: wait for the kernel before this one in the stream to
  // complete before touching memory, then let the next one be scheduled on SMs this grid leaves free
  const int b = blockIdx.y + z0;
  if (!g.Aarr && g.k <= 8192) {
    // this warp's chunks of A into L2 while the kernel before this one may still be finishing (waited for below,
    // before any load): prefetches only move lines into L2, the point of coherence, so the loads after
    // griddep_wait still read what that kernel wrote. All of them when the weights fit a third of L2, so that
    // HBM streams them through the previous kernel's tail and the wait; else the first SK_UNROLL. Rows of up to
    // 8192 columns only: measured back to back on one B200, the first chunks took 4096 x 4096 from 9.0 to 8.5 us
    // and 4096 x 14336 from 20.9 to 21.4 us
    const int lane_ = threadIdx.x & 31, w_ = threadIdx.x >> 5;
    const int sl = S > 1 ? (int)(blockIdx.x % (unsigned)S) : 0;
    const int r = (int)(blockIdx.x / (unsigned)S) * SK_ROWS + (lane_ >> 1);
    const int nch = g.k >> 5, c0 = (int)((long long)sl * nch / S), c1 = (int)((long long)(sl + 1) * nch / S);
    const bool whole = (long long)g.m * g.k * (long long)sizeof(T) * g.batch <= (48ll << 20);
    const int j_end = whole || c0 + w_ + SK_UNROLL * SK_WARPS > c1 ? c1 : c0 + w_ + SK_UNROLL * SK_WARPS;
    if (r < g.m) {
      const T *row = (const T *)g.A + (long long)b * g.sA + (long long)r * g.lda + (lane_ & 1) * 16;
      for (int j = c0 + w_; j < j_end; j += SK_WARPS) prefetch_l2(row + (long long)j * 32);
    }
  }
  griddep_wait();
  griddep_launch_dependents();
  const T *A = g.Aarr ? (const T *)g.Aarr[b] : (const T *)g.A + (long long)b * g.sA;
  const T *B = g.Barr ? (const T *)g.Barr[b] : (const T *)g.B + (long long)b * g.sB;
  const int osz = g.out_type == 0 ? 4 : 2;
  char *C = g.Carr ? (char *)g.Carr[b] : (char *)g.C + (long long)b * g.sC * osz;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gi = lane >> 2, ci = lane & 3;
  const int slice = S > 1 ? (int)(blockIdx.x % (unsigned)S) : 0;  // = the CTA's cluster rank
  const int row0 = (int)(blockIdx.x / (unsigned)S) * SK_ROWS;
  const int ra = row0 + gi, rb = row0 + gi + 8;
  const bool ok_a = ra < g.m, ok_b = rb < g.m, ok_col = gi < g.n;
  // rows past m and columns past n read row/column 0 (always valid) and are discarded
  const T *pa = A + (long long)(ok_a ? ra : 0) * g.lda + 8 * ci;
  const T *pb = A + (long long)(ok_b ? rb : 0) * g.lda + 8 * ci;
  const T *pB = B + (long long)(ok_col ? gi : 0) * g.ldb + 8 * ci;
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  const int nchunks = g.k >> 5;  // whole 32-wide chunks; the host guarantees k % 8 == 0
  const int c_lo = (int)((long long)slice * nchunks / S), c_hi = (int)((long long)(slice + 1) * nchunks / S);
  const bool vec = (((uintptr_t)A | (uintptr_t)B) & 15) == 0;  // pointer-array elements may be unaligned
  if (vec) {
    int j = c_lo + warp;
    for (; j + (SK_UNROLL - 1) * SK_WARPS < c_hi; j += SK_UNROLL * SK_WARPS) {
      uint4 va[SK_UNROLL], vb[SK_UNROLL], vB[SK_UNROLL];
#pragma unroll
      for (int u = 0; u < SK_UNROLL; ++u) {
        const long long off = (long long)(j + u * SK_WARPS) * 32;
        va[u] = ld_stream_v4(pa + off);
        vb[u] = ld_stream_v4(pb + off);
        vB[u] = ld_cached_v4(pB + off);
      }
#pragma unroll
      for (int u = 0; u < SK_UNROLL; ++u) {
        if (!ok_col) vB[u] = make_uint4(0, 0, 0, 0);
        mma16816<T>(d, va[u].x, vb[u].x, va[u].y, vb[u].y, vB[u].x, vB[u].y);
        mma16816<T>(d, va[u].z, vb[u].z, va[u].w, vb[u].w, vB[u].z, vB[u].w);
      }
    }
    for (; j < c_hi; j += SK_WARPS) {
      const long long off = (long long)j * 32;
      uint4 va = ld_stream_v4(pa + off), vb = ld_stream_v4(pb + off), vB = ld_cached_v4(pB + off);
      if (!ok_col) vB = make_uint4(0, 0, 0, 0);
      mma16816<T>(d, va.x, vb.x, va.y, vb.y, vB.x, vB.y);
      mma16816<T>(d, va.z, vb.z, va.w, vb.w, vB.z, vB.w);
    }
    // tail of k % 32 (a multiple of 8): lanes whose 8-wide group lies inside k load it, others zero
    const int kt = nchunks * 32;
    if (warp == 0 && kt < g.k && slice == S - 1) {
      const bool in = kt + 8 * ci < g.k;
      uint4 va = in ? ld_stream_v4(pa + kt) : make_uint4(0, 0, 0, 0);
      uint4 vb = in ? ld_stream_v4(pb + kt) : make_uint4(0, 0, 0, 0);
      uint4 vB = (in && ok_col) ? ld_cached_v4(pB + kt) : make_uint4(0, 0, 0, 0);
      mma16816<T>(d, va.x, vb.x, va.y, vb.y, vB.x, vB.y);
      mma16816<T>(d, va.z, vb.z, va.w, vb.w, vB.z, vB.w);
    }
  } else {
    // unaligned pointer-array element: scalar fp32 dot products, same reduction below
    float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
    const int c0 = 2 * ci;
    const int k_lo = (int)((long long)slice * g.k / S), k_hi = (int)((long long)(slice + 1) * g.k / S);
    for (int kk = k_lo + warp; kk < k_hi; kk += SK_WARPS) {
      const float x0 = ok_a ? to_f32(A[(long long)ra * g.lda + kk]) : 0.f;
      const float x1 = ok_b ? to_f32(A[(long long)rb * g.lda + kk]) : 0.f;
      const float y0 = c0 < g.n ? to_f32(B[(long long)c0 * g.ldb + kk]) : 0.f;
      const float y1 = c0 + 1 < g.n ? to_f32(B[(long long)(c0 + 1) * g.ldb + kk]) : 0.f;
      acc[0][0] = fmaf(x0, y0, acc[0][0]);
      acc[0][1] = fmaf(x0, y1, acc[0][1]);
      acc[1][0] = fmaf(x1, y0, acc[1][0]);
      acc[1][1] = fmaf(x1, y1, acc[1][1]);
    }
    d[0] = acc[0][0]; d[1] = acc[0][1]; d[2] = acc[1][0]; d[3] = acc[1][1];
  }
  // accumulator fragment: d0, d1 = (row g, cols 2c, 2c+1); d2, d3 = (row g+8, same cols)
  red[warp][gi][2 * ci] = d[0];
  red[warp][gi][2 * ci + 1] = d[1];
  red[warp][gi + 8][2 * ci] = d[2];
  red[warp][gi + 8][2 * ci + 1] = d[3];
  __syncthreads();
  const int r = threadIdx.x & 15, col = threadIdx.x >> 4;
  float sum = 0.f;
  if (threadIdx.x < SK_ROWS * 8) {
#pragma unroll
    for (int w = 0; w < SK_WARPS; ++w) sum += red[w][r][col];
  }
  if (S > 1) {
    if (threadIdx.x < SK_ROWS * 8) part[threadIdx.x] = sum;
    cluster_sync();  // every slice's sums are in its shared memory
    if (slice == 0 && threadIdx.x < SK_ROWS * 8) {
      sum = part[threadIdx.x];
      for (int q = 1; q < S; ++q) sum += ld_shared_cluster_f32(mapa_shared(smem_u32(&part[threadIdx.x]), (uint32_t)q));
    }
    cluster_sync();  // rank 0 has read them: the others may leave
    if (slice != 0) return;
  }
  if (threadIdx.x < SK_ROWS * 8) {
    const int row = row0 + r;
    if (row < g.m && col < g.n) {
      const long long idx = row + (long long)col * g.ldc;
      float v = g.alpha * sum;
      if (g.beta != 0.f) v += g.beta * load_out(C, idx, g.out_type);
      store_out(C, idx, v, g.out_type);
    }
  }
}

// Balanced form, built for weights with fewer than two 16-row blocks per SM (4096-row weights on 148 SMs: one CTA
// per block leaves some SMs with two blocks and some with one); opt-in, see tb200_skinny_bal_plan. The grid has G
// CTAs, two per SM, and CTA i takes
// the i-th of G equal contiguous ranges of the m / 16 x k / 32 units (16-row block, 32-wide chunk), so that every
// SM streams the same bytes. A range is cut at block boundaries into segments; its warps sum a segment as the
// per-block kernel does. A block inside one range is stored directly. A block shared by several CTAs (at most
// nslots) is finished by the last to arrive: each contributor parks its 16 x 8 partial tile in ws at its slot (its
// index among the block's CTAs), fences, and counts itself on cnt[block]; the last one adds the parked tiles in
// slot order (so the sum is the same whichever CTA arrives last), stores C and resets the counter to zero for the
// next launch. No CTA waits for another.
__device__ __forceinline__ long long bal_cta_of(long long x, long long U, long long G) {
  long long i = x * G / U;
  while (i + 1 < G && (i + 1) * U / G <= x) ++i;
  while (i > 0 && i * U / G > x) --i;
  return i;
}

template <typename T, int SK_WARPS, int SK_UNROLL>
__global__ void __launch_bounds__(SK_WARPS * 32, 2)
    tb200_gemm_skinny_bal_kernel(const tb200_gemm_t g, float *ws, unsigned *cnt, int nslots) {
  __shared__ float red[SK_WARPS][SK_ROWS][8];
  __shared__ int s_last;
  griddep_wait();
  griddep_launch_dependents();
  const T *A = (const T *)g.A;
  const T *B = (const T *)g.B;
  char *C = (char *)g.C;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gi = lane >> 2, ci = lane & 3;
  const long long nch = g.k >> 5;  // the host guarantees k % 32 == 0
  const long long blocks = (g.m + SK_ROWS - 1) / SK_ROWS;
  const long long U = blocks * nch, G = gridDim.x, i = blockIdx.x;
  const long long u1 = (i + 1) * U / G;
  const bool ok_col = gi < g.n;
  const T *pB = B + (long long)(ok_col ? gi : 0) * g.ldb + 8 * ci;
  const int r = threadIdx.x & 15, col = threadIdx.x >> 4;
  for (long long u = i * U / G; u < u1;) {
    const long long blk = u / nch;
    const int c0 = (int)(u - blk * nch);
    const int c1 = (int)(nch < c0 + (u1 - u) ? nch : c0 + (u1 - u));
    u += c1 - c0;
    const int row0 = (int)blk * SK_ROWS;
    const int ra = row0 + gi, rb = row0 + gi + 8;
    const bool ok_a = ra < g.m, ok_b = rb < g.m;
    const T *pa = A + (long long)(ok_a ? ra : 0) * g.lda + 8 * ci;
    const T *pb = A + (long long)(ok_b ? rb : 0) * g.lda + 8 * ci;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    int j = c0 + warp;
    for (; j + (SK_UNROLL - 1) * SK_WARPS < c1; j += SK_UNROLL * SK_WARPS) {
      uint4 va[SK_UNROLL], vb[SK_UNROLL], vB[SK_UNROLL];
#pragma unroll
      for (int q = 0; q < SK_UNROLL; ++q) {
        const long long off = (long long)(j + q * SK_WARPS) * 32;
        va[q] = ld_stream_v4(pa + off);
        vb[q] = ld_stream_v4(pb + off);
        vB[q] = ld_cached_v4(pB + off);
      }
#pragma unroll
      for (int q = 0; q < SK_UNROLL; ++q) {
        if (!ok_col) vB[q] = make_uint4(0, 0, 0, 0);
        mma16816<T>(d, va[q].x, vb[q].x, va[q].y, vb[q].y, vB[q].x, vB[q].y);
        mma16816<T>(d, va[q].z, vb[q].z, va[q].w, vb[q].w, vB[q].z, vB[q].w);
      }
    }
    for (; j < c1; j += SK_WARPS) {
      const long long off = (long long)j * 32;
      uint4 va = ld_stream_v4(pa + off), vb = ld_stream_v4(pb + off), vB = ld_cached_v4(pB + off);
      if (!ok_col) vB = make_uint4(0, 0, 0, 0);
      mma16816<T>(d, va.x, vb.x, va.y, vb.y, vB.x, vB.y);
      mma16816<T>(d, va.z, vb.z, va.w, vb.w, vB.z, vB.w);
    }
    red[warp][gi][2 * ci] = d[0];
    red[warp][gi][2 * ci + 1] = d[1];
    red[warp][gi + 8][2 * ci] = d[2];
    red[warp][gi + 8][2 * ci + 1] = d[3];
    __syncthreads();
    float sum = 0.f;
    if (threadIdx.x < SK_ROWS * 8) {
#pragma unroll
      for (int w = 0; w < SK_WARPS; ++w) sum += red[w][r][col];
    }
    bool store = c0 == 0 && c1 == nch;
    if (!store) {
      const long long first = bal_cta_of(blk * nch, U, G), last = bal_cta_of(blk * nch + nch - 1, U, G);
      const int slot = (int)(i - first), ncontrib = (int)(last - first + 1);
      if (threadIdx.x < SK_ROWS * 8) ws[((long long)blk * nslots + slot) * (SK_ROWS * 8) + threadIdx.x] = sum;
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) s_last = atomicAdd(&cnt[blk], 1u) == (unsigned)(ncontrib - 1);
      __syncthreads();
      store = s_last != 0;
      if (store) {
        __threadfence();
        if (threadIdx.x < SK_ROWS * 8) {
          sum = 0.f;
          for (int q = 0; q < ncontrib; ++q) sum += __ldcg(&ws[((long long)blk * nslots + q) * (SK_ROWS * 8) + threadIdx.x]);
        }
        if (threadIdx.x == 0) atomicExch(&cnt[blk], 0u);  // ready for the next launch
      }
    }
    if (store && threadIdx.x < SK_ROWS * 8) {
      const int row = row0 + r;
      if (row < g.m && col < g.n) {
        const long long idx = row + (long long)col * g.ldc;
        float v = g.alpha * sum;
        if (g.beta != 0.f) v += g.beta * load_out(C, idx, g.out_type);
        store_out(C, idx, v, g.out_type);
      }
    }
    __syncthreads();  // red is reused by the next segment
  }
}

}  // namespace

extern "C" int tb200_skinny_ok(const tb200_gemm_t *g) {
  if (g->in_type != TB200_F16 && g->in_type != TB200_BF16) return 0;
  if (g->n > 8 || g->opA != 1 || g->opB != 0 || g->k % 8 != 0) return 0;
  if (g->lda % 8 || g->ldb % 8) return 0;
  if (!g->Aarr && ((((uintptr_t)g->A) | ((uintptr_t)g->B)) & 15)) return 0;
  if (!g->Aarr && g->batch > 1 && ((g->sA % 8) || (g->sB % 8))) return 0;
  return 1;
}

// Kernel shape and k slices per 16-row block, from sweeps on the B200 (f16, n 1 and 8, CUDA-graph replay):
// * many blocks (at least six per SM): 4 warps x 8 chunks in flight, 128-thread CTAs, eight per SM, no
//   split. 14336 x 4096 and the 128256-row lm_head ran 15 % and 11 % faster than with 8 warps x 4 (5.2 and
//   6.4-6.5 TB/s), and lost with any split;
// * two to six blocks per SM: 8 warps x 4, no split (the 4 x 8 shape leaves these SMs short of warps:
//   6144 x 4096 ran 3.4 against 3.9 TB/s, 8192 x 1024 2.9 against 3.2);
// * fewer blocks: 16 warps x 2, and S the smallest power of two that gives a CTA to every other SM, each
//   warp keeping at least 2 chunks a slice: 4096 x 14336 and 4096 x 4096 unsplit (5.5 and 3.7 TB/s, 10 %
//   and 6 % faster than 8 x 4 with S = 2), 1024 x 4096 at S = 2.
// Smaller slices pay a per-CTA cost (launch, reductions, cluster barriers). TB200_SKINNY_SPLIT=1|2|4|8 forces
// S and TB200_SKINNY_CFG=4x8|8x4|16x2 the kernel shape (tests, bisecting; read per call); a forced S is
// taken where each warp keeps at least one chunk a slice.
enum { SK_CFG_4x8 = 0, SK_CFG_8x4 = 1, SK_CFG_16x2 = 2 };
static int skinny_plan(long long blocks, int k, int num_sms, int *S_out) {
  const int chunks = k >> 5;
  if (num_sms <= 0) num_sms = 148;
  const char *ce = getenv("TB200_SKINNY_CFG");
  int cfg = blocks >= 6LL * num_sms ? SK_CFG_4x8 : blocks >= 2LL * num_sms ? SK_CFG_8x4 : SK_CFG_16x2;
  if (ce && !strcmp(ce, "4x8")) cfg = SK_CFG_4x8;
  if (ce && !strcmp(ce, "8x4")) cfg = SK_CFG_8x4;
  if (ce && !strcmp(ce, "16x2")) cfg = SK_CFG_16x2;
  const int warps = cfg == SK_CFG_4x8 ? 4 : cfg == SK_CFG_8x4 ? 8 : 16;
  const char *e = getenv("TB200_SKINNY_SPLIT");
  const int want = e && *e ? atoi(e) : 0;
  int S = 1;
  if (want == 1 || want == 2 || want == 4 || want == 8) {
    S = chunks / want >= warps ? want : 1;
  } else if (cfg == SK_CFG_16x2) {
    while (S < 8 && blocks * S < num_sms / 2 && chunks / (2 * S) >= 2 * warps) S *= 2;
  }
  *S_out = S;
  return cfg;
}

template <typename T, int W, int U>
static cudaError_t launch_skinny_cfg(const tb200_gemm_t *g, int z0, int S, dim3 grid, cudaLaunchConfig_t cfg) {
  cfg.gridDim = grid;
  cfg.blockDim = dim3(W * 32, 1, 1);
  return cudaLaunchKernelEx(&cfg, tb200_gemm_skinny_kernel<T, W, U>, *g, z0, S);
}

template <typename T>
static cudaError_t launch_skinny_t(const tb200_gemm_t *g, int z0, int S, int shape, dim3 grid,
                                   const cudaLaunchConfig_t &cfg) {
  if (shape == SK_CFG_4x8) return launch_skinny_cfg<T, 4, 8>(g, z0, S, grid, cfg);
  if (shape == SK_CFG_8x4) return launch_skinny_cfg<T, 8, 4>(g, z0, S, grid, cfg);
  return launch_skinny_cfg<T, 16, 2>(g, z0, S, grid, cfg);
}

extern "C" __attribute__((visibility("default"))) int tb200_skinny_shape(long long blocks, int k, int num_sms, int *warps,
                                                                      int *unroll, int *slices) {
  int S = 1;
  const int cfg = skinny_plan(blocks, k, num_sms, &S);
  if (warps) *warps = cfg == SK_CFG_4x8 ? 4 : cfg == SK_CFG_8x4 ? 8 : 16;
  if (unroll) *unroll = cfg == SK_CFG_4x8 ? 8 : cfg == SK_CFG_8x4 ? 4 : 2;
  if (slices) *slices = S;
  return 0;
}

// The balanced decode's workspace keeps the same layout for every launch, so that no launch's parked tiles land
// where another launch keeps its counters: BAL_MAX_BLOCKS counters (zero between launches) first, then the parked
// tiles. At most BAL_MAX_BLOCKS 16-row blocks (65536 rows) take this kernel.
#define BAL_MAX_BLOCKS 4096
#define BAL_CNT_BYTES (BAL_MAX_BLOCKS * 4)

// The balanced decode's grid, slots per block and workspace bytes, or 0 when the GEMM is not one for it: batch 1,
// plain pointers, k % 32 == 0, at most BAL_MAX_BLOCKS blocks. Opt-in (TB200_SKINNY_BAL=1, read per call): on the
// B200 it ran slower than the per-block kernel on the 4096-row weights it was built for (4096 x 4096: 14.5 against
// 9.5-11 us; 4096 x 14336: 25 against 21 us). Each range ends in one or two segment tails (reduction, fence,
// counter) during which the CTA has no loads in flight, which costs more than the balance gains.
extern "C" size_t tb200_skinny_bal_plan(const tb200_gemm_t *g, int num_sms, int *grid, int *nslots) {
  if (!tb200_skinny_ok(g) || g->batch != 1 || g->Aarr || g->k % 32 != 0 || g->k <= 0) return 0;
  const char *e = getenv("TB200_SKINNY_BAL");
  if (!(e && *e == '1')) return 0;  // opt-in: measured slower than the per-block kernel (above)
  if (num_sms <= 0) num_sms = 148;
  const long long blocks = (g->m + SK_ROWS - 1) / SK_ROWS, nch = g->k / 32;
  if (blocks > BAL_MAX_BLOCKS) return 0;
  const long long U = blocks * nch;
  long long G = 2LL * num_sms;
  if (G > U / 32) G = U / 32;  // at least 32 chunks (two per warp) a CTA
  if (G < 2) return 0;
  const long long per = U / G;  // every range holds at least `per` units: a block meets at most this many CTAs
  const long long ns = (nch + per - 1) / per + 1;
  *grid = (int)G;
  *nslots = (int)ns;
  return (size_t)BAL_CNT_BYTES + (size_t)(blocks * ns) * SK_ROWS * 8 * sizeof(float);
}

extern "C" int tb200_launch_skinny_bal(const tb200_gemm_t *g, void *ws, size_t ws_bytes, cudaStream_t s) {
  int G = 0, ns = 0;
  const size_t need = tb200_skinny_bal_plan(g, tb200_num_sms(), &G, &ns);
  if (!need || !ws || ws_bytes < need || ((uintptr_t)ws & 255)) return (int)cudaErrorNotSupported;
  unsigned *cnt = (unsigned *)ws;
  float *parked = (float *)((char *)ws + BAL_CNT_BYTES);
  if (tb200_trace())
    fprintf(stderr, "[trace] launch tb200_gemm_skinny_bal<W=16,U=2> grid=(%d,1,1) block=(512,1,1) slots=%d m=%d n=%d k=%d\n",
            G, ns, g->m, g->n, g->k);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  int na = 0;
  if (tb200_pdl()) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.gridDim = dim3((unsigned)G, 1, 1);
  cfg.blockDim = dim3(512, 1, 1);
  cfg.stream = s;
  cfg.attrs = at;
  cfg.numAttrs = na;
  cudaError_t e = g->in_type == TB200_F16
                      ? cudaLaunchKernelEx(&cfg, tb200_gemm_skinny_bal_kernel<__half, 16, 2>, *g, parked, cnt, ns)
                      : cudaLaunchKernelEx(&cfg, tb200_gemm_skinny_bal_kernel<__nv_bfloat16, 16, 2>, *g, parked, cnt, ns);
  return (int)e;
}

extern "C" int tb200_launch_skinny(const tb200_gemm_t *g, cudaStream_t s) {
  if (!tb200_skinny_ok(g)) return tb200_launch_simt(g, s);
  const long long blocks = (g->m + SK_ROWS - 1) / SK_ROWS;
  int S = 1;
  const int shape = skinny_plan(blocks * (g->batch < 65535 ? g->batch : 65535), g->k, tb200_num_sms(), &S);
  const int threads = shape == SK_CFG_4x8 ? 128 : shape == SK_CFG_8x4 ? 256 : 512;
  const long long gx = blocks * S;
  if (gx > 0x7fffffffLL) return (int)cudaErrorInvalidConfiguration;
  for (int z0 = 0; z0 < g->batch; z0 += 65535) {
    const unsigned gy = (unsigned)(g->batch - z0 < 65535 ? g->batch - z0 : 65535);
    if (tb200_trace())
      fprintf(stderr, "[trace] launch tb200_gemm_skinny<W=%d,U=%d,S=%d> grid=(%lld,%u,1) block=(%d,1,1) m=%d n=%d k=%d out=%d\n",
              threads / 32, shape == SK_CFG_4x8 ? 8 : shape == SK_CFG_8x4 ? 4 : 2, S, gx, gy, threads, g->m, g->n, g->k,
              g->out_type);
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[2];
    int na = 0;
    if (S > 1) {  // the k slices of a block form one cluster
      at[na].id = cudaLaunchAttributeClusterDimension;
      at[na].val.clusterDim.x = (unsigned)S;
      at[na].val.clusterDim.y = 1;
      at[na].val.clusterDim.z = 1;
      ++na;
    }
    if (tb200_pdl()) {
      at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
      at[na].val.programmaticStreamSerializationAllowed = 1;
      ++na;
    }
    cfg.stream = s;
    cfg.attrs = at;
    cfg.numAttrs = na;
    const dim3 grid((unsigned)gx, gy, 1);
    cudaError_t e = g->in_type == TB200_F16 ? launch_skinny_t<__half>(g, z0, S, shape, grid, cfg)
                                            : launch_skinny_t<__nv_bfloat16>(g, z0, S, shape, grid, cfg);
    if (e != cudaSuccess) return (int)e;
  }
  return 0;
}
