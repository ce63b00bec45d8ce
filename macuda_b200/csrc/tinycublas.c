/* tinycublas.c - the cuBLAS v2 C ABI subset ggml-cuda calls, on the B200 kernels of this library.
 *
 * Host layer of libtinycublas_b200.so. It owns the handle, the type contract, the alpha/beta decoding
 * and the choice of kernel; the CUDA launchers live in the .cu files behind tb200_internal.h. The
 * file is compiled against CUDA's own cublas_v2.h, so the compiler checks every exported signature
 * against the real cuBLAS prototypes, as the reference does (cuda-shim/libtinycublas/cublas.c:9).
 *
 * Differences from the reference's host layer (cuda-shim/libtinycublas/cublas.c), by design:
 *   - pointer-array batches are read on the device (reference: device-to-host copy + stream sync +
 *     one launch per element, cublas.c:292-303);
 *   - no call synchronises the stream or reads device memory back, so every call is graph-capturable
 *     (the reference's split-K path bypassed capture, cublas.c:170); the one device allocation, the
 *     tensor maps of pointer-array batches, is made once per (handle, stream) outside any capture;
 *   - cublasSetMathMode is honoured for fp32 GEMMs (the reference stored it and always used TF32,
 *     cublas.c:218, :249);
 *   - the kernel plan reads the device's SM count (the reference hard-codes the RTX 5090's 170,
 *     cublas.c:73, :151).
 */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <stdint.h>
#include <cuda_runtime_api.h>
#include <cublas_v2.h>
#include "tb200_internal.h"
#include "tinycublas_b200.h"

#ifndef TB200_GIT_DESCRIBE
#define TB200_GIT_DESCRIBE "unknown"
#endif

/* Device scratch the library allocates for itself: one buffer per (handle, stream), so that two
 * streams sharing a handle never share scratch (the reference's per-handle split-K workspace did, and
 * raced: cublas.c:56-61). Made lazily, outside any stream capture, and grown when a call needs more. */
#define TB200_WS_SLOTS 8
struct tb200_ws {
  cudaStream_t stream;
  void *ptr;
  size_t bytes;
};

struct tb200_handle {
  cudaStream_t stream;
  cublasMath_t math_mode;
  int device;
  void *user_ws;
  size_t user_ws_bytes;
  struct tb200_ws ws[TB200_WS_SLOTS];
  struct tb200_ws dws[TB200_WS_SLOTS]; /* the balanced decode kernel's workspace, per stream */
  unsigned ws_allocs; /* allocations made, for the tests */
  /* buffers replaced by a larger one or given up by a stream: launches already queued may still read them, so
   * they are freed at cublasDestroy (after every stream drains), not on the GEMM path */
  struct tb200_ws retired[32];
  int n_retired;
};

/* keeps a replaced buffer until cublasDestroy; with the list full, waits for its stream and frees it now */
static void retire(struct tb200_handle *h, struct tb200_ws *w) {
  if (h->n_retired < (int)(sizeof h->retired / sizeof h->retired[0])) {
    h->retired[h->n_retired++] = *w;
  } else {
    cudaStreamSynchronize(w->stream);
    cudaFree(w->ptr);
  }
  w->ptr = NULL;
  w->bytes = 0;
}

/* scratch of at least `bytes` from one of the handle's per-stream slot arrays (`arr`) for its current stream, or
 * NULL (capturing, or out of memory: the caller then takes a path that needs none). zero: a new buffer is cleared
 * on the stream before its first use. */
static void *stream_slot(struct tb200_handle *h, struct tb200_ws *arr, size_t bytes, size_t min_bytes, int zero) {
  enum cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  int slot = -1;
  for (int i = 0; i < TB200_WS_SLOTS; i++)
    if (arr[i].ptr && arr[i].stream == h->stream) {
      slot = i;
      break;
    }
  if (slot >= 0 && arr[slot].bytes >= bytes) return arr[slot].ptr;
  if (cudaStreamIsCapturing(h->stream, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return NULL;
  if (slot < 0) {
    for (int i = 0; i < TB200_WS_SLOTS && slot < 0; i++)
      if (!arr[i].ptr) slot = i;
    if (slot < 0) slot = 0; /* all slots taken by other streams: the first one's buffer is retired below */
  }
  /* growth, or a slot taken over: launches queued earlier may still read the old buffer */
  if (arr[slot].ptr) retire(h, &arr[slot]);
  size_t want = bytes < min_bytes ? min_bytes : bytes;
  void *p = NULL;
  if (cudaMalloc(&p, want) != cudaSuccess) {
    (void)cudaGetLastError();
    return NULL;
  }
  if (zero && cudaMemsetAsync(p, 0, want, h->stream) != cudaSuccess) {
    (void)cudaGetLastError();
    cudaFree(p);
    return NULL;
  }
  arr[slot].stream = h->stream;
  arr[slot].ptr = p;
  arr[slot].bytes = want;
  h->ws_allocs++;
  return p;
}

/* the pointer-array tensor maps' scratch: at least 64 KB, grown when a larger batch comes, zeroed when made (its
 * fallback flag starts at zero and is never cleared) */
static void *handle_scratch(struct tb200_handle *h, size_t bytes) { return stream_slot(h, h->ws, bytes, 64u << 10, 1); }

/* the balanced decode kernel's workspace: one fixed 1 MB buffer per stream, zeroed once (its counters return to
 * zero at the end of every launch) */
#define TB200_DECODE_WS_BYTES (1u << 20)
static void *decode_scratch(struct tb200_handle *h, size_t bytes) {
  if (bytes > TB200_DECODE_WS_BYTES) return NULL;
  return stream_slot(h, h->dws, TB200_DECODE_WS_BYTES, TB200_DECODE_WS_BYTES, 1);
}

/* ---- environment knobs, read once (the reference's TINYCUBLAS_TC / TINYCUBLAS_GEMM bisect knobs,
 * cublas.c:79-81, under this library's own names) ---- */
static int env_flag(const char *name, int dflt) {
  const char *e = getenv(name);
  if (!e || !*e) return dflt;
  return *e != '0';
}
int tb200_trace(void) {
  static int v = -1;
  if (v < 0) v = env_flag("TB200_TRACE", 0);
  return v;
}
int tb200_pdl(void) { /* TB200_PDL=0: plain stream order between launches (bisect knob, read per launch) */
  return env_flag("TB200_PDL", 1);
}
static int tc_enabled(void) {     /* TB200_TC=0: no tensor-core kernel, everything on the SIMT kernel */
  static int v = -1;
  if (v < 0) v = env_flag("TB200_TC", 1);
  return v;
}
static int skinny_enabled(void) { /* TB200_SKINNY=0: decode shapes go to the tensor-core kernel */
  static int v = -1;
  if (v < 0) v = env_flag("TB200_SKINNY", 1);
  return v;
}

/* ---- type contract: reference cublas.c:107-134, restated ---- */
static int dtype_code(cudaDataType t) {
  return t == CUDA_R_32F ? TB200_F32 : t == CUDA_R_16F ? TB200_F16 : t == CUDA_R_16BF ? TB200_BF16 : -1;
}

/* IEEE binary16 bits -> float, exact (every half is a float) */
static float half_bits_to_float(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 0x1fu, f = h & 0x3ffu, bits;
  if (e == 0x1f) {
    bits = sign | 0x7f800000u | (f << 13);
  } else if (e == 0) {
    if (f == 0) {
      bits = sign;
    } else { /* subnormal: renormalise */
      int shift = 0;
      while (!(f & 0x400u)) { f <<= 1; shift++; }
      f &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 15 + 1 - shift) << 23) | (f << 13);
    }
  } else {
    bits = sign | ((e + 127 - 15) << 23) | (f << 13);
  }
  float out;
  memcpy(&out, &bits, 4);
  return out;
}

static int is_c16(cublasComputeType_t ct) { return ct == CUBLAS_COMPUTE_16F || ct == CUBLAS_COMPUTE_16F_PEDANTIC; }

/* alpha/beta live on the host in the compute type */
static float read_scalar(const void *p, cublasComputeType_t ct) {
  return is_c16(ct) ? half_bits_to_float(*(const uint16_t *)p) : *(const float *)p;
}

/* A and B of one type; a compute type cuBLAS defines for it; C as that compute type allows.
 *   f32:  32F, 32F_PEDANTIC, 32F_FAST_TF32, 32F_FAST_16F, 32F_FAST_16BF
 *   f16:  32F, 32F_PEDANTIC, or 16F / 16F_PEDANTIC with an f16 C
 *   bf16: 32F, 32F_PEDANTIC
 * Returns 0 and the codes, or -1 (NOT_SUPPORTED). *tf32 says whether an f32 GEMM may use TF32. */
static int gemm_contract(cudaDataType At, cudaDataType Bt, cudaDataType Ct, cublasComputeType_t ct, int *in, int *out,
                         int *tf32) {
  *in = dtype_code(At);
  *out = dtype_code(Ct);
  *tf32 = 0;
  if (*in < 0 || *out < 0 || dtype_code(Bt) != *in) return -1;
  int c32 = ct == CUBLAS_COMPUTE_32F || ct == CUBLAS_COMPUTE_32F_PEDANTIC;
  if (*in == TB200_F32) {
    if (ct == CUBLAS_COMPUTE_32F_FAST_TF32 || ct == CUBLAS_COMPUTE_32F_FAST_16F || ct == CUBLAS_COMPUTE_32F_FAST_16BF) {
      *tf32 = 1;
      return 0;
    }
    return c32 ? 0 : -1;
  }
  if (*in == TB200_F16) return (c32 || (is_c16(ct) && *out == TB200_F16)) ? 0 : -1;
  return c32 ? 0 : -1;
}

/* ---- planning ---- */
static int esize(int t) { return t == TB200_F32 ? 4 : 2; }

/* The persistent tensor-core kernel's tile: 128 x BN on one CTA (BN 32..256), or 256 x 256 / 256 x 128 on a
 * pair of CTAs (2-SM UMMA). Cost = waves of tiles over the SMs (pairs) x the time one SM spends on its
 * share of a tile, from the measured fraction of tensor peak each configuration sustains per SM: a
 * 128 x N x 16 UMMA re-reads its whole A and B from shared memory, which caps narrow single-CTA tiles,
 * while a pair tile streams half of B per SM. */
int tb200_tc_tile_n(int m, int n, int batch, int num_sms, int *pair) {
  static const int bns[6] = {256, 128, 64, 32, 256, 128};
  static const int cgs[6] = {1, 1, 1, 1, 2, 2};
  /* per-SM fraction of tensor peak each tile sustains, measured on the B200. The 256 x 128 pair tile ran
   * within 5 % of the 128 x 128 tile on the 4096 x 512 shapes (slower on Q, faster on down): equal
   * efficiency and the same area per SM, so the planner keeps the single-CTA tile on ties */
  static const double eff[6] = {0.57, 0.50, 0.35, 0.19, 0.80, 0.50};
  if (num_sms <= 0) num_sms = 148;
  int best = 256, best_pair = 0;
  double best_cost = 1e300;
  for (int i = 0; i < 6; i++) {
    const int bn = bns[i], cg = cgs[i];
    if (bn > 32 && n <= bn / 2) continue; /* a tile at least half full */
    const long long tiles = (long long)((m + 128 * cg - 1) / (128 * cg)) * ((n + bn - 1) / bn) * (long long)batch;
    const long long slots = num_sms / cg;
    const long long waves = (tiles + slots - 1) / slots;
    const double cost = (double)waves * bn / eff[i];
    if (cost < best_cost * 0.999) {
      best_cost = cost;
      best = bn;
      best_pair = cg == 2;
    }
  }
  if (pair) *pair = best_pair;
  return best;
}

/* The k split: two halves of a cluster per tile (two CTAs on a 128 x BN tile, or two CTA pairs on a 256 x 256
 * tile), each half with half of the k-blocks; each CTA adds the other half's partial sums for half of its
 * columns through distributed shared memory. One tile per cluster, so only for GEMMs whose tiles leave at
 * least half of the SMs idle. The planner compares modelled times: per tile a fixed cost plus a cost per
 * 64-deep k-block on one SM, fitted to f16 GEMMs measured on the B200 (4096 and 1024 rows, 128..512 columns,
 * k 4096 and 14336, CUDA-graph replay), and a floor of the compulsory bytes at 6 TB/s. It is taken when it
 * saves at least 5 %. Returns the split tile's width and sets *pair_out (2: single-CTA halves, 3: pair
 * halves), or returns 0. */
static double unsplit_kb_us(int bn, int pair) {
  if (pair) return bn == 256 ? 0.32 : 0.273;
  return bn == 256 ? 0.45 : bn == 128 ? 0.273 : bn == 64 ? 0.22 : 0.215;
}
static int ksplit_tile(int m, int n, int k, int batch, int num_sms, int bn0, int pair0, int *pair_out) {
  static const int bns[4] = {64, 128, 256, 256};
  static const int cgs[4] = {1, 1, 1, 2};
  static const double kb_us[4] = {0.225, 0.285, 0.46, 0.388}, fixed_us[4] = {6.0, 7.0, 6.9, 8.1};
  const long long nkb = ((long long)k + 63) / 64;
  if (nkb < 16 || num_sms < 4) return 0;
  /* f16 operands read once, f32 C written once */
  const double floor_us = ((double)m * k * 2 + (double)k * n * 2 + (double)m * n * 4) * batch / 6.0e6;
  const int cg0 = pair0 ? 2 : 1;
  const long long tiles0 = (long long)((m + 128 * cg0 - 1) / (128 * cg0)) * ((n + bn0 - 1) / bn0) * batch;
  const long long slots0 = num_sms / cg0;
  double t0 = (double)((tiles0 + slots0 - 1) / slots0) * (5.0 + (double)nkb * unsplit_kb_us(bn0, pair0));
  if (t0 < floor_us) t0 = floor_us;
  int best = 0;
  double best_t = 0.95 * t0;
  for (int i = 0; i < 4; i++) {
    const int bn = bns[i], cg = cgs[i];
    if (n <= bn / 2) continue; /* a tile at least half full */
    const long long tiles = (long long)((m + 128 * cg - 1) / (128 * cg)) * ((n + bn - 1) / bn) * batch;
    if (tiles * 2 * cg > num_sms) continue;
    double t = fixed_us[i] + (double)((nkb + 1) / 2) * kb_us[i];
    if (t < floor_us) t = floor_us;
    if (t < best_t) {
      best_t = t;
      best = bn;
      *pair_out = cg == 2 ? 3 : 2;
    }
  }
  return best;
}

int tb200_plan(int transa, int transb, int m, int n, int k, int batch, int in_type, int out_type, int tf32,
               int ptr_array, int aligned, int num_sms, int *tile_n, int *pair) {
  (void)out_type;
  if (tile_n) *tile_n = 0;
  if (pair) *pair = 0;
  if (m <= 0 || n <= 0 || batch <= 0) return TB200_KERNEL_NONE;
  if (k <= 0 || !tc_enabled()) return TB200_KERNEL_SIMT;
  int sixteen = in_type == TB200_F16 || in_type == TB200_BF16;
  if (sixteen && n <= 8 && transa == 1 && transb == 0 && k % 8 == 0 && aligned && skinny_enabled())
    return TB200_KERNEL_SKINNY;
  /* TF32 only with both operands K-major: an MN-major 32-bit operand needs the 128B swizzle with 32-byte
   * atoms (a layout this kernel does not stage); those GEMMs stay exact fp32 on the SIMT kernel */
  int tf32_ok = in_type == TB200_F32 && tf32 && transa == 1 && transb == 0;
  if ((sixteen || tf32_ok) && aligned) { /* pointer arrays included: per-element tensor maps on the device */
    int pr = 0;
    int bn = tb200_tc_tile_n(m, n, batch, num_sms, &pr);
    if (sixteen && !ptr_array) { /* the split kernel reads plain strided operands */
      int kpr = 0;
      const int ks = ksplit_tile(m, n, k, batch, num_sms <= 0 ? 148 : num_sms, bn, pr, &kpr);
      if (ks) {
        bn = ks;
        pr = kpr;
      }
    }
    if (tile_n) *tile_n = bn;
    if (pair) *pair = pr;
    return TB200_KERNEL_TC;
  }
  return TB200_KERNEL_SIMT;
}

/* base pointers 16-byte aligned, leading dimensions and strides whole multiples of 16 bytes: what a
 * TMA tensor map and 128-bit loads need */
static int operands_aligned(const tb200_gemm_t *g) {
  const long long es = esize(g->in_type);
  if (((long long)g->lda * es) % 16 || ((long long)g->ldb * es) % 16) return 0;
  if (g->Aarr || g->Barr) return 1; /* per-element pointers are checked by the kernels that read them */
  if (((uintptr_t)g->A & 15) || ((uintptr_t)g->B & 15)) return 0;
  if (g->batch > 1 && (((g->sA * es) % 16) || ((g->sB * es) % 16))) return 0;
  return 1;
}

/* TB200_TC_BN=32|64|128|256 forces a single-CTA tile of that width, TB200_TC_BN=pair the 256 x 256 pair
 * tile and TB200_TC_BN=pair128 the 256 x 128 pair tile (tests, bisecting; read per call) */
static void tile_override(int *tile_n, int *pair) {
  const char *e = getenv("TB200_TC_BN");
  if (e && (!strcmp(e, "pair") || !strcmp(e, "pair128"))) {
    *pair = 1;
    *tile_n = e[4] ? 128 : 256;
  } else {
    int v = e ? atoi(e) : 0;
    if (v == 32 || v == 64 || v == 128 || v == 256) {
      *tile_n = v;
      *pair = 0;
    }
  }
}

static const char *kernel_name(int kind) {
  return kind == TB200_KERNEL_SKINNY ? "skinny" : kind == TB200_KERNEL_TC ? "tc" : kind == TB200_KERNEL_SIMT ? "simt" : "none";
}

/* Plans and launches one validated GEMM on the handle's stream. A pointer-array batch on the tensor cores needs
 * scratch for its per-element tensor maps: the handle's per-stream buffer (allocated on first use), or with
 * noalloc the library's fixed device array (tb200_gemm_batched_ex_noalloc). */
static cublasStatus_t run_gemm_with(struct tb200_handle *h, tb200_gemm_t *g, int noalloc) {
  int tile_n = 0, pair = 0;
  int aligned = operands_aligned(g);
  int ptr_array = g->Aarr != NULL;
  int sms = tb200_num_sms();
  int kind = tb200_plan(g->opA, g->opB, g->m, g->n, g->k, g->batch, g->in_type, g->out_type, g->tf32, ptr_array,
                        aligned, sms, &tile_n, &pair);
  if (kind == TB200_KERNEL_TC) tile_override(&tile_n, &pair);
  if (tb200_trace())
    fprintf(stderr, "[trace] gemm%s %s op=%c%c m=%d n=%d k=%d batch=%d in=%d out=%d tf32=%d ptr=%d aligned=%d BN=%d pair=%d\n",
            noalloc ? "-noalloc" : "", kernel_name(kind), g->opA ? 'T' : 'N', g->opB ? 'T' : 'N', g->m, g->n, g->k,
            g->batch, g->in_type, g->out_type, g->tf32, ptr_array, aligned, tile_n, pair);
  int rc = 0;
  switch (kind) {
    case TB200_KERNEL_NONE: return CUBLAS_STATUS_SUCCESS;
    case TB200_KERNEL_SKINNY: {
      /* few 16-row blocks per SM: the balanced kernel, with its workspace (not on the allocation-free entry point,
       * and not during a capture that would have to allocate it) */
      int bal_grid = 0, bal_slots = 0;
      const size_t need = noalloc ? 0 : tb200_skinny_bal_plan(g, sms, &bal_grid, &bal_slots);
      void *dws = need ? decode_scratch(h, need) : NULL;
      rc = dws ? tb200_launch_skinny_bal(g, dws, TB200_DECODE_WS_BYTES, h->stream) : (int)cudaErrorNotSupported;
      if (rc == (int)cudaErrorNotSupported) rc = tb200_launch_skinny(g, h->stream);
      break;
    }
    case TB200_KERNEL_TC:
      if (ptr_array && noalloc) {
        rc = tb200_launch_tc_ptr_noalloc(g, tile_n, pair, sms, h->stream);
        if (rc == (int)cudaErrorNotSupported) rc = tb200_launch_simt(g, h->stream);
      } else if (ptr_array) {
        void *ws = handle_scratch(h, tb200_tc_ptr_ws_bytes(g->batch));
        rc = ws ? tb200_launch_tc_ptr(g, tile_n, pair, sms, ws, h->stream) : (int)cudaErrorNotSupported;
        if (rc == (int)cudaErrorNotSupported) rc = tb200_launch_simt(g, h->stream); /* no scratch: general kernel */
      } else {
        rc = tb200_launch_tc(g, tile_n, pair, sms, h->stream);
      }
      break;
    default: rc = tb200_launch_simt(g, h->stream); break;
  }
  if (rc != 0) {
    fprintf(stderr, "[tinycublas_b200] %s%s launch failed: %s\n", noalloc ? "tb200_gemm_batched_ex_noalloc: " : "",
            kernel_name(kind), cudaGetErrorString((cudaError_t)rc));
    return CUBLAS_STATUS_EXECUTION_FAILED;
  }
  return CUBLAS_STATUS_SUCCESS;
}

static cublasStatus_t run_gemm(struct tb200_handle *h, tb200_gemm_t *g) { return run_gemm_with(h, g, 0); }

static int op_code(cublasOperation_t op) { return op == CUBLAS_OP_N ? 0 : op == CUBLAS_OP_T ? 1 : -1; }
static int imax(int a, int b) { return a > b ? a : b; }

/* cuBLAS's argument rules: non-negative sizes, leading dimensions at least the stored row count */
static cublasStatus_t check_args(int oa, int ob, int m, int n, int k, int lda, int ldb, int ldc, int batch) {
  if (oa < 0 || ob < 0) return CUBLAS_STATUS_INVALID_VALUE;
  if (m < 0 || n < 0 || k < 0 || batch < 0) return CUBLAS_STATUS_INVALID_VALUE;
  if (lda < imax(1, oa == 0 ? m : k)) return CUBLAS_STATUS_INVALID_VALUE;
  if (ldb < imax(1, ob == 0 ? k : n)) return CUBLAS_STATUS_INVALID_VALUE;
  if (ldc < imax(1, m)) return CUBLAS_STATUS_INVALID_VALUE;
  return CUBLAS_STATUS_SUCCESS;
}

static cublasStatus_t gemm_common(cublasHandle_t handle, cublasOperation_t ta, cublasOperation_t tb, int m, int n, int k,
                                  const void *alpha, const void *A, const void *const *Aarr, cudaDataType At, int lda,
                                  long long sA, const void *B, const void *const *Barr, cudaDataType Bt, int ldb,
                                  long long sB, const void *beta, void *C, void *const *Carr, cudaDataType Ct, int ldc,
                                  long long sC, int batch, cublasComputeType_t ct) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  tb200_gemm_t g;
  memset(&g, 0, sizeof g);
  int tf32 = 0;
  if (gemm_contract(At, Bt, Ct, ct, &g.in_type, &g.out_type, &tf32)) return CUBLAS_STATUS_NOT_SUPPORTED;
  g.opA = op_code(ta);
  g.opB = op_code(tb);
  cublasStatus_t st = check_args(g.opA, g.opB, m, n, k, lda, ldb, ldc, batch);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  if (!alpha || !beta) return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0 || batch == 0) return CUBLAS_STATUS_SUCCESS;
  /* an f32 GEMM may use TF32 when the compute type says so or the handle's math mode asks for it */
  if (g.in_type == TB200_F32)
    g.tf32 = tf32 || (((int)h->math_mode & 0xf) == CUBLAS_TF32_TENSOR_OP_MATH && ct == CUBLAS_COMPUTE_32F);
  g.m = m;
  g.n = n;
  g.k = k;
  g.batch = batch;
  g.alpha = read_scalar(alpha, ct);
  g.beta = read_scalar(beta, ct);
  g.A = A; g.lda = lda; g.sA = sA; g.Aarr = Aarr;
  g.B = B; g.ldb = ldb; g.sB = sB; g.Barr = Barr;
  g.C = C; g.ldc = ldc; g.sC = sC; g.Carr = Carr;
  return run_gemm(h, &g);
}

/* ---- exported ABI ---- */

cublasStatus_t cublasCreate_v2(cublasHandle_t *handle) {
  if (!handle) return CUBLAS_STATUS_INVALID_VALUE;
  struct tb200_handle *h = (struct tb200_handle *)calloc(1, sizeof *h);
  if (!h) return CUBLAS_STATUS_ALLOC_FAILED;
  h->stream = NULL;
  h->math_mode = CUBLAS_DEFAULT_MATH;
  h->device = -1;
  (void)cudaGetDevice(&h->device); /* no context is created by this query */
  *handle = (cublasHandle_t)h;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasDestroy_v2(cublasHandle_t handle) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (h) {
    for (int i = 0; i < TB200_WS_SLOTS; i++) {
      if (h->ws[i].ptr) {
        cudaStreamSynchronize(h->ws[i].stream);
        cudaFree(h->ws[i].ptr);
      }
      if (h->dws[i].ptr) {
        cudaStreamSynchronize(h->dws[i].stream);
        cudaFree(h->dws[i].ptr);
      }
    }
    for (int i = 0; i < h->n_retired; i++) {
      cudaStreamSynchronize(h->retired[i].stream);
      cudaFree(h->retired[i].ptr);
    }
  }
  free(handle);
  return CUBLAS_STATUS_SUCCESS;
}

unsigned tb200_scratch_allocs(cublasHandle_t handle) {
  return handle ? ((struct tb200_handle *)handle)->ws_allocs : 0u;
}

cublasStatus_t cublasSetStream_v2(cublasHandle_t handle, cudaStream_t stream) {
  if (!handle) return CUBLAS_STATUS_NOT_INITIALIZED;
  struct tb200_handle *h = (struct tb200_handle *)handle;
  h->stream = stream;
  /* the stream's pointer-array scratch (64 KB: batches up to 255 elements), made now when this call is outside a
   * stream capture, so that such a batch captured later on this stream still runs on the tensor cores; nothing is
   * made during a capture, and a failed allocation only leaves it to the first pointer-array call */
  (void)handle_scratch(h, tb200_tc_ptr_ws_bytes(1));
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetMathMode(cublasHandle_t handle, cublasMath_t mode) {
  if (!handle) return CUBLAS_STATUS_NOT_INITIALIZED;
  ((struct tb200_handle *)handle)->math_mode = mode;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetWorkspace_v2(cublasHandle_t handle, void *workspace, size_t bytes) {
  if (!handle) return CUBLAS_STATUS_NOT_INITIALIZED;
  struct tb200_handle *h = (struct tb200_handle *)handle;
  h->user_ws = workspace;
  h->user_ws_bytes = bytes;
  return CUBLAS_STATUS_SUCCESS;
}

const char *cublasGetStatusString(cublasStatus_t s) {
  switch (s) {
    case CUBLAS_STATUS_SUCCESS: return "CUBLAS_STATUS_SUCCESS";
    case CUBLAS_STATUS_NOT_INITIALIZED: return "CUBLAS_STATUS_NOT_INITIALIZED";
    case CUBLAS_STATUS_ALLOC_FAILED: return "CUBLAS_STATUS_ALLOC_FAILED";
    case CUBLAS_STATUS_INVALID_VALUE: return "CUBLAS_STATUS_INVALID_VALUE";
    case CUBLAS_STATUS_NOT_SUPPORTED: return "CUBLAS_STATUS_NOT_SUPPORTED";
    case CUBLAS_STATUS_EXECUTION_FAILED: return "CUBLAS_STATUS_EXECUTION_FAILED";
    case CUBLAS_STATUS_INTERNAL_ERROR: return "CUBLAS_STATUS_INTERNAL_ERROR";
    default: return "CUBLAS_STATUS_UNKNOWN_ERROR";
  }
}

cublasStatus_t cublasSgemm_v2(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb, int m, int n, int k,
                              const float *alpha, const float *A, int lda, const float *B, int ldb, const float *beta,
                              float *C, int ldc) {
  return gemm_common(h, ta, tb, m, n, k, alpha, A, NULL, CUDA_R_32F, lda, 0, B, NULL, CUDA_R_32F, ldb, 0, beta, C, NULL,
                     CUDA_R_32F, ldc, 0, 1, CUBLAS_COMPUTE_32F);
}

cublasStatus_t cublasGemmEx(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb, int m, int n, int k,
                            const void *alpha, const void *A, cudaDataType At, int lda, const void *B, cudaDataType Bt,
                            int ldb, const void *beta, void *C, cudaDataType Ct, int ldc, cublasComputeType_t ct,
                            cublasGemmAlgo_t algo) {
  (void)algo;
  return gemm_common(h, ta, tb, m, n, k, alpha, A, NULL, At, lda, 0, B, NULL, Bt, ldb, 0, beta, C, NULL, Ct, ldc, 0, 1,
                     ct);
}

cublasStatus_t cublasGemmStridedBatchedEx(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb, int m, int n,
                                          int k, const void *alpha, const void *A, cudaDataType At, int lda,
                                          long long int sA, const void *B, cudaDataType Bt, int ldb, long long int sB,
                                          const void *beta, void *C, cudaDataType Ct, int ldc, long long int sC,
                                          int batch, cublasComputeType_t ct, cublasGemmAlgo_t algo) {
  (void)algo;
  return gemm_common(h, ta, tb, m, n, k, alpha, A, NULL, At, lda, sA, B, NULL, Bt, ldb, sB, beta, C, NULL, Ct, ldc, sC,
                     batch, ct);
}

cublasStatus_t cublasGemmBatchedEx(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb, int m, int n, int k,
                                   const void *alpha, const void *const Aarray[], cudaDataType At, int lda,
                                   const void *const Barray[], cudaDataType Bt, int ldb, const void *beta,
                                   void *const Carray[], cudaDataType Ct, int ldc, int batch, cublasComputeType_t ct,
                                   cublasGemmAlgo_t algo) {
  (void)algo;
  if (batch > 0 && (!Aarray || !Barray || !Carray)) return CUBLAS_STATUS_INVALID_VALUE;
  return gemm_common(h, ta, tb, m, n, k, alpha, NULL, Aarray, At, lda, 0, NULL, Barray, Bt, ldb, 0, beta, NULL, Carray,
                     Ct, ldc, 0, batch, ct);
}

cublasStatus_t cublasSgemmStridedBatched(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb, int m, int n,
                                         int k, const float *alpha, const float *A, int lda, long long int sA,
                                         const float *B, int ldb, long long int sB, const float *beta, float *C,
                                         int ldc, long long int sC, int batch) {
  return gemm_common(h, ta, tb, m, n, k, alpha, A, NULL, CUDA_R_32F, lda, sA, B, NULL, CUDA_R_32F, ldb, sB, beta, C,
                     NULL, CUDA_R_32F, ldc, sC, batch, CUBLAS_COMPUTE_32F);
}

cublasStatus_t cublasSgemmBatched(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb, int m, int n, int k,
                                  const float *alpha, const float *const Aarray[], int lda, const float *const Barray[],
                                  int ldb, const float *beta, float *const Carray[], int ldc, int batch) {
  if (batch > 0 && (!Aarray || !Barray || !Carray)) return CUBLAS_STATUS_INVALID_VALUE;
  return gemm_common(h, ta, tb, m, n, k, alpha, NULL, (const void *const *)Aarray, CUDA_R_32F, lda, 0, NULL,
                     (const void *const *)Barray, CUDA_R_32F, ldb, 0, beta, NULL, (void *const *)Carray, CUDA_R_32F, ldc,
                     0, batch, CUBLAS_COMPUTE_32F);
}

cublasStatus_t cublasStrsmBatched(cublasHandle_t handle, cublasSideMode_t side, cublasFillMode_t uplo,
                                  cublasOperation_t trans, cublasDiagType_t diag, int m, int n, const float *alpha,
                                  const float *const A[], int lda, float *const B[], int ldb, int batch) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (side != CUBLAS_SIDE_RIGHT || uplo != CUBLAS_FILL_MODE_UPPER || trans != CUBLAS_OP_N || diag != CUBLAS_DIAG_NON_UNIT)
    return CUBLAS_STATUS_NOT_SUPPORTED;
  if (m < 0 || n < 0 || batch < 0 || lda < imax(1, n) || ldb < imax(1, m) || !alpha) return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0 || batch == 0) return CUBLAS_STATUS_SUCCESS;
  if (!A || !B) return CUBLAS_STATUS_INVALID_VALUE;
  if (tb200_trace()) fprintf(stderr, "[trace] trsm_rupn m=%d n=%d batch=%d\n", m, n, batch);
  int rc = tb200_launch_trsm_rupn(A, B, m, n, lda, ldb, *alpha, batch, h->stream);
  return rc == 0 ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

cublasStatus_t tb200_gemm_ex_allgather(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                                       int m_local, int n, int k, const void *alpha, const void *A, cudaDataType Atype,
                                       int lda, const void *B, cudaDataType Btype, int ldb, void *const *C_replicas,
                                       int P, cudaDataType Ctype, int ldc, int row0, cublasComputeType_t ct) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  tb200_gemm_t g;
  memset(&g, 0, sizeof g);
  int tf32 = 0;
  if (gemm_contract(Atype, Btype, Ctype, ct, &g.in_type, &g.out_type, &tf32)) return CUBLAS_STATUS_NOT_SUPPORTED;
  g.opA = op_code(transa);
  g.opB = op_code(transb);
  if (!C_replicas || P < 1 || P > 8 || row0 < 0 || !alpha) return CUBLAS_STATUS_INVALID_VALUE;
  for (int q = 0; q < P; q++)
    if (!C_replicas[q]) return CUBLAS_STATUS_INVALID_VALUE;
  cublasStatus_t st = check_args(g.opA, g.opB, m_local, n, k, lda, ldb, ldc, 1);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  if ((long long)row0 + m_local > ldc) return CUBLAS_STATUS_INVALID_VALUE; /* rows stay inside each replica's column */
  if (m_local == 0 || n == 0) return CUBLAS_STATUS_SUCCESS;
  g.tf32 = tf32;
  g.m = m_local;
  g.n = n;
  g.k = k;
  g.batch = 1;
  g.alpha = read_scalar(alpha, ct);
  g.beta = 0.f;
  g.A = A; g.lda = lda;
  g.B = B; g.ldb = ldb;
  g.C = C_replicas[0]; g.ldc = ldc;
  g.nrep = P;
  g.row0 = row0;
  for (int q = 0; q < P; q++) g.rep[q] = C_replicas[q];
  if (!operands_aligned(&g) || !tb200_tc_ok(&g)) return CUBLAS_STATUS_NOT_SUPPORTED;
  int sms = tb200_num_sms(), pair = 0;
  int bn = tb200_tc_tile_n(m_local, n, 1, sms, &pair);
  if (tb200_trace())
    fprintf(stderr, "[trace] gemm tc-allgather m_local=%d n=%d k=%d P=%d row0=%d BN=%d pair=%d\n", m_local, n, k, P, row0,
            bn, pair);
  int rc = tb200_launch_tc(&g, bn, pair, sms, h->stream);
  if (rc == (int)cudaErrorNotSupported) return CUBLAS_STATUS_NOT_SUPPORTED;
  return rc == 0 ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

/* The N-sharded GEMM with its output exchange through NVLink multicast: this rank's m_local rows are stored
 * once per element to C_multicast (the multicast address of a buffer every rank holds, bound to one
 * multicast object), and the switch writes them into every rank's C at row offset row0. f32 C only (the
 * multimem store is f32), beta = 0. The caller orders the stores before any rank reads its C (a collective
 * after the launch). */
cublasStatus_t tb200_gemm_ex_multicast(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                                       int m_local, int n, int k, const void *alpha, const void *A, cudaDataType Atype,
                                       int lda, const void *B, cudaDataType Btype, int ldb, void *C_multicast,
                                       cudaDataType Ctype, int ldc, int row0, cublasComputeType_t ct) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  tb200_gemm_t g;
  memset(&g, 0, sizeof g);
  int tf32 = 0;
  if (gemm_contract(Atype, Btype, Ctype, ct, &g.in_type, &g.out_type, &tf32)) return CUBLAS_STATUS_NOT_SUPPORTED;
  if (g.out_type != TB200_F32) return CUBLAS_STATUS_NOT_SUPPORTED;
  g.opA = op_code(transa);
  g.opB = op_code(transb);
  if (!C_multicast || row0 < 0 || !alpha) return CUBLAS_STATUS_INVALID_VALUE;
  cublasStatus_t st = check_args(g.opA, g.opB, m_local, n, k, lda, ldb, ldc, 1);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  if ((long long)row0 + m_local > ldc) return CUBLAS_STATUS_INVALID_VALUE; /* rows stay inside C's columns */
  if (m_local == 0 || n == 0) return CUBLAS_STATUS_SUCCESS;
  g.tf32 = tf32;
  g.m = m_local;
  g.n = n;
  g.k = k;
  g.batch = 1;
  g.alpha = read_scalar(alpha, ct);
  g.beta = 0.f;
  g.A = A; g.lda = lda;
  g.B = B; g.ldb = ldb;
  g.C = C_multicast; g.ldc = ldc;
  g.mc = C_multicast;
  g.row0 = row0;
  if (!operands_aligned(&g) || !tb200_tc_ok(&g)) return CUBLAS_STATUS_NOT_SUPPORTED;
  int sms = tb200_num_sms(), pair = 0;
  int bn = tb200_tc_tile_n(m_local, n, 1, sms, &pair);
  if (tb200_trace())
    fprintf(stderr, "[trace] gemm tc-multicast m_local=%d n=%d k=%d row0=%d BN=%d pair=%d\n", m_local, n, k, row0, bn,
            pair);
  int rc = tb200_launch_tc(&g, bn, pair, sms, h->stream);
  if (rc == (int)cudaErrorNotSupported) return CUBLAS_STATUS_NOT_SUPPORTED;
  return rc == 0 ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

/* One launch of the tensor-core kernel for every group (expert) of a mixture-of-experts layer: group g
 * multiplies A_g = A + g * strideA with the columns [offsets[g], offsets[g + 1]) of B into the same columns
 * of C. offsets is a device array (the per-expert token counts come from the router on the GPU and never
 * reach the host). Same type contract and argument rules as cublasGemmStridedBatchedEx; the operands must
 * suit the tensor-core kernel (16-byte aligned, ld and strideA whole multiples of 16 bytes), otherwise
 * NOT_SUPPORTED. The kernel clamps the offsets to [0, n_total] and treats a decrease as an empty group. */
cublasStatus_t tb200_gemm_grouped_ex(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb, int m,
                                     int n_total, int k, int groups, const int *offsets, const void *alpha,
                                     const void *A, cudaDataType Atype, int lda, long long strideA, const void *B,
                                     cudaDataType Btype, int ldb, const void *beta, void *C, cudaDataType Ctype,
                                     int ldc, cublasComputeType_t computeType) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  tb200_gemm_t g;
  memset(&g, 0, sizeof g);
  int tf32 = 0;
  if (gemm_contract(Atype, Btype, Ctype, computeType, &g.in_type, &g.out_type, &tf32)) return CUBLAS_STATUS_NOT_SUPPORTED;
  g.opA = op_code(transa);
  g.opB = op_code(transb);
  cublasStatus_t st = check_args(g.opA, g.opB, m, n_total, k, lda, ldb, ldc, groups);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  if (!alpha || !beta || !offsets || groups > TB200_MAX_GROUPS || strideA < 0) return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n_total == 0 || groups == 0) return CUBLAS_STATUS_SUCCESS;
  if (g.in_type == TB200_F32)
    g.tf32 = tf32 || (((int)h->math_mode & 0xf) == CUBLAS_TF32_TENSOR_OP_MATH && computeType == CUBLAS_COMPUTE_32F);
  if (g.in_type == TB200_F32 && !g.tf32) return CUBLAS_STATUS_NOT_SUPPORTED; /* exact fp32: no grouped kernel */
  g.m = m;
  g.n = n_total;
  g.k = k;
  g.batch = groups;
  g.alpha = read_scalar(alpha, computeType);
  g.beta = read_scalar(beta, computeType);
  g.A = A; g.lda = lda; g.sA = strideA;
  g.B = B; g.ldb = ldb;
  g.C = C; g.ldc = ldc;
  g.grp_off = offsets;
  g.groups = groups;
  if (!operands_aligned(&g) || !tb200_tc_ok(&g)) return CUBLAS_STATUS_NOT_SUPPORTED;
  int sms = tb200_num_sms(), pair = 0;
  int avg_n = n_total / groups > 0 ? n_total / groups : 1;
  int bn = tb200_tc_tile_n(m, avg_n, groups, sms, &pair);
  tile_override(&bn, &pair);
  if (tb200_trace())
    fprintf(stderr, "[trace] gemm tc-grouped op=%c%c m=%d n_total=%d k=%d groups=%d BN=%d pair=%d\n", g.opA ? 'T' : 'N',
            g.opB ? 'T' : 'N', m, n_total, k, groups, bn, pair);
  int rc = tb200_launch_tc(&g, bn, pair, sms, h->stream);
  if (rc == (int)cudaErrorNotSupported) return CUBLAS_STATUS_NOT_SUPPORTED;
  if (rc != 0) {
    fprintf(stderr, "[tinycublas_b200] grouped launch failed: %s\n", cudaGetErrorString((cudaError_t)rc));
    return CUBLAS_STATUS_EXECUTION_FAILED;
  }
  return CUBLAS_STATUS_SUCCESS;
}

/* tb200_gemm_grouped_ex with the token gather fused into the GEMM's B loads: column j of B is column
 * token_ids[j] of X (k x n_src, ld ldx, under op N), so the per-expert copy of the tokens is never written.
 * The tensor-core kernel loads four token columns per TMA (tile::gather4) into its usual shared-memory
 * tile. 16-bit inputs only. */
cublasStatus_t tb200_gemm_grouped_gather_ex(cublasHandle_t handle, cublasOperation_t transa, int m, int n_total, int k,
                                            int groups, const int *offsets, const int *token_ids, const void *alpha,
                                            const void *A, cudaDataType Atype, int lda, long long strideA,
                                            const void *X, cudaDataType Xtype, int ldx, int n_src, const void *beta,
                                            void *C, cudaDataType Ctype, int ldc, cublasComputeType_t computeType) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  tb200_gemm_t g;
  memset(&g, 0, sizeof g);
  int tf32 = 0;
  if (gemm_contract(Atype, Xtype, Ctype, computeType, &g.in_type, &g.out_type, &tf32)) return CUBLAS_STATUS_NOT_SUPPORTED;
  g.opA = op_code(transa);
  g.opB = 0;
  cublasStatus_t st = check_args(g.opA, g.opB, m, n_total, k, lda, ldx, ldc, groups);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  if (!alpha || !beta || !offsets || !token_ids || groups > TB200_MAX_GROUPS || strideA < 0 || n_src < 1)
    return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n_total == 0 || groups == 0) return CUBLAS_STATUS_SUCCESS;
  if (g.in_type == TB200_F32) return CUBLAS_STATUS_NOT_SUPPORTED;
  g.m = m;
  g.n = n_total;
  g.k = k;
  g.batch = groups;
  g.alpha = read_scalar(alpha, computeType);
  g.beta = read_scalar(beta, computeType);
  g.A = A; g.lda = lda; g.sA = strideA;
  g.B = X; g.ldb = ldx;
  g.C = C; g.ldc = ldc;
  g.grp_off = offsets;
  g.groups = groups;
  g.gidx = token_ids;
  g.n_src = n_src;
  if (!operands_aligned(&g) || !tb200_tc_ok(&g)) return CUBLAS_STATUS_NOT_SUPPORTED;
  int sms = tb200_num_sms(), pair = 0;
  int avg_n = n_total / groups > 0 ? n_total / groups : 1;
  int bn = tb200_tc_tile_n(m, avg_n, groups, sms, &pair);
  tile_override(&bn, &pair); /* the launcher takes 32 or 64 columns, one CTA per tile */
  if (tb200_trace())
    fprintf(stderr, "[trace] gemm tc-grouped-gather op=%cN m=%d n_total=%d k=%d groups=%d n_src=%d BN=%d\n",
            g.opA ? 'T' : 'N', m, n_total, k, groups, n_src, bn <= 32 ? 32 : 64);
  int rc = tb200_launch_tc(&g, bn, pair, sms, h->stream);
  if (rc == (int)cudaErrorNotSupported) return CUBLAS_STATUS_NOT_SUPPORTED;
  if (rc != 0) {
    fprintf(stderr, "[tinycublas_b200] grouped gather launch failed: %s\n", cudaGetErrorString((cudaError_t)rc));
    return CUBLAS_STATUS_EXECUTION_FAILED;
  }
  return CUBLAS_STATUS_SUCCESS;
}

/* The routed layer's data movement around tb200_gemm_grouped_ex: tb200_moe_gather copies column
 * token_ids[p] of X (k elements of `type`, ld ldx, n_src columns) to column p of Xp (ld ldxp) for every
 * p < n_total, putting each expert's tokens one expert after another; tb200_moe_combine sums, for every
 * token t, weights[t * topk + j] * column positions[t * topk + j] of Cp over j in order into column t of Y
 * (f32). Ids and positions outside their range contribute zeros. On the handle's stream; no allocation. */
cublasStatus_t tb200_moe_gather(cublasHandle_t handle, const void *X, cudaDataType type, int k, int ldx, int n_src,
                                const int *token_ids, int n_total, void *Xp, int ldxp) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  const int code = dtype_code(type);
  if (code < 0) return CUBLAS_STATUS_NOT_SUPPORTED;
  if (k < 0 || n_src < 0 || n_total < 0 || ldx < (k > 1 ? k : 1) || ldxp < (k > 1 ? k : 1)) return CUBLAS_STATUS_INVALID_VALUE;
  if (k == 0 || n_total == 0) return CUBLAS_STATUS_SUCCESS;
  if (!X || !token_ids || !Xp) return CUBLAS_STATUS_INVALID_VALUE;
  const int es = code == TB200_F32 ? 4 : 2;
  int rc = tb200_launch_moe_gather(X, (long long)ldx * es, n_src, token_ids, n_total, k * es, Xp, (long long)ldxp * es,
                                   h->stream);
  return rc == 0 ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

cublasStatus_t tb200_moe_combine(cublasHandle_t handle, int m, const float *Cp, int ldc, int n_total,
                                 const int *positions, const float *weights, int topk, int n_tokens, float *Y,
                                 int ldy) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (m < 0 || n_total < 0 || topk < 0 || n_tokens < 0 || ldc < (m > 1 ? m : 1) || ldy < (m > 1 ? m : 1))
    return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n_tokens == 0) return CUBLAS_STATUS_SUCCESS;
  if (!Cp || !positions || !weights || !Y) return CUBLAS_STATUS_INVALID_VALUE;
  int rc = tb200_launch_moe_combine(Cp, m, ldc, n_total, positions, weights, topk, n_tokens, Y, ldy, h->stream);
  return rc == 0 ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

/* cublasGemmBatchedEx without any device allocation: same arguments, same plan and kernels (the dispatch above,
 * knobs included); where the pointer-array tensor-core path needs scratch it takes the library's fixed device
 * array (tb200_launch_tc_ptr_noalloc) instead of the handle's lazily allocated buffer. batchCount is bounded
 * by that array. */
cublasStatus_t tb200_gemm_batched_ex_noalloc(cublasHandle_t handle, cublasOperation_t transa,
                                             cublasOperation_t transb, int m, int n, int k, const void *alpha,
                                             const void *const Aarray[], cudaDataType Atype, int lda,
                                             const void *const Barray[], cudaDataType Btype, int ldb,
                                             const void *beta, void *const Carray[], cudaDataType Ctype, int ldc,
                                             int batchCount, cublasComputeType_t ct) {
  struct tb200_handle *h = (struct tb200_handle *)handle;
  if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (batchCount > tb200_noalloc_max_batch()) {
    fprintf(stderr,
            "[tinycublas_b200] tb200_gemm_batched_ex_noalloc: batchCount %d exceeds the %d its fixed scratch holds\n",
            batchCount, tb200_noalloc_max_batch());
    return CUBLAS_STATUS_INVALID_VALUE;
  }
  tb200_gemm_t g;
  memset(&g, 0, sizeof g);
  int tf32 = 0;
  if (gemm_contract(Atype, Btype, Ctype, ct, &g.in_type, &g.out_type, &tf32)) return CUBLAS_STATUS_NOT_SUPPORTED;
  g.opA = op_code(transa);
  g.opB = op_code(transb);
  cublasStatus_t st = check_args(g.opA, g.opB, m, n, k, lda, ldb, ldc, batchCount);
  if (st != CUBLAS_STATUS_SUCCESS) return st;
  if (!alpha || !beta) return CUBLAS_STATUS_INVALID_VALUE;
  if (m == 0 || n == 0 || batchCount == 0) return CUBLAS_STATUS_SUCCESS;
  if (!Aarray || !Barray || !Carray) return CUBLAS_STATUS_INVALID_VALUE;
  if (g.in_type == TB200_F32)
    g.tf32 = tf32 || (((int)h->math_mode & 0xf) == CUBLAS_TF32_TENSOR_OP_MATH && ct == CUBLAS_COMPUTE_32F);
  g.m = m;
  g.n = n;
  g.k = k;
  g.batch = batchCount;
  g.alpha = read_scalar(alpha, ct);
  g.beta = read_scalar(beta, ct);
  g.Aarr = Aarray; g.lda = lda;
  g.Barr = Barray; g.ldb = ldb;
  g.Carr = Carray; g.ldc = ldc;
  return run_gemm_with(h, &g, 1);
}

const char *tb200_version(void) { return "tinycublas_b200 " TB200_GIT_DESCRIBE " sm_100a"; }
