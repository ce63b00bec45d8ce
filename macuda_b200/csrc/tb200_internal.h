/* tb200_internal.h - the seam between the C host layer (tinycublas.c) and the CUDA launchers (*.cu).
 * Plain C types only; every launcher returns a cudaError_t as int and launches asynchronously. */
#ifndef TB200_INTERNAL_H
#define TB200_INTERNAL_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types, numbered as the reference's dtype_code (cuda-shim/libtinycublas/cublas.c:107) */
enum { TB200_F32 = 0, TB200_F16 = 1, TB200_BF16 = 2 };

/* One GEMM request, already validated: C = alpha * op(A) op(B) + beta * C, column-major.
 * Exactly one of (A, Aarr) is used: Aarr != NULL means a device array of batch pointers. Strides are
 * in elements of the operand's own type. */
typedef struct {
  int opA, opB;             /* 0 = N, 1 = T */
  int m, n, k, batch;
  float alpha, beta;
  const void *A; int lda; long long sA; const void *const *Aarr;
  const void *B; int ldb; long long sB; const void *const *Barr;
  void *C; int ldc; long long sC; void *const *Carr;
  int in_type, out_type;    /* TB200_F32 / F16 / BF16 */
  int tf32;                 /* f32 inputs only: 1 = TF32 tensor cores allowed */
  /* replicated output (N-sharded GEMM with the exchange fused into the epilogue): when nrep > 0 the
   * rows are stored at row offset row0 into each of the nrep replicas (device pointers valid in this
   * process, peers' buffers included) instead of C; tensor-core kernel only, beta == 0, batch == 1 */
  int nrep, row0;
  void *rep[8];
  /* the same with one multicast address instead of replicas: every f32 store of the epilogue goes to the
   * multicast object of all ranks' C (NVSwitch fans it out); row offset row0 */
  void *mc;
  /* the general kernel runs only if *run_if == run_if_gen (run_if NULL: always): the fallback launch behind a
   * pointer-array tensor-core launch, taken when some batch pointer is not 16-byte aligned (the prep kernel
   * then writes the call's generation number into the flag, which is never cleared) */
  const int *run_if;
  int run_if_gen;
  /* grouped GEMM (tensor-core kernel only): when groups > 0, group g multiplies batch element g of A (stride
   * sA) with columns [grp_off[g], grp_off[g + 1]) of B into the same columns of C; grp_off is a device array
   * of groups + 1 offsets read by the kernel (batch == groups, sB == sC == 0, n = all columns) */
  const int *grp_off;
  int groups;
  /* grouped GEMM with the token gather fused (16-bit, B under op N): column j of B is column gidx[j] of B's
   * n_src columns (gidx a device array of n columns; an id outside [0, n_src) gives a zero column) */
  const int *gidx;
  int n_src;
} tb200_gemm_t;

#define TB200_MAX_GROUPS 1024

int tb200_launch_simt(const tb200_gemm_t *g, cudaStream_t s);
int tb200_launch_skinny(const tb200_gemm_t *g, cudaStream_t s);
/* the balanced decode kernel (few 16-row blocks per SM): grid, slots and workspace bytes, 0 when not for this
 * GEMM; the launch takes a zero-initialised workspace of at least that size, owned by the caller per stream */
size_t tb200_skinny_bal_plan(const tb200_gemm_t *g, int num_sms, int *grid, int *nslots);
int tb200_launch_skinny_bal(const tb200_gemm_t *g, void *ws, size_t ws_bytes, cudaStream_t s);
int tb200_launch_tc(const tb200_gemm_t *g, int tile_n, int pair, int num_sms, cudaStream_t s);
/* pointer-array batches on the tensor cores: `ws` is device scratch of tb200_tc_ptr_ws_bytes(batch)
 * bytes owned by the caller for the duration of the launch */
size_t tb200_tc_ptr_ws_bytes(int batch);
int tb200_launch_tc_ptr(const tb200_gemm_t *g, int tile_n, int pair, int num_sms, void *ws, cudaStream_t s);
/* the same with the library's fixed device scratch instead of caller-provided scratch (no allocation) */
int tb200_noalloc_max_batch(void);
int tb200_launch_tc_ptr_noalloc(const tb200_gemm_t *g, int tile_n, int pair, int num_sms, cudaStream_t s);
int tb200_launch_trsm_rupn(const float *const *A, float *const *B, int rows, int n, int lda, int ldb, float alpha,
                           int batch, cudaStream_t s);

/* mixture-of-experts data movement (aux_kernels.cu): columns gathered into expert order; expert outputs
 * combined back into token order with the routing weights */
int tb200_launch_moe_gather(const void *X, long long ldx_bytes, int n_src, const int *ids, int n_total, int row_bytes,
                            void *Xp, long long ldp_bytes, cudaStream_t s);
int tb200_launch_moe_combine(const float *Cp, int m, long long ldc, int n_total, const int *pos, const float *w,
                             int topk, int n_tokens, float *Y, long long ldy, cudaStream_t s);

/* properties of the current device, cached per device ordinal */
int tb200_num_sms(void);

/* eligibility rules shared by the planner and the launchers */
int tb200_skinny_ok(const tb200_gemm_t *g);
int tb200_tc_ok(const tb200_gemm_t *g);

int tb200_trace(void);
/* launch the kernels with programmatic stream serialization (TB200_PDL=0 turns it off) */
int tb200_pdl(void);

#ifdef __cplusplus
}
#endif
#endif
