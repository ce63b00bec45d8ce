/* tinycublas_b200.h - the C ABI of libtinycublas_b200.so, the B200 (sm_100a) GEMM library.
 *
 * The library exports the cuBLAS v2 entry points that llama.cpp's ggml-cuda calls, with the exact
 * signatures of CUDA 12.9's cublas_v2.h, so it links in place of libcublas (or of macuda's
 * libtinycublas) without a source change on the caller's side. Every declaration below names the
 * reference interface it replaces, as path:line inside the Davinchy/macuda tree.
 *
 * Conventions shared by every GEMM entry point (the cuBLAS ones):
 *   C = alpha * op(A) * op(B) + beta * C, column-major, op(X) = X or X^T.
 *   A, B, C and pointer arrays are caller-owned DEVICE memory; alpha and beta are HOST pointers read
 *   in the compute type (half under CUBLAS_COMPUTE_16F*, float otherwise).
 *   Launches are asynchronous on the handle's stream. No entry point synchronises the host or reads
 *   device memory back. Device scratch is made only outside stream capture, and only where
 *   tb200_scratch_allocs says.
 *
 * Status codes:
 *   CUBLAS_STATUS_SUCCESS            launched (or nothing to do: m, n or batch is 0)
 *   CUBLAS_STATUS_NOT_INITIALIZED    NULL handle
 *   CUBLAS_STATUS_INVALID_VALUE      negative sizes, a leading dimension below its minimum, an
 *                                    operation other than N or T
 *   CUBLAS_STATUS_NOT_SUPPORTED      a type / compute-type combination outside the contract
 *                                    (reference cuda-shim/libtinycublas/cublas.c:118-134)
 *   CUBLAS_STATUS_EXECUTION_FAILED   the CUDA launch failed
 */
#ifndef TINYCUBLAS_B200_H
#define TINYCUBLAS_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>
#include <cublas_v2.h> /* cuBLAS types: cublasHandle_t, cublasStatus_t, cublasOperation_t, ... */

#ifdef __cplusplus
extern "C" {
#endif

/* ---- handle lifecycle ------------------------------------------------------------------------- */

/* replaces cuda-shim/libtinycublas/cublas.c:242-244. Allocates the handle on the host only; it
 * binds the legacy default stream and records the current device. Touches no device memory. */
cublasStatus_t cublasCreate_v2(cublasHandle_t *handle);

/* replaces cublas.c:245-247. Frees the handle and any scratch the library allocated for it (waiting for
 * the streams that used it). */
cublasStatus_t cublasDestroy_v2(cublasHandle_t handle);

/* replaces cublas.c:248. NULL selects the legacy default stream. Outside a stream capture, the first selection of
 * a stream also makes its pointer-array scratch (64 KB, for batches up to 255 elements), so that such a batch
 * captured later on that stream runs on the tensor cores. */
cublasStatus_t cublasSetStream_v2(cublasHandle_t handle, cudaStream_t stream);

/* replaces cublas.c:249. Unlike the reference (which stores and ignores it), the mode is honoured:
 * CUBLAS_TF32_TENSOR_OP_MATH lets fp32 GEMMs run on the TF32 tensor cores; the default and
 * CUBLAS_PEDANTIC_MATH keep them in fp32. */
cublasStatus_t cublasSetMathMode(cublasHandle_t handle, cublasMath_t mode);

/* replaces cublas.c:288 (a no-op there). Records a caller-owned device workspace; this library's
 * kernels do not need one, so the pointer is kept only for cublasGetWorkspace-style introspection. */
cublasStatus_t cublasSetWorkspace_v2(cublasHandle_t handle, void *workspace, size_t workspaceSizeInBytes);

/* replaces cublas.c:286-287 */
const char *cublasGetStatusString(cublasStatus_t status);

/* ---- GEMM ------------------------------------------------------------------------------------ */

/* replaces cublas.c:250-253. fp32 GEMM: fp32 FMA by default, TF32 tensor cores under
 * CUBLAS_TF32_TENSOR_OP_MATH (the reference always used TF32, cuda-shim/libtinycublas/gemm.cu:143-221). */
cublasStatus_t cublasSgemm_v2(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                              int m, int n, int k, const float *alpha, const float *A, int lda,
                              const float *B, int ldb, const float *beta, float *C, int ldc);

/* replaces cublas.c:254-259. In/out types f32, f16, bf16; fp32 accumulation always (also under
 * CUBLAS_COMPUTE_16F, which reads alpha/beta as half and requires an f16 C, as cuBLAS does). */
cublasStatus_t cublasGemmEx(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                            int m, int n, int k, const void *alpha, const void *A, cudaDataType Atype, int lda,
                            const void *B, cudaDataType Btype, int ldb, const void *beta, void *C,
                            cudaDataType Ctype, int ldc, cublasComputeType_t computeType, cublasGemmAlgo_t algo);

/* replaces cublas.c:261-280. Strides in elements of the respective type; a stride of 0 broadcasts
 * one matrix to the whole batch. One launch for the whole batch. */
cublasStatus_t cublasGemmStridedBatchedEx(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                                          int m, int n, int k, const void *alpha, const void *A, cudaDataType Atype,
                                          int lda, long long int strideA, const void *B, cudaDataType Btype, int ldb,
                                          long long int strideB, const void *beta, void *C, cudaDataType Ctype,
                                          int ldc, long long int strideC, int batchCount,
                                          cublasComputeType_t computeType, cublasGemmAlgo_t algo);

/* replaces cublas.c:308-313 (and its helper `batched`, cublas.c:292-303). The pointer arrays are
 * read ON THE DEVICE by the kernel: no device-to-host copy, no stream synchronisation, one launch. */
cublasStatus_t cublasGemmBatchedEx(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                                   int m, int n, int k, const void *alpha, const void *const Aarray[],
                                   cudaDataType Atype, int lda, const void *const Barray[], cudaDataType Btype,
                                   int ldb, const void *beta, void *const Carray[], cudaDataType Ctype, int ldc,
                                   int batchCount, cublasComputeType_t computeType, cublasGemmAlgo_t algo);

/* replaces cublas.c:289-291 */
cublasStatus_t cublasSgemmStridedBatched(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                                         int m, int n, int k, const float *alpha, const float *A, int lda,
                                         long long int strideA, const float *B, int ldb, long long int strideB,
                                         const float *beta, float *C, int ldc, long long int strideC, int batchCount);

/* replaces cublas.c:304-307 */
cublasStatus_t cublasSgemmBatched(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                                  int m, int n, int k, const float *alpha, const float *const Aarray[], int lda,
                                  const float *const Barray[], int ldb, const float *beta, float *const Carray[],
                                  int ldc, int batchCount);

/* replaces cublas.c:314-333 and the kernel gemm.cu:41-49. X * A = alpha * B in place in B, with A
 * upper-triangular, non-unit, not transposed (the case ggml's solve_tri issues); other cases return
 * NOT_SUPPORTED, as in the reference. Pointer arrays read on the device, one launch. */
cublasStatus_t cublasStrsmBatched(cublasHandle_t handle, cublasSideMode_t side, cublasFillMode_t uplo,
                                  cublasOperation_t trans, cublasDiagType_t diag, int m, int n, const float *alpha,
                                  const float *const A[], int lda, float *const B[], int ldb, int batchCount);

/* ---- library extensions (no cuBLAS counterpart) ------------------------------------------------ */

/* Which kernel family a GEMM of this shape and type goes to on a device with `num_sms` SMs, without
 * launching anything. Mirrors the role of the reference's test hook tinycublas_splitk_plan
 * (cublas.c:69-78): a pure function the host-only tests pin row by row.
 * Returns one of the TB200_KERNEL_* values; *tile_n receives the tensor-core tile width (0 if none) and
 * *pair the tile's mode: 0 one CTA per 128-row tile, 1 the 256-row tile of a CTA pair (2-SM UMMA), 2 and 3
 * the k split of those (two CTAs, or two CTA pairs, per tile, each half with half of the k-blocks; 16-bit
 * strided GEMMs whose tiles leave half of the SMs idle, with at least 1024 in k). */
enum { TB200_KERNEL_NONE = 0, TB200_KERNEL_SIMT = 1, TB200_KERNEL_SKINNY = 2, TB200_KERNEL_TC = 3 };
int tb200_plan(int transa, int transb, int m, int n, int k, int batch, int in_type, int out_type,
               int tf32, int ptr_array, int aligned, int num_sms, int *tile_n, int *pair);

/* Grouped GEMM for mixture-of-experts layers, in one launch: for every group (expert) g,
 *   C[:, offsets[g] : offsets[g+1]] = alpha * op(A_g) * op(B)[:, offsets[g] : offsets[g+1]] + beta * C[same],
 * with A_g = A + g * strideA (elements; 0 shares one A), B holding every group's tokens (columns) one group
 * after another, and C m x n_total. `offsets` is a DEVICE array of groups + 1 non-decreasing column offsets
 * (offsets[0] = 0, offsets[groups] = n_total), so per-expert token counts computed by a router on the GPU
 * need not reach the host, and an expert may get any number of tokens (none included). Types, compute
 * types, alpha/beta and argument rules as cublasGemmStridedBatchedEx (batchCount = groups <= 1024). Runs on
 * the tensor-core kernel only: operands 16-byte aligned with lda, ldb and strideA whole multiples of 16
 * bytes, f32 inputs only in TF32 mode; otherwise CUBLAS_STATUS_NOT_SUPPORTED. No counterpart in the
 * reference, whose only MoE form is cublasGemmBatchedEx with one n for every expert (cublas.c:292-313):
 * a routed layer's experts each get their own number of tokens. */
cublasStatus_t tb200_gemm_grouped_ex(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb, int m,
                                     int n_total, int k, int groups, const int *offsets, const void *alpha,
                                     const void *A, cudaDataType Atype, int lda, long long strideA, const void *B,
                                     cudaDataType Btype, int ldb, const void *beta, void *C, cudaDataType Ctype,
                                     int ldc, cublasComputeType_t computeType);

/* tb200_gemm_grouped_ex with the token gather fused into the GEMM: column j of B is column token_ids[j] of X
 * (k x n_src, ld ldx, op N), where token_ids is a DEVICE array of n_total ids (for a routed layer: each
 * expert's tokens one expert after another, as tb200_moe_gather would lay them out); an id outside
 * [0, n_src) gives a zero column of the product. Same result as tb200_moe_gather into a buffer followed by
 * tb200_gemm_grouped_ex on it, without writing and re-reading that buffer. 16-bit A and X only, operands
 * 16-byte aligned with lda, ldx, strideA multiples of 16 bytes; otherwise CUBLAS_STATUS_NOT_SUPPORTED.
 * n_src < 1 or a NULL token_ids: CUBLAS_STATUS_INVALID_VALUE. It needs no n_total x k buffer for the gathered
 * tokens, but on the B200 it runs slower than the two calls (a routed layer 202 against 175 us): the four-row
 * gather loads move B more slowly than whole tiles of a contiguous copy. No counterpart in the reference. */
cublasStatus_t tb200_gemm_grouped_gather_ex(cublasHandle_t handle, cublasOperation_t transa, int m, int n_total, int k,
                                            int groups, const int *offsets, const int *token_ids, const void *alpha,
                                            const void *A, cudaDataType Atype, int lda, long long strideA,
                                            const void *X, cudaDataType Xtype, int ldx, int n_src, const void *beta,
                                            void *C, cudaDataType Ctype, int ldc, cublasComputeType_t computeType);

/* The data movement of a routed mixture-of-experts layer around tb200_gemm_grouped_ex, on the handle's
 * stream, deterministic, no allocation. tb200_moe_gather: column p of Xp (ld ldxp) = column token_ids[p] of X
 * (k elements of `type`, ld ldx, n_src columns) for p < n_total, which lays out each expert's tokens one
 * expert after another (token_ids device array; an id outside [0, n_src) gives a zero column).
 * tb200_moe_combine: column t of Y (f32, ld ldy) = sum over j < topk, in j order, of
 * weights[t * topk + j] * column positions[t * topk + j] of Cp (f32, ld ldc, n_total columns) for
 * t < n_tokens (device arrays; a position outside [0, n_total) contributes nothing). No counterpart in the
 * reference. */
cublasStatus_t tb200_moe_gather(cublasHandle_t handle, const void *X, cudaDataType type, int k, int ldx, int n_src,
                                const int *token_ids, int n_total, void *Xp, int ldxp);
cublasStatus_t tb200_moe_combine(cublasHandle_t handle, int m, const float *Cp, int ldc, int n_total,
                                 const int *positions, const float *weights, int topk, int n_tokens, float *Y,
                                 int ldy);

/* The persistent tensor-core kernel's tile choice for an m x n x batch GEMM on `num_sms` SMs: returns the
 * tile width (32, 64, 128 or 256) and sets *pair (if not NULL) to 1 for the 256 x 256 tile of a CTA pair.
 * Pure function, pinned by host-only tests. */
int tb200_tc_tile_n(int m, int n, int batch, int num_sms, int *pair);

/* The decode kernel's shape for `blocks` 16-row blocks (m / 16 rounded up, times the batch) and depth k on
 * `num_sms` SMs: warps per CTA, 32-wide chunks of loads each warp keeps in flight, and k slices per block
 * (a cluster of that many CTAs; 1 = no split). Pure function of its arguments and the TB200_SKINNY_CFG /
 * TB200_SKINNY_SPLIT knobs, pinned by host-only tests. Returns 0. */
int tb200_skinny_shape(long long blocks, int k, int num_sms, int *warps, int *unroll, int *slices);

/* cublasGemmBatchedEx for callers that cannot let a library allocate device memory. No counterpart in the
 * reference (its pointer-array path copies the arrays to the host instead).
 *
 * Who needs it: a server that has handed all device memory to its own allocator up front, where a library's
 * cudaMalloc fails or fragments that memory; a latency-critical loop that cannot afford the implicit
 * synchronisation cudaMalloc and cudaFree bring. cublasGemmBatchedEx itself allocates device scratch once per
 * (handle, stream) for pointer arrays on the tensor cores.
 *
 * Same arguments (minus algo), plan and results as cublasGemmBatchedEx; it allocates nothing. Where device
 * scratch is needed it uses one fixed array inside the library (256 KB + 256 B, held by every GPU that loads
 * the library until the process exits), so batchCount is limited to tb200_noalloc_max_batch() (1024):
 * larger batches return CUBLAS_STATUS_INVALID_VALUE with a message on stderr.
 * The first call on a device looks up that array's device address (cudaGetSymbolAddress): make it before
 * any stream capture. All calls share the array and it keeps the last call's contents (each call rewrites the
 * tensor maps it uses and compares the fallback flag with its own call number, so nothing needs clearing):
 * calls whose launches overlap on the GPU - on different streams, or from different threads - race on it;
 * serialise them. */
cublasStatus_t tb200_gemm_batched_ex_noalloc(cublasHandle_t handle, cublasOperation_t transa,
                                             cublasOperation_t transb, int m, int n, int k, const void *alpha,
                                             const void *const Aarray[], cudaDataType Atype, int lda,
                                             const void *const Barray[], cudaDataType Btype, int ldb,
                                             const void *beta, void *const Carray[], cudaDataType Ctype, int ldc,
                                             int batchCount, cublasComputeType_t computeType);

/* The largest batchCount tb200_gemm_batched_ex_noalloc accepts. */
int tb200_noalloc_max_batch(void);

/* Test hook for tb200_gemm_batched_ex_noalloc (no counterpart in the reference): waits for the device and
 * returns 1 when the last such call on the current device found a batch pointer unfit for the tensor cores'
 * TMA loads (not 16-byte aligned; the general kernel then computed the batch), 0 when its tensor-core launch
 * computed it, -1 on error. */
int tb200_noalloc_last_fallback(void);

/* Device scratch allocations this handle has made so far (test hook, the counterpart of the reference's
 * tinycublas_splitk_ws_allocs, cublas.c:91-92). The library allocates scratch only for pointer-array
 * batches on the tensor cores (and for the opt-in balanced decode kernel): one buffer per (handle, stream),
 * made when cublasSetStream selects the stream or at the first such call on it, outside stream capture, and
 * grown when needed; a replaced buffer is kept until Destroy, which frees them all. */
unsigned tb200_scratch_allocs(cublasHandle_t handle);

/* Last error a kernel of this library recorded on the current device (0 = none): a bounded wait in
 * the tensor-core pipeline that gave up (1), or an internal inconsistency (2). Reading it clears it.
 * Synchronises the current device. */
int tb200_device_error(void);

/* Gather the row blocks of an N-sharded GEMM into C: `parts` holds P column-major blocks back to back,
 * block r of size rows x n with leading dimension rows (the NCCL all-gather output); block r lands in
 * rows [r*rows, (r+1)*rows) of C (ldc), and rows at or beyond m_total (the padding of the last block
 * when m is not a multiple of P) are dropped. elem_bytes is 2 or 4. Asynchronous on `stream`. */
cublasStatus_t tb200_gather_row_blocks(const void *parts, int P, int rows, int n, int elem_bytes, void *C,
                                       int ldc, int m_total, cudaStream_t stream);

/* The N-sharded GEMM with its output exchange fused into the epilogue (no reference counterpart: the
 * reference is single-GPU). This rank computes rows [row0, row0 + m_local) of C = alpha * op(A) op(B)
 * (A holds only those rows: m_local x k under op T) and stores them into each of the P replicas of C
 * (C_replicas: a HOST array of P device pointers valid in this process - this GPU's own C and the
 * peers' C mapped with tb200_ipc_open), each m x n with leading dimension ldc >= row0 + m_local.
 * Peers' replicas are written over NVLink by the tensor-core epilogue while later tiles compute.
 * beta is 0 (C is overwritten). Completion on a peer is known only after a cross-GPU synchronisation
 * that follows this launch on every rank (e.g. an NCCL collective on the same stream).
 * Returns NOT_SUPPORTED when the operands do not fit the tensor-core kernel (alignment, types). */
cublasStatus_t tb200_gemm_ex_allgather(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                                       int m_local, int n, int k, const void *alpha, const void *A, cudaDataType Atype,
                                       int lda, const void *B, cudaDataType Btype, int ldb, void *const *C_replicas,
                                       int P, cudaDataType Ctype, int ldc, int row0, cublasComputeType_t computeType);

/* The same N-sharded GEMM with the exchange through NVLink multicast (NVSwitch): C_multicast is the multicast
 * address of a buffer every rank holds (one multicast object bound to all of them); each element of this
 * rank's rows is stored once there and the switch writes it into every rank's C at row offset row0, so a
 * rank sends its own rows once instead of once per peer. f32 C, beta = 0; the caller orders the stores
 * before any rank reads C (a collective after the launch). No counterpart in the reference (single-GPU). */
cublasStatus_t tb200_gemm_ex_multicast(cublasHandle_t handle, cublasOperation_t transa, cublasOperation_t transb,
                                       int m_local, int n, int k, const void *alpha, const void *A, cudaDataType Atype,
                                       int lda, const void *B, cudaDataType Btype, int ldb, void *C_multicast,
                                       cudaDataType Ctype, int ldc, int row0, cublasComputeType_t computeType);

/* Set-up helpers for the replicas (not on the GEMM path): device memory another process of the node can
 * map. tb200_ipc_alloc returns the pointer and writes the 64-byte CUDA IPC handle to `handle`;
 * tb200_ipc_open maps a peer's handle into this process; tb200_ipc_close unmaps it; tb200_ipc_free
 * releases memory from tb200_ipc_alloc. */
cublasStatus_t tb200_ipc_alloc(size_t bytes, void **ptr, void *handle);
cublasStatus_t tb200_ipc_open(const void *handle, void **ptr);
cublasStatus_t tb200_ipc_close(void *ptr);
cublasStatus_t tb200_ipc_free(void *ptr);

/* The exchange step of a sharded GEMM on the copy engines (no counterpart in the reference, which is
 * single-GPU): copies this rank's block of C - rows [row0, row0 + rows) of columns [col0, col0 + ncols) of
 * replicas[self] (elem_bytes per element, leading dimension ldc, column-major) - into the same place of every
 * other replica (peers' C mapped with tb200_ipc_open), one cudaMemcpy2DAsync per peer, issued in ring order
 * from self + 1, peer q's on streams[q % nstreams] (nstreams = 1: one after another, every rank sending to a
 * different peer at each moment). No kernel and no SM time: the copies overlap the GEMMs that run meanwhile on other
 * streams. The caller orders the copies after the GEMM that wrote the block (an event), and every rank's
 * reads of its C after all peers' copies (a collective after the copies' streams). A contiguous batch slab
 * is the case ldc = rows = the slab's length, ncols = 1. */
cublasStatus_t tb200_push_block(void *const *replicas, int P, int self, long long row0, long long rows, long long col0,
                                long long ncols, long long ldc, int elem_bytes, const cudaStream_t *streams,
                                int nstreams);

/* HBM probes, the counterparts of gemm.cu:421-431: stream n4 16-byte writes of v, or n4 16-byte
 * reads folded into *sink. Asynchronous on `stream`. */
cublasStatus_t tb200_bw_write(void *p, long long n4, float v, cudaStream_t stream);
cublasStatus_t tb200_bw_read(const void *p, long long n4, float *sink, cudaStream_t stream);

/* Build identification: "tinycublas_b200 <git describe> sm_100a". */
const char *tb200_version(void);

#ifdef __cplusplus
}
#endif
#endif
