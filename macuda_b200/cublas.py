"""ctypes binding of the cuBLAS v2 C ABI subset that libtinycublas_b200.so exports.

This is the host-side mirror of the reference's interface for the GEMM path: the same entry points
(cublasCreate/Destroy/SetStream/SetMathMode, cublasGemmEx, cublasSgemm, cublasGemmStridedBatchedEx,
cublasGemmBatchedEx, ...; reference cuda-shim/libtinycublas/cublas.c:242-333), the same argument
meaning and the same status codes. It is what a Python caller (or a test) uses in place of a C
caller such as ggml-cuda (a C caller links -ltinycublas_b200 in place of -lcublas).

`CublasLib(path)` binds any library with that ABI, so the same code drives this library and, in the
tests and the benchmark's reference arm, the reference's own library built from its sources.
Pointers are plain integers (device addresses); alpha/beta are Python numbers converted to the
compute type (half under CUBLAS_COMPUTE_16F*, float otherwise) exactly as cuBLAS reads them.
"""
from __future__ import annotations

import ctypes
import os
import struct

HERE = os.path.dirname(os.path.abspath(__file__))
DEFAULT_LIB = os.path.join(HERE, "libtinycublas_b200.so")

# cudaDataType (library_types.h)
CUDA_R_32F, CUDA_R_16F, CUDA_R_16BF = 0, 2, 14
# cublasOperation_t
CUBLAS_OP_N, CUBLAS_OP_T, CUBLAS_OP_C = 0, 1, 2
# cublasComputeType_t
CUBLAS_COMPUTE_16F, CUBLAS_COMPUTE_16F_PEDANTIC = 64, 65
CUBLAS_COMPUTE_32F, CUBLAS_COMPUTE_32F_PEDANTIC = 68, 69
CUBLAS_COMPUTE_64F, CUBLAS_COMPUTE_64F_PEDANTIC = 70, 71
CUBLAS_COMPUTE_32I, CUBLAS_COMPUTE_32I_PEDANTIC = 72, 73
CUBLAS_COMPUTE_32F_FAST_16F, CUBLAS_COMPUTE_32F_FAST_16BF, CUBLAS_COMPUTE_32F_FAST_TF32 = 74, 75, 77
# cublasMath_t
CUBLAS_DEFAULT_MATH, CUBLAS_TENSOR_OP_MATH, CUBLAS_PEDANTIC_MATH, CUBLAS_TF32_TENSOR_OP_MATH = 0, 1, 2, 3
# cublasStatus_t
CUBLAS_STATUS_SUCCESS = 0
CUBLAS_STATUS_NOT_INITIALIZED = 1
CUBLAS_STATUS_ALLOC_FAILED = 3
CUBLAS_STATUS_INVALID_VALUE = 7
CUBLAS_STATUS_EXECUTION_FAILED = 13
CUBLAS_STATUS_INTERNAL_ERROR = 14
CUBLAS_STATUS_NOT_SUPPORTED = 15
# trsm enums
CUBLAS_SIDE_LEFT, CUBLAS_SIDE_RIGHT = 0, 1
CUBLAS_FILL_MODE_LOWER, CUBLAS_FILL_MODE_UPPER = 0, 1
CUBLAS_DIAG_NON_UNIT, CUBLAS_DIAG_UNIT = 0, 1
CUBLAS_GEMM_DEFAULT = -1

# kernel families reported by tb200_plan
TB200_KERNEL_NONE, TB200_KERNEL_SIMT, TB200_KERNEL_SKINNY, TB200_KERNEL_TC = 0, 1, 2, 3

STATUS_NAMES = {
    0: "CUBLAS_STATUS_SUCCESS", 1: "CUBLAS_STATUS_NOT_INITIALIZED", 3: "CUBLAS_STATUS_ALLOC_FAILED",
    7: "CUBLAS_STATUS_INVALID_VALUE", 13: "CUBLAS_STATUS_EXECUTION_FAILED", 14: "CUBLAS_STATUS_INTERNAL_ERROR",
    15: "CUBLAS_STATUS_NOT_SUPPORTED",
}

# the C declarations this binding needs: (name, restype, argtypes)
_vp, _i, _ll, _sz, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_size_t, ctypes.c_float
SIGNATURES = [
    ("cublasCreate_v2", _i, [ctypes.POINTER(_vp)]),
    ("cublasDestroy_v2", _i, [_vp]),
    ("cublasSetStream_v2", _i, [_vp, _vp]),
    ("cublasSetMathMode", _i, [_vp, _i]),
    ("cublasSetWorkspace_v2", _i, [_vp, _vp, _sz]),
    ("cublasGetStatusString", ctypes.c_char_p, [_i]),
    ("cublasSgemm_v2", _i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _vp, _i, _vp, _vp, _i]),
    ("cublasGemmEx", _i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _vp, _i, _i, _vp, _vp, _i, _i, _i, _i]),
    ("cublasGemmStridedBatchedEx", _i,
     [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _ll, _vp, _i, _i, _ll, _vp, _vp, _i, _i, _ll, _i, _i, _i]),
    ("cublasGemmBatchedEx", _i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _vp, _i, _i, _vp, _vp, _i, _i, _i, _i, _i]),
    ("cublasSgemmStridedBatched", _i,
     [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _ll, _vp, _i, _ll, _vp, _vp, _i, _ll, _i]),
    ("cublasSgemmBatched", _i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _vp, _i, _vp, _vp, _i, _i]),
    ("cublasStrsmBatched", _i, [_vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _i, _vp, _i, _i]),
]
EXTENSIONS = [
    ("tb200_plan", _i, [_i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    ("tb200_tc_tile_n", _i, [_i, _i, _i, _i, ctypes.POINTER(_i)]),
    ("tb200_skinny_shape", _i, [ctypes.c_longlong, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    ("tb200_device_error", _i, []),
    ("tb200_gather_row_blocks", _i, [_vp, _i, _i, _i, _i, _vp, _i, _i, _vp]),
    ("tb200_bw_write", _i, [_vp, _ll, _f, _vp]),
    ("tb200_bw_read", _i, [_vp, _ll, _vp, _vp]),
    ("tb200_version", ctypes.c_char_p, []),
    ("tb200_gemm_ex_allgather", _i,
     [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _vp, _i, _i, _vp, _i, _i, _i, _i, _i]),
    ("tb200_gemm_ex_multicast", _i,
     [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _vp, _i, _i, _vp, _i, _i, _i, _i]),
    ("tb200_ipc_alloc", _i, [_sz, ctypes.POINTER(_vp), _vp]),
    ("tb200_ipc_open", _i, [_vp, ctypes.POINTER(_vp)]),
    ("tb200_ipc_close", _i, [_vp]),
    ("tb200_ipc_free", _i, [_vp]),
    ("tb200_push_block", _i, [_vp, _i, _i, _ll, _ll, _ll, _ll, _ll, _i, _vp, _i]),
    ("tb200_scratch_allocs", ctypes.c_uint, [_vp]),
    ("tb200_gemm_batched_ex_noalloc", _i,
     [_vp, _i, _i, _i, _i, _i, _vp, _vp, _i, _i, _vp, _i, _i, _vp, _vp, _i, _i, _i, _i]),
    ("tb200_noalloc_max_batch", _i, []),
    ("tb200_noalloc_last_fallback", _i, []),
    ("tb200_gemm_grouped_ex", _i,
     [_vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _i, _i, _ll, _vp, _i, _i, _vp, _vp, _i, _i, _i]),
    ("tb200_gemm_grouped_gather_ex", _i,
     [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _i, _i, _ll, _vp, _i, _i, _i, _vp, _vp, _i, _i, _i]),
    ("tb200_moe_gather", _i, [_vp, _vp, _i, _i, _i, _i, _vp, _i, _vp, _i]),
    ("tb200_moe_combine", _i, [_vp, _i, _vp, _i, _i, _vp, _vp, _i, _i, _vp, _i]),
]


class CublasError(RuntimeError):
    def __init__(self, fn: str, status: int):
        super().__init__(f"{fn} returned {STATUS_NAMES.get(status, status)}")
        self.status = status


def half_bits(x: float) -> int:
    """IEEE binary16 bits of x, round to nearest even (struct's 'e' format)."""
    return struct.unpack("<H", struct.pack("<e", float(x)))[0]


def is_c16(compute_type: int) -> bool:
    return compute_type in (CUBLAS_COMPUTE_16F, CUBLAS_COMPUTE_16F_PEDANTIC)


def scalar(x: float, compute_type: int):
    """A host scalar in the compute type, as cuBLAS reads alpha/beta."""
    if is_c16(compute_type):
        return ctypes.c_uint16(half_bits(x))
    return ctypes.c_float(float(x))


class CublasLib:
    """A loaded library with the cuBLAS v2 subset ABI (this one, or the reference's)."""

    def __init__(self, path: str = DEFAULT_LIB, extensions: bool = True):
        if not os.path.exists(path):
            raise RuntimeError(
                f"{path} is missing: build it with `python -m macuda_b200.build` (nvcc, sm_100a). "
                "There is no CPU fallback for this library.")
        self.path = path
        self.lib = ctypes.CDLL(path, mode=os.RTLD_LOCAL | os.RTLD_NOW)
        for name, res, args in SIGNATURES + (EXTENSIONS if extensions else []):
            fn = getattr(self.lib, name)
            fn.restype = res
            fn.argtypes = args

    def handle(self) -> "Handle":
        return Handle(self)

    def version(self) -> str:
        return self.lib.tb200_version().decode()

    def plan(self, transa, transb, m, n, k, batch=1, in_type=1, out_type=0, tf32=0, ptr_array=0, aligned=1,
             num_sms=148):
        """(kernel family, tile width) - a CTA-pair tile is reported as 256 + its width (512 for 256 x 256,
        384 for 256 x 128); a k-split tile as minus that (two CTAs on a 128-row tile: -BN; two CTA pairs
        on a 256 x 256 tile: -512)"""
        tn, pr = ctypes.c_int(0), ctypes.c_int(0)
        kind = self.lib.tb200_plan(transa, transb, m, n, k, batch, in_type, out_type, tf32, ptr_array, aligned,
                                   num_sms, ctypes.byref(tn), ctypes.byref(pr))
        w = 256 + tn.value if pr.value in (1, 3) else tn.value
        return kind, (-w if pr.value >= 2 else w)

    def skinny_shape(self, m, k, batch=1, num_sms=148):
        """the decode kernel's (warps per CTA, chunks in flight per warp, k slices) for an m x n x k GEMM, n <= 8"""
        w, u, sl = ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int(0)
        self.lib.tb200_skinny_shape((m + 15) // 16 * batch, k, num_sms, ctypes.byref(w), ctypes.byref(u),
                                    ctypes.byref(sl))
        return w.value, u.value, sl.value

    def device_error(self) -> int:
        return self.lib.tb200_device_error()


class Handle:
    """cublasHandle_t with the entry points as methods; each returns the cublasStatus_t."""

    def __init__(self, lib: CublasLib):
        self._lib = lib
        self.lib = lib.lib
        self.h = ctypes.c_void_p()
        st = self.lib.cublasCreate_v2(ctypes.byref(self.h))
        if st != CUBLAS_STATUS_SUCCESS and not self.h:
            raise CublasError("cublasCreate_v2", st)
        self.create_status = st

    def close(self):
        if self.h:
            self.lib.cublasDestroy_v2(self.h)
            self.h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_stream(self, stream: int | None) -> int:
        return self.lib.cublasSetStream_v2(self.h, stream or None)

    def set_math_mode(self, mode: int) -> int:
        return self.lib.cublasSetMathMode(self.h, mode)

    def sgemm(self, ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
        a, b = ctypes.c_float(alpha), ctypes.c_float(beta)
        return self.lib.cublasSgemm_v2(self.h, ta, tb, m, n, k, ctypes.byref(a), A, lda, B, ldb, ctypes.byref(b), C, ldc)

    def gemm_ex(self, ta, tb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C, Ctype, ldc,
                compute_type=CUBLAS_COMPUTE_32F, algo=CUBLAS_GEMM_DEFAULT) -> int:
        a, b = scalar(alpha, compute_type), scalar(beta, compute_type)
        return self.lib.cublasGemmEx(self.h, ta, tb, m, n, k, ctypes.byref(a), A, Atype, lda, B, Btype, ldb,
                                     ctypes.byref(b), C, Ctype, ldc, compute_type, algo)

    def gemm_strided_batched_ex(self, ta, tb, m, n, k, alpha, A, Atype, lda, sA, B, Btype, ldb, sB, beta, C, Ctype,
                                ldc, sC, batch, compute_type=CUBLAS_COMPUTE_32F, algo=CUBLAS_GEMM_DEFAULT) -> int:
        a, b = scalar(alpha, compute_type), scalar(beta, compute_type)
        return self.lib.cublasGemmStridedBatchedEx(self.h, ta, tb, m, n, k, ctypes.byref(a), A, Atype, lda, sA, B,
                                                   Btype, ldb, sB, ctypes.byref(b), C, Ctype, ldc, sC, batch,
                                                   compute_type, algo)

    def gemm_grouped_ex(self, ta, tb, m, n_total, k, groups, offsets, alpha, A, Atype, lda, strideA, B, Btype, ldb,
                        beta, C, Ctype, ldc, compute_type=CUBLAS_COMPUTE_32F) -> int:
        """tb200_gemm_grouped_ex: offsets is a device pointer to groups + 1 int32 column offsets"""
        a, b = scalar(alpha, compute_type), scalar(beta, compute_type)
        return self.lib.tb200_gemm_grouped_ex(self.h, ta, tb, m, n_total, k, groups, offsets, ctypes.byref(a), A,
                                              Atype, lda, strideA, B, Btype, ldb, ctypes.byref(b), C, Ctype, ldc,
                                              compute_type)

    def gemm_grouped_gather_ex(self, ta, m, n_total, k, groups, offsets, token_ids, alpha, A, Atype, lda, strideA, X,
                               Xtype, ldx, n_src, beta, C, Ctype, ldc, compute_type=CUBLAS_COMPUTE_32F) -> int:
        """tb200_gemm_grouped_gather_ex: offsets (groups + 1) and token_ids (n_total) are device int32 arrays"""
        a, b = scalar(alpha, compute_type), scalar(beta, compute_type)
        return self.lib.tb200_gemm_grouped_gather_ex(self.h, ta, m, n_total, k, groups, offsets, token_ids,
                                                     ctypes.byref(a), A, Atype, lda, strideA, X, Xtype, ldx, n_src,
                                                     ctypes.byref(b), C, Ctype, ldc, compute_type)

    def gemm_batched_ex(self, ta, tb, m, n, k, alpha, Aarr, Atype, lda, Barr, Btype, ldb, beta, Carr, Ctype, ldc,
                        batch, compute_type=CUBLAS_COMPUTE_32F, algo=CUBLAS_GEMM_DEFAULT) -> int:
        a, b = scalar(alpha, compute_type), scalar(beta, compute_type)
        return self.lib.cublasGemmBatchedEx(self.h, ta, tb, m, n, k, ctypes.byref(a), Aarr, Atype, lda, Barr, Btype,
                                            ldb, ctypes.byref(b), Carr, Ctype, ldc, batch, compute_type, algo)

    def sgemm_strided_batched(self, ta, tb, m, n, k, alpha, A, lda, sA, B, ldb, sB, beta, C, ldc, sC, batch) -> int:
        a, b = ctypes.c_float(alpha), ctypes.c_float(beta)
        return self.lib.cublasSgemmStridedBatched(self.h, ta, tb, m, n, k, ctypes.byref(a), A, lda, sA, B, ldb, sB,
                                                  ctypes.byref(b), C, ldc, sC, batch)

    def sgemm_batched(self, ta, tb, m, n, k, alpha, Aarr, lda, Barr, ldb, beta, Carr, ldc, batch) -> int:
        a, b = ctypes.c_float(alpha), ctypes.c_float(beta)
        return self.lib.cublasSgemmBatched(self.h, ta, tb, m, n, k, ctypes.byref(a), Aarr, lda, Barr, ldb,
                                           ctypes.byref(b), Carr, ldc, batch)

    def strsm_batched(self, side, uplo, trans, diag, m, n, alpha, Aarr, lda, Barr, ldb, batch) -> int:
        a = ctypes.c_float(alpha)
        return self.lib.cublasStrsmBatched(self.h, side, uplo, trans, diag, m, n, ctypes.byref(a), Aarr, lda, Barr,
                                           ldb, batch)


def check(fn: str, status: int) -> None:
    if status != CUBLAS_STATUS_SUCCESS:
        raise CublasError(fn, status)


_default: CublasLib | None = None


def library() -> CublasLib:
    """The process-wide instance of this library (loaded on first use; raises if it is not built)."""
    global _default
    if _default is None:
        _default = CublasLib(DEFAULT_LIB)
    return _default
