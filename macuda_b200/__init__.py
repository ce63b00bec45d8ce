"""macuda_b200 - libtinycublas_b200: the cuBLAS GEMM subset ggml-cuda calls, written for B200 (sm_100a).

The product is the shared library macuda_b200/libtinycublas_b200.so (C ABI, declared in
include/tinycublas_b200.h). This package holds its sources (csrc/), its build recipe (build.py), a
ctypes binding of the ABI (cublas.py) and the multi-GPU N-sharded GEMM (dist.py).
"""
from .cublas import (CublasLib, CublasError, Handle, check, library, DEFAULT_LIB,  # noqa: F401
                     CUDA_R_32F, CUDA_R_16F, CUDA_R_16BF, CUBLAS_OP_N, CUBLAS_OP_T,
                     CUBLAS_COMPUTE_16F, CUBLAS_COMPUTE_32F, CUBLAS_COMPUTE_32F_FAST_TF32,
                     CUBLAS_STATUS_SUCCESS, CUBLAS_STATUS_NOT_SUPPORTED, CUBLAS_STATUS_INVALID_VALUE)

__all__ = ["CublasLib", "CublasError", "Handle", "check", "library", "DEFAULT_LIB"]
