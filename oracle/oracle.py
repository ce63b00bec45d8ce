"""TEST INFRASTRUCTURE: Python access to the CPU oracle (liboracle.so) and the reference arm.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline and reference legs import this
module. It is the checker, never the thing measured or shipped.

  gemm(...)            fp64 GEMM with cuBLAS semantics (gemm_oracle.c: orc_gemm), optionally on a
                       sample of rows and columns, returning the result and the per-element scale
                       |alpha| |op(A)_i| |op(B)_j| + |beta| |C0_ij| of the normalised error gate.
  check(...)           the gate: max |C - R| / scale <= 2^-10 (plus the output type's own rounding),
                       with non-finite outputs refused first, and the reference's own metric
                       max |C - R| / max |R| (cuda-shim/libtinycublas/bf16-20260921/
                       bench_gemm_contract.cu:44-49) reported beside it.
  ref_splitk_plan, ref_contract     the reference's host decisions restated (cublas.c:69-78, :118-134).
  cpu_gemm_f16_tn      the timed CPU baseline (stand-in for ggml-cpu's fp16 matmul).
  reference_library()  the reference's own libtinycublas, built from its sources by build_ref.sh.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libtinycublas_ref.so")

F32, F16, BF16 = 0, 1, 2
TOL = 2.0 ** -10
OUT_ROUND = {F32: 0.0, F16: 2.0 ** -11, BF16: 2.0 ** -8}
# the reference's own gate (bench_gemm_contract.cu:8-10, test_splitk.cu:8-9)
REF_METRIC_TOL = {F32: 2e-3, F16: 1e-2, BF16: 1e-2}

_lib = None


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB):
        subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True, capture_output=True)
    lib = ctypes.CDLL(LIB)
    vp, i, ll, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_double
    lib.orc_gemm.argtypes = [i, i, i, i, i, d, vp, vp, i, i, ll, vp, vp, i, i, ll, d, vp, vp, i, i, ll, i, vp, i, vp,
                             i, vp, vp]
    lib.orc_gemm.restype = None
    for name in ("orc_f32_to_f16", "orc_f32_to_bf16", "orc_f16_to_f32", "orc_bf16_to_f32"):
        getattr(lib, name).argtypes = [vp, vp, ll]
        getattr(lib, name).restype = None
    lib.orc_ref_splitk_plan.argtypes = [i, i, i, i, i]
    lib.orc_ref_splitk_plan.restype = i
    lib.orc_ref_contract.argtypes = [i, i, i, i]
    lib.orc_ref_contract.restype = i
    lib.orc_cpu_gemm_f16_tn.argtypes = [i, i, i, vp, i, vp, i, vp, i, i]
    lib.orc_cpu_gemm_f16_tn.restype = None
    lib.orc_trsm_rupn.argtypes = [vp, vp, i, i, i, i, d, vp]
    lib.orc_trsm_rupn.restype = None
    lib.orc_max_threads.restype = i
    lib.orc_half_bits_to_float.argtypes = [ctypes.c_uint16]
    lib.orc_half_bits_to_float.restype = ctypes.c_float
    lib.orc_float_to_half_bits.argtypes = [ctypes.c_float]
    lib.orc_float_to_half_bits.restype = ctypes.c_uint16
    _lib = lib
    return lib


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ---- conversions (round to nearest even) ----
def to_bits(x: np.ndarray, t: int) -> np.ndarray:
    """float32 array -> storage array of type t (float32 itself, or uint16 bit patterns)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if t == F32:
        return x
    out = np.empty(x.shape, dtype=np.uint16)
    fn = _load().orc_f32_to_f16 if t == F16 else _load().orc_f32_to_bf16
    fn(_ptr(x), _ptr(out), x.size)
    return out


def from_bits(b: np.ndarray, t: int) -> np.ndarray:
    """storage array of type t -> float32"""
    if t == F32:
        return np.asarray(b, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    out = np.empty(b.shape, dtype=np.float32)
    fn = _load().orc_f16_to_f32 if t == F16 else _load().orc_bf16_to_f32
    fn(_ptr(b), _ptr(out), b.size)
    return out


def _as_storage(a: np.ndarray, t: int) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if t == F32:
        assert a.dtype == np.float32
    else:
        assert a.dtype == np.uint16
    return a


def gemm(opA, opB, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta=0.0, C0=None, Ctype=F32, ldc=None, sA=0, sB=0,
         sC=0, batch=1, rows=None, cols=None, A_list=None, B_list=None, C_list=None):
    """fp64 reference. A/B/C0 are flat storage arrays (float32 or uint16 bits); with A_list/B_list/C_list
    (lists of such arrays, one per batch element) the pointer-array form is used. Returns (R, S) of
    shape [batch, ncols, nrows] (column-major per batch element, like C)."""
    lib = _load()
    ldc = ldc if ldc is not None else m
    r = None if rows is None else np.ascontiguousarray(rows, dtype=np.int32)
    c = None if cols is None else np.ascontiguousarray(cols, dtype=np.int32)
    nr = m if r is None else len(r)
    nc = n if c is None else len(c)
    R = np.empty((batch, nc, nr), dtype=np.float64)
    S = np.empty((batch, nc, nr), dtype=np.float64)
    keep = []

    def table(lst, t):
        if lst is None:
            return None
        arrs = [_as_storage(x, t) for x in lst]
        keep.extend(arrs)
        tab = (ctypes.c_void_p * len(arrs))(*[x.ctypes.data for x in arrs])
        keep.append(tab)
        return ctypes.cast(tab, ctypes.c_void_p)

    Ap, Bp, Cp = table(A_list, Atype), table(B_list, Btype), table(C_list, Ctype)
    A = None if A is None else _as_storage(A, Atype)
    B = None if B is None else _as_storage(B, Btype)
    C0 = None if C0 is None else _as_storage(C0, Ctype)
    lib.orc_gemm(opA, opB, m, n, k, float(alpha), _ptr(A), Ap, Atype, lda, sA, _ptr(B), Bp, Btype, ldb, sB,
                 float(beta), _ptr(C0), Cp, Ctype, ldc, sC, batch, _ptr(r), nr, _ptr(c), nc, _ptr(R), _ptr(S))
    return R, S


def extract(C: np.ndarray, Ctype: int, m: int, n: int, ldc: int, sC: int = 0, batch: int = 1, rows=None, cols=None):
    """Pull the m x n (or sampled) block of each batch element out of a flat C storage array, as fp64
    in the oracle's [batch, ncols, nrows] layout."""
    Cf = from_bits(C, Ctype).astype(np.float64)
    r = np.arange(m) if rows is None else np.asarray(rows)
    c = np.arange(n) if cols is None else np.asarray(cols)
    out = np.empty((batch, len(c), len(r)))
    for b in range(batch):
        base = b * sC
        idx = base + r[None, :] + c[:, None] * ldc
        out[b] = Cf[idx]
    return out


def check(got: np.ndarray, R: np.ndarray, S: np.ndarray, out_type: int, tol: float = TOL) -> dict:
    """The parity gate. got/R/S share the oracle's layout."""
    nonfinite = int(np.count_nonzero(~np.isfinite(got)))
    res = {"nonfinite": nonfinite, "tol": tol}
    if nonfinite:
        res.update(ok=False, norm_err=float("inf"), ref_metric=float("inf"))
        return res
    diff = np.abs(got - R)
    allowance = OUT_ROUND[out_type] * np.abs(R) + (2.0 ** -24 if out_type == F16 else 0.0)
    scale = np.maximum(S, 1e-300)
    norm = np.max(np.maximum(diff - allowance, 0.0) / scale) if diff.size else 0.0
    maxref = np.max(np.abs(R)) if R.size else 0.0
    ref_metric = float(np.max(diff) / maxref) if maxref > 0 else float(np.max(diff) if diff.size else 0.0)
    res.update(norm_err=float(norm), ref_metric=ref_metric,
               ok=bool(norm <= tol and ref_metric <= REF_METRIC_TOL[out_type]))
    return res


def ref_splitk_plan(m, n, k, batch, num_sms=170) -> int:
    return _load().orc_ref_splitk_plan(m, n, k, batch, num_sms)


def ref_contract(At, Bt, Ct, ct) -> int:
    return _load().orc_ref_contract(At, Bt, Ct, ct)


def trsm_rupn(A: np.ndarray, B: np.ndarray, rows: int, n: int, lda: int, ldb: int, alpha: float) -> np.ndarray:
    X = np.empty(rows * n, dtype=np.float64)
    _load().orc_trsm_rupn(_ptr(np.ascontiguousarray(A, np.float32)), _ptr(np.ascontiguousarray(B, np.float32)), rows,
                          n, lda, ldb, float(alpha), _ptr(X))
    return X


def cpu_gemm_f16_tn(m, n, k, A_bits: np.ndarray, lda: int, B_bits: np.ndarray, ldb: int, C: np.ndarray, ldc: int,
                    threads: int = 0) -> None:
    _load().orc_cpu_gemm_f16_tn(m, n, k, _ptr(A_bits), lda, _ptr(B_bits), ldb, _ptr(C), ldc, threads)


def max_threads() -> int:
    return _load().orc_max_threads()


def reference_library():
    """The reference's own libtinycublas (cublas.c + gemm.cu built for sm_100a), bound through the
    same ctypes binding as this library; None when it was not built."""
    if not os.path.exists(REF_LIB):
        return None
    from macuda_b200.cublas import CublasLib
    lib = CublasLib(REF_LIB, extensions=False)
    lib.lib.tinycublas_splitk_plan.argtypes = [ctypes.c_int] * 4
    lib.lib.tinycublas_splitk_plan.restype = ctypes.c_int
    lib.lib.tinycublas_ref_provenance.restype = ctypes.c_char_p
    return lib
