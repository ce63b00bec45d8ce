"""Shared helpers for the GPU parity tests: seeded inputs, device copies (torch as plumbing only),
and one call that runs a GEMM through the C ABI and checks it against the fp64 oracle."""
from __future__ import annotations

import numpy as np

from macuda_b200 import cublas as cb
from oracle import oracle as O

CUDA_TYPE = {O.F32: cb.CUDA_R_32F, O.F16: cb.CUDA_R_16F, O.BF16: cb.CUDA_R_16BF}


def storage(rng, count: int, t: int, sigma: float = 1.0) -> np.ndarray:
    """count values N(0, sigma^2), rounded to type t (float32 array, or uint16 bit patterns). Drawn in
    float32 (BASELINE-size operands hold up to 525M values)."""
    x = rng.standard_normal(count, dtype=np.float32)
    if sigma != 1.0:
        x *= np.float32(sigma)
    return O.to_bits(x, t)


def dev(a: np.ndarray):
    import torch
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).cuda()
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t, like: np.ndarray) -> np.ndarray:
    a = t.cpu().numpy()
    return a.view(np.uint16) if like.dtype == np.uint16 else a


def ptr_table(ptrs):
    import torch
    return torch.tensor(list(ptrs), dtype=torch.int64, device="cuda")


def sample_idx(rng, size: int, cap: int, extra=()):
    """all indices when small, else a seeded sample that always includes both ends and `extra`"""
    if size <= cap:
        return None
    extra = [int(e) for e in extra if 0 <= int(e) < size]
    idx = np.unique(np.concatenate([[0, size - 1], extra, rng.choice(size, cap - 2, replace=False)]))
    return idx.astype(np.int32)


def tile_edges(size: int, tiles=(32, 64, 128, 256)):
    """indices on both sides of the last boundary of every tile width: the first and last row (or column) of
    each width's last, possibly partial, tile and the one before it"""
    out = set()
    for t in tiles:
        last = (size - 1) // t * t
        out.update({last - 1, last, min(size - 1, last + t - 1), last - t})
    return sorted(i for i in out if 0 <= i < size)


def run_and_check(lib, h, *, opA=1, opB=0, m, n, k, in_t=O.F16, out_t=O.F32, alpha=1.0, beta=0.0, batch=1,
                  lda=None, ldb=None, ldc=None, sA=None, sB=None, sC=None, mode="strided", seed=0,
                  compute=cb.CUBLAS_COMPUTE_32F, a_sigma=0.02, sample=256, c_offset=0, broadcast_a=1, a_ptr_shift=0,
                  edges=False):
    """Build seeded operands, run one GEMM through the library's C ABI, check it against the oracle.
    mode: 'ex' (cublasGemmEx, batch 1), 'strided' (cublasGemmStridedBatchedEx), 'ptr' (cublasGemmBatchedEx,
    A pointers repeated `broadcast_a` times, as for GQA). Large shapes are checked on seeded row/column samples
    (`sample` of each); edges=True adds the rows and columns around the last boundary of every tile width.
    Returns the check dict (plus the status)."""
    import torch
    rng = np.random.default_rng(seed)
    a_rows, a_cols = (m, k) if opA == 0 else (k, m)
    b_rows, b_cols = (k, n) if opB == 0 else (n, k)
    lda = lda or max(1, a_rows)
    ldb = ldb or max(1, b_rows)
    ldc = ldc or max(1, m)
    sA = sA if sA is not None else lda * a_cols
    sB = sB if sB is not None else ldb * b_cols
    sC = sC if sC is not None else ldc * n
    nA = batch if mode != "ptr" else (batch + broadcast_a - 1) // broadcast_a
    A = storage(rng, max(1, sA * (nA - 1) + lda * a_cols + a_ptr_shift), in_t, a_sigma)
    B = storage(rng, max(1, sB * (batch - 1) + ldb * b_cols), in_t, 1.0)
    C0 = storage(rng, sC * (batch - 1) + ldc * n + c_offset, out_t, 1.0)
    dA, dB, dC = dev(A), dev(B), dev(C0)
    esA = 4 if in_t == O.F32 else 2
    esC = 4 if out_t == O.F32 else 2
    cbase = dC.data_ptr() + c_offset * esC
    ct_in, ct_out = CUDA_TYPE[in_t], CUDA_TYPE[out_t]
    if mode == "ex":
        assert batch == 1
        st = h.gemm_ex(opA, opB, m, n, k, alpha, dA.data_ptr(), ct_in, lda, dB.data_ptr(), ct_in, ldb, beta, cbase,
                       ct_out, ldc, compute)
    elif mode == "strided":
        st = h.gemm_strided_batched_ex(opA, opB, m, n, k, alpha, dA.data_ptr(), ct_in, lda, sA, dB.data_ptr(), ct_in,
                                       ldb, sB, beta, cbase, ct_out, ldc, sC, batch, compute)
    else:
        # a_ptr_shift: odd batch elements' A starts that many elements later (breaks 16-byte alignment)
        a_off = [(b // broadcast_a) * sA + (a_ptr_shift if b % 2 else 0) for b in range(batch)]
        a_ptrs = [dA.data_ptr() + o * esA for o in a_off]
        b_ptrs = [dB.data_ptr() + b * sB * esA for b in range(batch)]
        c_ptrs = [cbase + b * sC * esC for b in range(batch)]
        tA, tB, tC = ptr_table(a_ptrs), ptr_table(b_ptrs), ptr_table(c_ptrs)
        st = h.gemm_batched_ex(opA, opB, m, n, k, alpha, tA.data_ptr(), ct_in, lda, tB.data_ptr(), ct_in, ldb, beta,
                               tC.data_ptr(), ct_out, ldc, batch, compute)
    torch.cuda.synchronize()
    if st != 0:
        return {"ok": False, "status": st}
    got_all = host(dC, C0)[c_offset:]
    rows = sample_idx(rng, m, sample, tile_edges(m) if edges else ())
    cols = sample_idx(rng, n, sample, tile_edges(n) if edges else ())
    C0v = C0[c_offset:]
    if mode == "ptr":
        A_list = [A[o:o + lda * a_cols] for o in a_off]
        B_list = [B[b * sB:b * sB + ldb * b_cols] for b in range(batch)]
        C_list = [C0v[b * sC:b * sC + ldc * n] for b in range(batch)]
        R, S = O.gemm(opA, opB, m, n, k, alpha, None, in_t, lda, None, in_t, ldb, beta, None, out_t, ldc, batch=batch,
                      rows=rows, cols=cols, A_list=A_list, B_list=B_list, C_list=C_list)
    else:
        R, S = O.gemm(opA, opB, m, n, k, alpha, A, in_t, lda, B, in_t, ldb, beta, C0v, out_t, ldc, sA, sB, sC, batch,
                      rows=rows, cols=cols)
    got = O.extract(got_all, out_t, m, n, ldc, sC, batch, rows, cols)
    res = O.check(got, R, S, out_t)
    res["status"] = st
    # memory outside the m x n blocks must be untouched (ldc > m padding, the space before C's base)
    if c_offset:
        res["ok"] = res["ok"] and np.array_equal(host(dC, C0)[:c_offset], C0[:c_offset])
    if ldc > m:
        pad = np.ones(len(C0v), dtype=bool)
        for b in range(batch):
            for j in range(n):
                pad[b * sC + j * ldc:b * sC + j * ldc + m] = False
        res["pad_ok"] = bool(np.array_equal(got_all[pad], C0v[pad]))
        res["ok"] = res["ok"] and res["pad_ok"]
    return res
