"""tb200_gemm_batched_ex_noalloc: cublasGemmBatchedEx for callers that must not have the library allocate
device memory (a server whose allocator owns all device memory; a loop that cannot take cudaMalloc's
implicit synchronisation). It keeps its scratch in a fixed array inside the library instead of a
per-(handle, stream) cudaMalloc buffer.

Checked through the C ABI on two calls in a row (different inputs and batch sizes, so the second call runs
over the first call's leftovers in the shared array): against the fp64 oracle with the gate of the other
parity tests (oracle.check), and against the existing entry point, cublasGemmBatchedEx, within the same
tolerance. A call whose pointers the tensor cores cannot load (A 2 bytes off a 16-byte boundary, so the
general kernel computes it) is followed by an aligned call, which must be back on the tensor cores. This
file is named to be collected last, so a run that stops at the first failure has run every other test
before it; it also passes alone in a fresh process (its first call performs the library's per-device
set-up).
"""
import ctypes

import numpy as np
import pytest

from macuda_b200 import cublas as cb
from oracle import oracle as O
from tests.helpers import dev, ptr_table, storage

pytestmark = pytest.mark.gpu


def _sms():
    import torch
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def _problem(rng, m, n, k, batch, broadcast_a=1, a_shift=0):
    """Seeded operands of a pointer-array batch; element b's A starts a_shift elements late when b is odd."""
    nA = (batch + broadcast_a - 1) // broadcast_a
    A = storage(rng, nA * m * k + a_shift, O.F16, 0.02)  # element b: op(A) = A_b^T, A_b stored k x m (lda = k)
    B = storage(rng, batch * k * n, O.F16)  # element b: k x n (ldb = k)
    dA, dB = dev(A), dev(B)
    a_off = [(b // broadcast_a) * m * k + (a_shift if b % 2 else 0) for b in range(batch)]
    a_ptrs = ptr_table([dA.data_ptr() + o * 2 for o in a_off])
    b_ptrs = ptr_table([dB.data_ptr() + b * k * n * 2 for b in range(batch)])
    A_list = [A[o:o + m * k] for o in a_off]
    B_list = [B[b * k * n:(b + 1) * k * n] for b in range(batch)]
    return (dA, dB, a_ptrs, b_ptrs), A_list, B_list


def _run(lib, h, fn_name, m, n, k, batch, a_ptrs, b_ptrs):
    """One call through the C ABI into a NaN-poisoned output; returns the host copy of C."""
    import torch
    C = torch.full((batch * m * n,), float("nan"), device="cuda")
    c_ptrs = ptr_table([C.data_ptr() + b * m * n * 4 for b in range(batch)])
    one, zero = ctypes.c_float(1.0), ctypes.c_float(0.0)
    fn = getattr(lib.lib, fn_name)
    args = [h.h, cb.CUBLAS_OP_T, cb.CUBLAS_OP_N, m, n, k, ctypes.byref(one), a_ptrs.data_ptr(), cb.CUDA_R_16F, k,
            b_ptrs.data_ptr(), cb.CUDA_R_16F, k, ctypes.byref(zero), c_ptrs.data_ptr(), cb.CUDA_R_32F, m, batch,
            cb.CUBLAS_COMPUTE_32F]
    if fn_name == "cublasGemmBatchedEx":
        args.append(cb.CUBLAS_GEMM_DEFAULT)  # the no-alloc entry point takes no algo argument
    st = fn(*args)
    torch.cuda.synchronize()
    assert st == cb.CUBLAS_STATUS_SUCCESS, f"{fn_name}: status {st}"
    return C.cpu().numpy()


def _check_against_oracle_and_entry_point(lib, h, m, n, k, batch, bufs, A_list, B_list):
    _, _, a_ptrs, b_ptrs = bufs
    allocs_before = lib.lib.tb200_scratch_allocs(h.h)
    got = _run(lib, h, "tb200_gemm_batched_ex_noalloc", m, n, k, batch, a_ptrs, b_ptrs)
    assert lib.lib.tb200_scratch_allocs(h.h) == allocs_before, "the no-alloc entry point allocated scratch"
    fell_back = lib.lib.tb200_noalloc_last_fallback()
    assert np.isfinite(got).all(), "some element of C was never written"
    rows = np.unique(np.concatenate([np.arange(0, m, 7), [m - 1]])).astype(np.int32)
    R, S = O.gemm(1, 0, m, n, k, 1.0, None, O.F16, k, None, O.F16, k, batch=batch, rows=rows, A_list=A_list,
                  B_list=B_list)
    got_s = O.extract(got, O.F32, m, n, m, sC=m * n, batch=batch, rows=rows)
    res = O.check(got_s, R, S, O.F32)
    assert res["ok"], ("against the oracle", res)
    want = _run(lib, h, "cublasGemmBatchedEx", m, n, k, batch, a_ptrs, b_ptrs)
    res = O.check(got_s, O.extract(want, O.F32, m, n, m, sC=m * n, batch=batch, rows=rows), S, O.F32)
    assert res["ok"], ("against cublasGemmBatchedEx", res)
    return fell_back


def test_noalloc_matches_oracle_and_gemm_batched_ex_on_two_calls(lib):
    import torch
    assert torch.cuda.is_available()
    rng = np.random.default_rng(2024)
    h = lib.handle()
    # two calls in a row on the shared scratch: MoE-expert shape, then a GQA pointer batch with fewer
    # elements (the second call must not see the first one's leftover tensor maps)
    for (m, n, k, batch, bcast) in [(768, 32, 2048, 24, 1), (512, 256, 128, 6, 3)]:
        assert lib.plan(1, 0, m, n, k, batch, 1, 0, 0, 1, 1, _sms())[0] == cb.TB200_KERNEL_TC
        bufs, A_list, B_list = _problem(rng, m, n, k, batch, bcast)
        assert _check_against_oracle_and_entry_point(lib, h, m, n, k, batch, bufs, A_list, B_list) == 0
    h.close()


def test_noalloc_misaligned_call_then_aligned_call(lib):
    """The per-call flag in the shared array: a batch with A pointers 2 bytes off a 16-byte boundary is
    computed by the general kernel, and the aligned call after it goes back to the tensor cores."""
    rng = np.random.default_rng(77)
    h = lib.handle()
    m, n, k, batch = 256, 64, 512, 4
    bufs, A_list, B_list = _problem(rng, m, n, k, batch, a_shift=1)
    assert _check_against_oracle_and_entry_point(lib, h, m, n, k, batch, bufs, A_list, B_list) == 1
    bufs, A_list, B_list = _problem(rng, m, n, k, batch)
    assert _check_against_oracle_and_entry_point(lib, h, m, n, k, batch, bufs, A_list, B_list) == 0
    h.close()


def test_noalloc_rejects_batches_beyond_its_scratch(lib):
    h = lib.handle()
    one = ctypes.c_float(1.0)
    big = lib.lib.tb200_noalloc_max_batch() + 1
    # refused before any device work: the pointer arguments are never read
    st = lib.lib.tb200_gemm_batched_ex_noalloc(h.h, 1, 0, 64, 64, 64, ctypes.byref(one), 256, cb.CUDA_R_16F, 64, 256,
                                               cb.CUDA_R_16F, 64, ctypes.byref(one), 256, cb.CUDA_R_32F, 64, big,
                                               cb.CUBLAS_COMPUTE_32F)
    assert st == cb.CUBLAS_STATUS_INVALID_VALUE
    h.close()
