"""The oracle pinned before it is trusted (CPU only).

Pins: the reference's own host-test rows (contract, split-K plan), the reference's known-answer
GEMMs, the reference library's own plan function called directly, and numpy's IEEE conversions.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    with open(os.path.join(GOLD, name)) as f:
        return json.load(f)


def test_half_conversion_matches_numpy():
    rng = np.random.default_rng(1)
    x = np.concatenate([
        rng.normal(0, 1, 20000), rng.normal(0, 1e-5, 5000), rng.normal(0, 3e4, 5000),
        [0.0, -0.0, 65504.0, 65519.99, 65520.0, 1e9, -1e9, 2.0 ** -24, 2.0 ** -25, 2.0 ** -25 * 1.0001, 5.96e-8, 6.1e-5],
    ]).astype(np.float32)
    got = O.to_bits(x, O.F16)
    want = x.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, want)
    back = O.from_bits(got, O.F16)
    assert np.array_equal(back, want.view(np.float16).astype(np.float32))
    # every one of the 2^16 patterns decodes like numpy (NaNs compared as NaN)
    allbits = np.arange(65536, dtype=np.uint16)
    dec = O.from_bits(allbits, O.F16)
    ref = allbits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(dec), nan) and np.array_equal(dec[~nan], ref[~nan])


def test_bf16_conversion_round_to_nearest_even():
    rng = np.random.default_rng(2)
    x = rng.normal(0, 1, 50000).astype(np.float32)
    got = O.to_bits(x, O.BF16)
    u = x.view(np.uint32).astype(np.uint64)
    want = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)  # RNE on the top 16 bits
    assert np.array_equal(got, want)
    assert np.array_equal(O.from_bits(got, O.BF16), (got.astype(np.uint32) << 16).view(np.float32))


@pytest.mark.parametrize("row", load("reference_rows.json")["splitk_plan"]["rows"], ids=lambda r: r[0])
def test_oracle_plan_matches_reference_rows(row):
    what, m, n, k, batch, want = row
    assert O.ref_splitk_plan(m, n, k, batch, 170) == want, what


def test_reference_library_plan_function_matches_oracle():
    """The reference's own tinycublas_splitk_plan (built from cublas.c) is a pure host function:
    call it directly and compare with the restatement over a sweep of shapes."""
    ref = O.reference_library()
    if ref is None:
        pytest.skip("oracle/_ref not built (needs the reference tree; built by __graft_entry__.build)")
    rng = np.random.default_rng(3)
    shapes = [(int(m), int(n), int(k), int(b)) for m, n, k, b in
              zip(rng.integers(1, 20000, 400), rng.integers(1, 130, 400), rng.integers(1, 20000, 400),
                  rng.integers(1, 5, 400))]
    for row in load("reference_rows.json")["splitk_plan"]["rows"]:
        shapes.append(tuple(row[1:5]))
    for m, n, k, b in shapes:
        assert ref.lib.tinycublas_splitk_plan(m, n, k, b) == O.ref_splitk_plan(m, n, k, b, 170), (m, n, k, b)


@pytest.mark.parametrize("row", load("reference_rows.json")["contract"]["rows"], ids=lambda r: r[0])
def test_oracle_contract_matches_reference_rows(row):
    what, At, Bt, Ct, ct, want = row
    got = O.ref_contract(At, Bt, Ct, ct)
    assert (got == 0) == (want == 0), what


def test_known_answer_sgemm48_exact():
    ka = load("known_answers.json")["sgemm48"]
    A = np.array(ka["A"], dtype=np.float32)
    B = np.array(ka["B"], dtype=np.float32)
    R, S = O.gemm(0, 0, 48, 48, 48, 1.0, A, O.F32, 48, B, O.F32, 48)
    assert np.array_equal(R[0].reshape(-1), np.array(ka["C"], dtype=np.float64))


def test_known_answer_f16_4x4():
    ka = load("known_answers.json")["gemm16_4x4"]
    A = O.to_bits(np.array(ka["A"], np.float32), O.F16)
    B = O.to_bits(np.array(ka["B"], np.float32), O.F16)
    R, S = O.gemm(0, 0, 4, 4, 4, 1.0, A, O.F16, 4, B, O.F16, 4, Ctype=O.F16)
    assert np.array_equal(R[0].reshape(-1), np.array(ka["C"], dtype=np.float64))


def test_oracle_transposes_batch_and_sampling_against_numpy():
    rng = np.random.default_rng(4)
    m, n, k, batch = 37, 29, 53, 3
    for opA in (0, 1):
        for opB in (0, 1):
            lda = (m if opA == 0 else k) + 3
            ldb = (k if opB == 0 else n) + 1
            ldc = m + 2
            acols = k if opA == 0 else m
            bcols = n if opB == 0 else k
            sA, sB, sC = lda * acols + 5, ldb * bcols, ldc * n + 7
            A = rng.normal(size=sA * batch).astype(np.float32)
            B = rng.normal(size=sB * batch).astype(np.float32)
            C0 = rng.normal(size=sC * batch).astype(np.float32)
            R, S = O.gemm(opA, opB, m, n, k, 0.5, A, O.F32, lda, B, O.F32, ldb, 2.0, C0, O.F32, ldc, sA, sB, sC, batch)
            for b in range(batch):
                Am = A[b * sA:b * sA + lda * acols].reshape(acols, lda).T[:(m if opA == 0 else k)].astype(np.float64)
                Bm = B[b * sB:b * sB + ldb * bcols].reshape(bcols, ldb).T[:(k if opB == 0 else n)].astype(np.float64)
                opa = Am if opA == 0 else Am.T
                opb = Bm if opB == 0 else Bm.T
                Cm = C0[b * sC:b * sC + ldc * n].reshape(n, ldc).T[:m].astype(np.float64)
                want = 0.5 * opa @ opb + 2.0 * Cm
                assert np.allclose(R[b].T, want, rtol=1e-12, atol=1e-12)
            rows, cols = [0, 5, 36], [28, 3]
            Rs, _ = O.gemm(opA, opB, m, n, k, 0.5, A, O.F32, lda, B, O.F32, ldb, 2.0, C0, O.F32, ldc, sA, sB, sC,
                           batch, rows=rows, cols=cols)
            assert np.array_equal(Rs, R[:, cols][:, :, rows])


def test_check_refuses_nonfinite_and_mutants():
    """The gate must see a NaN, a 5% alpha error (the reference's matrix-control mutant) and a dropped
    k-slice (its drop_slice mutant); and must pass the exact answer."""
    rng = np.random.default_rng(5)
    m, n, k = 64, 16, 256
    A = O.to_bits(rng.normal(0, 0.02, m * k).astype(np.float32), O.F16)
    B = O.to_bits(rng.normal(0, 1, k * n).astype(np.float32), O.F16)
    R, S = O.gemm(1, 0, m, n, k, 1.0, A, O.F16, k, B, O.F16, k)
    assert O.check(R.copy(), R, S, O.F32)["ok"]
    bad = R.copy()
    bad[0, 3, 7] = np.nan
    assert not O.check(bad, R, S, O.F32)["ok"]
    assert not O.check(R * 1.05, R, S, O.F32)["ok"]
    Rpart, _ = O.gemm(1, 0, m, n, k - 32, 1.0, A, O.F16, k, B, O.F16, k)  # last 32 k dropped
    assert not O.check(Rpart, R, S, O.F32)["ok"]


def test_trsm_oracle_solves():
    rng = np.random.default_rng(6)
    rows, n = 7, 5
    A = np.triu(rng.normal(size=(n, n))) + 3 * np.eye(n)
    B = rng.normal(size=(rows, n))
    X = O.trsm_rupn(A.T.reshape(-1).astype(np.float32), B.T.reshape(-1).astype(np.float32), rows, n, n, rows, 0.5)
    Xm = X.reshape(n, rows).T
    assert np.allclose(Xm @ A.astype(np.float32).astype(np.float64), 0.5 * B.astype(np.float32), atol=1e-5)


def test_cpu_baseline_gemm_matches_oracle():
    rng = np.random.default_rng(7)
    m, n, k = 70, 13, 300
    A = O.to_bits(rng.normal(0, 0.02, m * k).astype(np.float32), O.F16)
    B = O.to_bits(rng.normal(0, 1, k * n).astype(np.float32), O.F16)
    C = np.zeros(m * n, dtype=np.float32)
    O.cpu_gemm_f16_tn(m, n, k, A, k, B, k, C, m, threads=2)
    R, S = O.gemm(1, 0, m, n, k, 1.0, A, O.F16, k, B, O.F16, k)
    got = O.extract(C, O.F32, m, n, m)
    assert O.check(got, R, S, O.F32)["ok"]
