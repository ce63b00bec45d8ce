"""The C-ABI boundary on the CPU: the library loads, exports what include/tinycublas_b200.h declares,
keeps the reference's type contract and cuBLAS's argument rules, and plans kernels as pinned.
Nothing here launches a kernel (every call returns before any CUDA work)."""
import ctypes
import json
import os
import re

import pytest

from macuda_b200 import cublas as cb
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tinycublas_b200.h")
GOLD = os.path.join(ROOT, "tests", "golden")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^[A-Za-z_][\w \*]*?\b(\w+)\s*\(", text, flags=re.M)
    return sorted(set(n for n in names if n not in ("if", "defined")))


def test_header_declares_the_reference_surface():
    names = declared_functions()
    # the linked surface ggml-cuda needs (reference cuda-shim/Makefile:100-109 coverage rule)
    for sym in ["cublasCreate_v2", "cublasDestroy_v2", "cublasSetStream_v2", "cublasSetMathMode", "cublasSgemm_v2",
                "cublasGemmEx", "cublasGemmStridedBatchedEx", "cublasGemmBatchedEx", "cublasSgemmStridedBatched",
                "cublasSgemmBatched", "cublasStrsmBatched", "cublasSetWorkspace_v2", "cublasGetStatusString"]:
        assert sym in names


def test_library_exports_every_declared_symbol(lib):
    exported = set()
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", lib.path], capture_output=True, text=True, check=True).stdout
    for line in out.splitlines():
        parts = line.split()
        if len(parts) == 3:
            exported.add(parts[2])
    missing = [n for n in declared_functions() if n not in exported]
    assert not missing, missing
    for n in declared_functions():
        assert hasattr(lib.lib, n)


def test_version_names_the_arch(lib):
    assert "sm_100a" in lib.version()


def test_status_strings(lib):
    assert lib.lib.cublasGetStatusString(0) == b"CUBLAS_STATUS_SUCCESS"
    assert lib.lib.cublasGetStatusString(15) == b"CUBLAS_STATUS_NOT_SUPPORTED"
    assert lib.lib.cublasGetStatusString(7) == b"CUBLAS_STATUS_INVALID_VALUE"


def test_null_handle_is_not_initialized(lib):
    one = ctypes.c_float(1.0)
    st = lib.lib.cublasGemmEx(None, 1, 0, 4, 4, 4, ctypes.byref(one), None, cb.CUDA_R_16F, 4, None, cb.CUDA_R_16F, 4,
                              ctypes.byref(one), None, cb.CUDA_R_32F, 4, cb.CUBLAS_COMPUTE_32F, -1)
    assert st == cb.CUBLAS_STATUS_NOT_INITIALIZED
    assert lib.lib.cublasSetStream_v2(None, None) == cb.CUBLAS_STATUS_NOT_INITIALIZED


def _contract_status(h, At, Bt, Ct, ct):
    """All three Ex entry points on an m = 0 problem: the contract is checked, nothing launches."""
    dummy = 256
    s1 = h.gemm_ex(1, 0, 0, 32, 32, 1.0, dummy, At, 32, dummy, Bt, 32, 0.0, dummy, Ct, 32, ct)
    s2 = h.gemm_strided_batched_ex(1, 0, 0, 32, 32, 1.0, dummy, At, 32, 1024, dummy, Bt, 32, 1024, 0.0, dummy, Ct, 32,
                                   1024, 2, ct)
    s3 = h.gemm_batched_ex(1, 0, 0, 32, 32, 1.0, dummy, At, 32, dummy, Bt, 32, 0.0, dummy, Ct, 32, 2, ct)
    return s1, s2, s3


with open(os.path.join(GOLD, "reference_rows.json")) as f:
    CONTRACT_ROWS = json.load(f)["contract"]["rows"]


@pytest.mark.parametrize("row", CONTRACT_ROWS, ids=lambda r: r[0])
def test_contract_rows_of_the_reference(lib, row):
    what, At, Bt, Ct, ct, want = row
    with lib.handle() as h:
        assert _contract_status(h, At, Bt, Ct, ct) == (want, want, want), what


def test_contract_equals_reference_on_every_type_combination(lib):
    types = [cb.CUDA_R_32F, cb.CUDA_R_16F, cb.CUDA_R_16BF, 1]  # 1 = CUDA_R_64F, never served
    computes = [64, 65, 68, 69, 70, 71, 72, 73, 74, 75, 77]
    with lib.handle() as h:
        for At in types:
            for Bt in types:
                for Ct in types:
                    for ct in computes:
                        want = cb.CUBLAS_STATUS_SUCCESS if O.ref_contract(At, Bt, Ct, ct) == 0 else \
                            cb.CUBLAS_STATUS_NOT_SUPPORTED
                        assert _contract_status(h, At, Bt, Ct, ct) == (want,) * 3, (At, Bt, Ct, ct)


@pytest.mark.parametrize("args,why", [
    (dict(m=-1), "negative m"), (dict(n=-1), "negative n"), (dict(k=-1), "negative k"),
    (dict(ta=2), "OP_C is not served"), (dict(lda=31), "lda < k under op T"),
    (dict(ldb=31), "ldb < k under op N"), (dict(ldc=31), "ldc < m"),
])
def test_invalid_arguments(lib, args, why):
    p = dict(ta=1, tb=0, m=32, n=32, k=32, lda=32, ldb=32, ldc=32)
    p.update(args)
    with lib.handle() as h:
        st = h.gemm_ex(p["ta"], p["tb"], p["m"], p["n"], p["k"], 1.0, 256, cb.CUDA_R_16F, p["lda"], 256, cb.CUDA_R_16F,
                       p["ldb"], 0.0, 256, cb.CUDA_R_32F, p["ldc"])
        assert st == cb.CUBLAS_STATUS_INVALID_VALUE, why


def test_empty_problems_succeed_without_a_device(lib):
    with lib.handle() as h:
        assert h.gemm_ex(1, 0, 0, 8, 8, 1.0, 256, cb.CUDA_R_16F, 8, 256, cb.CUDA_R_16F, 8, 0.0, 256, cb.CUDA_R_32F,
                         1) == 0
        assert h.gemm_ex(1, 0, 8, 0, 8, 1.0, 256, cb.CUDA_R_16F, 8, 256, cb.CUDA_R_16F, 8, 0.0, 256, cb.CUDA_R_32F,
                         8) == 0
        assert h.gemm_strided_batched_ex(1, 0, 8, 8, 8, 1.0, 256, cb.CUDA_R_16F, 8, 64, 256, cb.CUDA_R_16F, 8, 64, 0.0,
                                         256, cb.CUDA_R_32F, 8, 64, 0) == 0


def test_trsm_refuses_unserved_cases(lib):
    with lib.handle() as h:
        # the reference serves only side RIGHT, upper, no transpose, non-unit (cublas.c:317)
        assert h.strsm_batched(cb.CUBLAS_SIDE_LEFT, 1, 0, 0, 4, 4, 1.0, 256, 4, 256, 4, 2) == 15
        assert h.strsm_batched(cb.CUBLAS_SIDE_RIGHT, 0, 0, 0, 4, 4, 1.0, 256, 4, 256, 4, 2) == 15
        assert h.strsm_batched(cb.CUBLAS_SIDE_RIGHT, 1, 1, 0, 4, 4, 1.0, 256, 4, 256, 4, 2) == 15
        assert h.strsm_batched(cb.CUBLAS_SIDE_RIGHT, 1, 0, 1, 4, 4, 1.0, 256, 4, 256, 4, 2) == 15


# (transa, transb, m, n, k, batch, in, tf32, ptr, aligned) -> (kernel, BN) on 148 SMs; a CTA-pair tile is
# 256 + BN, a k-split tile minus that (-BN: two CTAs per 128-row tile; -512: two CTA pairs per 256 x 256 tile)
PLAN_ROWS = [
    ("config 1: ggml fp16 T,N 4096x512x4096: k split of the pair tile", (1, 0, 4096, 512, 4096, 1, 1, 0, 0, 1),
     (cb.TB200_KERNEL_TC, -512)),
    ("Q/O, 256 tokens: k split", (1, 0, 4096, 256, 4096, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, -128)),
    ("config 3 KQV folded: HBM-bound, unsplit", (1, 0, 128, 2048, 4096, 8, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, 128)),
    ("config 2 K/V 1024x512x4096: k split", (1, 0, 1024, 512, 4096, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, -64)),
    ("K/V in bf16: k split", (1, 0, 1024, 512, 4096, 1, 2, 0, 0, 1), (cb.TB200_KERNEL_TC, -64)),
    ("K/V with k < 1024 stays unsplit", (1, 0, 1024, 512, 960, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, 32)),
    ("K/V through pointer arrays stays unsplit", (1, 0, 1024, 512, 4096, 1, 1, 0, 1, 1), (cb.TB200_KERNEL_TC, 32)),
    ("config 2 gate/up 14336x512x4096: CTA-pair tile", (1, 0, 14336, 512, 4096, 1, 2, 0, 0, 1), (cb.TB200_KERNEL_TC, 512)),
    ("config 2 lm_head 128256x512x4096: CTA-pair tile", (1, 0, 128256, 512, 4096, 1, 1, 0, 0, 1),
     (cb.TB200_KERNEL_TC, 512)),
    ("config 2 down 4096x512x14336: k split of the pair tile", (1, 0, 4096, 512, 14336, 1, 1, 0, 0, 1),
     (cb.TB200_KERNEL_TC, -512)),
    ("down, 256 tokens: k split", (1, 0, 4096, 256, 14336, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, -128)),
    ("down, 128 tokens: k split", (1, 0, 4096, 128, 14336, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, -64)),
    ("down, 4 sequences of 512: enough tiles unsplit", (1, 0, 4096, 512, 14336, 4, 1, 0, 0, 1),
     (cb.TB200_KERNEL_TC, 512)),
    ("config 5 square 8192: CTA-pair tile", (1, 0, 8192, 8192, 8192, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, 512)),
    ("config 4 decode n=1", (1, 0, 4096, 1, 4096, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_SKINNY, 0)),
    ("config 4 decode n=8", (1, 0, 14336, 8, 4096, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_SKINNY, 0)),
    ("n=8 under op N A goes to the tensor cores", (0, 0, 4096, 8, 4096, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, 32)),
    ("n=9 leaves the skinny path", (1, 0, 4096, 9, 4096, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_TC, 32)),
    ("unaligned operands take the SIMT kernel", (1, 0, 48, 40, 72, 3, 1, 0, 0, 0), (cb.TB200_KERNEL_SIMT, 0)),
    ("fp32 without TF32 math stays fp32", (0, 0, 512, 512, 512, 1, 0, 0, 0, 1), (cb.TB200_KERNEL_SIMT, 0)),
    ("fp32 with TF32 math takes the tensor cores", (1, 0, 512, 512, 512, 1, 0, 1, 0, 1), (cb.TB200_KERNEL_TC, 32)),
    ("TF32 with an MN-major operand stays fp32", (0, 0, 512, 512, 512, 1, 0, 1, 0, 1), (cb.TB200_KERNEL_SIMT, 0)),
    ("pointer arrays, n=32 (MoE experts): tensor cores", (1, 0, 768, 32, 2048, 128, 1, 0, 1, 1), (cb.TB200_KERNEL_TC, 32)),
    ("pointer arrays, unaligned ld: SIMT", (1, 0, 768, 32, 2048, 128, 1, 0, 1, 0), (cb.TB200_KERNEL_SIMT, 0)),
    ("pointer arrays, n<=8: skinny", (1, 0, 768, 8, 2048, 128, 1, 0, 1, 1), (cb.TB200_KERNEL_SKINNY, 0)),
    ("k == 0 is a scale of C", (1, 0, 64, 64, 0, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_SIMT, 0)),
    ("empty", (1, 0, 0, 64, 64, 1, 1, 0, 0, 1), (cb.TB200_KERNEL_NONE, 0)),
]


@pytest.mark.parametrize("what,args,want", PLAN_ROWS, ids=[r[0] for r in PLAN_ROWS])
def test_plan_rows(lib, what, args, want):
    ta, tb, m, n, k, batch, it, tf32, ptr, aligned = args
    assert lib.plan(ta, tb, m, n, k, batch, it, 0, tf32, ptr, aligned, 148) == want, what


def test_tile_choice_is_a_compiled_configuration(lib):
    for m in (128, 1024, 4096, 14336, 128256):
        for n in (16, 32, 64, 100, 512, 2048, 16384):
            pair = ctypes.c_int(-1)
            bn = lib.lib.tb200_tc_tile_n(m, n, 1, 148, ctypes.byref(pair))
            assert bn in (32, 64, 128, 256) and pair.value in (0, 1)
            if pair.value:
                assert bn in (128, 256) and n > bn // 2


# decode kernel shape (warps x chunks in flight, k slices) on 148 SMs, as measured best on the B200: many 16-row
# blocks 4 x 8 unsplit, two to six per SM 8 x 4 unsplit, fewer 16 x 2 with the k split up to a CTA for every
# other SM
SKINNY_ROWS = [
    ((128256, 4096, 1), (4, 8, 1)),    # config 4 lm_head: 8016 blocks
    ((14336, 4096, 1), (4, 8, 1)),     # 896 blocks
    ((6144, 4096, 1), (8, 4, 1)),      # 384 blocks
    ((8192, 1024, 1), (8, 4, 1)),      # 512 blocks
    ((4096, 4096, 1), (16, 2, 1)),     # 256 blocks
    ((4096, 14336, 1), (16, 2, 1)),
    ((1024, 4096, 1), (16, 2, 2)),     # 64 blocks
    ((256, 4096, 1), (16, 2, 4)),      # 16 blocks
    ((256, 16384, 1), (16, 2, 8)),
    ((256, 512, 1), (16, 2, 1)),       # too shallow to split
    ((768, 2048, 128), (4, 8, 1)),     # config 5 MoE experts as a batch of decode GEMMs
]


@pytest.mark.parametrize("args,want", SKINNY_ROWS, ids=[f"{a[0]}x{a[1]}xb{a[2]}" for a, _ in SKINNY_ROWS])
def test_skinny_shape_rows(lib, monkeypatch, args, want):
    monkeypatch.delenv("TB200_SKINNY_CFG", raising=False)
    monkeypatch.delenv("TB200_SKINNY_SPLIT", raising=False)
    m, k, batch = args
    assert lib.skinny_shape(m, k, batch) == want


def test_skinny_shape_properties(lib, monkeypatch):
    """Over a grid of block counts, depths and SM counts: 4 x 8 from six blocks per SM, 8 x 4 from two, 16 x 2
    below; only the 16 x 2 shape splits k, and a split keeps at least 2 chunks of 32 per warp a slice and
    stops once the CTAs reach half the SMs."""
    monkeypatch.delenv("TB200_SKINNY_CFG", raising=False)
    monkeypatch.delenv("TB200_SKINNY_SPLIT", raising=False)
    for sms in (132, 148):
        for blocks in (1, 7, 16, 64, 73, 74, 200, 295, 296, 500, 887, 888, 5000):
            for k in (8, 256, 1024, 4096, 14336, 65536):
                w, u, S = lib.skinny_shape(blocks * 16, k, 1, sms)
                if blocks >= 6 * sms:
                    assert (w, u, S) == (4, 8, 1)
                elif blocks >= 2 * sms:
                    assert (w, u, S) == (8, 4, 1)
                else:
                    assert (w, u) == (16, 2) and S in (1, 2, 4, 8)
                    if S > 1:
                        assert (k // 32) // S >= 2 * 16 and blocks * (S // 2) < sms // 2


def test_skinny_shape_knobs(lib, monkeypatch):
    monkeypatch.setenv("TB200_SKINNY_CFG", "8x4")
    monkeypatch.setenv("TB200_SKINNY_SPLIT", "4")
    assert lib.skinny_shape(128256, 4096) == (8, 4, 4)
    monkeypatch.setenv("TB200_SKINNY_SPLIT", "8")
    assert lib.skinny_shape(4096, 1024) == (8, 4, 1)  # 32 chunks: 4 a slice, fewer than the 8 warps


def test_k_split_plan_properties(lib):
    """Over a grid of shapes and SM counts: the planner picks the k split (a negative width) only for 16-bit
    strided GEMMs with k >= 1024, with one tile per cluster fitting on the SMs (two CTAs per 128-row tile, or
    two CTA pairs per 256 x 256 tile), a tile at least half full; pointer arrays and fp32 never split."""
    seen = 0
    for sms in (132, 148, 160):
        for m in (256, 1024, 2048, 4096, 14336):
            for n in (16, 64, 128, 200, 512, 2048):
                for k in (512, 1024, 4096, 14336):
                    for batch in (1, 4):
                        kind, w = lib.plan(1, 0, m, n, k, batch, 1, 0, 0, 0, 1, sms)
                        assert kind == cb.TB200_KERNEL_SKINNY if n <= 8 else kind == cb.TB200_KERNEL_TC
                        if w < 0:
                            seen += 1
                            width = -w
                            pair = width > 256
                            bn = width - 256 if pair else width
                            rows = 256 if pair else 128
                            tiles = -(-m // rows) * -(-n // bn) * batch
                            assert k >= 1024 and bn in (64, 128, 256) and n > bn // 2
                            assert tiles * (4 if pair else 2) <= sms, (m, n, k, batch, sms, w)
                        # the same GEMM through pointer arrays, or in fp32 with TF32, never splits
                        assert lib.plan(1, 0, m, n, k, batch, 1, 0, 0, 1, 1, sms)[1] >= 0
                        assert lib.plan(1, 0, m, n, k, batch, 0, 0, 1, 0, 1, sms)[1] >= 0
    assert seen > 20


def test_grouped_gather_argument_rules(lib):
    """tb200_gemm_grouped_gather_ex refuses bad arguments before any device work: no token ids, no source
    columns, fp32 inputs (the fused gather is 16-bit only)."""
    with lib.handle() as h:
        assert h.gemm_grouped_gather_ex(1, 64, 64, 64, 2, 256, 0, 1.0, 256, cb.CUDA_R_16F, 64, 4096, 256,
                                        cb.CUDA_R_16F, 64, 8, 0.0, 256, cb.CUDA_R_32F, 64) == cb.CUBLAS_STATUS_INVALID_VALUE
        assert h.gemm_grouped_gather_ex(1, 64, 64, 64, 2, 256, 256, 1.0, 256, cb.CUDA_R_16F, 64, 4096, 256,
                                        cb.CUDA_R_16F, 64, 0, 0.0, 256, cb.CUDA_R_32F, 64) == cb.CUBLAS_STATUS_INVALID_VALUE
        assert h.gemm_grouped_gather_ex(1, 64, 64, 64, 2, 256, 256, 1.0, 256, cb.CUDA_R_32F, 64, 4096, 256,
                                        cb.CUDA_R_32F, 64, 8, 0.0, 256, cb.CUDA_R_32F, 64,
                                        cb.CUBLAS_COMPUTE_32F_FAST_TF32) == cb.CUBLAS_STATUS_NOT_SUPPORTED
        assert h.gemm_grouped_gather_ex(1, 64, 64, 64, 2, 256, 256, 1.0, 256, cb.CUDA_R_16F, 32, 4096, 256,
                                        cb.CUDA_R_16F, 64, 8, 0.0, 256, cb.CUDA_R_32F, 64) == cb.CUBLAS_STATUS_INVALID_VALUE


def test_grouped_gemm_argument_rules(lib):
    """tb200_gemm_grouped_ex refuses bad arguments before any device work (cuBLAS's rules, plus its own:
    at most 1024 groups, a device offsets array, fp32 inputs only in TF32 mode)."""
    with lib.handle() as h:
        args = dict(m=64, n_total=64, k=64, groups=4, offsets=256, alpha=1.0, A=256, Atype=cb.CUDA_R_16F, lda=64,
                    strideA=4096, B=256, Btype=cb.CUDA_R_16F, ldb=64, beta=0.0, C=256, Ctype=cb.CUDA_R_32F, ldc=64)

        def call(**kw):
            a = dict(args, **kw)
            return h.gemm_grouped_ex(1, 0, a["m"], a["n_total"], a["k"], a["groups"], a["offsets"], a["alpha"], a["A"],
                                     a["Atype"], a["lda"], a["strideA"], a["B"], a["Btype"], a["ldb"], a["beta"], a["C"],
                                     a["Ctype"], a["ldc"])
        assert call(groups=1025) == cb.CUBLAS_STATUS_INVALID_VALUE
        assert call(offsets=0) == cb.CUBLAS_STATUS_INVALID_VALUE
        assert call(lda=32) == cb.CUBLAS_STATUS_INVALID_VALUE  # op T: lda >= k
        assert call(m=-1) == cb.CUBLAS_STATUS_INVALID_VALUE
        assert call(strideA=-1) == cb.CUBLAS_STATUS_INVALID_VALUE
        assert call(Btype=cb.CUDA_R_16BF) == cb.CUBLAS_STATUS_NOT_SUPPORTED  # A and B types differ
        assert call(Atype=cb.CUDA_R_32F, Btype=cb.CUDA_R_32F) == cb.CUBLAS_STATUS_NOT_SUPPORTED  # exact fp32
        assert call(groups=0) == cb.CUBLAS_STATUS_SUCCESS and call(n_total=0) == cb.CUBLAS_STATUS_SUCCESS


def test_push_block_argument_rules(lib):
    """tb200_push_block (the copy-engine exchange) refuses bad arguments before any copy is issued, and does
    nothing for an empty block or a single rank."""
    import ctypes
    P = 4
    reps = (ctypes.c_void_p * P)(256, 512, 768, 1024)
    streams = (ctypes.c_void_p * P)(None, None, None, None)
    push = lib.lib.tb200_push_block
    inval = cb.CUBLAS_STATUS_INVALID_VALUE
    assert push(None, P, 0, 0, 16, 0, 8, 64, 4, streams, P) == inval          # no replica list
    assert push(reps, 0, 0, 0, 16, 0, 8, 64, 4, streams, P) == inval          # no ranks
    assert push(reps, P, P, 0, 16, 0, 8, 64, 4, streams, P) == inval          # self outside the group
    assert push(reps, P, 0, 60, 16, 0, 8, 64, 4, streams, P) == inval         # rows past the leading dimension
    assert push(reps, P, 0, -1, 16, 0, 8, 64, 4, streams, P) == inval
    assert push(reps, P, 0, 0, 16, -1, 8, 64, 4, streams, P) == inval
    assert push(reps, P, 0, 0, 16, 0, 8, 64, 8, streams, P) == inval          # element size 2 or 4 only
    assert push(reps, P, 0, 0, 16, 0, 8, 64, 4, None, P) == inval             # no streams
    assert push(reps, P, 0, 0, 16, 0, 8, 64, 4, streams, 0) == inval
    ok = cb.CUBLAS_STATUS_SUCCESS
    assert push(reps, P, 0, 0, 0, 0, 8, 64, 4, streams, P) == ok              # empty block: nothing to copy
    assert push(reps, P, 0, 0, 16, 0, 0, 64, 4, streams, P) == ok
    assert push(reps, 1, 0, 0, 16, 0, 8, 64, 4, streams, 1) == ok             # one rank: no peer
