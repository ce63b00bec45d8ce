"""Parity of every kernel family against the fp64 oracle, through the C ABI, on a B200.

Gate (oracle.check): max |C - C_ref| / (|alpha| |op(A)_i| |op(B)_j| + |beta| |C0_ij|) <= 2^-10, plus the
output type's own rounding for f16/bf16 C, with non-finite values refused first; and the reference's
own metric max |C - C_ref| / max |C_ref| <= 2e-3 (f32 C) or 1e-2 (16-bit C)
(cuda-shim/libtinycublas/bf16-20260921/bench_gemm_contract.cu:8-10).
"""
import json
import os

import numpy as np
import pytest

from macuda_b200 import cublas as cb
from oracle import oracle as O
from tests.helpers import dev, host, ptr_table, run_and_check, storage

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def h(lib):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    hh = lib.handle()
    yield hh
    hh.close()


def assert_ok(res, what=""):
    assert res.get("ok"), f"{what}: {res}"


def test_config1_ggml_fp16_tn(lib, h):
    """T,N 4096 x 512 x 4096, fp16 weights N(0, 0.02^2), activations N(0,1), f32 C."""
    assert lib.plan(1, 0, 4096, 512, 4096, 1, 1, 0, 0, 0, 1, 148)[0] == cb.TB200_KERNEL_TC
    assert_ok(run_and_check(lib, h, m=4096, n=512, k=4096, mode="ex", seed=11, sample=192), "config 1")
    assert lib.plan(1, 0, 1024, 512, 4096, 1, 1, 0, 0, 0, 1, 148)[0] == cb.TB200_KERNEL_TC
    assert_ok(run_and_check(lib, h, m=1024, n=512, k=4096, mode="ex", seed=13, sample=192), "config 2 K/V")


def test_config1_bf16(lib, h):
    assert_ok(run_and_check(lib, h, m=4096, n=512, k=4096, in_t=O.BF16, mode="ex", seed=12, sample=160), "bf16")


# the reference's 32-case matrix (bench_gemm_contract.cu:107-131): f16/bf16 x 4 transposes x {f32, same-type}
# C x (alpha, beta) in {(1, 0), (0.5, 2)}, at m 48, n 40, k 72, strided batch 3 - partial tiles everywhere
MATRIX = [(in_t, opA, opB, out_same, ab) for in_t in (O.F16, O.BF16) for opA in (0, 1) for opB in (0, 1)
          for out_same in (0, 1) for ab in (0, 1)]


@pytest.mark.parametrize("in_t,opA,opB,out_same,ab", MATRIX,
                         ids=[f"{'bf16' if c[0] == 2 else 'f16'}-{'NT'[c[1]]}{'NT'[c[2]]}-{'same' if c[3] else 'f32'}"
                              f"-{'a.5b2' if c[4] else 'a1b0'}" for c in MATRIX])
def test_contract_matrix(lib, h, in_t, opA, opB, out_same, ab):
    out_t = in_t if out_same else O.F32
    alpha, beta = (0.5, 2.0) if ab else (1.0, 0.0)
    res = run_and_check(lib, h, opA=opA, opB=opB, m=48, n=40, k=72, in_t=in_t, out_t=out_t, alpha=alpha, beta=beta,
                        batch=3, seed=7 + opA * 2 + opB)
    assert_ok(res)


# both operand majors, multi-tile shapes with tails in m, n and k, at every tile width of the tensor-core
# kernel (forced through TB200_TC_BN; the planner alone picks 32 for most small shapes)
TC_SHAPES = [
    (1, 0, 1000, 520, 700),
    (0, 0, 384, 300, 256),
    (0, 1, 512, 1000, 320),
    (1, 1, 300, 700, 136),
    (1, 0, 256, 24, 512),
]


@pytest.mark.parametrize("bn", [32, 64, 128, 256, "pair", "pair128"])
@pytest.mark.parametrize("opA,opB,m,n,k", TC_SHAPES)
def test_tensor_core_shapes(lib, h, monkeypatch, bn, opA, opB, m, n, k):
    assert lib.plan(opA, opB, m, n, k, 1, 1, 0, 0, 0, 1, 148)[0] == cb.TB200_KERNEL_TC
    monkeypatch.setenv("TB200_TC_BN", str(bn))
    assert_ok(run_and_check(lib, h, opA=opA, opB=opB, m=m, n=n, k=k, seed=m + n + k + len(str(bn))), f"BN {bn}")


@pytest.mark.parametrize("bn", [32, 128, 256, "pair", "pair128"])
def test_tensor_core_bf16_tf32_by_width(lib, h, monkeypatch, bn):
    monkeypatch.setenv("TB200_TC_BN", str(bn))
    assert_ok(run_and_check(lib, h, opA=1, opB=0, m=600, n=400, k=300, in_t=O.BF16, seed=5), "bf16")
    assert_ok(run_and_check(lib, h, opA=1, opB=0, m=600, n=400, k=300, in_t=O.F32, out_t=O.F32, a_sigma=1.0,
                            compute=cb.CUBLAS_COMPUTE_32F_FAST_TF32, seed=6), "tf32")


@pytest.mark.parametrize("bn", ["128", "pair", "pair128"])
def test_tensor_core_alpha_beta_and_16bit_out(lib, h, monkeypatch, bn):
    monkeypatch.setenv("TB200_TC_BN", bn)
    for out_t in (O.F32, O.F16, O.BF16):
        assert_ok(run_and_check(lib, h, m=700, n=300, k=512, out_t=out_t, alpha=-0.75, beta=0.5, seed=3), out_t)


# the k split, on single-CTA tiles (two CTAs per tile) and on the CTA-pair tile (two pairs per tile):
# TB200_KSPLIT=1 takes it wherever the tiles leave at least half of the SMs idle. Odd and tiny k-block counts,
# tails in m, n and k, both majors, bf16, alpha/beta with 16-bit C, strided batches; a GEMM with a single
# k-block stays on the unsplit kernel
KS_CASES = [
    dict(opA=1, opB=0, m=1000, n=300, k=4160),
    dict(opA=0, opB=1, m=520, n=200, k=136),
    dict(opA=1, opB=1, m=300, n=190, k=100),
    dict(opA=1, opB=0, m=256, n=129, k=64),
    dict(opA=1, opB=0, m=700, n=256, k=1000, in_t=O.BF16),
    dict(opA=1, opB=0, m=640, n=250, k=2048, out_t=O.F16, alpha=-0.75, beta=0.5),
    dict(opA=1, opB=0, m=640, n=250, k=2048, out_t=O.BF16, in_t=O.BF16, alpha=2.0, beta=-1.0),
    dict(opA=0, opB=0, m=300, n=200, k=520, batch=3),
]


@pytest.mark.parametrize("bn", [64, 128, 256, "pair"])
@pytest.mark.parametrize("case", KS_CASES, ids=[f"{c['m']}x{c['n']}x{c['k']}-{i}" for i, c in enumerate(KS_CASES)])
def test_k_split_cluster(lib, h, monkeypatch, bn, case):
    monkeypatch.setenv("TB200_KSPLIT", "1")
    monkeypatch.setenv("TB200_TC_BN", str(bn))
    assert_ok(run_and_check(lib, h, seed=case["m"] + case["k"] + len(str(bn)), **case), f"k split BN {bn}")


def test_pair_tile_large_and_batched(lib, h):
    """The CTA-pair (2-SM UMMA) tile as the planner picks it: gate/up shape, and a strided batch."""
    assert lib.plan(1, 0, 14336, 512, 4096, 1, 1, 0, 0, 0, 1, 148)[1] == 512
    assert_ok(run_and_check(lib, h, m=14336, n=512, k=4096, mode="ex", seed=17, sample=160), "gate/up")
    assert_ok(run_and_check(lib, h, m=1000, n=700, k=520, batch=3, seed=18), "batched")


@pytest.mark.parametrize("case", [
    dict(m=30001, n=777, k=4104, mode="ex"),                       # k % 128 = 8: the last stage's second chunk
    dict(m=8000, n=1000, k=1000, opA=0, opB=1, batch=2),           # lies past k; both operands MN-major
    dict(m=20000, n=600, k=2000, in_t=O.BF16, out_t=O.F16, alpha=0.5, beta=-1.0, mode="ex"),
], ids=["ragged-k-tail", "mn-major-batched", "bf16-alpha-beta"])
def test_pair_tile_two_chunks_per_stage(lib, h, monkeypatch, case):
    """The 256 x 256 pair tile with two k-chunks per stage (launches of three waves or more: 472, 256 and 237 pair
    tiles on 74 pairs), against the oracle."""
    monkeypatch.setenv("TB200_TC_BN", "pair")
    assert_ok(run_and_check(lib, h, seed=case["m"] + case["k"], sample=160, edges=True, **case), "two chunks a stage")


def test_strided_batch_and_broadcast(lib, h):
    # folded-GQA shape family of config 3 (small): KQ-like and KQV-like
    assert_ok(run_and_check(lib, h, m=512, n=256, k=128, batch=4, seed=21), "KQ-like")
    assert_ok(run_and_check(lib, h, opA=0, m=128, n=256, k=512, batch=4, seed=22), "KQV-like")
    assert_ok(run_and_check(lib, h, m=256, n=128, k=256, batch=3, sA=0, seed=23), "A broadcast (stride 0)")


@pytest.mark.parametrize("store", ["1", "0"])
def test_strided_batch_store_paths(lib, h, monkeypatch, store):
    """Strided batches through both epilogues: the per-lane stores (their default) and the rank-3 TMA-store map
    (TB200_TMA_STORE=1), ragged tiles, f32 and f16 C."""
    monkeypatch.setenv("TB200_TMA_STORE", store)
    assert_ok(run_and_check(lib, h, m=1000, n=300, k=136, batch=3, seed=24, edges=True), f"f32 C, store {store}")
    assert_ok(run_and_check(lib, h, m=520, n=264, k=256, batch=2, out_t=O.F16, seed=25, edges=True),
              f"f16 C, store {store}")


def test_ldc_padding_and_offset_base(lib, h):
    assert_ok(run_and_check(lib, h, m=200, n=72, k=256, ldc=203, c_offset=1, seed=31), "ldc 203, base+4B")


@pytest.mark.parametrize("n", [1, 2, 3, 4, 5, 7, 8])
def test_skinny_decode(lib, h, n):
    assert lib.plan(1, 0, 4096, n, 4096, 1, 1, 0, 0, 0, 1, 148)[0] == cb.TB200_KERNEL_SKINNY
    assert_ok(run_and_check(lib, h, m=4096, n=n, k=4096, seed=40 + n), f"n={n}")


@pytest.mark.parametrize("in_t,out_t,alpha,beta", [(O.BF16, O.F32, 1.0, 0.0), (O.F16, O.F16, 0.5, 2.0),
                                                    (O.BF16, O.BF16, -1.0, 1.0)])
def test_skinny_tails_and_epilogue(lib, h, in_t, out_t, alpha, beta):
    # m not a multiple of 16, k % 32 == 8 (tail chunk), strided batch
    assert_ok(run_and_check(lib, h, m=1000, n=6, k=1000, in_t=in_t, out_t=out_t, alpha=alpha, beta=beta, batch=2,
                            seed=50))


# the decode kernel's shapes and its k split across a cluster (TB200_SKINNY_CFG / TB200_SKINNY_SPLIT force the
# warps x chunks in flight and the slices per 16-row block):
# m not a multiple of 16, k % 32 in {8, 16, 24} (the tail in the last slice), every n, alpha/beta with
# 16-bit C, strided and pointer-array batches, and unaligned pointer-array elements (the scalar path)
SKINNY_SPLIT_CASES = [
    dict(m=1000, n=1, k=4104),
    dict(m=4096, n=8, k=4096),
    dict(m=520, n=5, k=4112, in_t=O.BF16, out_t=O.BF16, alpha=-1.0, beta=1.0),
    dict(m=300, n=3, k=4120, out_t=O.F16, alpha=0.5, beta=2.0, batch=3),
    dict(m=768, n=8, k=4096, batch=4, mode="ptr", broadcast_a=2),
    dict(m=256, n=2, k=4096, batch=4, mode="ptr", a_ptr_shift=2),
]


@pytest.mark.parametrize("cfg", ["4x8", "8x4", "16x2"])
@pytest.mark.parametrize("S", [1, 2, 4, 8])
@pytest.mark.parametrize("case", SKINNY_SPLIT_CASES,
                         ids=[f"{c['m']}x{c['n']}x{c['k']}-{i}" for i, c in enumerate(SKINNY_SPLIT_CASES)])
def test_skinny_k_split(lib, h, monkeypatch, cfg, S, case):
    """every kernel shape (TB200_SKINNY_CFG: warps x chunks in flight) with every k split"""
    monkeypatch.setenv("TB200_SKINNY_SPLIT", str(S))
    monkeypatch.setenv("TB200_SKINNY_CFG", cfg)
    assert_ok(run_and_check(lib, h, seed=case["m"] + case["k"] + S, **case), f"{cfg} S={S}")


# batch-1 decode GEMMs (cublasGemmEx): k not a multiple of 32, m not a multiple of 16, every n, alpha/beta with
# 16-bit C, bf16, a single 16-row block, few blocks (the k split across a cluster), and the same GEMM twice
DECODE_CASES = [
    dict(m=4096, n=1, k=4096),
    dict(m=14336, n=8, k=4096, sample=128),
    dict(m=4096, n=3, k=14336),
    dict(m=1000, n=7, k=1000, out_t=O.F16, alpha=0.5, beta=2.0),
    dict(m=520, n=2, k=4104, in_t=O.BF16, out_t=O.BF16, alpha=-1.0, beta=1.0),
    dict(m=64, n=8, k=4096),
    dict(m=16, n=1, k=8),
    dict(m=33, n=5, k=520, in_t=O.BF16),
]


@pytest.mark.parametrize("case", DECODE_CASES,
                         ids=[f"{c['m']}x{c['n']}x{c['k']}-{i}" for i, c in enumerate(DECODE_CASES)])
def test_decode_gemm_ex(lib, h, case):
    for rep in range(2):
        assert_ok(run_and_check(lib, h, mode="ex", seed=case["m"] + case["k"] + rep, **case), f"rep {rep}")


# the balanced decode kernel (equal ranges of 16-row blocks x 32-wide chunks, two CTAs per SM; blocks shared by
# several CTAs finished by the last to arrive), opt-in through TB200_SKINNY_BAL=1, on few- and many-block
# weights. Tails in m, every n, alpha/beta with 16-bit C, bf16, a single block, a tiny k, and each shape twice on
# the same stream (the per-block counters return to zero)
BAL_CASES = [
    dict(m=4096, n=1, k=4096),
    dict(m=4096, n=8, k=14336),
    dict(m=1000, n=7, k=1024, out_t=O.F16, alpha=0.5, beta=2.0),
    dict(m=520, n=2, k=4096, in_t=O.BF16, out_t=O.BF16, alpha=-1.0, beta=1.0),
    dict(m=14336, n=4, k=4096, sample=160),
    dict(m=16, n=3, k=4096),
    dict(m=33, n=5, k=2048, in_t=O.BF16),
    dict(m=1024, n=8, k=1024),
]


@pytest.mark.parametrize("case", BAL_CASES, ids=[f"{c['m']}x{c['n']}x{c['k']}-{i}" for i, c in enumerate(BAL_CASES)])
def test_decode_balanced(lib, h, monkeypatch, case):
    monkeypatch.setenv("TB200_SKINNY_BAL", "1")
    for rep in range(2):
        assert_ok(run_and_check(lib, h, mode="ex", seed=case["m"] + case["n"] + case["k"] + rep, **case), f"rep {rep}")


def test_decode_balanced_workspace_across_sizes(lib, monkeypatch):
    """one stream's balanced-decode workspace serves launches of every size in turn: few blocks, then many (whose
    counters must not be where a smaller launch parked its partial tiles), then few again"""
    monkeypatch.setenv("TB200_SKINNY_BAL", "1")
    with lib.handle() as hh:
        for i, m in enumerate([64, 4096, 16, 14336, 1024, 4096, 48]):
            assert_ok(run_and_check(lib, hh, m=m, n=1 + i % 8, k=4096, mode="ex", sample=192, seed=600 + i), f"m={m}")


def test_decode_balanced_two_streams(lib, monkeypatch):
    """the balanced kernel's workspace is per (handle, stream): two streams of one handle interleave decode GEMMs"""
    import torch
    monkeypatch.setenv("TB200_SKINNY_BAL", "1")
    from tests.helpers import dev, host
    rng = np.random.default_rng(71)
    m, n, k = 4096, 4, 4096
    A = storage(rng, m * k, O.F16, 0.02)
    Bs = [storage(rng, k * n, O.F16) for _ in range(2)]
    dA, dBs = dev(A), [dev(b) for b in Bs]
    Cs = [torch.full((m * n,), float("nan"), device="cuda") for _ in range(2)]
    streams = [torch.cuda.Stream() for _ in range(2)]
    with lib.handle() as hh:
        for it in range(6):
            j = it % 2
            hh.set_stream(streams[j].cuda_stream)
            assert hh.gemm_ex(1, 0, m, n, k, 1.0, dA.data_ptr(), cb.CUDA_R_16F, k, dBs[j].data_ptr(), cb.CUDA_R_16F, k,
                              0.0, Cs[j].data_ptr(), cb.CUDA_R_32F, m) == 0
        torch.cuda.synchronize()
    rows = np.arange(0, m, 13, dtype=np.int32)
    for j in range(2):
        R, S = O.gemm(1, 0, m, n, k, 1.0, A, O.F16, k, Bs[j], O.F16, k, rows=rows)
        assert_ok(O.check(O.extract(Cs[j].cpu().numpy(), O.F32, m, n, m, rows=rows), R, S, O.F32), f"stream {j}")


def test_skinny_pointer_arrays_gqa(lib, h):
    assert_ok(run_and_check(lib, h, m=768, n=8, k=2048, batch=8, mode="ptr", broadcast_a=4, seed=60), "ptr n=8")


@pytest.mark.parametrize("bn", [None, "64", "pair", "pair128"])
def test_pointer_arrays_tensor_cores(lib, h, monkeypatch, bn):
    """cublasGemmBatchedEx on the tensor cores: per-element tensor maps built on the device."""
    if bn:
        monkeypatch.setenv("TB200_TC_BN", bn)
    assert lib.plan(1, 0, 768, 32, 2048, 16, 1, 0, 0, 1, 1, 148)[0] == cb.TB200_KERNEL_TC
    assert_ok(run_and_check(lib, h, m=768, n=32, k=2048, batch=16, mode="ptr", seed=63), "MoE experts")
    assert_ok(run_and_check(lib, h, m=512, n=256, k=128, batch=8, mode="ptr", broadcast_a=4, seed=64), "GQA KQ")
    assert_ok(run_and_check(lib, h, opA=0, m=128, n=256, k=512, batch=8, mode="ptr", broadcast_a=4, seed=65),
              "GQA KQV (MN-major A)")
    assert_ok(run_and_check(lib, h, m=300, n=200, k=136, batch=5, mode="ptr", in_t=O.BF16, out_t=O.BF16, alpha=0.5,
                            beta=-1.0, seed=66), "bf16 out, alpha/beta, tails")


def test_pointer_arrays_misaligned_element_falls_back(lib, h):
    """An element pointer off 16-byte alignment cannot feed TMA: the tensor-core launch stands down on the
    device and the general kernel queued behind it computes the batch - no host sync, same result."""
    assert_ok(run_and_check(lib, h, m=256, n=64, k=256, batch=4, mode="ptr", a_ptr_shift=2, seed=67),
              "A pointers of odd elements shifted by 4 bytes")
    assert_ok(run_and_check(lib, h, m=256, n=64, k=256, batch=4, mode="ptr", seed=68), "aligned again")


def test_pointer_array_scratch_is_per_stream(lib):
    import torch
    with lib.handle() as hh:
        run_and_check(lib, hh, m=256, n=64, k=256, batch=4, mode="ptr", seed=69)
        run_and_check(lib, hh, m=256, n=64, k=256, batch=3, mode="ptr", seed=70)
        assert lib.lib.tb200_scratch_allocs(hh.h) == 1
        s2 = torch.cuda.Stream()
        hh.set_stream(s2.cuda_stream)
        with torch.cuda.stream(s2):
            res = run_and_check(lib, hh, m=256, n=64, k=256, batch=4, mode="ptr", seed=71)
        assert res["ok"], res
        assert lib.lib.tb200_scratch_allocs(hh.h) == 2
    with lib.handle() as hh:  # strided GEMMs never allocate
        run_and_check(lib, hh, m=512, n=256, k=256, batch=3, seed=72)
        assert lib.lib.tb200_scratch_allocs(hh.h) == 0


def test_pointer_arrays_general(lib, h):
    assert_ok(run_and_check(lib, h, m=768, n=32, k=512, batch=6, mode="ptr", seed=61), "ptr n=32")
    assert_ok(run_and_check(lib, h, opA=0, m=128, n=64, k=256, batch=4, mode="ptr", broadcast_a=2, seed=62), "GQA")


def test_unaligned_operands_take_the_general_kernel(lib, h):
    # the reference's align cases (bench_gemm_contract.cu:133-139): ldc 33, C base + 16 bytes; plus odd lda/ldb
    assert_ok(run_and_check(lib, h, m=32, n=32, k=32, ldc=33, seed=70), "ldc 33")
    assert_ok(run_and_check(lib, h, m=32, n=32, k=32, c_offset=4, seed=71), "C base + 16 B")
    assert_ok(run_and_check(lib, h, m=45, n=37, k=51, lda=53, ldb=55, seed=72), "odd lda/ldb")
    assert_ok(run_and_check(lib, h, opA=0, opB=1, m=45, n=37, k=51, lda=47, ldb=41, in_t=O.BF16, out_t=O.BF16,
                            alpha=2.0, beta=-1.0, batch=2, seed=73), "odd, batched, bf16")


def test_compute16f_f16_out(lib, h):
    assert_ok(run_and_check(lib, h, opA=0, opB=0, m=256, n=128, k=512, in_t=O.F16, out_t=O.F16,
                            compute=cb.CUBLAS_COMPUTE_16F, alpha=1.0, beta=0.0, seed=80), "COMPUTE_16F")


def test_known_answer_f16_4x4_compute16f(lib, h):
    import torch
    ka = json.load(open(os.path.join(GOLD, "known_answers.json")))["gemm16_4x4"]
    A = O.to_bits(np.array(ka["A"], np.float32), O.F16)
    B = O.to_bits(np.array(ka["B"], np.float32), O.F16)
    C = np.zeros(16, np.uint16)
    dA, dB, dC = dev(A), dev(B), dev(C)
    st = h.gemm_ex(0, 0, 4, 4, 4, 1.0, dA.data_ptr(), cb.CUDA_R_16F, 4, dB.data_ptr(), cb.CUDA_R_16F, 4, 0.0,
                   dC.data_ptr(), cb.CUDA_R_16F, 4, cb.CUBLAS_COMPUTE_16F)
    torch.cuda.synchronize()
    assert st == 0
    assert np.array_equal(O.from_bits(host(dC, C), O.F16), np.array(ka["C"], np.float32))


def test_known_answer_sgemm48_exact_fp32_and_tf32(lib):
    """link_smoke.c:41-52: small integers, exact in fp32 and in TF32, across a multi-block grid; as NN (the
    reference's call, fp32 kernel under either math mode) and as TN (the TF32 tensor-core path)."""
    import torch
    ka = json.load(open(os.path.join(GOLD, "known_answers.json")))["sgemm48"]
    A = np.array(ka["A"], np.float32)
    B = np.array(ka["B"], np.float32)
    want = np.array(ka["C"], np.float32)
    At = np.ascontiguousarray(A.reshape(48, 48).T)  # stored A^T (column-major), so op T gives A back
    for mode in (cb.CUBLAS_DEFAULT_MATH, cb.CUBLAS_TF32_TENSOR_OP_MATH):
        for ta, a in ((0, A), (1, At.reshape(-1))):
            with lib.handle() as hh:
                assert hh.set_math_mode(mode) == 0
                C = np.full(48 * 48, np.nan, np.float32)
                dA, dB, dC = dev(a), dev(B), dev(C)
                assert hh.sgemm(ta, 0, 48, 48, 48, 1.0, dA.data_ptr(), 48, dB.data_ptr(), 48, 0.0, dC.data_ptr(),
                                48) == 0
                torch.cuda.synchronize()
                assert np.array_equal(host(dC, C), want), (mode, ta)


def test_sgemm_fp32_and_tf32(lib, h):
    assert_ok(run_and_check(lib, h, opA=0, opB=1, m=300, n=200, k=250, in_t=O.F32, out_t=O.F32, a_sigma=1.0,
                            alpha=1.5, beta=-0.5, seed=90), "fp32 SIMT")
    res = run_and_check(lib, h, opA=1, opB=0, m=512, n=256, k=512, in_t=O.F32, out_t=O.F32, a_sigma=1.0,
                        compute=cb.CUBLAS_COMPUTE_32F_FAST_TF32, seed=91)
    assert_ok(res, "TF32 tensor cores")
    assert res["norm_err"] > 1e-7, "TF32 rounding should be visible: was the fp32 path taken?"
    res = run_and_check(lib, h, opA=0, opB=1, m=300, n=200, k=250, in_t=O.F32, out_t=O.F32, a_sigma=1.0,
                        compute=cb.CUBLAS_COMPUTE_32F_FAST_TF32, seed=92)
    assert_ok(res, "TF32 requested with MN-major operands: exact fp32 kernel")


def test_k_zero_scales_c(lib, h):
    assert_ok(run_and_check(lib, h, m=64, n=48, k=0, alpha=1.0, beta=0.5, out_t=O.F32, seed=95), "k=0")


def test_trsm_batched(lib, h):
    import torch
    rng = np.random.default_rng(100)
    rows, n, batch = 37, 20, 3
    As, Bs = [], []
    for _ in range(batch):
        A = np.triu(rng.normal(size=(n, n))).astype(np.float32) + 4 * np.eye(n, dtype=np.float32)
        As.append(np.asfortranarray(A).reshape(-1, order="F").copy())
        Bs.append(rng.normal(size=rows * n).astype(np.float32))
    dAs = [dev(a) for a in As]
    dBs = [dev(b) for b in Bs]
    tA, tB = ptr_table([d.data_ptr() for d in dAs]), ptr_table([d.data_ptr() for d in dBs])
    st = h.strsm_batched(cb.CUBLAS_SIDE_RIGHT, cb.CUBLAS_FILL_MODE_UPPER, 0, cb.CUBLAS_DIAG_NON_UNIT, rows, n, 0.5,
                         tA.data_ptr(), n, tB.data_ptr(), rows, batch)
    torch.cuda.synchronize()
    assert st == 0
    for b in range(batch):
        X = O.trsm_rupn(As[b], Bs[b], rows, n, n, rows, 0.5)
        got = dBs[b].cpu().numpy().astype(np.float64)
        assert np.max(np.abs(got - X)) <= 1e-4 * max(1.0, np.max(np.abs(X)))


def test_deterministic(lib, h):
    import torch
    rng = np.random.default_rng(110)
    # unsplit tensor-core tile, the k split (fixed order of the two slices' sums), decode
    for (m, n, k) in [(4096, 512, 1024), (1024, 512, 4096), (4096, 8, 4096)]:
        A, B = storage(rng, m * k, O.F16, 0.02), storage(rng, k * n, O.F16)
        dA, dB = dev(A), dev(B)
        outs = []
        for _ in range(3):
            dC = torch.full((m * n,), float("nan"), device="cuda")
            assert h.gemm_ex(1, 0, m, n, k, 1.0, dA.data_ptr(), cb.CUDA_R_16F, k, dB.data_ptr(), cb.CUDA_R_16F, k, 0.0,
                             dC.data_ptr(), cb.CUDA_R_32F, m) == 0
            outs.append(dC.cpu().numpy())
        assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


def test_dependent_chain_in_one_stream(lib, h):
    """Each GEMM reads the previous one's output, issued back to back on one stream with no host sync:
    kernels are launched with programmatic stream serialization, so a kernel may be scheduled before the
    one it depends on has finished and must wait (griddepcontrol.wait) before reading. Outputs start as
    NaN, so a read too early shows up as a non-finite value or a mismatch. Links: tensor-core chain, then
    decode links skinny (T,N, n=8) -> tensor core (N,N, n=8) -> skinny. Every link is checked against the
    oracle computed from the previous link's actual device output."""
    import torch
    rng = np.random.default_rng(140)
    n_tc, n_dec = 256, 8
    # (opA, m, k, n): op T weights are stored k x m, op N weights m x k; the input is the previous output
    links = [(1, 2048, 4096, n_tc), (1, 4096, 2048, n_tc), (1, 1024, 4096, n_tc),
             (1, 4096, 1024, n_dec), (0, 2048, 4096, n_dec), (1, 4096, 2048, n_dec)]
    assert lib.plan(1, 0, 4096, n_dec, 1024)[0] == cb.TB200_KERNEL_SKINNY
    assert lib.plan(0, 0, 2048, n_dec, 4096)[0] == cb.TB200_KERNEL_TC
    x_tc = storage(rng, 4096 * n_tc, O.F16)
    x_dec = storage(rng, 1024 * n_dec, O.F16)
    W = [storage(rng, m * k, O.F16, 0.02) for (_, m, k, _) in links]
    dW = [dev(w) for w in W]
    outs = [torch.full((m * n,), float("nan"), dtype=torch.float16, device="cuda") for (_, m, _, n) in links]
    src = [dev(x_tc)] + outs[:2] + [dev(x_dec)] + outs[3:5]
    for i, (opA, m, k, n) in enumerate(links):
        lda = k if opA == 1 else m
        assert h.gemm_ex(opA, 0, m, n, k, 1.0, dW[i].data_ptr(), cb.CUDA_R_16F, lda, src[i].data_ptr(), cb.CUDA_R_16F,
                         k, 0.0, outs[i].data_ptr(), cb.CUDA_R_16F, m) == 0
    torch.cuda.synchronize()
    inputs = [x_tc] + [host(o, x_tc) for o in outs[:2]] + [x_dec] + [host(o, x_tc) for o in outs[3:5]]
    for i, (opA, m, k, n) in enumerate(links):
        lda = k if opA == 1 else m
        rows = np.arange(0, m, 5, dtype=np.int32)
        R, S = O.gemm(opA, 0, m, n, k, 1.0, W[i], O.F16, lda, inputs[i], O.F16, k, 0.0, None, O.F16, m, rows=rows)
        got = O.extract(host(outs[i], x_tc), O.F16, m, n, m, rows=rows)
        assert_ok(O.check(got, R, S, O.F16), f"link {i}")


def _grouped_case(lib, h, rng, m, k, counts, in_t=O.F16, out_t=O.F32, alpha=1.0, beta=0.0, opA=1, offsets=None,
                  guard=64):
    """One tb200_gemm_grouped_ex call; every group's columns checked against the oracle on sampled rows,
    and a guard region after C checked untouched. counts: tokens per group (offsets = their prefix)."""
    import torch
    G = len(counts)
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32) if offsets is None else np.asarray(offsets, np.int32)
    n_total = int(np.sum(counts))
    lda = k if opA == 1 else m
    A = storage(rng, G * m * k, in_t, 0.02)
    B = storage(rng, max(1, k * n_total), in_t)
    C0 = storage(rng, m * n_total + guard, out_t)
    dA, dB, dC = dev(A), dev(B), dev(C0)
    d_off = torch.from_numpy(offs).cuda()
    ct = {O.F16: cb.CUDA_R_16F, O.BF16: cb.CUDA_R_16BF, O.F32: cb.CUDA_R_32F}
    st = h.gemm_grouped_ex(opA, 0, m, n_total, k, G, d_off.data_ptr(), alpha, dA.data_ptr(), ct[in_t], lda, m * k,
                           dB.data_ptr(), ct[in_t], k, beta, dC.data_ptr(), ct[out_t], m)
    torch.cuda.synchronize()
    assert st == cb.CUBLAS_STATUS_SUCCESS, st
    C = host(dC, C0)
    assert np.array_equal(C[m * n_total:], C0[m * n_total:]), "the guard region after C was written"
    rows = np.unique(np.concatenate([np.arange(0, m, 11), [m - 1]])).astype(np.int32)
    clamped = np.maximum.accumulate(np.clip(offs, 0, n_total))
    for g in range(G):
        c0, c1 = int(clamped[g]), int(clamped[g + 1])
        if c1 <= c0:
            continue
        n = c1 - c0
        Ag = A[g * m * k:(g + 1) * m * k]
        Bg = B[c0 * k:c1 * k]
        Cg0 = C0[c0 * m:c1 * m]
        R, S = O.gemm(opA, 0, m, n, k, alpha, Ag, in_t, lda, Bg, in_t, k, beta, Cg0, out_t, m, rows=rows)
        res = O.check(O.extract(C[c0 * m:c1 * m], out_t, m, n, m, rows=rows), R, S, out_t)
        assert res["ok"], f"group {g} (columns {c0}..{c1}): {res}"


def _grouped_gather_case(lib, h, rng, m, k, counts, n_src, ids=None, in_t=O.F16, out_t=O.F32, alpha=1.0, beta=0.0,
                         opA=1, guard=64):
    """One tb200_gemm_grouped_gather_ex call (B = columns ids of X, fused): every group's columns checked
    against the oracle run on the gathered B (zero columns for ids outside [0, n_src)), and a guard region
    after C checked untouched."""
    import torch
    G = len(counts)
    offs = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    n_total = int(np.sum(counts))
    ids = rng.integers(0, n_src, n_total).astype(np.int32) if ids is None else np.asarray(ids, np.int32)
    lda = k if opA == 1 else m
    A = storage(rng, G * m * k, in_t, 0.02)
    X = storage(rng, k * n_src, in_t)
    C0 = storage(rng, m * n_total + guard, out_t)
    dA, dX, dC = dev(A), dev(X), dev(C0)
    d_off, d_ids = torch.from_numpy(offs).cuda(), torch.from_numpy(ids).cuda()
    ct = {O.F16: cb.CUDA_R_16F, O.BF16: cb.CUDA_R_16BF, O.F32: cb.CUDA_R_32F}
    st = h.gemm_grouped_gather_ex(opA, m, n_total, k, G, d_off.data_ptr(), d_ids.data_ptr(), alpha, dA.data_ptr(),
                                  ct[in_t], lda, m * k, dX.data_ptr(), ct[in_t], k, n_src, beta, dC.data_ptr(),
                                  ct[out_t], m)
    torch.cuda.synchronize()
    assert st == cb.CUBLAS_STATUS_SUCCESS, st
    C = host(dC, C0)
    assert np.array_equal(C[m * n_total:], C0[m * n_total:]), "the guard region after C was written"
    Xc = X.reshape(n_src, k)
    B = np.stack([Xc[t] if 0 <= t < n_src else np.zeros(k, Xc.dtype) for t in ids]).ravel() if n_total else Xc[:0].ravel()
    rows = np.unique(np.concatenate([np.arange(0, m, 11), [m - 1]])).astype(np.int32)
    for g in range(G):
        c0, c1 = int(offs[g]), int(offs[g + 1])
        if c1 <= c0:
            continue
        n = c1 - c0
        R, S = O.gemm(opA, 0, m, n, k, alpha, A[g * m * k:(g + 1) * m * k], in_t, lda, B[c0 * k:c1 * k], in_t, k,
                      beta, C0[c0 * m:c1 * m], out_t, m, rows=rows)
        res = O.check(O.extract(C[c0 * m:c1 * m], out_t, m, n, m, rows=rows), R, S, out_t)
        assert res["ok"], f"group {g} (columns {c0}..{c1}): {res}"


@pytest.mark.parametrize("bn", ["32", "64"])
def test_grouped_gather_moe_routing(lib, h, monkeypatch, bn):
    """The fused gather on config 5's expert shape (768 x 2048, 128 experts, 4096 routed copies of 512
    tokens): skewed counts with empty experts, every tile width the fused path takes."""
    monkeypatch.setenv("TB200_TC_BN", bn)
    rng = np.random.default_rng(160)
    counts = rng.multinomial(4096, rng.dirichlet(np.full(128, 0.3)))
    counts[[0, 17, 127]] = 0
    _grouped_gather_case(lib, h, rng, 768, 2048, counts, n_src=512)


@pytest.mark.parametrize("in_t,out_t,alpha,beta,opA", [(O.BF16, O.F32, 1.0, 0.0, 1), (O.F16, O.F16, 0.5, 0.75, 1),
                                                       (O.F16, O.F32, 1.0, 0.0, 0)])
def test_grouped_gather_types_epilogue_majors_and_bad_ids(lib, h, in_t, out_t, alpha, beta, opA):
    """tails in m, n and k (k = 200: the last k-chunk half outside X), empty groups, and token ids outside
    [0, n_src) - negative, n_src itself, far past it - which give zero columns (C = beta C0 there)."""
    rng = np.random.default_rng(161)
    counts = [37, 0, 70, 1, 64, 29]
    n_src = 90
    ids = rng.integers(0, n_src, sum(counts)).astype(np.int32)
    ids[[0, 5, 40, 100, 200]] = [-1, n_src, 1 << 30, -(1 << 30), n_src - 1]
    _grouped_gather_case(lib, h, rng, 1000, 200, counts, n_src, ids=ids, in_t=in_t, out_t=out_t, alpha=alpha,
                         beta=beta, opA=opA)


def test_grouped_gemm_moe_unbalanced_routing(lib, h):
    """Config 5's expert shape (768 x 2048, 128 experts) with 4096 routed tokens spread unevenly: skewed
    counts, empty experts included, each expert's n different and mostly not a multiple of the tile."""
    rng = np.random.default_rng(150)
    p = rng.dirichlet(np.full(128, 0.3))
    counts = rng.multinomial(4096, p)
    counts[[0, 17, 127]] = 0
    assert (counts == 0).sum() >= 3 and counts.max() > 3 * counts.mean()
    _grouped_case(lib, h, rng, 768, 2048, counts)


@pytest.mark.parametrize("in_t,out_t,alpha,beta,opA", [(O.BF16, O.F32, 1.0, 0.0, 1), (O.F16, O.F16, 0.5, 0.75, 1),
                                                       (O.F16, O.F32, 1.0, 0.0, 0)])
def test_grouped_gemm_types_epilogue_and_majors(lib, h, in_t, out_t, alpha, beta, opA):
    rng = np.random.default_rng(151)
    _grouped_case(lib, h, rng, 1000, 512, [37, 0, 300, 1, 64, 129], in_t=in_t, out_t=out_t, alpha=alpha, beta=beta,
                  opA=opA)


def test_grouped_gemm_clamps_malformed_offsets(lib, h):
    """Offsets past n_total or decreasing: the kernel clamps them (a decrease is an empty group) and never
    writes outside C."""
    rng = np.random.default_rng(152)
    counts = [40, 40, 40, 40]  # n_total = 160
    _grouped_case(lib, h, rng, 256, 256, counts, offsets=[0, 60, 30, 500, 160])


def test_two_streams_no_shared_state(lib):
    """The reference's BURST arm (splitk-20260923/test_splitk.cu:153-175) with two streams fails 8/8 because
    its split-K workspace is per handle. Here: 8 decode GEMMs and 8 prefill GEMMs on two streams and two
    handles, no sync in between, every output checked."""
    import torch
    rng = np.random.default_rng(120)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    h1, h2 = lib.handle(), lib.handle()
    h1.set_stream(s1.cuda_stream)
    h2.set_stream(s2.cuda_stream)
    m, k = 2048, 2048
    B = storage(rng, k * 32, O.F16)
    dB = dev(B)
    As = [storage(rng, m * k, O.F16, 0.02) for _ in range(8)]
    dAs = [dev(a) for a in As]
    outs = [torch.full((m * 32,), float("nan"), device="cuda") for _ in range(8)]
    torch.cuda.synchronize()
    for i in range(8):
        hh, n = (h1, 8) if i % 2 == 0 else (h2, 32)
        assert hh.gemm_ex(1, 0, m, n, k, 1.0, dAs[i].data_ptr(), cb.CUDA_R_16F, k, dB.data_ptr(), cb.CUDA_R_16F, k,
                          0.0, outs[i].data_ptr(), cb.CUDA_R_32F, m) == 0
    torch.cuda.synchronize()
    for i in range(8):
        n = 8 if i % 2 == 0 else 32
        R, S = O.gemm(1, 0, m, n, k, 1.0, As[i], O.F16, k, B, O.F16, k, rows=np.arange(0, m, 7, dtype=np.int32))
        got = O.extract(outs[i].cpu().numpy(), O.F32, m, n, m, rows=np.arange(0, m, 7))
        assert_ok(O.check(got, R, S, O.F32), f"burst {i}")
    h1.close()
    h2.close()


def test_graph_capture_replays(lib):
    import torch
    rng = np.random.default_rng(130)
    m, n, k = 1024, 256, 512
    A, B = storage(rng, m * k, O.F16, 0.02), storage(rng, k * n, O.F16)
    dA, dB = dev(A), dev(B)
    dC = torch.zeros(m * n, device="cuda")
    s = torch.cuda.Stream()
    hh = lib.handle()
    hh.set_stream(s.cuda_stream)
    def issue():
        assert hh.gemm_ex(1, 0, m, n, k, 1.0, dA.data_ptr(), cb.CUDA_R_16F, k, dB.data_ptr(), cb.CUDA_R_16F, k, 0.0,
                          dC.data_ptr(), cb.CUDA_R_32F, m) == 0
        assert hh.gemm_ex(1, 0, m, 4, k, 1.0, dA.data_ptr(), cb.CUDA_R_16F, k, dB.data_ptr(), cb.CUDA_R_16F, k, 1.0,
                          dC.data_ptr(), cb.CUDA_R_32F, m) == 0

    with torch.cuda.stream(s):
        issue()  # the first call of a kernel variant on a device sets its attributes: do it before capturing
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        assert hh.gemm_ex(1, 0, m, n, k, 1.0, dA.data_ptr(), cb.CUDA_R_16F, k, dB.data_ptr(), cb.CUDA_R_16F, k, 0.0,
                          dC.data_ptr(), cb.CUDA_R_32F, m) == 0
        assert hh.gemm_ex(1, 0, m, 4, k, 1.0, dA.data_ptr(), cb.CUDA_R_16F, k, dB.data_ptr(), cb.CUDA_R_16F, k, 1.0,
                          dC.data_ptr(), cb.CUDA_R_32F, m) == 0
    dC.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    R, S = O.gemm(1, 0, m, n, k, 1.0, A, O.F16, k, B, O.F16, k)
    R4, _ = O.gemm(1, 0, m, 4, k, 1.0, A, O.F16, k, B, O.F16, k)
    R[:, :4, :] += R4
    got = O.extract(dC.cpu().numpy(), O.F32, m, n, m)
    assert_ok(O.check(got, R, 2 * S, O.F32), "graph replay")
    del g
    hh.close()


def test_graph_capture_pointer_arrays(lib):
    """After the first call on a stream made its scratch, pointer-array GEMMs capture and replay."""
    import torch
    from tests.helpers import storage as st_
    rng = np.random.default_rng(131)
    m, n, k, batch = 256, 64, 512, 6
    A = st_(rng, m * k * batch, O.F16, 0.02)
    B = st_(rng, k * n * batch, O.F16)
    dA, dB = dev(A), dev(B)
    dC = torch.zeros(m * n * batch, device="cuda")
    tA = ptr_table([dA.data_ptr() + b * m * k * 2 for b in range(batch)])
    tB = ptr_table([dB.data_ptr() + b * k * n * 2 for b in range(batch)])
    tC = ptr_table([dC.data_ptr() + b * m * n * 4 for b in range(batch)])
    s = torch.cuda.Stream()
    hh = lib.handle()
    hh.set_stream(s.cuda_stream)

    def issue():
        assert hh.gemm_batched_ex(1, 0, m, n, k, 1.0, tA.data_ptr(), cb.CUDA_R_16F, k, tB.data_ptr(), cb.CUDA_R_16F, k,
                                  0.0, tC.data_ptr(), cb.CUDA_R_32F, m, batch) == 0

    with torch.cuda.stream(s):
        issue()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        issue()
    dC.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    R, S = O.gemm(1, 0, m, n, k, 1.0, A, O.F16, k, B, O.F16, k, sA=m * k, sB=k * n, batch=batch)
    got = O.extract(dC.cpu().numpy(), O.F32, m, n, m, sC=m * n, batch=batch)
    assert_ok(O.check(got, R, S, O.F32), "pointer-array graph replay")
    del g
    hh.close()


def test_graph_capture_pointer_arrays_first_call(lib):
    """cublasSetStream made the stream's pointer-array scratch outside the capture, so the first pointer-array
    call on that stream can be inside one (a warm-up strided GEMM of the same tile sets the kernel's attributes)."""
    import torch
    from tests.helpers import storage as st_
    rng = np.random.default_rng(137)
    m, n, k, batch = 256, 64, 512, 6
    A = st_(rng, m * k * batch, O.F16, 0.02)
    B = st_(rng, k * n * batch, O.F16)
    dA, dB = dev(A), dev(B)
    dC = torch.zeros(m * n * batch, device="cuda")
    tA = ptr_table([dA.data_ptr() + b * m * k * 2 for b in range(batch)])
    tB = ptr_table([dB.data_ptr() + b * k * n * 2 for b in range(batch)])
    tC = ptr_table([dC.data_ptr() + b * m * n * 4 for b in range(batch)])
    s = torch.cuda.Stream()
    hh = lib.handle()
    hh.set_stream(s.cuda_stream)
    assert lib.lib.tb200_scratch_allocs(hh.h) == 1, "cublasSetStream did not make the stream's scratch"
    with torch.cuda.stream(s):
        assert hh.gemm_strided_batched_ex(1, 0, m, n, k, 1.0, dA.data_ptr(), cb.CUDA_R_16F, k, m * k, dB.data_ptr(),
                                          cb.CUDA_R_16F, k, k * n, 0.0, dC.data_ptr(), cb.CUDA_R_32F, m, m * n, batch) == 0
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        assert hh.gemm_batched_ex(1, 0, m, n, k, 1.0, tA.data_ptr(), cb.CUDA_R_16F, k, tB.data_ptr(), cb.CUDA_R_16F, k,
                                  0.0, tC.data_ptr(), cb.CUDA_R_32F, m, batch) == 0
    assert lib.lib.tb200_scratch_allocs(hh.h) == 1
    dC.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    R, S = O.gemm(1, 0, m, n, k, 1.0, A, O.F16, k, B, O.F16, k, sA=m * k, sB=k * n, batch=batch)
    got = O.extract(dC.cpu().numpy(), O.F32, m, n, m, sC=m * n, batch=batch)
    assert_ok(O.check(got, R, S, O.F32), "pointer-array first call inside a capture")
    del g
    hh.close()


def test_no_device_error_recorded(lib):
    assert lib.device_error() == 0


def test_reference_arm_agrees_with_oracle(lib, h):
    """The reference's own library (cublas.c + gemm.cu built here for sm_100a) on the same config-1
    GEMM: it must pass the same gate, which pins the oracle against the real reference."""
    ref = O.reference_library()
    if ref is None:
        pytest.skip("oracle/_ref not built")
    import torch
    rng = np.random.default_rng(140)
    m, n, k = 4096, 512, 4096
    A, B = storage(rng, m * k, O.F16, 0.02), storage(rng, k * n, O.F16)
    dA, dB = dev(A), dev(B)
    outs = {}
    for name, L in (("ours", lib), ("reference", ref)):
        dC = torch.full((m * n,), float("nan"), device="cuda")
        hh = L.handle()
        assert hh.gemm_ex(1, 0, m, n, k, 1.0, dA.data_ptr(), cb.CUDA_R_16F, k, dB.data_ptr(), cb.CUDA_R_16F, k, 0.0,
                          dC.data_ptr(), cb.CUDA_R_32F, m) == 0
        torch.cuda.synchronize()
        outs[name] = dC.cpu().numpy()
        hh.close()
    rows = np.arange(0, m, 29, dtype=np.int32)
    cols = np.arange(0, n, 7, dtype=np.int32)
    R, S = O.gemm(1, 0, m, n, k, 1.0, A, O.F16, k, B, O.F16, k, rows=rows, cols=cols)
    for name, C in outs.items():
        assert_ok(O.check(O.extract(C, O.F32, m, n, m, rows=rows, cols=cols), R, S, O.F32), name)
    # ours vs the reference directly: both are fp32-accumulate GEMMs of the same inputs
    diff = np.max(np.abs(outs["ours"] - outs["reference"])) / np.max(np.abs(outs["reference"]))
    assert diff < 1e-4, diff
