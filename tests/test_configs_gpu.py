"""Parity at the BASELINE configurations' own sizes (configs 3, 4 and 5; configs 1 and 2 are in
test_gemm_gpu.py), each GEMM as ggml issues it and checked against the fp64 oracle on seeded row and column
samples, with the gate of oracle.check."""
import numpy as np
import pytest

from macuda_b200 import cublas as cb
from oracle import oracle as O
from tests.helpers import dev, host, run_and_check, storage

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h(lib):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    hh = lib.handle()
    yield hh
    hh.close()


def assert_ok(res, what=""):
    assert res.get("ok"), f"{what}: {res}"


# config 3: 32 query heads / 8 KV heads, head_dim 128, 512 queries, 4096 keys, fp16 N(0, 1), f32 C
def test_config3_kq_strided_folded(lib, h):
    """KQ with the 4 query heads of each KV head folded into n: m 4096 keys, n 2048, k 128, batch 8."""
    assert_ok(run_and_check(lib, h, m=4096, n=2048, k=128, batch=8, a_sigma=1.0, sample=128, seed=300), "KQ folded")


def test_config3_kq_pointer_gqa(lib, h):
    """KQ as 32 pointer-array elements, each KV head's pointer repeated for its 4 query heads."""
    assert_ok(run_and_check(lib, h, m=4096, n=512, k=128, batch=32, mode="ptr", broadcast_a=4, a_sigma=1.0,
                            sample=96, seed=301), "KQ pointer GQA")


@pytest.mark.parametrize("mode", ["strided", "ptr"])
def test_config3_kqv_softmax_weights(lib, h, mode):
    """KQV: C (128 x 512 per head) = V^T P with P softmax-shaped (each query's weights over the 4096 keys are
    uniform positive numbers normalised to sum 1, stored fp16), V fp16 N(0, 1); strided form with the 4
    query heads of a KV head folded into n (batch 8), and pointer form (batch 32, V pointer repeated 4x)."""
    import torch
    rng = np.random.default_rng(302)
    Hq, Hkv, D, Tq, Tk = 32, 8, 128, 512, 4096
    V = storage(rng, Hkv * Tk * D, O.F16)  # per KV head: k = Tk x m = D (op T, lda = Tk)
    u = rng.uniform(0.0, 1.0, (Hq, Tq, Tk)).astype(np.float32)
    P = O.to_bits((u / u.sum(axis=2, keepdims=True)).astype(np.float32).ravel(), O.F16)  # k = Tk x n per head
    dV, dP = dev(V), dev(P)
    C = torch.full((Hq * D * Tq,), float("nan"), device="cuda")
    if mode == "strided":
        g = Hq // Hkv
        st = h.gemm_strided_batched_ex(1, 0, D, g * Tq, Tk, 1.0, dV.data_ptr(), cb.CUDA_R_16F, Tk, Tk * D, dP.data_ptr(),
                                       cb.CUDA_R_16F, Tk, g * Tq * Tk, 0.0, C.data_ptr(), cb.CUDA_R_32F, D, D * g * Tq,
                                       Hkv)
    else:
        tab = lambda ptrs: torch.tensor(ptrs, dtype=torch.int64, device="cuda")
        pa = tab([dV.data_ptr() + (b // 4) * Tk * D * 2 for b in range(Hq)])
        pb = tab([dP.data_ptr() + b * Tq * Tk * 2 for b in range(Hq)])
        pc = tab([C.data_ptr() + b * D * Tq * 4 for b in range(Hq)])
        st = h.gemm_batched_ex(1, 0, D, Tq, Tk, 1.0, pa.data_ptr(), cb.CUDA_R_16F, Tk, pb.data_ptr(), cb.CUDA_R_16F, Tk,
                               0.0, pc.data_ptr(), cb.CUDA_R_32F, D, Hq)
    torch.cuda.synchronize()
    assert st == 0
    got = C.cpu().numpy()
    cols = np.unique(np.concatenate([[0, Tq - 1], rng.choice(Tq, 62, replace=False)])).astype(np.int32)
    for b in range(0, Hq, 5):  # a spread of heads, each against its own KV head
        A = V[(b // 4) * Tk * D:(b // 4 + 1) * Tk * D]
        B = P[b * Tq * Tk:(b + 1) * Tq * Tk]
        R, S = O.gemm(1, 0, D, Tq, Tk, 1.0, A, O.F16, Tk, B, O.F16, Tk, cols=cols)
        res = O.check(O.extract(got[b * D * Tq:(b + 1) * D * Tq], O.F32, D, Tq, D, cols=cols), R, S, O.F32)
        assert_ok(res, f"head {b}")


# config 4: decode n in {1, 2, 4, 8} against the weight shapes (4096^2 is in test_gemm_gpu.py; 128256 x 4096
# runs the same kernel as 14336 x 4096 with more row blocks)
@pytest.mark.parametrize("m,k", [(14336, 4096), (4096, 14336)])
@pytest.mark.parametrize("n", [1, 8])
def test_config4_decode_shapes(lib, h, m, k, n):
    assert lib.plan(1, 0, m, n, k)[0] == cb.TB200_KERNEL_SKINNY
    assert_ok(run_and_check(lib, h, m=m, n=n, k=k, mode="ex", sample=192, seed=310 + n + m % 97), f"{m}x{k} n={n}")


# config 5: MoE experts as pointer arrays (128 experts, 32 tokens each), and squares
@pytest.mark.parametrize("m,k", [(768, 2048), (2048, 768)])
def test_config5_moe_pointer_arrays(lib, h, m, k):
    assert lib.plan(1, 0, m, 32, k, 128, 1, 0, 0, 1, 1, 148)[0] == cb.TB200_KERNEL_TC
    assert_ok(run_and_check(lib, h, m=m, n=32, k=k, batch=128, mode="ptr", sample=64, seed=320 + m), f"{m}x32x{k}")


@pytest.mark.parametrize("in_t", [O.F16, O.BF16])
def test_config5_square_4096(lib, h, in_t):
    assert_ok(run_and_check(lib, h, m=4096, n=4096, k=4096, in_t=in_t, mode="ex", sample=96, seed=330), "4096^3")
