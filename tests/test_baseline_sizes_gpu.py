"""Parity at every BASELINE size the benchmark times, each GEMM as ggml issues it (T, N, f32 C), checked
against the fp64 oracle on seeded row and column samples that always include the rows and columns around
the last boundary of every tile width (so the last, possibly partial, m-tile and n-tile of each kernel
configuration are checked), with the gate of oracle.check.

* configs[1] (the headline step) in both 16-bit input types, each projection on the kernel configuration the
  planner picks for it on a 148-SM B200: lm_head 128256 x 512 x 4096 on the 256 x 256 CTA-pair tile over
  about a thousand tiles (several waves of the persistent scheduler), down 4096 x 512 x 14336 on the split
  pair tile, gate/up, Q/O and K/V.
* config 5 squares 8192^3 and 16384^3, f16 and bf16.
* config 4 decode against the vocabulary-sized weight, 128256 x 4096, at n = 1 and 8.

The reference's habit: value checks over many blocks (cuda-shim/test/link_smoke.c:38-46) against an fp64
host result (cuda-shim/libtinycublas/splitk-20260923/test_splitk.cu:139-140).
"""
import pytest

from macuda_b200 import cublas as cb
from oracle import oracle as O
from tests.helpers import run_and_check

pytestmark = pytest.mark.gpu

TYPES = [O.F16, O.BF16]
TNAME = {O.F16: "f16", O.BF16: "bf16"}


@pytest.fixture(scope="module")
def h(lib):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    hh = lib.handle()
    yield hh
    hh.close()


def sms():
    import torch
    return torch.cuda.get_device_properties(0).multi_processor_count


# (name, m, k, the planner's choice on 148 SMs: (kernel, tile) as CublasLib.plan reports it)
PROJECTIONS = [
    ("q_o", 4096, 4096, None),
    ("k_v", 1024, 4096, None),
    ("gate_up", 14336, 4096, (cb.TB200_KERNEL_TC, 512)),
    ("down", 4096, 14336, None),
    ("lm_head", 128256, 4096, (cb.TB200_KERNEL_TC, 512)),
]


@pytest.mark.parametrize("in_t", TYPES, ids=[TNAME[t] for t in TYPES])
@pytest.mark.parametrize("name,m,k,plan", PROJECTIONS, ids=[p[0] for p in PROJECTIONS])
def test_config1_projection_at_size(lib, h, name, m, k, plan, in_t):
    kind, tile = lib.plan(1, 0, m, 512, k, 1, in_t, O.F32, 0, 0, 1, sms())
    assert kind == cb.TB200_KERNEL_TC
    if plan is not None and sms() == 148:
        assert (kind, tile) == plan, (name, kind, tile)
    res = run_and_check(lib, h, m=m, n=512, k=k, in_t=in_t, mode="ex", sample=224, edges=True,
                        seed=900 + m % 1000 + k % 97 + in_t)
    assert res.get("ok"), f"{name} {TNAME[in_t]} ({kind}, tile {tile}): {res}"


def test_down_takes_the_split_pair_tile(lib):
    """down 4096 x 512 x 14336 is planned on two CTA pairs per 256 x 256 tile (k split) on a 148-SM B200; the
    test above checks it as planned."""
    if sms() != 148:
        pytest.skip("plan rows are for 148 SMs")
    assert lib.plan(1, 0, 4096, 512, 14336, 1, 1, 0, 0, 0, 1, 148) == (cb.TB200_KERNEL_TC, -512)


@pytest.mark.parametrize("in_t", TYPES, ids=[TNAME[t] for t in TYPES])
@pytest.mark.parametrize("S", [8192, 16384])
def test_config5_square_at_size(lib, h, S, in_t):
    res = run_and_check(lib, h, m=S, n=S, k=S, in_t=in_t, mode="ex", sample=160, edges=True, seed=950 + S % 991 + in_t)
    assert res.get("ok"), f"{S}^3 {TNAME[in_t]}: {res}"


@pytest.mark.parametrize("n", [1, 8])
@pytest.mark.parametrize("in_t", TYPES, ids=[TNAME[t] for t in TYPES])
def test_config4_decode_vocabulary_weight(lib, h, n, in_t):
    assert lib.plan(1, 0, 128256, n, 4096, 1, in_t)[0] == cb.TB200_KERNEL_SKINNY
    res = run_and_check(lib, h, m=128256, n=n, k=4096, in_t=in_t, mode="ex", sample=512, edges=True,
                        seed=970 + n + in_t)
    assert res.get("ok"), f"128256 x {n} x 4096 {TNAME[in_t]}: {res}"
