"""Failure detection of the tensor-core kernel, without a GPU fault: every pipeline wait is bounded, and a wait
that runs out sets the kernel's abort flag, lets every copy in flight land, frees tensor memory and records an
error word that tb200_device_error() returns (and clears). The test makes one wait run out: TB200_TEST_STALL=1
has the MMA thread first wait on a barrier that nothing arrives at, and TB200_WAIT_BUDGET_CYC shortens the
pipeline waits' budget to about a millisecond (the drain waits keep theirs). The context stays usable: the next
GEMM on the same stream is checked against the oracle."""
import pytest

from tests.helpers import run_and_check

pytestmark = pytest.mark.gpu


def test_wait_that_runs_out_records_an_error_and_the_context_survives(lib, monkeypatch):
    import torch
    assert torch.cuda.is_available()
    h = lib.handle()
    assert lib.device_error() == 0  # nothing recorded before (also clears the word)
    # a small single-CTA GEMM: two 128 x 128 tiles, no k split
    monkeypatch.setenv("TB200_TC_BN", "128")
    monkeypatch.setenv("TB200_KSPLIT", "0")
    monkeypatch.setenv("TB200_WAIT_BUDGET_CYC", "2000000")
    monkeypatch.setenv("TB200_TEST_STALL", "1")
    res = run_and_check(lib, h, m=256, n=128, k=256, mode="ex", seed=41)
    assert res["status"] == 0  # the launch itself succeeded; the kernel gave up on the device
    assert lib.device_error() == 1, "the wait that nothing completes did not record its error"
    monkeypatch.delenv("TB200_TEST_STALL")
    monkeypatch.delenv("TB200_WAIT_BUDGET_CYC")
    for seed in (42, 43):  # the same shape, then the planner's own choice, on the same stream
        if seed == 43:
            monkeypatch.delenv("TB200_TC_BN")
            monkeypatch.delenv("TB200_KSPLIT")
        res = run_and_check(lib, h, m=256, n=128, k=256, mode="ex", seed=seed)
        assert res["ok"], res
    assert lib.device_error() == 0
    h.close()
