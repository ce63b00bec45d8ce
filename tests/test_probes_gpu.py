"""The HBM bandwidth probes tb200_bw_write / tb200_bw_read (reference cuda-shim/libtinycublas/gemm.cu:421-431,
driven by cuda-shim/test/bw_bench.c:19-28): the write probe fills every 16-byte word of a buffer with one
value; the read probe streams a buffer and keeps a word only when its thread's sum equals a sentinel, so
that the loads cannot be dropped."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SENTINEL = np.float32(1.234567e30)  # the read probe's sentinel sum (aux_kernels.cu)


def test_write_probe_fills_the_buffer(lib):
    import torch
    n4 = (64 << 20) // 16 + 3  # not a multiple of the grid: the grid-stride tail is covered
    buf = torch.full(((n4 + 16) * 4,), -1.0, device="cuda", dtype=torch.float32)  # 16 words past the range
    st = lib.lib.tb200_bw_write(buf.data_ptr(), n4, ctypes.c_float(2.5), None)
    torch.cuda.synchronize()
    assert st == 0
    assert bool((buf[:n4 * 4] == 2.5).all()), "some word was not written"
    assert bool((buf[n4 * 4:] == -1.0).all()), "a word past the range was written"
    # a second pattern over a prefix only
    st = lib.lib.tb200_bw_write(buf.data_ptr(), 1000, ctypes.c_float(-7.0), None)
    torch.cuda.synchronize()
    assert st == 0
    assert bool((buf[:4000] == -7.0).all()) and bool((buf[4000:n4 * 4] == 2.5).all())


def test_read_probe_reads_and_keeps_the_sentinel(lib):
    import torch
    sink = torch.zeros(1, device="cuda")
    # many words whose per-thread sums are far from the sentinel: the sink stays untouched
    buf = torch.ones((32 << 20) // 4, device="cuda")
    assert lib.lib.tb200_bw_read(buf.data_ptr(), buf.numel() // 4, sink.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert float(sink.item()) == 0.0
    # one word whose components sum to the sentinel: its thread stores the sum, so the loads really happened
    one = torch.tensor([float(SENTINEL), 0.0, 0.0, 0.0], device="cuda")
    assert lib.lib.tb200_bw_read(one.data_ptr(), 1, sink.data_ptr(), None) == 0
    torch.cuda.synchronize()
    assert np.float32(sink.item()) == SENTINEL
    # an empty range launches nothing
    assert lib.lib.tb200_bw_read(one.data_ptr(), 0, sink.data_ptr(), None) == 0


def test_probe_bandwidth_is_plausible(lib):
    """512 MiB each way: both probes run at a sizeable fraction of HBM (a probe that skipped its loads or
    stores would show an impossible rate, one that faulted would fail the sync)."""
    import torch
    n4 = (512 << 20) // 16
    buf = torch.empty(n4 * 4, device="cuda")
    sink = torch.zeros(1, device="cuda")
    s = torch.cuda.current_stream()
    rates = {}
    for name in ("write", "read"):
        def call():
            if name == "write":
                return lib.lib.tb200_bw_write(buf.data_ptr(), n4, ctypes.c_float(1.0), ctypes.c_void_p(s.cuda_stream))
            return lib.lib.tb200_bw_read(buf.data_ptr(), n4, sink.data_ptr(), ctypes.c_void_p(s.cuda_stream))
        assert call() == 0
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(10):
            call()
        e1.record(s)
        torch.cuda.synchronize()
        rates[name] = n4 * 16 * 10 / (e0.elapsed_time(e1) * 1e-3) / 1e9
    assert 1000 < rates["write"] < 12000, rates
    assert 1000 < rates["read"] < 12000, rates
