"""The device side of the N-sharded GEMM on one GPU: tb200_gather_row_blocks against its host mirror
(macuda_b200.dist.gather_row_blocks_host), f32 and 16-bit, with and without padding rows."""
import numpy as np
import pytest

from macuda_b200.dist import gather_row_blocks_host, shard_rows

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,P,n,elem", [(4096, 8, 512, 4), (1000, 3, 7, 4), (130, 4, 33, 2), (11, 2, 5, 2)])
def test_gather_row_blocks_matches_host_mirror(lib, m, P, n, elem):
    import torch
    _, _, mp = shard_rows(m, P, 0)
    rng = np.random.default_rng(m + P)
    if elem == 4:
        parts = rng.normal(size=P * mp * n).astype(np.float32)
        dparts = torch.from_numpy(parts).cuda()
        C = np.full(m * n + 3, -7.0, np.float32)
    else:
        parts = rng.integers(0, 65535, size=P * mp * n).astype(np.uint16)
        dparts = torch.from_numpy(parts.view(np.int16)).cuda()
        C = np.full(m * n + 3, 77, np.uint16)
    dC = torch.from_numpy(C.view(np.int16) if elem == 2 else C).cuda()
    st = lib.lib.tb200_gather_row_blocks(dparts.data_ptr(), P, mp, n, elem, dC.data_ptr(), m, m, None)
    torch.cuda.synchronize()
    assert st == 0
    got = dC.cpu().numpy()
    got = got.view(np.uint16) if elem == 2 else got
    want = gather_row_blocks_host(parts, P, mp, n, m, C.copy(), m)
    assert np.array_equal(got, want)
