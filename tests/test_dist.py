"""The N-sharded GEMM's host logic on CPU with two gloo ranks: shard arithmetic, the all-gather and
the row-block layout that the device gather kernel implements; and a rank that fails before its
collective (the other rank must get an error within its process-group timeout, not hang).
The GPU gather kernel itself is checked against the same host mirror in test_dist_gpu."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from macuda_b200.dist import gather_row_blocks_host, shard_rows


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_rows_cover_every_row_once():
    for m in (1, 7, 8, 128256, 14336, 1000):
        for world in (1, 2, 3, 4, 8):
            seen = []
            for r in range(world):
                first, rows, mp_ = shard_rows(m, world, r)
                assert mp_ == -(-m // world) and 0 <= rows <= mp_
                seen.extend(range(first, first + rows))
            assert seen == list(range(m))


def _worker(rank, world, port, m, n, k, fail_rank, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    try:
        rng = np.random.default_rng(0)
        W = rng.normal(size=(m, k))  # output features x in features (row i = output feature i)
        X = rng.normal(size=(k, n))
        first, rows, mpr = shard_rows(m, world, rank)
        local = np.zeros((n, mpr))  # column-major mp x n block: [column][row]
        local[:, :rows] = (W[first:first + rows] @ X).T
        if rank == fail_rank:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # the message is flushed before the process vanishes
            os._exit(0)  # leaves between steps, before joining the collective
        parts = [torch.zeros(n * mpr, dtype=torch.float64) for _ in range(world)]
        try:
            dist.all_gather(parts, torch.from_numpy(local.reshape(-1).copy()))
        except Exception as ex:  # the peer never joined: the timeout must surface as an error
            q.put((rank, "error:" + type(ex).__name__))
            return
        flat = torch.cat(parts).numpy()
        C = np.full(m * n, np.nan)
        gather_row_blocks_host(flat, world, mpr, n, m, C, m)
        want = (W @ X).T.reshape(-1)  # column-major m x n
        q.put((rank, bool(np.allclose(C, want))))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _run(world, m, n, k, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, m, n, k, fail_rank, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


@pytest.mark.parametrize("m", [64, 11])
def test_two_rank_sharded_gemm_layout(m):
    out = _run(2, m, 5, 7)
    assert out == {0: True, 1: True}, out


def test_rank_that_never_joins_surfaces_as_error():
    out = _run(2, 16, 3, 4, fail_rank=1)
    assert out[1] == "left"
    assert isinstance(out[0], str) and out[0].startswith("error:"), out
