"""The sharded GEMMs on every visible GPU, up to 8 (skipped with fewer than 2): every exchange, every
rank's full C - including the rows its peers computed and delivered (over NCCL, by P2P stores from the
peers' epilogues, or by the peers' copy engines) - checked against the fp64 oracle on seeded row samples.
m is not a multiple of the rank count, so the last rank owns fewer rows. The batch-sharded form splits a
strided batch of 5 elements (a ragged share) and checks every element of every rank's C."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, m, n, k, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok, info, used = False, "", mode
    try:
        from macuda_b200 import cublas as cb
        from macuda_b200.dist import (BatchShardedGemm, CopyEngineShardedGemm, CopyStreams, FusedShardedGemm,
                                      ShardedGemm, shard_rows, step_barrier)
        from oracle import oracle as O
        lib = cb.library()
        h = lib.handle()
        stream = torch.cuda.Stream()
        h.set_stream(stream.cuda_stream)
        rng = np.random.default_rng(7)
        W = O.to_bits(rng.normal(0, 0.02, m * k).astype(np.float32), O.F16)  # m rows of k: op T, lda = k
        X = O.to_bits(rng.normal(0, 1, k * n).astype(np.float32), O.F16)
        first, rows, _ = shard_rows(m, world, rank)
        w_local = torch.from_numpy(W[first * k:(first + rows) * k].view(np.int16).copy()).cuda()
        x = torch.from_numpy(X.view(np.int16)).cuda()
        if mode == "batch":
            nb_total = 5
            Wb = O.to_bits(rng.normal(0, 0.02, nb_total * m * k).astype(np.float32), O.F16)
            Xb = O.to_bits(rng.normal(0, 1, nb_total * k * n).astype(np.float32), O.F16)
            b0, nb, _ = shard_rows(nb_total, world, rank)
            copies = CopyStreams(world)
            wl = torch.from_numpy(Wb[b0 * m * k:(b0 + max(nb, 1)) * m * k].view(np.int16).copy()).cuda()
            xl = torch.from_numpy(Xb[b0 * k * n:(b0 + max(nb, 1)) * k * n].view(np.int16).copy()).cuda()
            g = BatchShardedGemm(lib, h, m, n, k, nb_total, rank, world, wl, m * k, xl, k * n, cb.CUDA_R_16F, copies)
            g.c.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            st = 0
            for _ in range(2):
                st = st or g.run(None, stream)
                copies.join(stream)
                step_barrier(stream)
            torch.cuda.synchronize()
            C = g.c.cpu().numpy()
            rows_s = np.unique(np.concatenate([np.arange(0, m, 41), [m - 1]])).astype(np.int32)
            res = {"ok": True}
            for b in range(nb_total):
                R, S = O.gemm(1, 0, m, n, k, 1.0, Wb[b * m * k:(b + 1) * m * k], O.F16, k, Xb[b * k * n:(b + 1) * k * n],
                              O.F16, k, rows=rows_s)
                r = O.check(O.extract(C[b * m * n:(b + 1) * m * n], O.F32, m, n, m, rows=rows_s), R, S, O.F32)
                if not r["ok"]:
                    res = dict(r, element=b)
            ok, info = (st == 0 and res["ok"]), f"st={st} {res}"
            g.close()
            h.close()
            q.put((rank, ok, info, used))
            dist.destroy_process_group()
            return
        if mode == "ce":
            copies = CopyStreams(world)
            g = CopyEngineShardedGemm(lib, h, m, n, k, rank, world, w_local, cb.CUDA_R_16F, copies)
            g.c.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            st = 0
            # the second pass, in three column chunks pushed one peer after another (ring order), overwrites the
            # first in place
            for chunks, cs in ((1, copies), (3, CopyStreams(world, lanes=1))):
                g.copies = cs
                st = st or g.run(x, stream, chunks=chunks)
                cs.join(stream)
                step_barrier(stream)
            torch.cuda.synchronize()
            C = g.c.cpu().numpy()
        elif mode in ("multicast", "p2p"):
            g = FusedShardedGemm(lib, h, m, n, k, rank, world, w_local, cb.CUDA_R_16F,
                                 exchange="auto" if mode == "multicast" else "p2p")  # auto: multicast if present
            used = g.exchange
            g.c.fill_(float("nan"))
            torch.cuda.synchronize()
            dist.barrier()
            for _ in range(2):  # twice: the second run overwrites the first in place
                st = g.run(x, stream)
                step_barrier(stream)
            torch.cuda.synchronize()
            C = g.c.cpu().numpy()
        else:
            g = ShardedGemm(lib, h, m, n, k, rank, world, w_local, cb.CUDA_R_16F)
            comm = torch.cuda.Stream()
            st = g.run(x, stream, comm)
            torch.cuda.synchronize()
            C = g.c.cpu().numpy()
        rows_s = np.unique(np.concatenate([np.arange(0, m, 37), [first, m - 1]])).astype(np.int32)
        R, S = O.gemm(1, 0, m, n, k, 1.0, W, O.F16, k, X, O.F16, k, rows=rows_s)
        res = O.check(O.extract(C, O.F32, m, n, m, rows=rows_s), R, S, O.F32)
        ok, info = (st == 0 and res["ok"]), f"st={st} {res}"
        if mode in ("multicast", "p2p", "ce"):
            g.close()
        h.close()
    except Exception as ex:
        info = repr(ex)
    q.put((rank, ok, info, used))
    dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["ce", "batch", "multicast", "p2p", "allgather"])
def test_sharded_gemm_on_all_gpus(mode):
    import torch
    world = min(torch.cuda.device_count(), 8)
    if world < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    m, n, k = 4300, 512, 2048
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, m, n, k, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for rank, ok, info, used in out:
        assert ok, f"rank {rank}: {info}"
    if mode == "multicast" and any(u != "multicast" for _, _, _, u in out):
        pytest.skip("no NVLink multicast on this box (the p2p exchange ran and passed)")
