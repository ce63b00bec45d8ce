"""N-sharded GEMM across the GPUs of one node: each rank computes its rows of C, every rank ends with all of C.

The reference is single-GPU. For the largest GEMMs (lm_head, FFN, big squares) this library splits the
weight's output features - cuBLAS m under ggml's (T, N) call - across P ranks, one process per GPU;
rank r owns weight rows [r*mp, r*mp + rows_r) with mp = ceil(m / P) (the last rank may own fewer).
Two ways to replicate C:

  FusedShardedGemm (default): the exchange is done by the tensor-core epilogue while later tiles still
    compute. By default every rank's C is mapped into every other rank (CUDA IPC) and the epilogue stores
    this rank's rows into all P replicas over NVLink P2P (tb200_gemm_ex_allgather). exchange="multicast"
    instead stores each element once to an NVLink multicast address (NVSwitch; every rank's C in symmetric
    memory bound to one multicast object) and the switch writes it into every rank's C
    (tb200_gemm_ex_multicast). That sends a rank's rows once instead of once per peer, but every rank then
    also receives its own rows back through its NVLink port: inbound traffic is all of C instead of
    (P-1)/P of it, and inbound is the bound of an all-gather, so P2P is the default (measured at P = 2:
    0.586 vs 0.778 ms per step). Either way one 4-byte NCCL all-reduce per step tells each rank that its
    peers' stores have landed.
  CopyEngineShardedGemm: the GEMM writes this rank's rows straight into its own full C (ldc = m), and the
    copy engines push that row block into every peer's C (tb200_push_block: one cudaMemcpy2DAsync per peer,
    each on its own stream). No SM time goes to the exchange, so it overlaps whatever the SMs run next -
    in the benchmark's step, the projections that run whole on every rank. `wait` joins the copies into the
    caller's stream; then the same 4-byte NCCL all-reduce tells each rank that its peers' copies have landed.
    BatchShardedGemm does the same for a strided batch split across ranks (whole batch elements per rank:
    KV-head groups of an attention GEMM, experts of an MoE layer): each rank's C slab is contiguous and is
    pushed whole.
  ShardedGemm: the GEMM writes a local mp x n block, an NCCL all-gather on a communication stream
    concatenates the P blocks, and tb200_gather_row_blocks lays them out as the column-major C.

`gather_row_blocks_host` is the host mirror of the device gather (the layout contract the tests pin).
"""
from __future__ import annotations

import numpy as np


def shard_rows(m: int, world: int, rank: int):
    """(first row, rows owned, rows per block) of rank `rank` when m rows are split across `world` ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    mp = -(-m // world)
    first = min(m, rank * mp)
    rows = max(0, min(m, first + mp) - first)
    return first, rows, mp


def gather_row_blocks_host(parts: np.ndarray, P: int, rows: int, n: int, m_total: int, C: np.ndarray, ldc: int):
    """Host mirror of tb200_gather_row_blocks: parts is the flat all-gather output (P blocks of rows x n,
    column-major, ld = rows); block r goes to rows [r*rows, (r+1)*rows) of the flat column-major C."""
    blocks = parts.reshape(P, n, rows)  # [block][column][row]
    for r in range(P):
        for i in range(rows):
            row = r * rows + i
            if row >= m_total:
                break
            C[row + np.arange(n) * ldc] = blocks[r, :, i]
    return C


class ShardedGemm:
    """One N-sharded GEMM C (m x n, f32 or 16-bit) = W^T X, as ggml issues it, on this rank's GPU.

    w_local: this rank's weight rows, stored k x rows (op T, lda = k) - a torch tensor on this GPU.
    Buffers for the local block, the all-gather output and the final C are allocated once here, so
    that `run` allocates nothing. `run` enqueues the GEMM on `stream` and the all-gather + gather on
    `comm`, and records an event the caller's next consumer of C can wait on (`done`).
    """

    def __init__(self, lib, handle, m: int, n: int, k: int, rank: int, world: int, w_local, dtype_code: int,
                 out_dtype=None, group=None):
        import torch
        self.lib, self.h = lib, handle
        self.m, self.n, self.k = m, n, k
        self.rank, self.world, self.group = rank, world, group
        self.first, self.rows, self.mp = shard_rows(m, world, rank)
        self.w = w_local
        self.dtype_code = dtype_code
        out_dtype = out_dtype or torch.float32
        self.elem = torch.empty((), dtype=out_dtype).element_size()
        self.c_local = torch.zeros(self.mp * n, device="cuda", dtype=out_dtype)
        self.gathered = torch.empty(world * self.mp * n, device="cuda", dtype=out_dtype)
        self.c = torch.empty(m * n, device="cuda", dtype=out_dtype)
        self.ready = torch.cuda.Event()
        self.done = torch.cuda.Event()

    def run(self, x, stream, comm) -> int:
        """x: activations stored k x n (op N, ldb = k), torch tensor on this GPU."""
        import torch
        import torch.distributed as dist
        from . import cublas as cb
        ctype_out = {4: cb.CUDA_R_32F, 2: cb.CUDA_R_16F}[self.elem]
        st = 0
        if self.rows > 0:
            st = self.h.gemm_ex(cb.CUBLAS_OP_T, cb.CUBLAS_OP_N, self.rows, self.n, self.k, 1.0, self.w.data_ptr(),
                                self.dtype_code, self.k, x.data_ptr(), self.dtype_code, self.k, 0.0,
                                self.c_local.data_ptr(), ctype_out, self.mp, cb.CUBLAS_COMPUTE_32F)
        self.ready.record(stream)
        comm.wait_event(self.ready)
        with torch.cuda.stream(comm):
            dist.all_gather_into_tensor(self.gathered, self.c_local, group=self.group)
            st2 = self.lib.lib.tb200_gather_row_blocks(self.gathered.data_ptr(), self.world, self.mp, self.n,
                                                       self.elem, self.c.data_ptr(), self.m, self.m, comm.cuda_stream)
        self.done.record(comm)
        return st or st2


class _DeviceArray:
    """A raw device allocation exposed to torch through __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr: int, count: int, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None, "stream": None}


class IpcReplicas:
    """A device buffer of `nbytes` on every rank, each mapped into every other rank of the group (CUDA IPC):
    `reps[q]` is rank q's buffer as a pointer valid in this process (`own` = reps[rank]). Collective: every
    rank constructs it with the same size, and closes it."""

    def __init__(self, lib, nbytes: int, rank: int, world: int, group=None):
        import ctypes

        import torch.distributed as dist
        self.lib, self.rank, self.world, self.group = lib, rank, world, group
        own = ctypes.c_void_p()
        hbuf = ctypes.create_string_buffer(64)
        st = lib.lib.tb200_ipc_alloc(nbytes, ctypes.byref(own), hbuf)
        if st != 0:
            raise RuntimeError(f"tb200_ipc_alloc: status {st}")
        self.own = own.value
        handles = [None] * world
        dist.all_gather_object(handles, hbuf.raw, group=group)
        self.reps, self.opened = [], []
        for r in range(world):
            if r == rank:
                self.reps.append(self.own)
                continue
            p = ctypes.c_void_p()
            st = lib.lib.tb200_ipc_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(p))
            if st != 0:
                raise RuntimeError(f"tb200_ipc_open (rank {r}): status {st}")
            self.reps.append(p.value)
            self.opened.append(p.value)
        self.array = (ctypes.c_void_p * world)(*self.reps)

    def close(self):
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.opened:
            self.lib.lib.tb200_ipc_close(p)
        self.opened = []
        dist.barrier(group=self.group)  # every peer has unmapped this rank's buffer before it is freed
        if self.own:
            self.lib.lib.tb200_ipc_free(self.own)
            self.own = 0


class CopyStreams:
    """Streams for the copy-engine exchange, and an event per stream that `join` records and makes another
    stream wait on. lanes = world (default): one stream per peer, every peer's copy at once; lanes = 1: one
    stream, the copies one after another in ring order from this rank (each rank sends to a different peer
    at each moment)."""

    def __init__(self, world: int, lanes: int = None):
        import ctypes

        import torch
        lanes = world if lanes is None else max(1, min(lanes, world))
        self.lanes = lanes
        self.streams = [torch.cuda.Stream() for _ in range(lanes)]
        self.array = (ctypes.c_void_p * lanes)(*[s.cuda_stream for s in self.streams])
        self.events = [torch.cuda.Event() for _ in range(world)]
        self.ready = torch.cuda.Event()

    def after(self, stream):
        """Order the copies enqueued next after everything enqueued on `stream` so far."""
        self.ready.record(stream)
        for s in self.streams:
            s.wait_event(self.ready)

    def join(self, stream):
        """Make `stream` wait for every copy enqueued so far."""
        for s, e in zip(self.streams, self.events):
            e.record(s)
            stream.wait_event(e)


class CopyEngineShardedGemm:
    """N-sharded GEMM with the exchange on the copy engines.

    Rank r's GEMM writes its rows [first, first + rows) of C straight into its own full C (leading dimension
    m) and tb200_push_block copies that row block into every peer's C. `run` splits the columns into `chunks`
    GEMMs so that the copies of one chunk overlap the next chunk's math (1 = one GEMM, then the copies). The
    copies go on `copies` (a CopyStreams shared by the step; it may be replaced between steps); then
    `copies.join(stream)` and `step_barrier` complete the exchange."""

    exchange = "ce"

    def __init__(self, lib, handle, m: int, n: int, k: int, rank: int, world: int, w_local, dtype_code: int,
                 copies: "CopyStreams", group=None, chunks: int = 1):
        import torch
        self.lib, self.h = lib, handle
        self.m, self.n, self.k = m, n, k
        self.rank, self.world, self.group = rank, world, group
        self.first, self.rows, self.mp = shard_rows(m, world, rank)
        self.w = w_local
        self.dtype_code = dtype_code
        self.copies = copies
        self.chunks = max(1, chunks)
        self.esize = torch.empty((), dtype=torch.float16).element_size()
        self.buf = IpcReplicas(lib, m * n * 4, rank, world, group)
        self.c = torch.as_tensor(_DeviceArray(self.buf.own, m * n), device="cuda")

    def run(self, x, stream=None, chunks: int = None) -> int:
        from . import cublas as cb
        chunks = self.chunks if chunks is None else max(1, chunks)
        if self.rows == 0:
            return 0
        step = -(-self.n // chunks)
        for col0 in range(0, self.n, step):
            nc = min(step, self.n - col0)
            st = self.h.gemm_ex(cb.CUBLAS_OP_T, cb.CUBLAS_OP_N, self.rows, nc, self.k, 1.0, self.w.data_ptr(),
                                self.dtype_code, self.k, x.data_ptr() + col0 * self.k * self.esize, self.dtype_code,
                                self.k, 0.0, self.buf.own + (self.first + col0 * self.m) * 4, cb.CUDA_R_32F, self.m,
                                cb.CUBLAS_COMPUTE_32F)
            if st != 0:
                return st
            self.copies.after(stream)
            st = self.lib.lib.tb200_push_block(self.buf.array, self.world, self.rank, self.first, self.rows, col0, nc,
                                               self.m, 4, self.copies.array, self.copies.lanes)
            if st != 0:
                return st
        return 0

    def close(self):
        self.c = None
        self.buf.close()


class BatchShardedGemm:
    """A strided-batched GEMM (T, N, f32 C) split across ranks by whole batch elements: rank r computes
    elements [b0, b0 + nb) (bshard of them per rank, the last rank possibly fewer) into its slab of its own
    full C and the copy engines push the slab into every peer's C. The slabs are contiguous because C's batch
    stride is m * n: they all-gather straight into C. A, B: this rank's elements only (strides sA, sB)."""

    exchange = "ce"

    def __init__(self, lib, handle, m: int, n: int, k: int, batch: int, rank: int, world: int, A_local, sA: int,
                 B_local, sB: int, dtype_code: int, copies: "CopyStreams", group=None):
        import torch
        self.lib, self.h = lib, handle
        self.m, self.n, self.k, self.batch = m, n, k, batch
        self.rank, self.world = rank, world
        self.b0, self.nb, self.bshard = shard_rows(batch, world, rank)
        self.A, self.sA, self.B, self.sB = A_local, sA, B_local, sB
        self.dtype_code = dtype_code
        self.copies = copies
        self.buf = IpcReplicas(lib, batch * m * n * 4, rank, world, group)
        self.c = torch.as_tensor(_DeviceArray(self.buf.own, batch * m * n), device="cuda")

    def compute(self, stream=None) -> int:
        from . import cublas as cb
        if self.nb == 0:
            return 0
        return self.h.gemm_strided_batched_ex(cb.CUBLAS_OP_T, cb.CUBLAS_OP_N, self.m, self.n, self.k, 1.0,
                                              self.A.data_ptr(), self.dtype_code, self.k, self.sA, self.B.data_ptr(),
                                              self.dtype_code, self.k, self.sB, 0.0,
                                              self.buf.own + self.b0 * self.m * self.n * 4, cb.CUDA_R_32F, self.m,
                                              self.m * self.n, self.nb, cb.CUBLAS_COMPUTE_32F)

    def push(self, stream=None) -> int:
        if self.nb == 0:
            return 0
        self.copies.after(stream)
        slab = self.m * self.n
        return self.lib.lib.tb200_push_block(self.buf.array, self.world, self.rank, self.b0 * slab, self.nb * slab, 0, 1,
                                             self.batch * slab, 4, self.copies.array, self.copies.lanes)

    def run(self, x=None, stream=None) -> int:
        return self.compute(stream) or self.push(stream)

    def close(self):
        self.c = None
        self.buf.close()


class FusedShardedGemm:
    """N-sharded GEMM with the output exchange fused into the tensor-core epilogue.

    exchange="multicast": every rank's full C (m x n, f32) is one symmetric-memory buffer (torch's CUDA
    symmetric memory, bound to an NVLink multicast object); `run` launches tb200_gemm_ex_multicast, whose
    epilogue stores each element of this rank's rows once to the multicast address.
    exchange="p2p": every rank allocates its C with tb200_ipc_alloc, the 64-byte IPC handles are
    all-gathered, each rank maps every peer's C (tb200_ipc_open), and `run` launches
    tb200_gemm_ex_allgather, whose epilogue stores this rank's rows into all P replicas.
    exchange="auto": multicast when every rank has a multicast address, else p2p. Default: "p2p".
    No all-gather call, no layout kernel. After the last GEMM of a step, `step_barrier` (a 4-byte NCCL
    all-reduce on the compute stream) tells every rank that all peers' kernels, and so their stores into
    its C, have completed.
    """

    def __init__(self, lib, handle, m: int, n: int, k: int, rank: int, world: int, w_local, dtype_code: int,
                 group=None, exchange: str = "p2p"):
        import ctypes

        import torch
        import torch.distributed as dist
        self.lib, self.h = lib, handle
        self.m, self.n, self.k = m, n, k
        self.rank, self.world, self.group = rank, world, group
        self.first, self.rows, self.mp = shard_rows(m, world, rank)
        self.w = w_local
        self.dtype_code = dtype_code
        self.mc, self._symm, self.own, self.opened = 0, None, 0, []
        if exchange not in ("auto", "multicast", "p2p"):
            raise ValueError(f"exchange {exchange!r}")
        if exchange != "p2p":
            buf, hdl, mc = None, None, 0
            try:
                import torch.distributed._symmetric_memory as symm_mem
                buf = symm_mem.empty(m * n, dtype=torch.float32, device=torch.device("cuda", torch.cuda.current_device()))
                hdl = symm_mem.rendezvous(buf, group if group is not None else dist.group.WORLD)
                mc = int(getattr(hdl, "multicast_ptr", 0) or 0)
            except Exception:
                mc = 0
            have = torch.tensor([1 if mc else 0], dtype=torch.int32, device="cuda")
            dist.all_reduce(have, op=dist.ReduceOp.MIN, group=group)  # every rank takes the same exchange
            if int(have.item()) == 1:
                self.mc, self._symm, self.c = mc, (buf, hdl), buf
                self.exchange = "multicast"
                return
            if exchange == "multicast":
                raise RuntimeError("NVLink multicast is not available on every rank")
            del buf, hdl
        self.exchange = "p2p"
        own = ctypes.c_void_p()
        hbuf = ctypes.create_string_buffer(64)
        st = lib.lib.tb200_ipc_alloc(m * n * 4, ctypes.byref(own), hbuf)
        if st != 0:
            raise RuntimeError(f"tb200_ipc_alloc: status {st}")
        handles = [None] * world
        dist.all_gather_object(handles, hbuf.raw, group=group)
        self.reps, self.opened = [], []
        for r in range(world):
            if r == rank:
                self.reps.append(own.value)
                continue
            p = ctypes.c_void_p()
            st = lib.lib.tb200_ipc_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(p))
            if st != 0:
                raise RuntimeError(f"tb200_ipc_open (rank {r}): status {st}")
            self.reps.append(p.value)
            self.opened.append(p.value)
        self.own = own.value
        self.rep_array = (ctypes.c_void_p * world)(*self.reps)
        self.c = torch.as_tensor(_DeviceArray(self.own, m * n), device="cuda")

    def run(self, x, stream=None) -> int:
        import ctypes
        from . import cublas as cb
        if self.rows == 0:
            return 0
        one = ctypes.c_float(1.0)
        if self.mc:
            return self.lib.lib.tb200_gemm_ex_multicast(
                self.h.h, cb.CUBLAS_OP_T, cb.CUBLAS_OP_N, self.rows, self.n, self.k, ctypes.byref(one),
                self.w.data_ptr(), self.dtype_code, self.k, x.data_ptr(), self.dtype_code, self.k, self.mc,
                cb.CUDA_R_32F, self.m, self.first, cb.CUBLAS_COMPUTE_32F)
        return self.lib.lib.tb200_gemm_ex_allgather(
            self.h.h, cb.CUBLAS_OP_T, cb.CUBLAS_OP_N, self.rows, self.n, self.k, ctypes.byref(one), self.w.data_ptr(),
            self.dtype_code, self.k, x.data_ptr(), self.dtype_code, self.k, self.rep_array, self.world, cb.CUDA_R_32F,
            self.m, self.first, cb.CUBLAS_COMPUTE_32F)

    def close(self):
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        if self._symm is not None:  # symmetric memory: released once no rank can still write into it
            self._symm, self.c, self.mc = None, None, 0
            dist.barrier(group=self.group)
            return
        for p in self.opened:
            self.lib.lib.tb200_ipc_close(p)
        self.opened = []
        dist.barrier(group=self.group)  # every peer has unmapped this rank's C before it is freed
        if self.own:
            self.lib.lib.tb200_ipc_free(self.own)
            self.own = 0


def step_barrier(stream, group=None, _flag={}):
    """A 4-byte NCCL all-reduce on `stream`: when it completes on a rank, every rank's earlier kernels on
    its stream - and so every peer store into this rank's replicas - have completed."""
    import torch
    import torch.distributed as dist
    dev = torch.cuda.current_device()
    if dev not in _flag:
        _flag[dev] = torch.zeros(1, dtype=torch.int32, device="cuda")
    with torch.cuda.stream(stream):
        dist.all_reduce(_flag[dev], group=group)


class ReplicatedGemm:
    """The whole GEMM on this rank (the full weight, the full C): every rank computes the same C and nothing
    is exchanged. For projections whose shards would be too small to use the GPU, or whose C costs more to
    exchange than to compute again (see pick_fastest)."""

    exchange = "replicated"

    def __init__(self, lib, handle, m: int, n: int, k: int, w_full, dtype_code: int):
        import torch
        self.lib, self.h = lib, handle
        self.m, self.n, self.k = m, n, k
        self.w = w_full
        self.dtype_code = dtype_code
        self.c = torch.empty(m * n, device="cuda", dtype=torch.float32)

    def run(self, x, stream=None) -> int:
        from . import cublas as cb
        return self.h.gemm_ex(cb.CUBLAS_OP_T, cb.CUBLAS_OP_N, self.m, self.n, self.k, 1.0, self.w.data_ptr(),
                              self.dtype_code, self.k, x.data_ptr(), self.dtype_code, self.k, 0.0, self.c.data_ptr(),
                              cb.CUDA_R_32F, self.m, cb.CUBLAS_COMPUTE_32F)

    def close(self):
        self.c = None


def pick_fastest(candidates: dict, x, stream, group=None, warmup: int = 3, iters: int = 10) -> str:
    """Time each candidate's run(x, stream) on this rank (CUDA events around `iters` back-to-back calls after
    `warmup`), take the maximum over ranks, and return the key of the fastest: the same on every rank.
    Every rank must call it with the same candidates in the same order."""
    import torch
    import torch.distributed as dist
    keys = list(candidates)
    times = torch.zeros(len(keys), dtype=torch.float64, device="cuda")
    for i, key in enumerate(keys):
        c = candidates[key]
        for _ in range(warmup):
            if c.run(x, stream) != 0:
                raise RuntimeError(f"{key}: GEMM failed")
        torch.cuda.synchronize()
        dist.barrier(group=group)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(iters):
            c.run(x, stream)
        e1.record(stream)
        torch.cuda.synchronize()
        times[i] = e0.elapsed_time(e1) / iters
        dist.barrier(group=group)  # peers' stores into this rank's buffers are done before the next candidate
    dist.all_reduce(times, op=dist.ReduceOp.MAX, group=group)
    return keys[int(torch.argmin(times).item())]

