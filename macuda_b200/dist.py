"""N-sharded GEMM across the GPUs of one node: each rank computes its rows of C, NCCL all-gathers them.

The reference is single-GPU. For the largest GEMMs (lm_head, FFN, big squares) this library splits the
weight's output features - cuBLAS m under ggml's (T, N) call - across P ranks, one process per GPU:

  rank r owns weight rows [r*mp, r*mp + rows_r) with mp = ceil(m / P) (the last rank may own fewer);
  it runs cublasGemmEx(T, N, rows_r, n, k) into a local column-major block of mp x n (ldc = mp);
  an NCCL all-gather over NVLink concatenates the P blocks ([P][mp x n]) on a communication stream;
  tb200_gather_row_blocks lays them out as the column-major m x n C (ldc >= m), dropping the padding rows.

Nothing here touches another GPU's memory directly: peer data arrives through NCCL into local memory.
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
