#!/usr/bin/env python3
"""Benchmark of libtinycublas_b200 on its headline workload (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--dtype f16|bf16]

Workload: the Llama-3.1-8B-shaped prefill projection set at 512 tokens, issued as
ggml-cuda issues it: cublasGemmEx(T, N, m = out features, n = 512, k = in features, fp16 weights
N(0, 0.02^2), fp16 activations N(0, 1), f32 C, COMPUTE_32F). One step = the 8 projections Q 4096->4096,
K 4096->1024, V 4096->1024, O 4096->4096, gate and up 4096->14336, down 14336->4096, lm_head
4096->128256 (761.2 GFLOP). Synthetic seeded data of those shapes; weights are random, not a checkpoint.
Inputs are larger than L2 (1.9 GB touched per step), so no flush is needed between steps.

At N > 1 (torchrun, one process per GPU, NCCL): every projection is N-sharded along m (the weight's
output features); each rank computes its m/N rows and its GEMM epilogue stores them into every rank's
C over NVLink P2P (CUDA IPC mappings, macuda_b200.dist.FusedShardedGemm), with one 4-byte NCCL
all-reduce per step as the completion barrier. --exchange multicast stores each element once to an
NVLink multicast address instead (symmetric memory; slower for this all-gather, see macuda_b200/dist.py);
--exchange allgather uses an NCCL all-gather + layout kernel. Total work is fixed, so scaling is
"strong".

Keys beyond the base contract: roofline (dominant kernel = the lm_head GEMM), cpu_baseline (the
oracle's multithreaded fp16 GEMM on the host, a stand-in for ggml-cpu), e2e (the same step through the
public API with host buffers: H2D of the step's activations and D2H of the last token's logits), per
projection figures, decode (n <= 8) HBM bandwidth figures (config 4), and configs 3 and 5 figures
(attention batched GEMMs, MoE pointer-array GEMMs, squares).

--impl reference runs the same step through the reference's own libtinycublas (its cublas.c and gemm.cu,
compiled from source for sm_100a by oracle/build_ref.sh): the reference's implementation of this path
is GPU code, so it is timed on the same B200.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TOKENS = 512
HIDDEN, KV, FFN, VOCAB = 4096, 1024, 14336, 128256
# (name, m = out features, k = in features, which activation feeds it)
PROJECTIONS = [
    ("q", HIDDEN, HIDDEN, "x"), ("k", KV, HIDDEN, "x"), ("v", KV, HIDDEN, "x"), ("o", HIDDEN, HIDDEN, "x"),
    ("gate", FFN, HIDDEN, "x"), ("up", FFN, HIDDEN, "x"), ("down", HIDDEN, FFN, "h"), ("lm_head", VOCAB, HIDDEN, "x"),
]
STEP_FLOP = sum(2.0 * m * TOKENS * k for _, m, k, _ in PROJECTIONS)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d["bf16_tflops_sustained"], "source": "measured"}
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms while running."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.samples = []
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), line.strip()))

    def mark(self, begin: bool):
        if begin:
            self.t0 = time.time()
        else:
            self.t1 = time.time()

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = [s for t, s in self.samples if self.t0 is None or (self.t0 - 0.15 <= t <= (self.t1 or t) + 0.15)]
        if not rows:
            rows = [s for _, s in self.samples]
        sm, smax, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            p = [x.strip() for x in r.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                smax = max(smax, float(p[2]))
            except ValueError:
                continue
            for name, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons), "samples": len(sm)}


def make_inputs(torch, rank, world, dtype, seed=1234):
    """Weights (each projection's full matrix, the same on every rank, stored k x m: op T, lda = k; "w" is
    this rank's m/world rows of it) and activations."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    acts = {
        "x": (torch.randn(TOKENS, HIDDEN, device="cuda", generator=g)).to(dtype).contiguous(),  # B: k x n, ldb = k
        "h": (torch.randn(TOKENS, FFN, device="cuda", generator=g)).to(dtype).contiguous(),
    }
    from macuda_b200.dist import shard_rows
    layers = []
    for name, m, k, src in PROJECTIONS:
        first, rows, mp = shard_rows(m, world, rank)
        gw = torch.Generator(device="cuda")
        gw.manual_seed(seed * 131 + sum(map(ord, name)) * 7)
        w_full = (torch.randn(m, k, device="cuda", generator=gw) * 0.02).to(dtype)  # row r = output feature r
        w = w_full if world == 1 else w_full[first:first + max(rows, 1)].clone()
        c = torch.empty(m * TOKENS, device="cuda", dtype=torch.float32) if world == 1 else None
        layers.append({"name": name, "m": m, "mp": rows, "k": k, "src": src, "w": w, "w_full": w_full, "c_local": c})
    return acts, layers


def gemm_call(h, cb, layer, act, ctype, out_ptr, ldc):
    k, mp = layer["k"], layer["mp"]
    return h.gemm_ex(cb.CUBLAS_OP_T, cb.CUBLAS_OP_N, mp, TOKENS, k, 1.0, layer["w"].data_ptr(), ctype, k,
                     act.data_ptr(), ctype, k, 0.0, out_ptr, cb.CUDA_R_32F, ldc, cb.CUBLAS_COMPUTE_32F)


def run_cpu_baseline():
    """The oracle's fp16 GEMM on the host cores, on a bounded sample of the workload: the Q, K, V and O
    projections of one step (41.9 GFLOP)."""
    import numpy as np
    from oracle import oracle as O
    rng = np.random.default_rng(5)
    x = O.to_bits(rng.normal(0, 1, HIDDEN * TOKENS).astype(np.float32), O.F16)
    total, t = 0.0, 0.0
    for name, m, k, _ in PROJECTIONS[:4]:
        w = O.to_bits(rng.normal(0, 0.02, m * k).astype(np.float32), O.F16)
        c = np.empty(m * TOKENS, np.float32)
        t0 = time.perf_counter()
        O.cpu_gemm_f16_tn(m, TOKENS, k, w, k, x, k, c, m, 0)
        t += time.perf_counter() - t0
        total += 2.0 * m * TOKENS * k
    cores = O.max_threads()
    return {"value": round(total / t / 1e12, 5), "unit": "TFLOP/s", "cores": cores, "kind": "port",
            "sample": "Q, K, V, O projections of one step (41.9 GFLOP), fp16 in, f32 out, oracle/gemm_oracle.c "
                      "orc_cpu_gemm_f16_tn (F16C + AVX2 FMA + OpenMP; stand-in for ggml-cpu, absent from the tree)",
            "seconds": round(t, 3)}


def decode_figures(torch, lib, cb, dtype_code, dtype):
    """Config 4: n in {1, 2, 4, 8} against the four weight shapes, HBM GB/s of the skinny kernel.
    Weight copies rotate so that the bytes touched per pass exceed twice L2."""
    out = {}
    h = lib.handle()
    s = torch.cuda.current_stream()
    h.set_stream(s.cuda_stream)
    for (m, k) in [(4096, 4096), (14336, 4096), (4096, 14336), (128256, 4096)]:
        wbytes = m * k * 2
        copies = max(1, min(16, (300 << 20) // wbytes + 1))
        ws = [torch.randn(m, k, device="cuda").mul_(0.02).to(dtype) for _ in range(copies)]
        for n in (1, 2, 4, 8):
            x = torch.randn(n, k, device="cuda").to(dtype)
            c = torch.empty(m * n, device="cuda")
            reps = max(4 * copies, 20)

            def one(i):
                return h.gemm_ex(1, 0, m, n, k, 1.0, ws[i % copies].data_ptr(), dtype_code, k, x.data_ptr(),
                                 dtype_code, k, 0.0, c.data_ptr(), cb.CUDA_R_32F, m, cb.CUBLAS_COMPUTE_32F)
            for i in range(copies):
                one(i)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            e0.record(s)
            for i in range(reps):
                one(i)
            e1.record(s)
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / reps
            byts = m * k * 2 + n * k * 2 + m * n * 4
            out[f"{m}x{k}_n{n}"] = {"us": round(us, 2), "GB/s": round(byts / us / 1e3, 1)}
        del ws
    h.close()
    return out


def config_figures(torch, lib, cb, dtype_code, dtype, only=None, reps_override=None):
    """Configs 3 and 5: attention batched GEMMs (strided with the GQA heads folded into n, and pointer arrays
    with each KV head's pointer repeated for its 4 query heads), MoE expert GEMMs (pointer arrays over 128
    experts, 32 tokens each) and square GEMMs, all T,N with f32 C as ggml issues them. Per case: device
    time (CUDA events around back-to-back calls, median of 3 repeats), TFLOP/s, compulsory bytes / time, and
    the fraction of the measured peak of its bound (HBM copy bandwidth, or burst bf16 tensor throughput).
    only: run just the case of that name (bench.py --case, for profiling one kernel)."""
    pk = peaks()
    out = {}
    h = lib.handle()
    s = torch.cuda.current_stream()
    h.set_stream(s.cuda_stream)
    f32 = cb.CUDA_R_32F

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, device="cuda") * scale).to(dtype)

    def table(ptrs):
        return torch.tensor(ptrs, dtype=torch.int64, device="cuda")

    def measure(name, call, reps, flop, byts, bound):
        if only is not None and name != only:
            return
        if reps_override:
            reps = reps_override
        for _ in range(2):
            st = call()
            if st != 0:
                out[name] = {"status": st}
                return
        torch.cuda.synchronize()
        ts = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(reps):
                call()
            e1.record(s)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / reps)
        us = statistics.median(ts)
        tf, gbs = flop / us / 1e6, byts / us / 1e3
        frac = gbs / pk["hbm_gbs"] if bound == "hbm" else tf / pk["bf16_tflops"]
        out[name] = {"us": round(us, 2), "TFLOP/s": round(tf, 1), "GB/s": round(gbs, 1), "bound": bound,
                     "frac_of_measured_peak": round(frac, 3)}

    # config 3: 32 query heads / 8 KV heads, head_dim 128, 512 queries, 4096 keys
    Hq, Hkv, D, Tq, Tk = 32, 8, 128, 512, 4096
    g = Hq // Hkv
    K = rnd(Hkv, Tk, D)          # per KV head: k = D x m = Tk (op T, lda = D)
    Q = rnd(Hq, Tq, D)           # per query head: k = D x n = Tq (ldb = D); heads of a group are adjacent
    V = rnd(Hkv, D, Tk)          # per KV head: k = Tk x m = D (op T, lda = Tk)
    P = rnd(Hq, Tq, Tk)          # per query head: k = Tk x n = Tq (ldb = Tk)
    Ckq = torch.empty(Hq * Tk * Tq, device="cuda")
    Ckqv = torch.empty(Hq * D * Tq, device="cuda")
    flop3 = 2.0 * Tk * Tq * D * Hq
    b_kq = (K.numel() + Q.numel()) * 2 + Ckq.numel() * 4
    b_kqv = (V.numel() + P.numel()) * 2 + Ckqv.numel() * 4
    measure("c3_kq_strided_folded", lambda: h.gemm_strided_batched_ex(
        1, 0, Tk, g * Tq, D, 1.0, K.data_ptr(), dtype_code, D, Tk * D, Q.data_ptr(), dtype_code, D, g * Tq * D, 0.0,
        Ckq.data_ptr(), f32, Tk, Tk * g * Tq, Hkv), 10, flop3, b_kq, "hbm")
    measure("c3_kqv_strided_folded", lambda: h.gemm_strided_batched_ex(
        1, 0, D, g * Tq, Tk, 1.0, V.data_ptr(), dtype_code, Tk, D * Tk, P.data_ptr(), dtype_code, Tk, g * Tq * Tk, 0.0,
        Ckqv.data_ptr(), f32, D, D * g * Tq, Hkv), 10, flop3, b_kqv, "hbm")
    es = 2
    kq_a = table([K.data_ptr() + (b // g) * Tk * D * es for b in range(Hq)])
    kq_b = table([Q.data_ptr() + b * Tq * D * es for b in range(Hq)])
    kq_c = table([Ckq.data_ptr() + b * Tk * Tq * 4 for b in range(Hq)])
    kqv_a = table([V.data_ptr() + (b // g) * D * Tk * es for b in range(Hq)])
    kqv_b = table([P.data_ptr() + b * Tq * Tk * es for b in range(Hq)])
    kqv_c = table([Ckqv.data_ptr() + b * D * Tq * 4 for b in range(Hq)])
    measure("c3_kq_pointer_gqa", lambda: h.gemm_batched_ex(
        1, 0, Tk, Tq, D, 1.0, kq_a.data_ptr(), dtype_code, D, kq_b.data_ptr(), dtype_code, D, 0.0, kq_c.data_ptr(), f32,
        Tk, Hq), 10, flop3, b_kq, "hbm")
    measure("c3_kqv_pointer_gqa", lambda: h.gemm_batched_ex(
        1, 0, D, Tq, Tk, 1.0, kqv_a.data_ptr(), dtype_code, Tk, kqv_b.data_ptr(), dtype_code, Tk, 0.0, kqv_c.data_ptr(),
        f32, D, Hq), 10, flop3, b_kqv, "hbm")
    del K, Q, V, P, Ckq, Ckqv

    # config 5 MoE: 128 experts, hidden 2048, expert FFN 768, 32 tokens per expert (balanced top-8 routing)
    E, Hd, Fe, Te = 128, 2048, 768, 32
    Wgu = rnd(E, Fe, Hd, scale=0.02)   # per expert: k = Hd x m = Fe (op T, lda = Hd)
    Wd = rnd(E, Hd, Fe, scale=0.02)    # per expert: k = Fe x m = Hd
    Xe = rnd(E, Te, Hd)                # tokens gathered per expert: k = Hd x n = Te
    He = rnd(E, Te, Fe)
    Cgu = torch.empty(E * Fe * Te, device="cuda")
    Cd = torch.empty(E * Hd * Te, device="cuda")
    flop5 = 2.0 * Fe * Te * Hd * E
    pa = table([Wgu.data_ptr() + e * Fe * Hd * es for e in range(E)])
    pb = table([Xe.data_ptr() + e * Te * Hd * es for e in range(E)])
    pc = table([Cgu.data_ptr() + e * Fe * Te * 4 for e in range(E)])
    measure("c5_moe_gate_up_pointer", lambda: h.gemm_batched_ex(
        1, 0, Fe, Te, Hd, 1.0, pa.data_ptr(), dtype_code, Hd, pb.data_ptr(), dtype_code, Hd, 0.0, pc.data_ptr(), f32,
        Fe, E), 10, flop5, (Wgu.numel() + Xe.numel()) * 2 + Cgu.numel() * 4, "hbm")
    pa = table([Wd.data_ptr() + e * Hd * Fe * es for e in range(E)])
    pb = table([He.data_ptr() + e * Te * Fe * es for e in range(E)])
    pc = table([Cd.data_ptr() + e * Hd * Te * 4 for e in range(E)])
    measure("c5_moe_down_pointer", lambda: h.gemm_batched_ex(
        1, 0, Hd, Te, Fe, 1.0, pa.data_ptr(), dtype_code, Fe, pb.data_ptr(), dtype_code, Fe, 0.0, pc.data_ptr(), f32,
        Hd, E), 10, flop5, (Wd.numel() + He.numel()) * 2 + Cd.numel() * 4, "hbm")
    # the same experts through the grouped GEMM (one launch, per-expert token counts on the device): balanced
    # routing as above, then a skewed routing of the same 4096 token-slots (Dirichlet(0.3) shares, seeded)
    import numpy as np
    Xall = Xe.reshape(E * Te, Hd)  # the tokens of all experts, one expert after another: k = Hd x n = 4096
    Call = torch.empty(E * Te * Fe, device="cuda")
    skew = np.random.default_rng(5).multinomial(E * Te, np.random.default_rng(6).dirichlet(np.full(E, 0.3)))
    grouped = hasattr(lib.lib, "tb200_gemm_grouped_ex")  # this library's extension; the reference has none
    for label, counts in (("balanced", np.full(E, Te)), ("skewed", skew)) if grouped else ():
        offs = torch.from_numpy(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)).cuda()
        used = int(np.count_nonzero(counts))  # an expert without tokens never reads its weights
        measure(f"c5_moe_gate_up_grouped_{label}", lambda: h.gemm_grouped_ex(
            1, 0, Fe, E * Te, Hd, E, offs.data_ptr(), 1.0, Wgu.data_ptr(), dtype_code, Hd, Fe * Hd, Xall.data_ptr(),
            dtype_code, Hd, 0.0, Call.data_ptr(), f32, Fe), 10, flop5,
            (used * Fe * Hd + Xe.numel()) * 2 + Call.numel() * 4, "hbm")
        if f"c5_moe_gate_up_grouped_{label}" in out:
            out[f"c5_moe_gate_up_grouped_{label}"]["experts_with_tokens"] = used
    if grouped:
        # a routed layer end to end with the skewed routing, top-8 over 128 experts for 512 tokens: tokens
        # gathered into expert order, up projection (all experts, one launch), down projection (its 16-bit
        # input stands in for the activation's output), outputs combined back per token with the weights
        T, topk = 512, 8
        rng = np.random.default_rng(7)
        share = rng.dirichlet(np.full(E, 0.3))
        ex = np.stack([rng.choice(E, topk, replace=False, p=share) for _ in range(T)]).astype(np.int32)
        wts = rng.uniform(0.1, 1.0, (T, topk)).astype(np.float32)
        wts /= wts.sum(axis=1, keepdims=True)
        order = np.argsort(ex.ravel(), kind="stable")
        pos = np.empty(T * topk, np.int32)
        pos[order] = np.arange(T * topk, dtype=np.int32)
        offs = torch.from_numpy(np.concatenate([[0], np.cumsum(np.bincount(ex.ravel(), minlength=E))])
                                .astype(np.int32)).cuda()
        ids = torch.from_numpy((order // topk).astype(np.int32)).cuda()
        d_pos, d_w = torch.from_numpy(pos).cuda(), torch.from_numpy(wts.ravel().copy()).cuda()
        Xtok = rnd(T, Hd)
        Xp = torch.empty(T * topk, Hd, device="cuda", dtype=dtype)
        Cup = torch.empty(T * topk * Fe, device="cuda")
        Hp = rnd(T * topk, Fe)
        Cdn = torch.empty(T * topk * Hd, device="cuda")
        Y = torch.empty(T * Hd, device="cuda")
        n_tot = T * topk
        used = int(np.count_nonzero(np.bincount(ex.ravel(), minlength=E)))

        def layer():
            st = lib.lib.tb200_moe_gather(h.h, Xtok.data_ptr(), dtype_code, Hd, Hd, T, ids.data_ptr(), n_tot,
                                          Xp.data_ptr(), Hd)
            st = st or h.gemm_grouped_ex(1, 0, Fe, n_tot, Hd, E, offs.data_ptr(), 1.0, Wgu.data_ptr(), dtype_code, Hd,
                                         Fe * Hd, Xp.data_ptr(), dtype_code, Hd, 0.0, Cup.data_ptr(), f32, Fe)
            st = st or h.gemm_grouped_ex(1, 0, Hd, n_tot, Fe, E, offs.data_ptr(), 1.0, Wd.data_ptr(), dtype_code, Fe,
                                         Hd * Fe, Hp.data_ptr(), dtype_code, Fe, 0.0, Cdn.data_ptr(), f32, Hd)
            return st or lib.lib.tb200_moe_combine(h.h, Hd, Cdn.data_ptr(), Hd, n_tot, d_pos.data_ptr(),
                                                   d_w.data_ptr(), topk, T, Y.data_ptr(), Hd)
        layer_bytes = (2 * used * Fe * Hd + T * Hd + 2 * n_tot * Hd + n_tot * Fe) * 2 + (n_tot * (Fe + 2 * Hd)
                                                                                          + T * Hd) * 4
        measure("c5_moe_routed_layer_skewed", layer, 10, 2 * flop5, layer_bytes, "hbm")
        if "c5_moe_routed_layer_skewed" in out:
            out["c5_moe_routed_layer_skewed"]["experts_with_tokens"] = used
            out["c5_moe_routed_layer_skewed"]["launches"] = "gather + grouped up + grouped down + combine"

        def layer_fused():  # the gather inside the up projection's B loads
            st = h.gemm_grouped_gather_ex(1, Fe, n_tot, Hd, E, offs.data_ptr(), ids.data_ptr(), 1.0, Wgu.data_ptr(),
                                          dtype_code, Hd, Fe * Hd, Xtok.data_ptr(), dtype_code, Hd, T, 0.0,
                                          Cup.data_ptr(), f32, Fe)
            st = st or h.gemm_grouped_ex(1, 0, Hd, n_tot, Fe, E, offs.data_ptr(), 1.0, Wd.data_ptr(), dtype_code, Fe,
                                         Hd * Fe, Hp.data_ptr(), dtype_code, Fe, 0.0, Cdn.data_ptr(), f32, Hd)
            return st or lib.lib.tb200_moe_combine(h.h, Hd, Cdn.data_ptr(), Hd, n_tot, d_pos.data_ptr(),
                                                   d_w.data_ptr(), topk, T, Y.data_ptr(), Hd)
        # the expert-order copy of the tokens is neither written nor read back
        measure("c5_moe_routed_layer_skewed_fused", layer_fused, 10, 2 * flop5, layer_bytes - 2 * n_tot * Hd * 2, "hbm")
        if "c5_moe_routed_layer_skewed_fused" in out:
            out["c5_moe_routed_layer_skewed_fused"]["experts_with_tokens"] = used
            out["c5_moe_routed_layer_skewed_fused"]["launches"] = "grouped up with the gather fused + grouped down + combine"
    del Wgu, Wd, Xe, He, Cgu, Cd, Xall, Call

    # config 5 squares, both 16-bit input types
    for S in (4096, 8192, 16384) if only is None or only.startswith("c5_square") else ():
        for tname, tdt, tcode in (("f16", torch.float16, cb.CUDA_R_16F), ("bf16", torch.bfloat16, cb.CUDA_R_16BF)):
            A = (torch.randn(S, S, device="cuda") * 0.02).to(tdt)
            B = torch.randn(S, S, device="cuda").to(tdt)
            C = torch.empty(S * S, device="cuda")
            measure(f"c5_square_{S}_{tname}", lambda: h.gemm_ex(
                1, 0, S, S, S, 1.0, A.data_ptr(), tcode, S, B.data_ptr(), tcode, S, 0.0, C.data_ptr(), f32, S,
                cb.CUBLAS_COMPUTE_32F), 3 if S == 16384 else 10, 2.0 * S ** 3, 2 * S * S * 2 + S * S * 4, "tensor")
            del A, B, C
    torch.cuda.empty_cache()
    h.close()
    return out


def run_case(args):
    """--case NAME: one config 3/5 figure alone (its inputs, 2 warm-up calls, 3 x --steps timed calls)."""
    import torch
    from macuda_b200 import cublas as cb
    if args.impl == "reference":
        from oracle import oracle as O
        lib = O.reference_library()
    else:
        lib = cb.library()
    dtype = torch.float16 if args.dtype == "f16" else torch.bfloat16
    ctype = cb.CUDA_R_16F if args.dtype == "f16" else cb.CUDA_R_16BF
    out = config_figures(torch, lib, cb, ctype, dtype, only=args.case, reps_override=args.steps)
    if args.case not in out:
        print(json.dumps({"case": args.case, "error": "no such case (see configs_3_5 in a full run)"}))
        return 1
    print(json.dumps({"case": args.case, "impl": args.impl, **out[args.case]}))
    return 0


def run_single(args):
    """--gemm MxNxK: one ggml-style T,N GEMM (f32 C) repeated, for profiling one kernel in isolation.
    Weight copies rotate so that the weights touched per pass exceed twice L2."""
    import torch
    from macuda_b200 import cublas as cb
    m, n, k = (int(x) for x in args.gemm.lower().split("x"))
    if args.impl == "reference":
        from oracle import oracle as O
        lib = O.reference_library()
    else:
        lib = cb.library()
    dtype = torch.float16 if args.dtype == "f16" else torch.bfloat16
    ctype = cb.CUDA_R_16F if args.dtype == "f16" else cb.CUDA_R_16BF
    copies = max(1, min(16, -(-(300 << 20) // (m * k * 2))))
    ws = [(torch.randn(m, k, device="cuda") * 0.02).to(dtype) for _ in range(copies)]
    x = torch.randn(n, k, device="cuda").to(dtype)
    c = torch.empty(m * n, device="cuda")
    h = lib.handle()
    s = torch.cuda.Stream()
    h.set_stream(s.cuda_stream)

    def one(i):
        st = h.gemm_ex(1, 0, m, n, k, 1.0, ws[i % copies].data_ptr(), ctype, k, x.data_ptr(), ctype, k, 0.0,
                       c.data_ptr(), cb.CUDA_R_32F, m, cb.CUBLAS_COMPUTE_32F)
        if st != 0:
            raise RuntimeError(f"cublasGemmEx status {st}")
    for i in range(args.warmup):
        one(i)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for i in range(args.steps):
        one(i)
    e1.record(s)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    flop = 2.0 * m * n * k
    byts = m * k * 2 + n * k * 2 + m * n * 4
    plan = lib.plan(1, 0, m, n, k) if args.impl == "ours" else None
    print(json.dumps({"gemm": f"{m}x{n}x{k}", "impl": args.impl, "dtype": args.dtype, "us": round(us, 2),
                      "TFLOP/s": round(flop / us / 1e6, 1), "GB/s": round(byts / us / 1e3, 1), "plan": plan,
                      "weight_copies": copies, "steps": args.steps}))
    h.close()
    return 0


def run(args):
    import torch
    import torch.distributed as dist
    from macuda_b200 import cublas as cb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        os.environ["NCCL_DEBUG"] = "WARN"  # keep NCCL's version banner off stdout: one JSON line only
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    if args.impl == "reference":
        from oracle import oracle as O
        lib = O.reference_library()
        if lib is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref/libtinycublas_ref.so was not built "
                                  "(needs the reference tree at build time)"}))
            return 0
        launched = world
        if world > 1:  # the reference is single-GPU: rank 0 alone runs it
            dist.barrier()
            if rank != 0:
                dist.destroy_process_group()
                return 0
            world = 1
    else:
        lib = cb.library()
    dtype = torch.float16 if args.dtype == "f16" else torch.bfloat16
    ctype = cb.CUDA_R_16F if args.dtype == "f16" else cb.CUDA_R_16BF
    acts, layers = make_inputs(torch, rank, world, dtype)
    stream = torch.cuda.Stream()
    comm = torch.cuda.Stream() if world > 1 else None
    h = lib.handle()
    h.set_stream(stream.cuda_stream)
    sharded = []
    fused = world > 1 and args.exchange != "allgather"
    any_shard = True
    if world > 1:
        from macuda_b200.dist import FusedShardedGemm, ReplicatedGemm, ShardedGemm, pick_fastest, step_barrier
        for L in layers:
            if fused:
                # N-sharded (rows exchanged by the epilogue) or whole on every rank (nothing exchanged): the
                # faster of the two, timed on every rank (max over ranks) during set-up
                cands = {"sharded": FusedShardedGemm(lib, h, L["m"], TOKENS, L["k"], rank, world, L["w"], ctype,
                                                     exchange={"fused": "p2p"}.get(args.exchange, args.exchange)),
                         "whole": ReplicatedGemm(lib, h, L["m"], TOKENS, L["k"], L["w_full"], ctype)}
                choice = pick_fastest(cands, acts[L["src"]], stream) if args.shard == "auto" else args.shard
                for key, c in cands.items():
                    if key != choice:
                        c.close()
                sharded.append(cands[choice])
            else:
                sharded.append(ShardedGemm(lib, h, L["m"], TOKENS, L["k"], rank, world, L["w"], ctype))
        any_shard = any(getattr(g, "exchange", "allgather") != "replicated" for g in sharded)
    for L in layers:
        L.pop("w_full", None)  # whole weights stay only where a projection runs whole on every rank
    # Inside the timed region the only events are the two around the dominant GEMM (lm_head, the roofline
    # kernel): an event between two kernels would also stop the next one from being scheduled while the
    # previous one finishes (programmatic dependent launch). The per-projection breakdown comes from a
    # separate pass after the timed region, with an event before every GEMM.
    dom = layers.index(next(L for L in layers if L["name"] == "lm_head"))
    marks = [[torch.cuda.Event(enable_timing=True) for _ in range(len(layers) + 1)] for _ in range(args.steps)]
    per_gemm_ms = [0.0] * len(layers)
    launches_per_step = len(layers) * (2 if world > 1 and not fused else 1)

    def step(ev=None, only=None):
        for i, L in enumerate(layers):
            act = acts[L["src"]]
            if ev is not None and (only is None or i == only):
                ev[i].record(stream)
            if world == 1:
                st = gemm_call(h, cb, L, act, ctype, L["c_local"].data_ptr(), L["m"])
            elif fused:  # this rank's rows, stored by the epilogue into every rank's C
                st = sharded[i].run(act, stream)
            else:  # this rank's rows, then the all-gather + layout on the comm stream (overlaps the next GEMM)
                st = sharded[i].run(act, stream, comm)
            if ev is not None and (i == len(layers) - 1 if only is None else i == only):
                ev[i + 1].record(stream)
            if st != 0:
                raise RuntimeError(f"{L['name']}: status {st}")
        if fused and any_shard:
            step_barrier(stream)  # every peer's stores into this rank's C have landed
        elif world > 1 and not fused:
            stream.wait_stream(comm)

    # warm-up
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    clocks = ClockSampler(local) if not args.no_clocks else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if clocks:
        clocks.mark(True)
    e0.record(stream)
    for j in range(args.steps):
        step(marks[j], only=dom)
    e1.record(stream)
    torch.cuda.synchronize()
    if clocks:
        clocks.mark(False)
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clock_info = clocks.stop() if clocks else None

    dom_ms = sum(marks[j][dom].elapsed_time(marks[j][dom + 1]) for j in range(args.steps)) / args.steps
    # the per-projection breakdown, after the timed region: an event before every GEMM
    n_bd = min(args.steps, 20)
    for j in range(n_bd):
        step(marks[j])
    torch.cuda.synchronize()
    for j in range(n_bd):
        for i in range(len(layers)):
            per_gemm_ms[i] += marks[j][i].elapsed_time(marks[j][i + 1]) / n_bd
    value = STEP_FLOP / (ms * 1e-3) / 1e12
    gemm_only_ms = sum(per_gemm_ms)  # this rank's GEMMs alone (the all-gathers overlap on the comm stream)
    if world > 1:
        t = torch.tensor([gemm_only_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gemm_only_ms = float(t.item())

    pk = peaks()
    L = layers[dom]
    dom_flop = 2.0 * L["mp"] * TOKENS * L["k"]
    dom_tflops = dom_flop / (dom_ms * 1e-3) / 1e12
    traffic = None
    prof = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if os.path.exists(prof) and world == 1 and args.impl == "ours":
        try:
            with open(prof) as f:
                traffic = json.load(f).get("lm_head_dram_bytes")
        except Exception:
            traffic = None
    roofline = {"bound": "tensor", "achieved": round(dom_tflops, 2), "peak": pk["bf16_tflops_sustained"],
                "unit": "TFLOP/s", "frac": round(dom_tflops / pk["bf16_tflops_sustained"], 4), "traffic": traffic,
                "kernel": "lm_head GEMM (%d x %d x %d)" % (L["mp"], TOKENS, L["k"]),
                "peak_source": pk["source"] + " bf16 sustained (cuBLAS 8192^3, MEASURED_PEAKS.json)",
                "frac_of_burst": round(dom_tflops / pk["bf16_tflops"], 4),
                "algorithmic_bytes": L["mp"] * L["k"] * 2 + TOKENS * L["k"] * 2 + L["mp"] * TOKENS * 4}

    shapes = {Lx["name"]: {"m": Lx["mp"], "n": TOKENS, "k": Lx["k"], "us": round(per_gemm_ms[i] * 1e3, 2),
                           "TFLOP/s": round(2.0 * Lx["mp"] * TOKENS * Lx["k"] / (per_gemm_ms[i] * 1e-3) / 1e12, 1)}
              for i, Lx in enumerate(layers)}

    # e2e through the public API with host buffers: each step copies its activations from pinned host
    # memory (double-buffered on a copy stream, overlapping the previous step) and reads back the last
    # token's logits
    e2e = None
    hx = [acts["x"].cpu().pin_memory(), acts["h"].cpu().pin_memory()]
    dev_bufs = [[torch.empty_like(acts["x"]), torch.empty_like(acts["h"])] for _ in range(2)]
    logits = torch.empty(VOCAB, dtype=torch.float32).pin_memory()
    copy = torch.cuda.Stream()
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    lm = layers[dom]
    n_e2e = max(3, min(args.steps, 100))

    def e2e_step(i):
        b = i % 2
        with torch.cuda.stream(copy):
            copy.wait_event(free[b])
            dev_bufs[b][0].copy_(hx[0], non_blocking=True)
            dev_bufs[b][1].copy_(hx[1], non_blocking=True)
            ready[b].record(copy)
        stream.wait_event(ready[b])
        for j, L2 in enumerate(layers):
            act = dev_bufs[b][0] if L2["src"] == "x" else dev_bufs[b][1]
            if world == 1:
                st = gemm_call(h, cb, L2, act, ctype, L2["c_local"].data_ptr(), L2["m"])
            elif fused:
                st = sharded[j].run(act, stream)
            else:
                st = sharded[j].run(act, stream, comm)
            if st != 0:
                raise RuntimeError("e2e gemm failed")
        if fused and any_shard:
            step_barrier(stream)
        elif world > 1 and not fused:
            stream.wait_stream(comm)
        free[b].record(stream)
        c_lm = lm["c_local"] if world == 1 else sharded[dom].c
        with torch.cuda.stream(stream):
            logits.copy_(c_lm[(TOKENS - 1) * lm["m"]:TOKENS * lm["m"]], non_blocking=True)

    for i in range(3):
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    t_wall = time.perf_counter()
    for i in range(n_e2e):
        e2e_step(i)
    f1.record(stream)
    torch.cuda.synchronize()
    t_wall = time.perf_counter() - t_wall
    e2e_ms = f0.elapsed_time(f1) / n_e2e
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": round(STEP_FLOP / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "h2d_bytes_per_step": int(hx[0].numel() * 2 + hx[1].numel() * 2), "d2h_bytes_per_step": VOCAB * 4,
           "ms_per_step": round(e2e_ms, 4), "wall_ms_per_step": round(t_wall * 1e3 / n_e2e, 4), "steps": n_e2e}

    cpu = None
    if rank == 0 and world == 1 and args.impl == "ours" and not args.no_cpu_baseline:
        try:
            cpu = run_cpu_baseline()
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"error": str(ex)[:200]}

    decode = None
    if rank == 0 and world == 1 and not args.no_decode:
        decode = decode_figures(torch, lib, cb, ctype, dtype)
    configs = None
    if rank == 0 and world == 1 and not args.no_configs:
        configs = config_figures(torch, lib, cb, ctype, dtype)

    if fused:
        for g in sharded:
            g.close()
    h.close()
    if rank == 0:
        line = {
            "metric": "GEMM TFLOP/s (Llama-3.1-8B prefill projection set, 512 tokens, fp16 -> f32, ggml's T,N call)",
            "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": args.dtype, "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) activations; no checkpoint)",
            "config": {"workload": "llama3.1-8b prefill projections q,k,v,o,gate,up,down,lm_head @ 512 tokens "
                                   "(BASELINE configs[1])", "tokens": TOKENS, "step_gflop": round(STEP_FLOP / 1e9, 1),
                       "parallelism": ((f"x{world}: " + ", ".join(
                                           f"{L['name']} " + ("whole on every rank" if g.exchange == "replicated"
                                                              else "N-sharded, rows exchanged by " +
                                                              ("NVLink multicast" if g.exchange == "multicast" else
                                                               "P2P") + " stores from the GEMM epilogue")
                                           for L, g in zip(layers, sharded)) +
                                        ("; one NCCL barrier per step" if any_shard else "")) if fused else
                                       f"N-shard x{world}, C exchanged by NCCL all-gather + layout kernel")
                                      if world > 1 else "single GPU",
                       "l2": "inputs larger than L2 (1.9 GB per step); no flush"},
            "frac_of_peak": round(value / pk["bf16_tflops_sustained"], 4),
            "roofline": roofline, "shapes": shapes,
            "shapes_note": "per-projection device time from %d further steps after the timed region, an event before "
                           "every GEMM (events between kernels stop the next one being scheduled early, so these "
                           "sum to more than ms_per_step)" % n_bd,
            "gpu_launches": launches_per_step * args.steps,
            "gemm_only": {"ms_per_step": round(gemm_only_ms, 4),
                          "TFLOP/s": round(STEP_FLOP / (gemm_only_ms * 1e-3) / 1e12, 2),
                          "note": "sum of the per-projection times (max over ranks); at N > 1 the all-gathers run "
                                  "on a second stream and the step time includes them"},
        }
        if args.impl == "reference":
            line["impl"] = "reference"
            line["n_gpus"] = launched
            line["note"] = "the reference library is single-GPU: rank 0 ran the whole step on one GPU"
            line["cpu_baseline"] = {"value": line["value"], "unit": "TFLOP/s", "cores": 0, "kind": "reference",
                                    "sample": "the whole step through the reference's own libtinycublas (cublas.c + "
                                              "gemm.cu compiled from source for sm_100a) on one B200; the reference's "
                                              "implementation of this path is GPU code, it has no CPU implementation"}
            line["e2e"] = {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
            line["gpu_launches"] = None
        else:
            line["cpu_baseline"] = cpu
            line["e2e"] = e2e
        if clock_info:
            line["clocks"] = clock_info
        if decode:
            line["decode"] = decode
        if configs:
            line["configs_3_5"] = configs
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    elif dist.is_initialized():  # the reference arm under torchrun: rank 0 ran alone
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--dtype", choices=["f16", "bf16"], default="f16")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-configs", action="store_true", help="skip the config 3 and 5 figures")
    ap.add_argument("--no-clocks", action="store_true")
    ap.add_argument("--gemm", default=None, help="MxNxK: time one T,N GEMM alone (profiling)")
    ap.add_argument("--case", default=None, help="run one config 3/5 figure alone, by its name in configs_3_5 "
                                                 "(profiling); --steps sets its back-to-back calls")
    ap.add_argument("--shard", choices=["auto", "sharded", "whole"], default="auto",
                    help="N > 1, fused exchange: per projection N-sharded or whole on every rank (auto: the faster, "
                         "timed on every rank at set-up)")
    ap.add_argument("--exchange", choices=["fused", "multicast", "p2p", "allgather"], default="fused",
                    help="N > 1: how the sharded C is replicated (fused = p2p stores from the epilogue)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.gemm:
        return run_single(args)
    if args.case:
        return run_case(args)
    return run(args)


if __name__ == "__main__":
    sys.exit(main())
