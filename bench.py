#!/usr/bin/env python3
"""Benchmark of libtinycublas_b200 on its headline workload (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--dtype f16|bf16]

Workload: the Llama-3.1-8B-shaped prefill projection set at 512 tokens, issued as
ggml-cuda issues it: cublasGemmEx(T, N, m = out features, n = 512, k = in features, fp16 weights
N(0, 0.02^2), fp16 activations N(0, 1), f32 C, COMPUTE_32F). One step = the 8 projections Q 4096->4096,
K 4096->1024, V 4096->1024, O 4096->4096, gate and up 4096->14336, down 14336->4096, lm_head
4096->128256 (761.2 GFLOP). Synthetic seeded data of those shapes; weights are random, not a checkpoint.
Inputs are larger than L2 (1.9 GB touched per step), so no flush is needed between steps.

At N > 1 (torchrun, one process per GPU, NCCL) each projection is either N-sharded along m (the weight's
output features: each rank computes its m/N rows) or run whole on every rank, and every rank ends the step
holding every projection's full C. A sharded projection's rows reach the peers one of two ways: the copy
engines push them after the GEMM (CUDA IPC mappings, macuda_b200.dist.CopyEngineShardedGemm; these shards
run first, so their copies cross NVLink while the SMs run what follows), or the GEMM epilogue stores them
into every peer's C (FusedShardedGemm). One 4-byte NCCL all-reduce per step is the completion barrier. The
plan - which projections are sharded, and how - is chosen at set-up by timing candidate plans as whole steps
on every rank (max over ranks; --exchange auto, the default). --exchange ce keeps to copy-engine plans,
--exchange fused decides per projection between epilogue stores and whole, --exchange multicast stores
through an NVLink multicast address, --exchange allgather uses an NCCL all-gather + layout kernel. Total work is fixed, so scaling is "strong". After the timed region every
rank checks sampled rows of every projection's C - rows of every peer's shard included - against fp64 on the
device ("parity", max over ranks), and `sharded_shapes` gives per-shape figures split across the N ranks
(lm_head, FFN, squares N-sharded; config 3 attention by KV-head groups and config 5 MoE by experts), each
with its one-GPU time, compute-only and end-to-end scaling and the link bound R.

Keys beyond the base contract: roofline (dominant kernel = the lm_head GEMM, against the burst tensor peak:
the timed region lasts milliseconds), cpu_baseline (the oracle's multithreaded fp16 GEMM on the host, a
stand-in for ggml-cpu), e2e (the same step through the public API with host buffers: H2D of the step's
activations and D2H of the last token's logits), parity, per projection figures, decode (n <= 8) HBM
bandwidth figures (config 4), the HBM probes, and configs 3 and 5 figures (attention batched GEMMs, MoE
pointer-array and grouped GEMMs, squares).

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

    def __init__(self, device_index: int, period_ms: int = 100):
        self.dev = device_index
        self.period_ms = period_ms
        self.samples = []
        self.proc = None
        self.t0 = self.t1 = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(self.period_ms)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
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

    def window(self, t0, t1):
        """median SM clock and the throttle reasons of the samples taken between wall times t0 and t1"""
        return self._summary([s for t, s in list(self.samples) if t0 <= t <= t1])

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
        return self._summary(rows)

    @staticmethod
    def _summary(rows):
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


def bind_to_gpu_cpus(torch, dev):
    """Run this process on the host CPUs local to GPU `dev` (its PCI device's local_cpulist in sysfs), so that the
    pinned host buffers of the e2e leg sit on the GPU's NUMA node. Returns the CPU list, or None when unknown."""
    try:
        pr = torch.cuda.get_device_properties(dev)
        bdf = "%04x:%02x:%02x.0" % (pr.pci_domain_id, pr.pci_bus_id, pr.pci_device_id)
        with open(f"/sys/bus/pci/devices/{bdf}/local_cpulist") as f:
            text = f.read().strip()
        cpus = set()
        for part in text.split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            return text
    except Exception:
        pass
    return None


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
        check = parity_rows(m, max(world, 8), seed + len(layers))
        layers.append({"name": name, "m": m, "mp": rows, "first": first, "k": k, "src": src, "w": w, "w_full": w_full,
                       "c_local": c, "check_rows": torch.tensor(check, device="cuda"),
                       "w_check": w_full[check].clone()})
    return acts, layers


def parity_rows(m, world, seed):
    """Rows of C the parity check reads: the first, middle and last row of every rank's shard (of `world`
    shards, so every peer's rows are covered at any N up to it) and 24 seeded others."""
    import numpy as np
    from macuda_b200.dist import shard_rows
    rows = set()
    for r in range(world):
        first, cnt, _ = shard_rows(m, world, r)
        if cnt:
            rows |= {first, first + cnt // 2, first + cnt - 1}
    rows |= set(np.random.default_rng(seed).choice(m, 24, replace=False).tolist())
    return sorted(rows)


def check_rows(torch, C, m, n, rows, W_rows, X):
    """The parity gate on sampled rows of a T,N GEMM's column-major f32 C (ldc = m), against fp64 on the device:
    R = W_rows X^T; max |C - R| / (|W_i| |X_j|) <= 2^-10 (north star) and the reference's own metric
    max |C - R| / max |R| <= 2e-3 (cuda-shim/libtinycublas/bf16-20260921/bench_gemm_contract.cu:8-10), non-finite
    values refused first. The checker only: it never feeds the measured path."""
    got = C[: m * n].view(n, m)[:, rows].t().double()
    W, Xd = W_rows.double(), X.double()
    R = W @ Xd.t()
    S = W.norm(dim=1)[:, None] * Xd.norm(dim=1)[None, :]
    finite = bool(torch.isfinite(got).all().item())
    d = (got - R).abs()
    norm = float((d / S.clamp_min(1e-300)).max().item()) if finite else float("inf")
    refm = float((d.max() / R.abs().max().clamp_min(1e-300)).item()) if finite else float("inf")
    return {"ok": finite and norm <= 2.0 ** -10 and refm <= 2e-3, "norm_err": norm, "ref_metric": refm}


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
    """Config 4: n in {1, 2, 4, 8} against the four weight shapes, HBM GB/s of the skinny kernel (median of three
    repeats of back-to-back calls). Weight copies rotate so that the bytes touched per pass exceed twice L2."""
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
            times = []
            for _ in range(3):  # median of three repeats of back-to-back calls
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record(s)
                for i in range(reps):
                    one(i)
                e1.record(s)
                torch.cuda.synchronize()
                times.append(e0.elapsed_time(e1) * 1e3 / reps)
            us = statistics.median(times)
            byts = m * k * 2 + n * k * 2 + m * n * 4
            out[f"{m}x{k}_n{n}"] = {"us": round(us, 2), "GB/s": round(byts / us / 1e3, 1)}
        del ws
    h.close()
    return out


def config_figures(torch, lib, cb, dtype_code, dtype, only=None, reps_override=None, clocks=None):
    """Configs 3 and 5: attention batched GEMMs (strided with the GQA heads folded into n, and pointer arrays
    with each KV head's pointer repeated for its 4 query heads), MoE expert GEMMs (pointer arrays over 128
    experts, 32 tokens each) and square GEMMs, all T,N with f32 C as ggml issues them. Per case: device
    time (CUDA events around back-to-back calls, median of 3 repeats), TFLOP/s, compulsory bytes / time, and
    the fraction of the measured peak of its bound (HBM copy bandwidth, or burst bf16 tensor throughput).
    only: run just the case of that name (bench.py --case, for profiling one kernel). clocks: a running
    ClockSampler; the square cases, timed for about half a second each, then carry the median SM clock of their
    own window and their time scaled to the maximum clock (us x MHz / max MHz), which compares the two input
    types at equal clocks."""
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
        w0 = time.time()
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(reps):
                call()
            e1.record(s)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / reps)
        w1 = time.time()
        us = statistics.median(ts)
        tf, gbs = flop / us / 1e6, byts / us / 1e3
        frac = gbs / pk["hbm_gbs"] if bound == "hbm" else tf / pk["bf16_tflops"]
        out[name] = {"us": round(us, 2), "TFLOP/s": round(tf, 1), "GB/s": round(gbs, 1), "bound": bound,
                     "frac_of_measured_peak": round(frac, 3)}
        if clocks is not None and name.startswith("c5_square"):
            time.sleep(0.12)  # the sampler's last reading of the window
            c = clocks.window(w0, w1)
            if c:
                out[name]["clocks"] = c
                out[name]["us_at_max_clock"] = round(us * c["sm_mhz"] / max(c["sm_max_mhz"], 1.0), 2)

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
            # about 0.15 s per repeat: enough clock samples per case
            measure(f"c5_square_{S}_{tname}", lambda: h.gemm_ex(
                1, 0, S, S, S, 1.0, A.data_ptr(), tcode, S, B.data_ptr(), tcode, S, 0.0, C.data_ptr(), f32, S,
                cb.CUBLAS_COMPUTE_32F), {4096: 1500, 8192: 200, 16384: 25}[S], 2.0 * S ** 3, 2 * S * S * 2 + S * S * 4,
                "tensor")
            del A, B, C
    torch.cuda.empty_cache()
    h.close()
    return out


# measured peer-to-peer copy bandwidth per direction between two B200s of this pool over NVLink 5 (GB/s): the
# link figure of the scaling bound R
PEER_GBS = 770.0


def probe_figures(torch, lib):
    """The HBM probes (tb200_bw_write / tb200_bw_read, the counterparts of the reference's bandwidth probes,
    cuda-shim/libtinycublas/gemm.cu:421-431 driven by cuda-shim/test/bw_bench.c): 1 GiB streamed one way,
    20 launches each, GB/s from CUDA events."""
    import ctypes
    n4 = (1 << 30) // 16
    buf = torch.empty(n4 * 4, device="cuda")
    sink = torch.zeros(1, device="cuda")
    s = torch.cuda.current_stream()
    out = {}
    for name in ("write", "read"):
        def call():
            if name == "write":
                return lib.lib.tb200_bw_write(buf.data_ptr(), n4, ctypes.c_float(1.0), ctypes.c_void_p(s.cuda_stream))
            return lib.lib.tb200_bw_read(buf.data_ptr(), n4, sink.data_ptr(), ctypes.c_void_p(s.cuda_stream))
        for _ in range(3):
            call()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(20):
            call()
        e1.record(s)
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / 20
        out[name] = {"GB/s": round(n4 * 16 / us / 1e3, 1), "us": round(us, 1), "bytes": n4 * 16}
    del buf
    return out


def sharded_figures(torch, lib, cb, h, stream, rank, world, copies, ring):
    """Per-shape figures at N > 1 (3 and 5): each case once on one GPU (the whole GEMM,
    every rank timing it on its own GPU), then split across the N ranks:
      * N-sharded along m (the weight's output features): lm_head, FFN gate/up and down, squares
        4096/8192/16384 in f16 and bf16. Each rank computes its rows into its own full C (ldc = m) and either the
        copy engines push them into every peer's C (tb200_push_block), the columns in `chunks` GEMMs so the
        copies of one chunk overlap the next chunk's math, or the GEMM epilogue stores them into every peer's C
        (tb200_gemm_ex_allgather); both are timed and the faster is reported as e2e;
      * batch-sharded (whole batch elements per rank): config 3 attention by KV-head groups (strided with the 4
        query heads of each KV head folded into n; pointer arrays with each KV head's pointer repeated for its
        query heads), config 5 MoE by experts (pointer arrays, and the grouped GEMM). Each rank's C slab is
        contiguous and is pushed whole.
    Times are device times on the compute stream (CUDA events, max over ranks): `n1_us` the whole GEMM on one
    GPU, `compute_us` this rank's part alone, `e2e_us` its part plus the exchange until every rank holds all of
    C (the copies joined and one NCCL barrier). compute_scaling = n1 / (N compute), e2e_scaling = n1 / (N e2e).
    R = n1 * B / ((N - 1) * C bytes), B = PEER_GBS: the efficiency bound of a perfectly overlapped exchange (each
    rank receives (N-1)/N of C over its link while computing 1/N of the work). parity: sampled rows of C as rank
    0..N-1 hold it after the exchange (every rank's part included), against fp64 on the device, max over ranks."""
    import ctypes

    import torch.distributed as dist
    from macuda_b200.dist import IpcReplicas, shard_rows, step_barrier
    f32 = cb.CUDA_R_32F
    out = {}

    def timed(fn, reps):
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.barrier()
        return float(t.item())

    def gen(shape, seed, scale, dt):
        g = torch.Generator(device="cuda")
        g.manual_seed(seed)  # the same on every rank: every rank holds the same operands
        return (torch.randn(*shape, device="cuda", generator=g) * scale).to(dt)

    def reduce_parity(r):
        t = torch.tensor([r["norm_err"], r["ref_metric"], 0.0 if r["ok"] else 1.0], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return {"ok": float(t[2].item()) == 0.0, "norm_err": float("%.3e" % t[0].item()),
                "ref_metric": float("%.3e" % t[1].item())}

    def merge(a, b):
        return {"ok": a["ok"] and b["ok"], "norm_err": max(a["norm_err"], b["norm_err"]),
                "ref_metric": max(a["ref_metric"], b["ref_metric"])}

    def record(name, flop, c_bytes, bound, t1, tc, te, par, extra=None):
        rec = {"n1_us": round(t1 * 1e3, 1), "compute_us": round(tc * 1e3, 1), "e2e_us": round(te * 1e3, 1),
               "compute_scaling": round(t1 / (world * tc), 3), "e2e_scaling": round(t1 / (world * te), 3),
               "R": round(t1 * 1e-3 * PEER_GBS * 1e9 / ((world - 1) * c_bytes), 3), "bound": bound,
               "TFLOP/s_e2e": round(flop / (te * 1e-3) / 1e12, 1), "TFLOP/s_n1": round(flop / (t1 * 1e-3) / 1e12, 1),
               "C_bytes": int(c_bytes), "parity": reduce_parity(par)}
        if extra:
            rec.update(extra)
        out[name] = rec

    def reps_for(t_ms):
        return int(max(3, min(40, 25.0 / max(t_ms, 1e-3))))

    # ---- N-sharded along m: lm_head, FFN, squares ----
    cases = [("lm_head", 128256, 512, 4096, "f16", (1, 2, 4)), ("ffn_gate_up", 14336, 512, 4096, "f16", (1, 2)),
             ("ffn_down", 4096, 512, 14336, "f16", (1, 2))]
    for S in (4096, 8192, 16384):
        for tn in ("f16", "bf16"):
            cases.append((f"square_{S}_{tn}", S, S, S, tn, (1, 4, 8) if S > 4096 else (1, 4)))
    for ci, (name, m, n, k, tn, chunk_opts) in enumerate(cases):
        dt = torch.float16 if tn == "f16" else torch.bfloat16
        code = cb.CUDA_R_16F if tn == "f16" else cb.CUDA_R_16BF
        A = gen((m, k), 7000 + ci, 0.02, dt)   # stored k x m (op T, lda = k): row i = output feature i
        B = gen((n, k), 7100 + ci, 1.0, dt)    # stored k x n (op N, ldb = k)
        first, rows, _ = shard_rows(m, world, rank)
        C1 = torch.empty(m * n, device="cuda")
        buf = IpcReplicas(lib, m * n * 4, rank, world)
        esz = 2

        def whole():
            return h.gemm_ex(1, 0, m, n, k, 1.0, A.data_ptr(), code, k, B.data_ptr(), code, k, 0.0, C1.data_ptr(), f32,
                             m, cb.CUBLAS_COMPUTE_32F)

        def part(col0=0, nc=n):
            if rows == 0:
                return 0
            return h.gemm_ex(1, 0, rows, nc, k, 1.0, A.data_ptr() + first * k * esz, code, k,
                             B.data_ptr() + col0 * k * esz, code, k, 0.0, buf.own + (first + col0 * m) * 4, f32, m,
                             cb.CUBLAS_COMPUTE_32F)

        def sharded(chunks, cs):
            step = -(-n // chunks)
            for col0 in range(0, n, step):
                nc = min(step, n - col0)
                if part(col0, nc) != 0:
                    raise RuntimeError(f"{name}: GEMM failed")
                cs.after(stream)
                if rows and lib.lib.tb200_push_block(buf.array, world, rank, first, rows, col0, nc, m, 4, cs.array,
                                                     cs.lanes) != 0:
                    raise RuntimeError(f"{name}: push failed")
            cs.join(stream)
            step_barrier(stream)

        one = ctypes.c_float(1.0)

        def sharded_p2p():  # the GEMM epilogue stores the rows into every replica (peers' over NVLink)
            if rows and lib.lib.tb200_gemm_ex_allgather(
                    h.h, 1, 0, rows, n, k, ctypes.byref(one), A.data_ptr() + first * k * esz, code, k, B.data_ptr(),
                    code, k, buf.array, world, f32, m, first, cb.CUBLAS_COMPUTE_32F) != 0:
                raise RuntimeError(f"{name}: sharded GEMM failed")
            step_barrier(stream)

        t1 = timed(whole, reps_for(2.0 * m * n * k / 1.2e15 * 1e3))
        reps = reps_for(t1)
        tc = timed(part, reps)
        best = None
        for ch in chunk_opts:
            for cname, cs in (("every peer at once", copies), ("ring", ring)):
                te = timed(lambda: sharded(ch, cs), reps)
                if best is None or te < best[0]:
                    best = (te, ch, cname, cs)
        t_ce = best[0]
        t_p2p = timed(sharded_p2p, reps)
        if t_p2p < best[0]:
            best = (t_p2p, "p2p", None, None)
            sharded_p2p()
        else:
            sharded(best[1], best[3])
        torch.cuda.synchronize()
        dist.barrier()
        rws = torch.tensor(parity_rows(m, world, 11 + ci), device="cuda")
        Cfull = torch.as_tensor(_Dev(buf.own, m * n), device="cuda")
        par = check_rows(torch, Cfull, m, n, rws, A[rws], B)
        record(name, 2.0 * m * n * k, m * n * 4, "tensor", t1, tc, best[0], par,
               {"m": m, "n": n, "k": k, "dtype": tn, "sharded": "m (weight rows)",
                "exchange": "p2p epilogue stores" if best[1] == "p2p" else
                f"copy engines ({best[2]}), {best[1]} column chunk(s)",
                "e2e_us_copy_engines": round(t_ce * 1e3, 1), "e2e_us_p2p_epilogue": round(t_p2p * 1e3, 1)})
        del Cfull
        buf.close()
        del A, B, C1
        torch.cuda.empty_cache()

    # ---- batch-sharded: config 3 attention (KV-head groups), config 5 MoE (experts) ----
    dt, code = torch.float16, cb.CUDA_R_16F
    Hq, Hkv, D, Tq, Tk = 32, 8, 128, 512, 4096
    g = Hq // Hkv
    K = gen((Hkv, Tk, D), 7201, 1.0, dt)
    Q = gen((Hq, Tq, D), 7202, 1.0, dt)
    V = gen((Hkv, D, Tk), 7203, 1.0, dt)
    u = torch.rand(Hq, Tq, Tk, device="cuda", generator=torch.Generator(device="cuda").manual_seed(7204))
    P_ = (u / u.sum(dim=2, keepdim=True)).to(dt)  # softmax-shaped weights
    del u

    def table(ptrs):
        return torch.tensor(ptrs, dtype=torch.int64, device="cuda")

    def batch_case(name, nbatch, slab, flop, c_bytes, bound, whole_fn, part_fn, check_fn, extra):
        """whole_fn(C base): the whole batch; part_fn(C base, b0, nb): batch elements [b0, b0 + nb) into their
        slabs of the full C; check_fn(C tensor, b) -> parity dict of element b."""
        b0, nb, _ = shard_rows(nbatch, world, rank)
        total = nbatch * slab
        C1 = torch.empty(total, device="cuda")
        buf = IpcReplicas(lib, total * 4, rank, world)

        def sharded(cs):
            if nb and part_fn(buf.own, b0, nb) != 0:
                raise RuntimeError(f"{name}: GEMM failed")
            cs.after(stream)
            if nb and lib.lib.tb200_push_block(buf.array, world, rank, b0 * slab, nb * slab, 0, 1, total, 4,
                                               cs.array, cs.lanes) != 0:
                raise RuntimeError(f"{name}: push failed")
            cs.join(stream)
            step_barrier(stream)

        t1 = timed(lambda: whole_fn(C1.data_ptr()), 10)
        reps = reps_for(t1)
        tc = timed(lambda: part_fn(buf.own, b0, nb) if nb else 0, reps)
        te_c = timed(lambda: sharded(copies), reps)
        te_r = timed(lambda: sharded(ring), reps)
        te, cs_best = (te_c, copies) if te_c <= te_r else (te_r, ring)
        extra = dict(extra, exchange="copy engines (" + ("every peer at once" if cs_best is copies else "ring") + ")")
        sharded(cs_best)
        torch.cuda.synchronize()
        dist.barrier()
        Cfull = torch.as_tensor(_Dev(buf.own, total), device="cuda")
        par = {"ok": True, "norm_err": 0.0, "ref_metric": 0.0}
        for r in range(world):  # the first and last element of every rank's share
            rb0, rnb, _ = shard_rows(nbatch, world, r)
            for b in {rb0, rb0 + rnb - 1} if rnb else ():
                par = merge(par, check_fn(Cfull, b))
        record(name, flop, c_bytes, bound, t1, tc, te, par, dict(extra, batch=nbatch, sharded="batch"))
        del Cfull
        buf.close()
        del C1

    def gemm_cols(C, b, m, n, slab, W_t, X_t, nrows=48):
        """parity of element b (m x n, column-major at b * slab) on seeded rows: W_t (m x k rows), X_t (n x k)"""
        rws = torch.tensor(sorted(set([0, m - 1] + torch.randperm(m, generator=torch.Generator().manual_seed(b))[
            :nrows].tolist())), device="cuda")
        return check_rows(torch, C[b * slab:(b + 1) * slab], m, n, rws, W_t[rws], X_t)

    flop3 = 2.0 * Tk * Tq * D * Hq
    # KQ, strided, the 4 query heads of a KV head folded into n: element = KV head (8)
    batch_case("c3_kq_strided_folded", Hkv, Tk * g * Tq, flop3, Hq * Tk * Tq * 4, "hbm",
               lambda C: h.gemm_strided_batched_ex(1, 0, Tk, g * Tq, D, 1.0, K.data_ptr(), code, D, Tk * D, Q.data_ptr(),
                                                   code, D, g * Tq * D, 0.0, C, f32, Tk, Tk * g * Tq, Hkv),
               lambda C, b0, nb: h.gemm_strided_batched_ex(
                   1, 0, Tk, g * Tq, D, 1.0, K.data_ptr() + b0 * Tk * D * 2, code, D, Tk * D,
                   Q.data_ptr() + b0 * g * Tq * D * 2, code, D, g * Tq * D, 0.0, C + b0 * Tk * g * Tq * 4, f32, Tk,
                   Tk * g * Tq, nb),
               lambda C, b: gemm_cols(C, b, Tk, g * Tq, Tk * g * Tq, K[b], Q[b * g:(b + 1) * g].reshape(g * Tq, D)),
               {"m": Tk, "n": g * Tq, "k": D, "split": "KV heads"})
    batch_case("c3_kqv_strided_folded", Hkv, D * g * Tq, flop3, Hq * D * Tq * 4, "hbm",
               lambda C: h.gemm_strided_batched_ex(1, 0, D, g * Tq, Tk, 1.0, V.data_ptr(), code, Tk, D * Tk,
                                                   P_.data_ptr(), code, Tk, g * Tq * Tk, 0.0, C, f32, D, D * g * Tq, Hkv),
               lambda C, b0, nb: h.gemm_strided_batched_ex(
                   1, 0, D, g * Tq, Tk, 1.0, V.data_ptr() + b0 * D * Tk * 2, code, Tk, D * Tk,
                   P_.data_ptr() + b0 * g * Tq * Tk * 2, code, Tk, g * Tq * Tk, 0.0, C + b0 * D * g * Tq * 4, f32, D,
                   D * g * Tq, nb),
               lambda C, b: gemm_cols(C, b, D, g * Tq, D * g * Tq, V[b], P_[b * g:(b + 1) * g].reshape(g * Tq, Tk)),
               {"m": D, "n": g * Tq, "k": Tk, "split": "KV heads"})
    # pointer arrays, element = query head (32), whole KV-head groups per rank (world divides 8)
    kq_a = table([K.data_ptr() + (q // g) * Tk * D * 2 for q in range(Hq)])
    kq_b = table([Q.data_ptr() + q * Tq * D * 2 for q in range(Hq)])
    kqv_a = table([V.data_ptr() + (q // g) * D * Tk * 2 for q in range(Hq)])
    kqv_b = table([P_.data_ptr() + q * Tq * Tk * 2 for q in range(Hq)])

    def ctab(C, slab, b0, nb):
        return table([C + (b0 + i) * slab * 4 for i in range(nb)])

    tabs = {}

    def ptr_call(key, a, b, m, n, k, lda, slab, C, b0, nb):
        if (key, C, b0) not in tabs:
            tabs[(key, C, b0)] = ctab(C, slab, b0, nb)
        return h.gemm_batched_ex(1, 0, m, n, k, 1.0, a.data_ptr() + b0 * 8, code, lda, b.data_ptr() + b0 * 8, code, lda,
                                 0.0, tabs[(key, C, b0)].data_ptr(), f32, m, nb)

    batch_case("c3_kq_pointer_gqa", Hq, Tk * Tq, flop3, Hq * Tk * Tq * 4, "hbm",
               lambda C: ptr_call("kq", kq_a, kq_b, Tk, Tq, D, D, Tk * Tq, C, 0, Hq),
               lambda C, b0, nb: ptr_call("kq", kq_a, kq_b, Tk, Tq, D, D, Tk * Tq, C, b0, nb),
               lambda C, b: gemm_cols(C, b, Tk, Tq, Tk * Tq, K[b // g], Q[b]),
               {"m": Tk, "n": Tq, "k": D, "split": "query heads, whole KV-head groups per rank"})
    batch_case("c3_kqv_pointer_gqa", Hq, D * Tq, flop3, Hq * D * Tq * 4, "hbm",
               lambda C: ptr_call("kqv", kqv_a, kqv_b, D, Tq, Tk, Tk, D * Tq, C, 0, Hq),
               lambda C, b0, nb: ptr_call("kqv", kqv_a, kqv_b, D, Tq, Tk, Tk, D * Tq, C, b0, nb),
               lambda C, b: gemm_cols(C, b, D, Tq, D * Tq, V[b // g], P_[b]),
               {"m": D, "n": Tq, "k": Tk, "split": "query heads, whole KV-head groups per rank"})
    del K, Q, V, P_, kq_a, kq_b, kqv_a, kqv_b
    tabs.clear()

    # config 5 MoE: 128 experts, hidden 2048, expert FFN 768, 32 tokens each (balanced top-8 routing)
    E, Hd, Fe, Te = 128, 2048, 768, 32
    Wgu = gen((E, Fe, Hd), 7301, 0.02, dt)
    Wd = gen((E, Hd, Fe), 7302, 0.02, dt)
    Xe = gen((E, Te, Hd), 7303, 1.0, dt)
    He = gen((E, Te, Fe), 7304, 1.0, dt)
    flop5 = 2.0 * Fe * Te * Hd * E
    for nm, W, X, m, k in (("c5_moe_gate_up_pointer", Wgu, Xe, Fe, Hd), ("c5_moe_down_pointer", Wd, He, Hd, Fe)):
        pa = table([W.data_ptr() + e * m * k * 2 for e in range(E)])
        pb = table([X.data_ptr() + e * Te * k * 2 for e in range(E)])
        batch_case(nm, E, m * Te, flop5, E * m * Te * 4, "hbm",
                   lambda C, pa=pa, pb=pb, m=m, k=k, nm=nm: ptr_call(nm, pa, pb, m, Te, k, k, m * Te, C, 0, E),
                   lambda C, b0, nb, pa=pa, pb=pb, m=m, k=k, nm=nm: ptr_call(nm, pa, pb, m, Te, k, k, m * Te, C, b0, nb),
                   lambda C, b, W=W, X=X, m=m: gemm_cols(C, b, m, Te, m * Te, W[b], X[b]),
                   {"m": m, "n": Te, "k": k, "split": "experts"})
    offs_full = torch.arange(0, (E + 1) * Te, Te, dtype=torch.int32, device="cuda")
    batch_case("c5_moe_gate_up_grouped_balanced", E, Fe * Te, flop5, E * Fe * Te * 4, "hbm",
               lambda C: h.gemm_grouped_ex(1, 0, Fe, E * Te, Hd, E, offs_full.data_ptr(), 1.0, Wgu.data_ptr(), code, Hd,
                                           Fe * Hd, Xe.data_ptr(), code, Hd, 0.0, C, f32, Fe),
               lambda C, b0, nb: h.gemm_grouped_ex(1, 0, Fe, nb * Te, Hd, nb, offs_full.data_ptr(), 1.0,
                                                   Wgu.data_ptr() + b0 * Fe * Hd * 2, code, Hd, Fe * Hd,
                                                   Xe.data_ptr() + b0 * Te * Hd * 2, code, Hd, 0.0,
                                                   C + b0 * Te * Fe * 4, f32, Fe),
               lambda C, b: gemm_cols(C, b, Fe, Te, Fe * Te, Wgu[b], Xe[b]),
               {"m": Fe, "n": Te, "k": Hd, "split": "experts (grouped GEMM, offsets on the device)"})
    del Wgu, Wd, Xe, He
    tabs.clear()
    torch.cuda.empty_cache()
    return out


class _Dev:
    """A raw device range seen by torch through __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr, count):
        self.__cuda_array_interface__ = {"shape": (count,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None, "stream": None}



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


# candidate plans at N > 1: which projections are N-sharded and how their rows reach the peers ("ce": the copy
# engines push them after the GEMM, to every peer at once, overlapping the projections that follow; "ring": the
# same pushes one peer after another in ring order; "ring2": two such rings at once; "p2p": the GEMM
# epilogue stores them into the
# peers' C over NVLink); the others run whole on every rank. A plan uses one copy-engine mode. Each is timed as a
# whole step on every rank at set-up and the fastest kept. The copy engines win with one peer and lose with more
# (their pushes to several peers at once ran at 300-400 GB/s in all against 585-677 GB/s to one; along a ring
# 472-489 GB/s at P = 8), the epilogue stores hold ~550-590 GB/s: so both are candidates, alone and mixed.
_ALL = ("q", "k", "v", "o", "gate", "up", "down", "lm_head")
PLANS = [
    {},
    {"lm_head": "ce"}, {"lm_head": "ring"}, {"lm_head": "ring2"}, {"lm_head": "p2p"},
    {"lm_head": "ring", "gate": "ring", "up": "ring"}, {"lm_head": "ring2", "gate": "ring2", "up": "ring2"},
    {"lm_head": "ce", "gate": "ce", "up": "ce"}, {"lm_head": "p2p", "gate": "ce", "up": "ce"},
    {"lm_head": "p2p", "gate": "p2p", "up": "p2p"},
    {"lm_head": "ce", "gate": "ce", "up": "ce", "down": "ce"}, {"lm_head": "p2p", "down": "p2p"},
    {"lm_head": "ce", "gate": "ce", "up": "ce", "down": "ce", "q": "ce", "o": "ce"},
    {n: "ce" for n in _ALL}, {n: "p2p" for n in _ALL},
]


def plan_name(plan):
    return "+".join(f"{n}:{m}" for n, m in plan.items()) or "none"


def run(args):
    import torch
    import torch.distributed as dist
    from macuda_b200 import cublas as cb

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    all_cpus = os.sched_getaffinity(0)
    host_cpus = bind_to_gpu_cpus(torch, local)
    if world > 1:
        from datetime import timedelta
        # NCCL's initialisation lines (communicator size, ranks, transports) go to stderr, so that the rank count
        # can be read from the log; stdout carries only the JSON line
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
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
    names = [L["name"] for L in layers]
    stream = torch.cuda.Stream()
    h = lib.handle()
    h.set_stream(stream.cuda_stream)
    exchange = args.exchange if world > 1 else "none"
    if exchange in ("fused", "p2p"):
        exchange = "p2p"
    runners = [None] * len(layers)
    order = list(range(len(layers)))
    copies, comm = None, None
    finish = lambda: None  # noqa: E731  completes the step's exchange on the compute stream
    finish_barrier = False  # whether finish() ends with a barrier of every rank
    if world > 1:
        from macuda_b200.dist import (CopyEngineShardedGemm, CopyStreams, FusedShardedGemm, ReplicatedGemm,
                                      ShardedGemm, pick_fastest, step_barrier)
        if exchange in ("auto", "ce"):
            copies = CopyStreams(world)
            lanes = {"ce": copies, "ring": CopyStreams(world, lanes=1), "ring2": CopyStreams(world, lanes=2)}
            plans = [pl for pl in PLANS if exchange == "auto" or all(v in lanes for v in pl.values())]
            if args.shard == "sharded":
                plans = [{n: ("ce" if exchange == "ce" else "p2p") for n in names}]
            elif args.shard == "whole":
                plans = [{}]
            used = {m for pl in plans for m in pl.values()}
            ce = [CopyEngineShardedGemm(lib, h, L["m"], TOKENS, L["k"], rank, world, L["w"], ctype, copies)
                  if used & set(lanes) else None for L in layers]
            pp = [FusedShardedGemm(lib, h, L["m"], TOKENS, L["k"], rank, world, L["w"], ctype, exchange="p2p")
                  if "p2p" in used else None for L in layers]
            whole = [ReplicatedGemm(lib, h, L["m"], TOKENS, L["k"], L["w_full"], ctype) for L in layers]

            def plan_order(plan):
                """copy-engine shards first (their copies overlap what follows), then epilogue shards, then whole"""
                rank_of = {"ce": 0, "ring": 0, "ring2": 0, "p2p": 1}
                return sorted(range(len(layers)), key=lambda i: (rank_of.get(plan.get(names[i]), 2), i))

            def runner_of(plan, i):
                mode = plan.get(names[i])
                return ce[i] if mode in lanes else pp[i] if mode == "p2p" else whole[i]

            def copies_of(plan):
                modes = [m for m in plan.values() if m in lanes]
                return lanes[modes[0]] if modes else copies

            def plan_step(plan):
                cs = copies_of(plan)
                for i in plan_order(plan):
                    g = runner_of(plan, i)
                    if g is ce[i]:
                        g.copies = cs
                    if g.run(acts[layers[i]["src"]], stream) != 0:
                        raise RuntimeError(f"{names[i]}: GEMM failed")
                if set(plan.values()) & set(lanes):
                    cs.join(stream)
                if plan:
                    step_barrier(stream)

            if len(plans) > 1:
                # every candidate plan timed as a whole step on every rank (max over ranks), the fastest kept: the
                # same choice everywhere
                times = torch.zeros(len(plans), dtype=torch.float64, device="cuda")
                for pi, plan in enumerate(plans):
                    for _ in range(3):
                        plan_step(plan)
                    torch.cuda.synchronize()
                    dist.barrier()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record(stream)
                    for _ in range(10):
                        plan_step(plan)
                    e1.record(stream)
                    torch.cuda.synchronize()
                    times[pi] = e0.elapsed_time(e1) / 10
                    dist.barrier()
                dist.all_reduce(times, op=dist.ReduceOp.MAX)
                plan = plans[int(torch.argmin(times).item())]
                plan_times = {plan_name(pl): round(float(t), 4) for pl, t in zip(plans, times.tolist())}
            else:
                plan, plan_times = plans[0], None
            for i in range(len(layers)):
                keep = runner_of(plan, i)
                for g in (ce[i], pp[i], whole[i]):
                    if g is not None and g is not keep:
                        g.close()
                runners[i] = keep
            order = plan_order(plan)
            sharded_set = tuple(n for n in names if n in plan)
            plan_modes = dict(plan)
            copies = copies_of(plan)
            for i in range(len(layers)):
                if runners[i] is ce[i]:
                    runners[i].copies = copies
            if plan:
                finish_barrier = True

                def finish():
                    if set(plan.values()) & set(lanes):
                        copies.join(stream)
                    step_barrier(stream)
        elif exchange in ("p2p", "multicast"):
            plan_times = None
            for i, L in enumerate(layers):
                # N-sharded (rows exchanged by the epilogue) or whole on every rank (nothing exchanged): the
                # faster of the two, timed on every rank (max over ranks) during set-up
                cands = {"sharded": FusedShardedGemm(lib, h, L["m"], TOKENS, L["k"], rank, world, L["w"], ctype,
                                                     exchange=exchange),
                         "whole": ReplicatedGemm(lib, h, L["m"], TOKENS, L["k"], L["w_full"], ctype)}
                choice = pick_fastest(cands, acts[L["src"]], stream) if args.shard == "auto" else args.shard
                for key, c in cands.items():
                    if key != choice:
                        c.close()
                runners[i] = cands[choice]
            sharded_set = tuple(n for n, g in zip(names, runners) if g.exchange != "replicated")
            plan_modes = {n: exchange for n in sharded_set}
            if sharded_set:
                finish_barrier = True

                def finish():
                    step_barrier(stream)  # every peer's stores into this rank's C have landed
        else:  # NCCL all-gather + layout kernel, every projection sharded
            plan_times = None
            comm = torch.cuda.Stream()
            runners = [ShardedGemm(lib, h, L["m"], TOKENS, L["k"], rank, world, L["w"], ctype) for L in layers]
            sharded_set = tuple(names)
            plan_modes = {n: "allgather" for n in names}

            def finish():
                stream.wait_stream(comm)
    else:
        sharded_set, plan_times, plan_modes = (), None, {}
    for L in layers:
        L.pop("w_full", None)  # whole weights stay only where a projection runs whole on every rank

    def launch(i, act):
        L = layers[i]
        if world == 1:
            return gemm_call(h, cb, L, act, ctype, L["c_local"].data_ptr(), L["m"])
        if exchange == "allgather":  # this rank's rows, then the all-gather + layout on the comm stream
            return runners[i].run(act, stream, comm)
        return runners[i].run(act, stream)

    def step(src, marks=None, before=None, pre_finish=None):
        """One step: every projection once, in `order` (the N-sharded ones first, so that their exchange
        overlaps the rest), then the exchange's completion. marks: {i: (event, event)} recorded around GEMM i;
        before: {i: f} called just before GEMM i is enqueued; pre_finish: called before the completion."""
        for i in order:
            if before is not None and i in before:
                before[i]()
            if marks is not None and i in marks:
                marks[i][0].record(stream)
            st = launch(i, src[layers[i]["src"]])
            if marks is not None and i in marks:
                marks[i][1].record(stream)
            if st != 0:
                raise RuntimeError(f"{names[i]}: status {st}")
        if pre_finish is not None:
            pre_finish()
        finish()

    # Inside the timed region the only events are the two around the dominant GEMM (lm_head, the roofline
    # kernel): an event between two kernels would also stop the next one from being scheduled while the
    # previous one finishes (programmatic dependent launch). The per-projection breakdown comes from a
    # separate pass after the timed region, with events around every GEMM.
    dom = names.index("lm_head")
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    marks = [{dom: (ev(), ev())} for _ in range(args.steps)]
    launches_per_step = len(layers) * (2 if exchange == "allgather" else 1)

    for _ in range(args.warmup):
        step(acts)
    torch.cuda.synchronize()
    clocks = ClockSampler(local) if not args.no_clocks else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    if clocks:
        clocks.mark(True)
    e0.record(stream)
    for j in range(args.steps):
        step(acts, marks[j])
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
    dom_ms = sum(marks[j][dom][0].elapsed_time(marks[j][dom][1]) for j in range(args.steps)) / args.steps

    # the per-projection breakdown, after the timed region: events around every GEMM
    n_bd = min(args.steps, 20)
    per_gemm_ms = [0.0] * len(layers)
    bd = [{i: (ev(), ev()) for i in range(len(layers))} for _ in range(n_bd)]
    for j in range(n_bd):
        step(acts, bd[j])
    torch.cuda.synchronize()
    for j in range(n_bd):
        for i in range(len(layers)):
            per_gemm_ms[i] += bd[j][i][0].elapsed_time(bd[j][i][1]) / n_bd
    value = STEP_FLOP / (ms * 1e-3) / 1e12
    gemm_only_ms = sum(per_gemm_ms)  # this rank's GEMMs alone (the exchange's copies run on other streams)
    if world > 1:
        t = torch.tensor([gemm_only_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        gemm_only_ms = float(t.item())

    def m_run(i):  # rows the GEMM of projection i computes on this rank
        return layers[i]["mp"] if names[i] in sharded_set else layers[i]["m"]

    pk = peaks()
    L = layers[dom]
    dom_flop = 2.0 * m_run(dom) * TOKENS * L["k"]
    dom_tflops = dom_flop / (dom_ms * 1e-3) / 1e12
    traffic = None
    prof = os.path.join(ROOT, "profiles", "roofline_traffic.json")
    if os.path.exists(prof) and world == 1 and args.impl == "ours":
        try:
            with open(prof) as f:
                traffic = json.load(f).get("lm_head_dram_bytes")
        except Exception:
            traffic = None
    # the timed region lasts milliseconds (args.steps steps of well under 1 ms): the burst peak is the denominator
    roofline = {"bound": "tensor", "achieved": round(dom_tflops, 2), "peak": pk["bf16_tflops"],
                "unit": "TFLOP/s", "frac": round(dom_tflops / pk["bf16_tflops"], 4), "traffic": traffic,
                "kernel": "lm_head GEMM (%d x %d x %d)" % (m_run(dom), TOKENS, L["k"]),
                "peak_source": ("measured bf16 burst (cuBLAS 8192^3, MEASURED_PEAKS.json)" if pk["source"] == "measured"
                                else "fallback bf16 burst (1.59 PFLOP/s, an earlier measurement on this pool: "
                                     "MEASURED_PEAKS.json was absent)") +
                               ": the timed region is %.1f ms long, far from the seconds-long loop of the sustained "
                               "figure" % (ms * args.steps),
                "frac_of_sustained": round(dom_tflops / pk["bf16_tflops_sustained"], 4),
                "algorithmic_bytes": m_run(dom) * L["k"] * 2 + TOKENS * L["k"] * 2 + m_run(dom) * TOKENS * 4}

    shapes = {names[i]: {"m": m_run(i), "n": TOKENS, "k": layers[i]["k"],
                         "ran": ("N-sharded" if names[i] in sharded_set else "whole on every rank") if world > 1
                         else "single GPU",
                         "us": round(per_gemm_ms[i] * 1e3, 2),
                         "TFLOP/s": round(2.0 * m_run(i) * TOKENS * layers[i]["k"] / (per_gemm_ms[i] * 1e-3) / 1e12, 1)}
              for i in range(len(layers))}

    # e2e through the public API with host buffers: each step copies its activations from pinned host
    # memory (double-buffered on a host-to-device stream, overlapping the previous step) and reads back the
    # last token's logits (on a stream of their own, after lm_head, so that the next step's activation copy does
    # not queue behind it; the next step's lm_head, which overwrites that C, waits for the read). At N > 1 each
    # rank copies 1/N of the packed activations over its own host link and the copy engines push that slice
    # into every peer's buffer (CUDA IPC) while the step runs; the step's barrier, which waits for this rank's
    # pushes, tells every rank that the next step's inputs are whole, and a buffer is refilled only after the
    # barrier that follows its last reader.
    logits = torch.empty(VOCAB, dtype=torch.float32).pin_memory()
    h2d, d2h = torch.cuda.Stream(), torch.cuda.Stream()
    lm_done, read_done = torch.cuda.Event(), torch.cuda.Event()
    n_e2e = max(3, min(args.steps, 100))

    def c_of(i):
        return layers[i]["c_local"] if world == 1 else runners[i].c

    nxt_of_dom = order[order.index(dom) + 1] if order.index(dom) + 1 < len(order) else None
    e2e_ipc = []
    if world == 1:
        hx = {"x": acts["x"].cpu().pin_memory(), "h": acts["h"].cpu().pin_memory()}
        dev_bufs = [{"x": torch.empty_like(acts["x"]), "h": torch.empty_like(acts["h"])} for _ in range(2)]
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        h2d_bytes = int(hx["x"].numel() * 2 + hx["h"].numel() * 2)

        def stage(b):
            with torch.cuda.stream(h2d):
                h2d.wait_event(free[b])
                dev_bufs[b]["x"].copy_(hx["x"], non_blocking=True)
                dev_bufs[b]["h"].copy_(hx["h"], non_blocking=True)
                ready[b].record(h2d)
    else:
        from macuda_b200.dist import CopyStreams, IpcReplicas, _DeviceArray, step_barrier
        nx, nh = acts["x"].numel(), acts["h"].numel()
        esz = acts["x"].element_size()
        chunk = -(-(nx + nh) // world)
        packed = torch.zeros(world * chunk, dtype=acts["x"].dtype, device="cuda")
        packed[:nx] = acts["x"].reshape(-1)
        packed[nx:nx + nh] = acts["h"].reshape(-1)
        hshard = packed[rank * chunk:(rank + 1) * chunk].cpu().pin_memory()
        del packed
        e2e_ipc = [IpcReplicas(lib, world * chunk * esz, rank, world) for _ in range(2)]
        full = [torch.as_tensor(_DeviceArray(r.own, world * chunk, "<i2"), device="cuda").view(acts["x"].dtype)
                for r in e2e_ipc]
        dev_bufs = [{"x": f[:nx].view(acts["x"].shape), "h": f[nx:nx + nh].view(acts["h"].shape)} for f in full]
        # the plan's copy streams when it has them: the input pushes then queue behind the step's exchange on
        # the same engines instead of running alongside it (on streams of their own they slowed it: copy-engine
        # pushes to several peers at once do not add up)
        in_lanes = copies if copies is not None else CopyStreams(world, lanes=1)
        bar_done = torch.cuda.Event()
        bar_done.record(stream)
        h2d_bytes = int(chunk * esz)

        def stage(b):  # this rank's slice from the host, at the start of the step before the one that reads it
            with torch.cuda.stream(h2d):
                h2d.wait_event(bar_done)  # every rank has passed the barrier after buffer b's last reader
                full[b][rank * chunk:(rank + 1) * chunk].copy_(hshard, non_blocking=True)

        def push(b):
            """The slice to every peer, queued on the copy streams after this step's exchange (which is the
            step's longest path: the pushes ahead of it, waiting for the host copy, delayed it), then the compute
            stream waits for them before the step's barrier."""
            in_lanes.after(h2d)
            if lib.lib.tb200_push_block(e2e_ipc[b].array, world, rank, rank * chunk, chunk, 0, 1, world * chunk, esz,
                                        in_lanes.array, in_lanes.lanes) != 0:
                raise RuntimeError("tb200_push_block failed")
            in_lanes.join(stream)

    def e2e_step(i):
        b = i % 2
        if world == 1:
            stage(b)
            stream.wait_event(ready[b])
        after_lm = lambda: lm_done.record(stream)  # noqa: E731
        before = {dom: lambda: stream.wait_event(read_done)}  # the previous step's read of this C has finished
        if nxt_of_dom is not None:
            before[nxt_of_dom] = after_lm
        if world == 1:
            step(dev_bufs[b], before=before)
            if nxt_of_dom is None:
                after_lm()
            free[b].record(stream)
        else:
            stage(1 - b)  # the next step's inputs, while this step runs
            step(dev_bufs[b], before=before, pre_finish=lambda: push(1 - b))
            if not finish_barrier:
                step_barrier(stream)
            bar_done.record(stream)
        with torch.cuda.stream(d2h):  # lm_head's C is complete after its GEMM (and, at N > 1, the barrier)
            d2h.wait_event(lm_done if world == 1 else bar_done)
            logits.copy_(c_of(dom)[(TOKENS - 1) * VOCAB:TOKENS * VOCAB], non_blocking=True)
            read_done.record(d2h)

    if world > 1:  # the first step's inputs, staged before the loop
        stage(0)
        push(0)
        step_barrier(stream)
        bar_done.record(stream)
    # this box's host-to-device rate for one step's worth of this rank's inputs (pinned, one copy, 5 times): the
    # e2e figure follows it wherever the copies outlast the step
    probe_src = torch.empty(h2d_bytes, dtype=torch.uint8).pin_memory()
    probe_dst = torch.empty(h2d_bytes, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    p0, p1 = ev(), ev()
    with torch.cuda.stream(h2d):
        probe_dst.copy_(probe_src, non_blocking=True)
        p0.record(h2d)
        for _ in range(5):
            probe_dst.copy_(probe_src, non_blocking=True)
        p1.record(h2d)
    torch.cuda.synchronize()
    h2d_gbps = h2d_bytes * 5 / (p0.elapsed_time(p1) * 1e-3) / 1e9
    del probe_src, probe_dst
    for i in range(4):  # an even count: the timed steps go on alternating the two input buffers
        e2e_step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
        torch.cuda.synchronize()
    f0, f1 = ev(), ev()
    f0.record(stream)
    t_wall = time.perf_counter()
    for i in range(n_e2e):
        e2e_step(i)
    stream.wait_event(read_done)  # the last step's logits are on the host inside the timed region
    f1.record(stream)
    torch.cuda.synchronize()
    t_wall = time.perf_counter() - t_wall
    e2e_ms = f0.elapsed_time(f1) / n_e2e
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e = {"value": round(STEP_FLOP / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
           "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": VOCAB * 4,
           "ms_per_step": round(e2e_ms, 4), "wall_ms_per_step": round(t_wall * 1e3 / n_e2e, 4), "steps": n_e2e,
           "host_cpus": host_cpus, "h2d_probe_GBps": round(h2d_gbps, 1),
           "inputs": "all activations from this GPU's pinned host memory" if world == 1 else
                     f"1/{world} of the activations from each rank's pinned host memory (h2d_bytes_per_step, per "
                     f"rank), pushed to every peer by the copy engines over NVLink"}
    if e2e_ipc:
        del dev_bufs, full
        for r in e2e_ipc:
            r.close()

    # parity of every projection's C as every rank holds it after the last step (each peer's rows included),
    # against fp64 on sampled rows
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    par = {"ok": True, "norm_err": 0.0, "ref_metric": 0.0, "rows_per_projection": 0}
    for i in range(len(layers)):
        Li = layers[i]
        r = check_rows(torch, c_of(i), Li["m"], TOKENS, Li["check_rows"], Li["w_check"], acts[Li["src"]])
        par["ok"] = par["ok"] and r["ok"]
        par["norm_err"] = max(par["norm_err"], r["norm_err"])
        par["ref_metric"] = max(par["ref_metric"], r["ref_metric"])
        par["rows_per_projection"] = max(par["rows_per_projection"], int(Li["check_rows"].numel()))
    if world > 1:
        t = torch.tensor([par["norm_err"], par["ref_metric"], 0.0 if par["ok"] else 1.0], device="cuda",
                         dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        par.update(norm_err=float(t[0].item()), ref_metric=float(t[1].item()), ok=float(t[2].item()) == 0.0)
    par.update(ranks_checked=world, tol=2.0 ** -10, columns="all %d" % TOKENS,
               how="every rank: the first, middle and last row of each of 8 row shards (every peer's rows at any "
                   "N <= 8) plus 24 seeded rows of each projection's C, against fp64 W_rows X^T on the device; "
                   "max over ranks")
    par["norm_err"] = float("%.3e" % par["norm_err"])
    par["ref_metric"] = float("%.3e" % par["ref_metric"])

    cpu = None
    if rank == 0 and world == 1 and args.impl == "ours" and not args.no_cpu_baseline:
        try:
            os.sched_setaffinity(0, all_cpus)  # the CPU baseline takes every host core it can
            cpu = run_cpu_baseline()
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"error": str(ex)[:200]}

    decode = None
    if rank == 0 and world == 1 and not args.no_decode:
        decode = decode_figures(torch, lib, cb, ctype, dtype)
    probes = None
    if rank == 0 and world == 1 and args.impl == "ours":
        probes = probe_figures(torch, lib)
    configs = None
    if rank == 0 and world == 1 and not args.no_configs:
        cs = ClockSampler(local, period_ms=20) if not args.no_clocks else None
        if cs:
            cs.start()
            time.sleep(0.3)
        try:
            configs = config_figures(torch, lib, cb, ctype, dtype, clocks=cs)
        finally:
            if cs:
                cs.stop()
    sharded = None
    if world > 1 and args.impl == "ours" and not args.no_sharded_shapes:
        sharded = sharded_figures(torch, lib, cb, h, stream, rank, world, CopyStreams(world),
                                  CopyStreams(world, lanes=1))

    for g in runners:
        if g is not None and hasattr(g, "close"):
            g.close()
    h.close()
    if rank == 0:
        how = {"ce": "N-sharded, rows pushed to every peer at once by the copy engines",
               "ring": "N-sharded, rows pushed by the copy engines to one peer after another (ring order)",
               "ring2": "N-sharded, rows pushed by the copy engines along two rings of peers at once",
               "p2p": "N-sharded, rows stored into every peer's C by the GEMM epilogue (P2P)",
               "multicast": "N-sharded, rows stored through an NVLink multicast address by the GEMM epilogue",
               "allgather": "N-sharded, C exchanged by NCCL all-gather + layout kernel"}
        if world == 1:
            par_note = "single GPU"
        else:
            par_note = f"x{world}: " + ", ".join(f"{names[i]} " + how.get(plan_modes.get(names[i]), "whole on every rank")
                                                 for i in order)
            if plan_modes:
                par_note += "; copy-engine shards run first so their copies overlap the rest; one NCCL barrier per step"
        line = {
            "metric": "GEMM TFLOP/s (Llama-3.1-8B prefill projection set, 512 tokens, %s -> f32, ggml's T,N call)"
                      % args.dtype,
            "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": args.dtype, "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) activations; no checkpoint)",
            "config": {"workload": "llama3.1-8b prefill projections q,k,v,o,gate,up,down,lm_head @ 512 tokens "
                                   "(BASELINE configs[1])", "tokens": TOKENS, "step_gflop": round(STEP_FLOP / 1e9, 1),
                       "parallelism": par_note, "exchange": exchange if world > 1 else None,
                       "l2": "inputs larger than L2 (1.9 GB per step); no flush"},
            "frac_of_peak": round(value / pk["bf16_tflops"], 4),
            # every fraction of a peak in this line (frac_of_peak, roofline, the configs' frac_of_measured_peak)
            # divides by these: MEASURED_PEAKS.json's figures, or the profiling recipe's fallback when it is absent
            "peaks": {"source": pk["source"], "hbm_gbs": pk["hbm_gbs"], "bf16_tflops": pk["bf16_tflops"],
                      "bf16_tflops_sustained": pk["bf16_tflops_sustained"]},
            "parity": par,
            "roofline": roofline, "shapes": shapes,
            "shapes_note": "per-projection device time from %d further steps after the timed region, events around "
                           "every GEMM (events between kernels stop the next one being scheduled early, so these "
                           "sum to more than ms_per_step); m is the rows the GEMM computed on each rank" % n_bd,
            "gpu_launches": launches_per_step * args.steps,
            "gemm_only": {"ms_per_step": round(gemm_only_ms, 4),
                          "TFLOP/s": round(STEP_FLOP / (gemm_only_ms * 1e-3) / 1e12, 2),
                          "note": "sum of the per-projection GEMM times (max over ranks); at N > 1 the exchange runs "
                                  "on other streams or engines and the step time includes it"},
        }
        if plan_times:
            line["plan_search_ms"] = plan_times
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
        if probes:
            line["hbm_probes"] = probes
        if configs:
            line["configs_3_5"] = configs
        if sharded:
            line["sharded_shapes"] = sharded
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
                    help="N > 1: which projections are N-sharded (the rest run whole on every rank); auto: the fastest "
                         "plan, timed on every rank at set-up")
    ap.add_argument("--exchange", choices=["auto", "ce", "fused", "multicast", "p2p", "allgather"], default="auto",
                    help="N > 1: how the sharded C is replicated (auto = the fastest plan of copy-engine and epilogue "
                         "shards, timed at set-up; ce = copy-engine plans only; fused = p2p = per projection, epilogue "
                         "stores or whole)")
    ap.add_argument("--no-sharded-shapes", action="store_true",
                    help="N > 1: skip the per-shape sharded figures (squares, lm_head, FFN, configs 3 and 5)")
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
