"""The drop-in claim from C: tests/c_caller/ggml_calls.c makes ggml-cuda's cuBLAS calls through CUDA's own
cublas_v2.h and is linked with -ltinycublas_b200 where ggml-cuda links -lcublas. On the CPU: it builds,
and every cuBLAS symbol it imports resolves to this library (no libcublas anywhere). On the GPU: it runs,
and every element of every call matches the host's exact integer arithmetic."""
import os
import subprocess

import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "c_caller")
EXE = os.path.join(HERE, "ggml_calls")


def _build():
    r = subprocess.run(["make", "-s", "-C", HERE], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    return EXE


def test_c_caller_links_against_this_library(lib):
    exe = _build()
    deps = subprocess.run(["ldd", exe], capture_output=True, text=True).stdout
    assert "libtinycublas_b200.so" in deps
    assert "libcublas" not in deps
    undefined = subprocess.run(["nm", "-D", "--undefined-only", exe], capture_output=True, text=True).stdout
    wanted = {line.split()[-1] for line in undefined.splitlines() if "cublas" in line}
    assert {"cublasCreate_v2", "cublasGemmEx", "cublasGemmBatchedEx", "cublasGemmStridedBatchedEx",
            "cublasSgemm_v2", "cublasSetStream_v2", "cublasSetMathMode", "cublasDestroy_v2"} <= wanted
    exported = subprocess.run(["nm", "-D", "--defined-only", lib.path], capture_output=True, text=True).stdout
    have = {line.split()[-1] for line in exported.splitlines()}
    assert wanted <= have, wanted - have


@pytest.mark.gpu
def test_c_caller_runs_exact():
    exe = _build()
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "ALL OK" in r.stdout, r.stdout + r.stderr
