"""Build recipe for libtinycublas_b200.so (sm_100a), in-tree.

    python -m macuda_b200.build            # build if any source is newer than the library
    python -m macuda_b200.build --force    # rebuild everything

Each .cu file is compiled by nvcc for sm_100a only (-gencode arch=compute_100a,code=sm_100a), the C
host layer by gcc against CUDA's own cublas_v2.h, and everything is linked into one shared library
with the static CUDA runtime. A linker version script exports exactly the cuBLAS ABI subset and the
documented tb200_* extensions; -Bsymbolic binds the library's internal calls to its own definitions
even when the process has also loaded NVIDIA's libcublas (as PyTorch does). The static symbol table is
stripped (the exported dynamic symbols stay): it names nvcc's temporary files, whose names carry a
process id, and without it two builds of the same sources are byte-identical (tests/test_build.py).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libtinycublas_b200.so")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

CU_SOURCES = ["gemm_tc.cu", "gemm_simt.cu", "gemm_skinny.cu", "aux_kernels.cu"]
C_SOURCES = ["tinycublas.c"]
HEADERS = ["tb200_internal.h", "tb200_device.cuh", "exports.map"]


def _git_describe() -> str:
    try:
        out = subprocess.run(["git", "-C", ROOT, "describe", "--always", "--dirty"], capture_output=True, text=True,
                             timeout=10)
        return out.stdout.strip() or "unknown"
    except Exception:
        return "unknown"


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.stderr.strip() and os.environ.get("TB200_BUILD_VERBOSE"):
        sys.stderr.write(r.stderr)


def _stale(outputs: list[str], inputs: list[str]) -> bool:
    if not all(os.path.exists(o) for o in outputs):
        return True
    newest_in = max(os.path.getmtime(i) for i in inputs)
    oldest_out = min(os.path.getmtime(o) for o in outputs)
    return newest_in > oldest_out


def build(force: bool = False, verbose: bool = False, lib_path: str = None, build_dir: str = None) -> str:
    """Compile and link the library if needed; returns its path. lib_path / build_dir put a build somewhere
    else than the package (the reproducible-build test builds a second copy and compares the bytes)."""
    LIB_OUT = lib_path or LIB
    BUILD_DIR = build_dir or BUILD
    srcs = [os.path.join(CSRC, f) for f in CU_SOURCES + C_SOURCES + HEADERS]
    srcs.append(os.path.join(ROOT, "include", "tinycublas_b200.h"))
    srcs.append(os.path.abspath(__file__))
    if not force and not _stale([LIB_OUT], srcs):
        return LIB_OUT
    if shutil.which(NVCC) is None and not os.path.exists(NVCC):
        raise RuntimeError(f"nvcc not found at {NVCC}")
    os.makedirs(BUILD_DIR, exist_ok=True)
    os.makedirs(os.path.dirname(os.path.abspath(LIB_OUT)), exist_ok=True)
    inc = ["-I", CSRC, "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA_HOME, "include")]
    jobs = []
    for f in CU_SOURCES:
        obj = os.path.join(BUILD_DIR, f + ".o")
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
               "--expt-relaxed-constexpr", *inc, "-c", os.path.join(CSRC, f), "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        jobs.append((cmd, obj))
    for f in C_SOURCES:
        obj = os.path.join(BUILD_DIR, f + ".o")
        cmd = ["gcc", "-O2", "-fPIC", "-std=c11", "-Wall", "-Wextra", "-Wno-unused-parameter",
               f'-DTB200_GIT_DESCRIBE="{_git_describe()}"', *inc, "-c", os.path.join(CSRC, f), "-o", obj]
        jobs.append((cmd, obj))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(lambda j: _run(j[0]), jobs))
    tmp = LIB_OUT + ".tmp"
    link = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *[o for _, o in jobs],
            "-Xlinker", "-Bsymbolic", "-Xlinker", "--version-script=" + os.path.join(CSRC, "exports.map"),
            "-Xlinker", "--no-undefined", "-Xlinker", "--strip-all", "-lpthread", "-ldl", "-lrt"]
    _run(link)
    os.replace(tmp, LIB_OUT)
    return LIB_OUT


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
