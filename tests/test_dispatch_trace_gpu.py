"""Trace-based dispatch assertions (as the reference greps its `[trace] launch` lines for each projection,
cuda-shim/test/splitk_check.sh:1-32): the configs[1] projections and a decode GEMM issued with
TB200_TRACE=1 in a child process, and each launch line's kernel configuration and grid checked on a
148-SM B200."""
import os
import re
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r'''
import sys, torch
sys.path.insert(0, sys.argv[1])
from macuda_b200 import cublas as cb
lib = cb.library()
h = lib.handle()
for name, m, n, k in [("q", 4096, 512, 4096), ("k", 1024, 512, 4096), ("v", 1024, 512, 4096),
                      ("o", 4096, 512, 4096), ("gate", 14336, 512, 4096), ("up", 14336, 512, 4096),
                      ("down", 4096, 512, 14336), ("lm_head", 128256, 512, 4096), ("decode", 4096, 1, 4096)]:
    W = torch.zeros(m * k, dtype=torch.float16, device="cuda")
    X = torch.zeros(k * n, dtype=torch.float16, device="cuda")
    C = torch.empty(m * n, device="cuda")
    print(f"== {name}", file=sys.stderr, flush=True)
    assert h.gemm_ex(1, 0, m, n, k, 1.0, W.data_ptr(), cb.CUDA_R_16F, k, X.data_ptr(), cb.CUDA_R_16F, k, 0.0,
                     C.data_ptr(), cb.CUDA_R_32F, m) == 0
    torch.cuda.synchronize()
'''

# projection -> (kernel configuration in the launch line, grid x) on 148 SMs (74 CTA pairs); KS=2 is the k
# split (one cluster per tile: two CTAs, or with CG=2 two CTA pairs); the decode kernel's W warps x U chunks
# in flight and S k slices
EXPECTED = {
    "q": ("tb200_gemm_tc<f16,BN=256,KC=1,CG=2,KS=2>", 128),
    "k": ("tb200_gemm_tc<f16,BN=64,KC=2,CG=1,KS=2>", 128),
    "v": ("tb200_gemm_tc<f16,BN=64,KC=2,CG=1,KS=2>", 128),
    "o": ("tb200_gemm_tc<f16,BN=256,KC=1,CG=2,KS=2>", 128),
    "gate": ("tb200_gemm_tc<f16,BN=256,KC=1,CG=2>", 148),
    "up": ("tb200_gemm_tc<f16,BN=256,KC=1,CG=2>", 148),
    "down": ("tb200_gemm_tc<f16,BN=256,KC=1,CG=2,KS=2>", 128),
    "lm_head": ("tb200_gemm_tc<f16,BN=256,KC=2,CG=2>", 148),  # 1002 pair tiles: two k-chunks a stage
    "decode": ("tb200_gemm_skinny<W=16,U=2,S=1>", 256),
}


def test_projection_launches_as_traced(lib):
    import torch
    if torch.cuda.get_device_properties(0).multi_processor_count != 148:
        pytest.skip("the expected grids are for a 148-SM B200")
    env = dict(os.environ, TB200_TRACE="1")
    env.pop("TB200_TC_BN", None)
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], capture_output=True, text=True, env=env, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    seen, cur = {}, None
    for line in r.stderr.splitlines():
        if line.startswith("== "):
            cur = line[3:].strip()
        elif "[trace] launch" in line and cur is not None:
            m = re.search(r"launch (\S+) grid=\((\d+),", line)
            seen.setdefault(cur, []).append((m.group(1), int(m.group(2))))
    for name, (kern, grid) in EXPECTED.items():
        assert seen.get(name) == [(kern, grid)], f"{name}: {seen.get(name)}"
