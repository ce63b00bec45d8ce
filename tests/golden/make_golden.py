"""Writes the golden fixtures the oracle and the library are pinned against.

    python tests/golden/make_golden.py

reference_rows.json   rows transcribed from the reference's own host tests (file:line cited per table):
                      the type contract (cuda-shim/test/cublas_contract.c:36-50) and the split-K plan
                      (cuda-shim/test/splitk_dispatch.c:19-31), each with the outcome the reference expects.
known_answers.json    the reference's value-checked known-answer GEMMs (cuda-shim/test/link_smoke.c),
                      with the expected C computed here in exact integer arithmetic, independently of
                      the oracle: the 48x48x48 Sgemm on small integers (:41-52, checked for exact
                      equality there) and the 4x4x4 f16-out COMPUTE_16F GemmEx (:59-75).
Neither file depends on anything outside this script.
"""
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))

# cudaDataType and cublasComputeType_t values (CUDA 12.9 library_types.h / cublas_api.h)
R32F, R16F, R16BF = 0, 2, 14
C16F, C32F, C64F, C32I, C32F_TF32 = 64, 68, 70, 72, 77
SUCCESS, NOT_SUPPORTED = 0, 15

CONTRACT = {
    "source": "cuda-shim/test/cublas_contract.c:36-50",
    "columns": ["what", "Atype", "Btype", "Ctype", "computeType", "expected_status"],
    "rows": [
        ["bf16 x bf16 -> f32, COMPUTE_32F (ggml's bf16)", R16BF, R16BF, R32F, C32F, SUCCESS],
        ["bf16 x bf16 -> bf16, COMPUTE_32F", R16BF, R16BF, R16BF, C32F, SUCCESS],
        ["f16 x f16 -> f16, COMPUTE_16F (ggml's f16)", R16F, R16F, R16F, C16F, SUCCESS],
        ["f16 x f16 -> f32, COMPUTE_32F", R16F, R16F, R32F, C32F, SUCCESS],
        ["f32 x f32 -> f32, COMPUTE_32F_FAST_TF32", R32F, R32F, R32F, C32F_TF32, SUCCESS],
        ["f16 x bf16 (mismatched A/B)", R16F, R16BF, R32F, C32F, NOT_SUPPORTED],
        ["bf16 x f16 (mismatched A/B)", R16BF, R16F, R32F, C32F, NOT_SUPPORTED],
        ["f32 x f16 (mismatched A/B)", R32F, R16F, R32F, C32F, NOT_SUPPORTED],
        ["bf16 with COMPUTE_16F", R16BF, R16BF, R32F, C16F, NOT_SUPPORTED],
        ["f16 COMPUTE_16F with an f32 C", R16F, R16F, R32F, C16F, NOT_SUPPORTED],
        ["f32 with COMPUTE_64F", R32F, R32F, R32F, C64F, NOT_SUPPORTED],
        ["f32 with COMPUTE_32I", R32F, R32F, R32F, C32I, NOT_SUPPORTED],
        ["bf16 with COMPUTE_32F_FAST_TF32", R16BF, R16BF, R32F, C32F_TF32, NOT_SUPPORTED],
    ],
}

PLAN = {
    "source": "cuda-shim/test/splitk_dispatch.c:19-31 (plan for the RTX 5090's 170 SMs, cublas.c:69-78)",
    "num_sms": 170,
    "columns": ["what", "m", "n", "k", "batch", "expected_S"],
    "rows": [
        ["k/v (3B decode)", 256, 32, 2048, 1, 16],
        ["q/o (3B decode)", 2048, 32, 2048, 1, 8],
        ["down (3B decode)", 2048, 32, 11008, 1, 8],
        ["gate/up (3B decode): gx 172, never split", 11008, 32, 2048, 1, 1],
        ["diffusion mix: gy 4, never split", 1280, 256, 1280, 1, 1],
        ["boundary gx 169 splits", 169 * 64, 32, 2048, 1, 2],
        ["boundary gx 170 does not", 170 * 64, 32, 2048, 1, 1],
        ["boundary n 64 (gy 1) splits", 2048, 64, 2048, 1, 8],
        ["boundary n 65 (gy 2) does not", 2048, 65, 2048, 1, 1],
        ["k 2047 cannot keep 4 tiles in 16 slices", 256, 32, 2047, 1, 8],
        ["k 255: 4 tiles need k >= 256 for S 2", 2048, 32, 255, 1, 1],
        ["workspace bound: batch 3 of q/o is 12 MiB", 2048, 32, 2048, 3, 1],
        ["workspace bound: batch 2 of q/o is 8 MiB", 2048, 32, 2048, 2, 8],
    ],
}


def sgemm48():
    N = 48
    A = [(i % 7) - 3 for i in range(N * N)]
    B = [((i * 5) % 4) - 1 for i in range(N * N)]
    C = [0] * (N * N)
    for col in range(N):
        for row in range(N):
            C[row + col * N] = sum(A[row + k * N] * B[k + col * N] for k in range(N))
    return {"source": "cuda-shim/test/link_smoke.c:41-52", "op": "NN", "m": N, "n": N, "k": N, "lda": N,
            "ldb": N, "ldc": N, "alpha": 1.0, "beta": 0.0, "type": "f32", "compute": C32F, "check": "exact",
            "A": A, "B": B, "C": C}


def gemm16_4x4():
    M = 4
    A = [(i % 7) - 3 for i in range(M * M)]
    B = [((i * 5) % 4) - 1 for i in range(M * M)]
    C = [0] * (M * M)
    for col in range(M):
        for row in range(M):
            C[row + col * M] = sum(A[row + k * M] * B[k + col * M] for k in range(M))
    return {"source": "cuda-shim/test/link_smoke.c:59-75", "op": "NN", "m": M, "n": M, "k": M, "lda": M,
            "ldb": M, "ldc": M, "alpha": 1.0, "beta": 0.0, "type": "f16", "out": "f16", "compute": C16F,
            "check": "rel 1e-2 + abs 1e-2 (link_smoke.c:71)", "A": A, "B": B, "C": C}


def main():
    with open(os.path.join(HERE, "reference_rows.json"), "w") as f:
        json.dump({"contract": CONTRACT, "splitk_plan": PLAN}, f, indent=1)
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump({"sgemm48": sgemm48(), "gemm16_4x4": gemm16_4x4()}, f)
    print("wrote reference_rows.json, known_answers.json")


if __name__ == "__main__":
    main()
