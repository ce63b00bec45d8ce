"""A routed mixture-of-experts layer through the library's extension entry points: tokens gathered into
expert order (tb200_moe_gather), every expert in one grouped GEMM with its own token count
(tb200_gemm_grouped_ex) - or both in one launch with the gather fused into the GEMM's loads
(tb200_gemm_grouped_gather_ex) - expert outputs combined back into token order with the routing weights
(tb200_moe_combine); checked against an fp64 restatement of the layer, Y[:, t] = sum_j w_tj W_{e_tj}^T x_t."""
import numpy as np
import pytest

from macuda_b200 import cublas as cb
from oracle import oracle as O
from tests.helpers import dev, storage

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def h(lib):
    import torch
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    hh = lib.handle()
    yield hh
    hh.close()


def _routing(rng, T, E, topk):
    """Skewed top-k routing: each token's topk distinct experts drawn from Dirichlet(0.3) shares, weights
    normalised to sum 1. Returns experts [T, topk], weights [T, topk], and the expert-order permutation:
    token_ids [n_total], offsets [E + 1], positions [T, topk] (where token t's j-th copy sits)."""
    share = rng.dirichlet(np.full(E, 0.3))
    experts = np.stack([rng.choice(E, topk, replace=False, p=share) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, (T, topk)).astype(np.float32)
    w /= w.sum(axis=1, keepdims=True)
    order = np.argsort(experts.ravel(), kind="stable")  # (t, j) pairs in expert order
    token_ids = (order // topk).astype(np.int32)
    positions = np.empty(T * topk, np.int32)
    positions[order] = np.arange(T * topk, dtype=np.int32)
    offsets = np.concatenate([[0], np.cumsum(np.bincount(experts.ravel(), minlength=E))]).astype(np.int32)
    return experts, w, token_ids, offsets, positions.reshape(T, topk)


@pytest.mark.parametrize("fused", [False, True], ids=["gather+grouped", "grouped_gather"])
@pytest.mark.parametrize("in_t", [O.F16, O.BF16])
def test_routed_moe_layer(lib, h, in_t, fused):
    import torch
    rng = np.random.default_rng(400)
    E, topk, T, Hd, F = 32, 4, 384, 1024, 512
    experts, w, token_ids, offsets, positions = _routing(rng, T, E, topk)
    assert (np.diff(offsets) == 0).any() or np.diff(offsets).max() > 3 * np.diff(offsets).mean()  # uneven
    n_total = T * topk
    X = storage(rng, Hd * T, in_t)                  # token t: column t, Hd features
    W = storage(rng, E * F * Hd, in_t, 0.02)         # expert e: k = Hd x m = F (op T, lda = Hd)
    dX, dW = dev(X), dev(W)
    ct = {O.F16: cb.CUDA_R_16F, O.BF16: cb.CUDA_R_16BF}[in_t]
    d_ids = torch.from_numpy(token_ids).cuda()
    d_off = torch.from_numpy(offsets).cuda()
    d_pos = torch.from_numpy(positions.ravel().copy()).cuda()
    d_w = torch.from_numpy(w.ravel().copy()).cuda()
    Xp = torch.empty(Hd * n_total, dtype=torch.int16, device="cuda")
    C = torch.full((F * n_total,), float("nan"), device="cuda")
    Y = torch.full((F * T,), float("nan"), device="cuda")
    L = lib.lib
    if fused:  # the gather inside the grouped GEMM's B loads
        assert h.gemm_grouped_gather_ex(1, F, n_total, Hd, E, d_off.data_ptr(), d_ids.data_ptr(), 1.0, dW.data_ptr(),
                                        ct, Hd, F * Hd, dX.data_ptr(), ct, Hd, T, 0.0, C.data_ptr(), cb.CUDA_R_32F,
                                        F) == 0
    else:
        assert L.tb200_moe_gather(h.h, dX.data_ptr(), ct, Hd, Hd, T, d_ids.data_ptr(), n_total, Xp.data_ptr(), Hd) == 0
        assert h.gemm_grouped_ex(1, 0, F, n_total, Hd, E, d_off.data_ptr(), 1.0, dW.data_ptr(), ct, Hd, F * Hd,
                                 Xp.data_ptr(), ct, Hd, 0.0, C.data_ptr(), cb.CUDA_R_32F, F) == 0
    assert L.tb200_moe_combine(h.h, F, C.data_ptr(), F, n_total, d_pos.data_ptr(), d_w.data_ptr(), topk, T,
                               Y.data_ptr(), F) == 0
    torch.cuda.synchronize()
    got = Y.cpu().numpy().reshape(T, F)  # column t of Y = row t here
    assert np.isfinite(got).all()
    # fp64 restatement on sampled output rows, with the gate's normalisation (|w| |W_e row| |x_t| per term)
    rows = np.arange(0, F, 7)
    Xf = O.from_bits(X, in_t).astype(np.float64).reshape(T, Hd)
    Wf = O.from_bits(W, in_t).astype(np.float64).reshape(E, F, Hd)[:, rows, :]
    ref = np.zeros((T, rows.size))
    scale = np.zeros((T, rows.size))
    wn = np.linalg.norm(Wf, axis=2)  # [E, rows]
    xn = np.linalg.norm(Xf, axis=1)  # [T]
    for j in range(topk):
        e = experts[:, j]
        ref += w[:, j:j + 1] * np.einsum("trk,tk->tr", Wf[e], Xf)
        scale += np.abs(w[:, j:j + 1]) * wn[e] * xn[:, None]
    err = np.abs(got[:, rows] - ref) / np.maximum(scale, 1e-30)
    assert err.max() <= 2.0 ** -10, f"max normalised error {err.max():.3e}"


def test_moe_gather_unaligned_and_out_of_range_ids(lib, h):
    """The byte path (a leading dimension that breaks 16-byte alignment) and ids outside the source: zero
    columns, nothing read outside X."""
    import torch
    rng = np.random.default_rng(401)
    k, ldx, n_src = 37, 41, 50
    X = rng.integers(-30000, 30000, ldx * n_src, dtype=np.int16)
    ids = np.array([3, 49, -1, 50, 0, 7, 1000, 49], dtype=np.int32)
    dX = torch.from_numpy(X).cuda()
    d_ids = torch.from_numpy(ids).cuda()
    Xp = torch.full((k * ids.size,), 12345, dtype=torch.int16, device="cuda")
    assert lib.lib.tb200_moe_gather(h.h, dX.data_ptr(), cb.CUDA_R_16F, k, ldx, n_src, d_ids.data_ptr(), ids.size,
                                    Xp.data_ptr(), k) == 0
    got = Xp.cpu().numpy().reshape(ids.size, k)
    for p, t in enumerate(ids):
        want = X[t * ldx:t * ldx + k] if 0 <= t < n_src else np.zeros(k, np.int16)
        assert np.array_equal(got[p], want), p
