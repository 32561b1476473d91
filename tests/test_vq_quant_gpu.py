"""GPU parity of the VQ quantiser (graft_vq_quantize) against its CPU checker
(oracle/vq_quant.py) and against the reference's own quantiser's golden
vectors (tests/golden/vq_quant_ref_*.npz): bit-exact codes, codebook and
scales; then the quantised matrix through the VQ GEMV."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from oracle import vq_quant as vq
from conftest import GOLDEN, TOL, norm_rel

pytestmark = pytest.mark.gpu


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("M,K,sub,iters,seed", [
    (64, 512, 4096, 25, 0),        # sampled
    (32, 256, 1 << 20, 25, 3),     # every pair in the sample
    (7, 96, 100, 5, 11),           # ragged rows, tiny sample
    (256, 4096, 200_000, 25, 0),   # the reference's sample size
])
def test_quantize_bit_exact(lib, M, K, sub, iters, seed):
    import torch
    import kernels_b200 as kb
    rng = np.random.default_rng(M + K)
    W = rng.normal(0, 0.02, (M, K)).astype(np.float32)
    W[0, :32] = 0.0                                      # an all-zero group
    IDX, Cb, S = kb.vq_quantize(torch.from_numpy(W).cuda(), iters=iters, sub=sub, seed=seed)
    ridx, rC16, rS16, _ = vq.quantize(W, iters=iters, sub=sub, seed=seed)
    assert np.array_equal(host(S).view(np.uint16), rS16)
    assert np.array_equal(host(Cb).view(np.uint16), rC16)
    assert np.array_equal(host(IDX), ridx)


@pytest.mark.parametrize("name,M,K,sub", [("s4096", 64, 512, 4096), ("s8192", 96, 1024, 8192)])
def test_quantize_matches_reference_golden(lib, name, M, K, sub):
    """The reference's pq_quantize.quantize_matrix (run under tests/golden/mlx_np.py
    with the same draws) produced these; the CUDA quantiser must give the same."""
    import torch
    import kernels_b200 as kb
    g = np.load(GOLDEN / f"vq_quant_ref_{name}.npz")
    rng = np.random.default_rng(M + K)
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    W[1, 32:64] = 0.0
    W[M - 1, :32] = 0.0
    IDX, Cb, S = kb.vq_quantize(torch.from_numpy(W).cuda(), iters=25, sub=sub, seed=0)
    assert np.array_equal(host(S).view(np.uint16), g["S"])
    assert np.array_equal(host(Cb).view(np.uint16), g["C"])
    assert np.array_equal(host(IDX), g["idx"])


def test_quantised_matrix_through_the_vq_gemv(lib):
    import torch
    import kernels_b200 as kb
    M, K = 1024, 2048
    rng = np.random.default_rng(9)
    W = torch.from_numpy(rng.normal(0, 0.02, (M, K)).astype(np.float32)).cuda()
    IDX, Cb, S = kb.vq_quantize(W)
    x = torch.from_numpy(rng.normal(0, 1, K).astype(np.float16)).cuda()
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    kb.gemv_vq_ex(IDX, Cb, S, 32, x, y, kb.vq_params(M, K))
    ref = oracle.gemv_vq(host(IDX), host(Cb).view(np.uint16), host(S).view(np.uint16), 32,
                         host(x).view(np.uint16))
    assert norm_rel(host(y), ref) <= TOL
    # and the quantised product is close to the unquantised one
    exact = host(W).astype(np.float64) @ host(x).astype(np.float64)
    assert norm_rel(host(y), exact) < 0.15


def test_quantize_rejects_bad_params(lib):
    import torch
    import kernels_b200 as kb
    W = torch.zeros((4, 48), dtype=torch.float32, device="cuda")
    with pytest.raises(kb.GraftError):
        kb.vq_quantize(W)                                  # K % 32 != 0
    with pytest.raises(kb.GraftError):
        kb.vq_quantize(torch.zeros((4, 64), dtype=torch.float32, device="cuda"), sub=0)
