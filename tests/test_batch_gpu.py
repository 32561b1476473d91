"""GPU parity of the batched int4 GEMV (graft_gemm_int4_sb_f16, B = 1..16
tokens per call) against the fp64 oracle, token by token."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL, TOL_ELEM, elem_rel, norm_rel

pytestmark = pytest.mark.gpu


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("M,K,G", [(4096, 4096, 64), (14336, 4096, 64), (300, 2880, 32),
                                   (2000, 2880, 64), (77, 1024, 128), (1000, 14336, 64)])
@pytest.mark.parametrize("B", [1, 3, 8, 12, 16])
def test_batched_vs_oracle(lib, M, K, G, B):
    import torch
    import kernels_b200 as kb
    from kernels_b200 import synth
    w = synth.int4_weights(M, K, G, seed=M + B)
    X = torch.stack([synth.activations(K, seed=100 + b) for b in range(B)])
    Y = torch.full((B, M), float("nan"), dtype=torch.float16, device="cuda")
    P = kb.gemv_params(M, K, G)
    kb.gemm_int4_sb_f16(w["W"], w["SB"], X, Y, B, P)
    Wn, SBn = host(w["W"]).view(np.uint32), host(w["SB"]).view(np.uint16)
    got = host(Y).astype(np.float32)
    assert np.isfinite(got).all()
    for b in range(B):
        ref = oracle.gemv_int4_sb(Wn, SBn, host(X[b]).view(np.uint16), G)
        assert norm_rel(got[b], ref) <= TOL, b
        assert elem_rel(got[b], ref) <= TOL_ELEM, b


def test_batched_matches_the_gemv(lib):
    """B tokens in one call give what B batch-1 calls give (within fp32 rounding)."""
    import torch
    import kernels_b200 as kb
    from kernels_b200 import synth
    M, K, G, B = 6144, 4096, 64, 8
    w = synth.int4_weights(M, K, G, seed=1)
    X = torch.stack([synth.activations(K, seed=200 + b) for b in range(B)])
    P = kb.gemv_params(M, K, G)
    Y = torch.empty((B, M), dtype=torch.float16, device="cuda")
    kb.gemm_int4_sb_f16(w["W"], w["SB"], X, Y, B, P)
    for b in range(B):
        y1 = torch.empty(M, dtype=torch.float16, device="cuda")
        kb.gemv_int4_sb_f16out(w["W"], w["SB"], X[b], y1, P)
        d = (Y[b].float() - y1.float()).abs().max().item()
        assert d <= 2e-3 * y1.float().abs().max().item(), b


def test_batched_rejects_bad_batch(lib):
    import torch
    import kernels_b200 as kb
    P = kb.gemv_params(64, 256, 64)
    t = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    with pytest.raises(kb.GraftError):
        kb.gemm_int4_sb_f16(t, t, t, t, 17, P)
    with pytest.raises(kb.GraftError):
        kb.gemm_int4_sb_f16(t, t, t, t, 0, P)
