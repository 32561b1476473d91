"""GPU: the batched int4 GEMV on the tcgen05 tensor cores (graft_gemm_set_tcgen05(1))
against the fp64 oracle, token by token: partial row tiles, 9..16 tokens, and
the config-1 lm_head shape (row-sampled); and that it agrees with the mma.sync
tile engine it stands in for."""
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


@pytest.fixture
def tc(lib):
    import kernels_b200 as kb
    was = kb.gemm_set_tcgen05(True)
    yield kb
    kb.gemm_set_tcgen05(was)


def run(kb, M, K, B, seed, rows=None):
    import torch
    from kernels_b200 import synth
    G = 64
    w = synth.int4_weights(M, K, G, seed=seed)
    X = torch.stack([synth.activations(K, seed=seed + 100 + b) for b in range(B)])
    Y = torch.full((B, M), float("nan"), dtype=torch.float16, device="cuda")
    P = kb.gemv_params(M, K, G)
    kb.gemm_int4_sb_f16(w["W"], w["SB"], X, Y, B, P)
    got = host(Y).astype(np.float32)
    assert np.isfinite(got).all()
    assert kb.device_errors(clear=True)["int4"] == 0
    sel = np.arange(M) if rows is None else rows
    Wn = host(w["W"]).view(np.uint32).reshape(M, -1)[sel]
    SBn = host(w["SB"]).view(np.uint16).reshape(M, -1)[sel]
    for b in range(B):
        ref = oracle.gemv_int4_sb(Wn, SBn, host(X[b]).view(np.uint16), G)
        assert norm_rel(got[b][sel], ref) <= TOL, b
        assert elem_rel(got[b][sel], ref) <= TOL_ELEM, b
    return w, X, got


@pytest.mark.parametrize("M,K,B", [(256, 512, 16), (300, 1024, 12), (4096, 4096, 16),
                                   (14336, 4096, 9), (1000, 2048, 13)])
def test_tcgen05_vs_oracle(tc, M, K, B):
    run(tc, M, K, B, seed=M + B)


def test_tcgen05_lmhead_row_sample(tc):
    """128256 x 4096 at 16 tokens (the config-1 lm_head), checked on 2048
    rows spread over every tile position."""
    M = 128256
    rows = np.unique(np.linspace(0, M - 1, 2048).astype(np.int64))
    run(tc, M, 4096, 16, seed=7, rows=rows)


def test_tcgen05_matches_tile_engine(tc):
    import torch
    kb = tc
    w, X, got = run(kb, 6144, 4096, 16, seed=3)
    kb.gemm_set_tcgen05(False)
    Y = torch.empty((16, 6144), dtype=torch.float16, device="cuda")
    P = kb.gemv_params(6144, 4096, 64)
    kb.gemm_int4_sb_f16(w["W"], w["SB"], X, Y, 16, P)
    ref = host(Y).astype(np.float32)
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max()
