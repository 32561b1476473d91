"""GPU parity of the VQ codebook GEMV and codeword decode (C ABI)."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL, TOL_ELEM, elem_rel, golden, norm_rel

pytestmark = pytest.mark.gpu


def dev(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def test_vq_wide_vs_reference_golden(lib):
    import torch
    import kernels_b200 as kb
    g = golden("vq_s32")
    M, K = (int(v) for v in g["shape"])
    P = kb.vq_params(M, K)
    y = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
    kb.gemv_vq_wide(dev(g["IDX"]), dev(g["C"]), dev(g["S"]), dev(g["x"]), y, P)
    assert norm_rel(host(y), g["y"]) <= TOL


def test_codebook_decode_bit_exact(lib):
    import torch
    import kernels_b200 as kb
    rng = np.random.default_rng(5)
    IDX = rng.integers(0, 256, size=100003, dtype=np.uint8)
    Cb = rng.normal(0, 0.02, (256, 2)).astype(np.float16).view(np.uint16)
    out = torch.empty(2 * IDX.size, dtype=torch.int16, device="cuda")
    kb.vq_decode(dev(IDX), dev(Cb), out, IDX.size)
    assert np.array_equal(host(out).view(np.uint16), oracle.vq_decode(IDX, Cb))


@pytest.mark.parametrize("M,K", [(4096, 4096), (14336, 4096)])   # config 2
@pytest.mark.parametrize("y_f16", [True, False])
def test_baseline_rowscale(lib, M, K, y_f16):
    import torch
    import kernels_b200 as kb
    from kernels_b200 import synth
    w = synth.vq_weights(M, K, seed=1)
    x = synth.activations(K, seed=1)
    P = kb.vq_params(M, K)
    y = torch.empty(M, dtype=torch.float16 if y_f16 else torch.float32, device="cuda")
    kb.gemv_vq_ex(w["IDX"], w["C"], w["S"], K, x, y, P)
    ref = oracle.gemv_vq(host(w["IDX"]), host(w["C"]).view(np.uint16),
                         host(w["S"]).view(np.uint16).reshape(M, 1), K,
                         host(x).view(np.uint16))
    got = host(y).astype(np.float32)
    assert norm_rel(got, ref) <= TOL
    assert elem_rel(got, ref) <= TOL_ELEM
    if not y_f16:
        assert norm_rel(got, ref) <= 5e-5


@pytest.mark.parametrize("M,K", [(1, 32), (77, 2880), (300, 1024), (5, 16384)])
def test_edge_shapes_per32_scales(lib, M, K):
    import torch
    import kernels_b200 as kb
    rng = np.random.default_rng(M + K)
    IDX = rng.integers(0, 256, size=(M, K // 2), dtype=np.uint8)
    Cb = rng.normal(0, 0.5, (256, 2)).astype(np.float16).view(np.uint16)
    S = rng.uniform(0.5, 1.5, (M, K // 32)).astype(np.float16).view(np.uint16)
    x = rng.normal(0, 1, K).astype(np.float16).view(np.uint16)
    P = kb.vq_params(M, K)
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    kb.gemv_vq_wide(dev(IDX), dev(Cb), dev(S), dev(x), y, P)
    assert norm_rel(host(y), oracle.gemv_vq(IDX, Cb, S, 32, x)) <= TOL
