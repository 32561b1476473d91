"""GPU parity of the CUDA-core GEMV engine (register-direct fp32 FMAs, no
tensor cores) against the fp64 oracle, for the int4 and VQ entry points; the
tensor engine is covered by test_int4_gpu.py / test_vq_gpu.py."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL, norm_rel

pytestmark = pytest.mark.gpu


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.fixture
def cuda_core(lib):
    import kernels_b200 as kb
    kb.set_gemv_engine("cuda-core")
    assert kb.get_gemv_engine() == "cuda-core"
    yield kb
    kb.set_gemv_engine("tensor")


@pytest.mark.parametrize("M,K,G", [(4096, 4096, 64), (14336, 4096, 64), (300, 2880, 32),
                                   (77, 4096, 128)])
def test_int4_cuda_core(cuda_core, M, K, G):
    import torch
    from kernels_b200 import synth
    kb = cuda_core
    w = synth.int4_weights(M, K, G, seed=3)
    x = synth.activations(K, seed=3)
    P = kb.gemv_params(M, K, G)
    y16 = torch.empty(M, dtype=torch.float16, device="cuda")
    kb.gemv_int4_sb_f16out(w["W"], w["SB"], x, y16, P)
    xs = torch.empty(K // 32, dtype=torch.float32, device="cuda")
    y32 = torch.empty(M, dtype=torch.float32, device="cuda")
    kb.xsum32(x, xs, P)
    kb.gemv_int4_wide_unroll(w["W"], w["SB"], None, x, y32, xs, P)
    ref = oracle.gemv_int4_sb(host(w["W"]).view(np.uint32), host(w["SB"]).view(np.uint16),
                              host(x).view(np.uint16), G)
    assert norm_rel(host(y32), ref) <= TOL
    assert norm_rel(host(y16).astype(np.float32), ref) <= TOL


@pytest.mark.parametrize("M,K,sg", [(4096, 4096, None), (14336, 4096, None), (300, 1024, 32),
                                    (77, 2880, 32)])
def test_vq_cuda_core(cuda_core, M, K, sg):
    import torch
    from kernels_b200 import synth
    kb = cuda_core
    sgv = K if sg is None else sg
    w = synth.vq_weights(M, K, seed=4, scale_group=sgv)
    x = synth.activations(K, seed=4)
    P = kb.vq_params(M, K)
    y = torch.empty(M, dtype=torch.float32, device="cuda")
    kb.gemv_vq_ex(w["IDX"], w["C"], w["S"], sgv, x, y, P)
    S = host(w["S"]).view(np.uint16).reshape(M, -1)
    ref = oracle.gemv_vq(host(w["IDX"]), host(w["C"]).view(np.uint16), S, sgv,
                         host(x).view(np.uint16))
    assert norm_rel(host(y), ref) <= TOL

