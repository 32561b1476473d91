"""GPU parity of the int4 group-affine GEMV (C ABI) against the reference's
golden outputs and the fp64 oracle, including the BASELINE shapes at full size."""
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


def run_v6(kb, W, SB, x, P):
    import torch
    xs = torch.empty(P.K // 32, dtype=torch.float32, device="cuda")
    y = torch.full((P.M,), float("nan"), dtype=torch.float32, device="cuda")
    kb.xsum32(x, xs, P)
    kb.gemv_int4_wide_unroll(W, SB, None, x, y, xs, P)
    return host(y), host(xs)


@pytest.mark.parametrize("name", ["int4_sep_g64", "int4_sep_g32", "int4_sep_g128"])
def test_simd_separate_scales_vs_reference_golden(lib, name):
    import torch
    import kernels_b200 as kb
    g = golden(name)
    M, K, G = (int(v) for v in g["shape"])
    P = kb.gemv_params(M, K, G)
    x = dev(g["x"])
    xs = torch.empty(K // 32, dtype=torch.float32, device="cuda")
    y = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
    kb.xsum32(x, xs, P)
    assert np.array_equal(host(xs), oracle.xsum32(g["x"]))   # same fp32 order: bit-exact
    kb.gemv_int4_simd(dev(g["W"]), dev(g["S"]), dev(g["B"]), x, y, xs, P)
    got = host(y)
    assert np.isfinite(got).all()
    assert norm_rel(got, g["y"]) <= TOL


def test_wide_unroll_vs_reference_golden_k2880(lib):
    import kernels_b200 as kb
    g = golden("int4_sb_k2880")
    M, K, G = (int(v) for v in g["shape"])
    P = kb.gemv_params(M, K, G)
    got, _ = run_v6(kb, dev(g["W"]), dev(g["SB"]), dev(g["x"]), P)
    assert norm_rel(got, g["y"]) <= TOL


def baseline_case(kb, M, K, G=64, seed=0):
    from kernels_b200 import synth
    w = synth.int4_weights(M, K, G, seed=seed)
    x = synth.activations(K, seed=seed)
    return w, x


@pytest.mark.parametrize("M,K", [(4096, 4096),                  # config 0
                                 (14336, 4096), (4096, 14336),    # config 1
                                 (6144, 4096), (128256, 4096),
                                 (2880, 2880)])                    # MoE projection shape
def test_baseline_shapes_f16out_and_f32(lib, M, K):
    import torch
    import kernels_b200 as kb
    w, x = baseline_case(kb, M, K)
    P = kb.gemv_params(M, K, 64)
    y16 = torch.empty(M, dtype=torch.float16, device="cuda")
    kb.gemv_int4_sb_f16out(w["W"], w["SB"], x, y16, P)
    got32, _ = run_v6(kb, w["W"], w["SB"], x, P)
    ref = oracle.gemv_int4_sb(host(w["W"]).view(np.uint32), host(w["SB"]).view(np.uint16),
                              host(x).view(np.uint16), 64)
    assert norm_rel(host(y16).astype(np.float32), ref) <= TOL
    assert elem_rel(host(y16).astype(np.float32), ref) <= TOL_ELEM
    assert norm_rel(got32, ref) <= TOL
    # fp32 accumulation: the fp32 output is far inside the tolerance
    assert norm_rel(got32, ref) <= 5e-5
    assert elem_rel(got32, ref) <= TOL_ELEM


@pytest.mark.parametrize("B", [1, 8])
def test_config4_lmhead_full_shape(lib, B):
    """BASELINE config 4's lm_head, 201088 x 2880, at full size on one GPU: the
    batch-1 GEMV (scale rows of 180 B, not 16-byte strided, so it runs through
    the batched kernel's per-tile scale copies) and the batch-8 probe."""
    import torch
    import kernels_b200 as kb
    from kernels_b200 import synth
    M, K = 201088, 2880
    w, _ = baseline_case(kb, M, K, seed=4)
    P = kb.gemv_params(M, K, 64)
    X = torch.stack([synth.activations(K, seed=70 + b) for b in range(B)])
    Y = torch.full((B, M), float("nan"), dtype=torch.float16, device="cuda")
    if B == 1:
        kb.gemv_int4_sb_f16out(w["W"], w["SB"], X[0], Y[0], P)
    else:
        kb.gemm_int4_sb_f16(w["W"], w["SB"], X, Y, B, P)
    got = host(Y).astype(np.float32)
    Wn, SBn = host(w["W"]).view(np.uint32), host(w["SB"]).view(np.uint16)
    for b in range(B):
        ref = oracle.gemv_int4_sb(Wn, SBn, host(X[b]).view(np.uint16), 64)
        assert np.isfinite(got[b]).all(), b
        assert norm_rel(got[b], ref) <= TOL, b
        assert elem_rel(got[b], ref) <= TOL_ELEM, b


@pytest.mark.parametrize("M,K,G", [(20000, 4096, 32), (9000, 14336, 64), (60013, 4096, 128),
                                   (60001, 2048, 64)])
def test_tall_shapes_one_token_mode(lib, M, K, G):
    """Tall matrices whose scale rows are 16-byte strided and which give at
    least 6 units (16-row tile x K-part) per warp on 148 SMs run the batched
    kernel's one-token mode rather than the batch-1 tile GEMV: every group size
    it takes, long rows, and row counts that end in a partial 16-row tile."""
    import torch
    import kernels_b200 as kb
    w, x = baseline_case(kb, M, K, G=G, seed=M % 97)
    P = kb.gemv_params(M, K, G)
    y = torch.full((M,), float("nan"), dtype=torch.float16, device="cuda")
    kb.gemv_int4_sb_f16out(w["W"], w["SB"], x, y, P)
    got = host(y).astype(np.float32)
    ref = oracle.gemv_int4_sb(host(w["W"]).view(np.uint32), host(w["SB"]).view(np.uint16),
                              host(x).view(np.uint16), G)
    assert np.isfinite(got).all()
    assert norm_rel(got, ref) <= TOL
    assert elem_rel(got, ref) <= TOL_ELEM
    assert kb.device_errors(clear=True)["int4"] == 0


@pytest.mark.parametrize("M,K,G", [(1, 32, 32), (7, 64, 32), (33, 96, 96), (130, 2880, 64),
                                   (257, 512, 128), (61, 1024, 256), (9, 65536, 64),
                                   (5000, 160, 32)])
def test_edge_shapes(lib, M, K, G):
    """Tails in M, one-chunk rows, ragged chunk counts, non-power-of-two group
    (G = 96), very long rows."""
    import kernels_b200 as kb
    rng = np.random.default_rng(M * 7 + K)
    W = rng.integers(0, 2**32, size=(M, K // 8), dtype=np.uint64).astype(np.uint32)
    S = np.abs(rng.normal(0, 0.02, (M, K // G))).astype(np.float16)
    B = rng.normal(0, 0.1, (M, K // G)).astype(np.float16)
    x = rng.normal(0, 1, K).astype(np.float16)
    P = kb.gemv_params(M, K, G)
    SB = np.stack([S, B], -1)
    got, _ = run_v6(kb, dev(W), dev(SB.view(np.uint16)), dev(x.view(np.uint16)), P)
    ref = oracle.gemv_int4_sb(W, SB.view(np.uint16), x.view(np.uint16), G)
    assert norm_rel(got, ref) <= TOL
    assert elem_rel(got, ref) <= TOL_ELEM


def test_deterministic_and_stream_ordered(lib):
    import torch
    import kernels_b200 as kb
    w, x = baseline_case(kb, 6144, 4096, seed=3)
    P = kb.gemv_params(6144, 4096, 64)
    s = torch.cuda.Stream()
    outs = []
    with torch.cuda.stream(s):
        for _ in range(3):
            y = torch.empty(6144, dtype=torch.float16, device="cuda")
            kb.gemv_int4_sb_f16out(w["W"], w["SB"], x, y, P)
            outs.append(y)
    s.synchronize()
    assert all(torch.equal(outs[0], o) for o in outs[1:])


def test_misaligned_activation_rejected(lib):
    import torch
    import kernels_b200 as kb
    P = kb.gemv_params(64, 512, 64)
    buf = torch.zeros(2048, dtype=torch.uint8, device="cuda")
    y = torch.empty(64, dtype=torch.float16, device="cuda")
    with pytest.raises(kb.GraftError, match="16-byte aligned"):
        kb.gemv_int4_sb_f16out(buf, buf, buf.data_ptr() + 2, y, P)


def test_stream_read_reads_and_leaves_sink(lib):
    import torch
    import kernels_b200 as kb
    src = torch.zeros(1 << 20, dtype=torch.int32, device="cuda")
    sink = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    kb.stream_read(src, sink, src.numel() // 4)
    assert host(sink)[0] == 7
