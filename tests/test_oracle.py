"""CPU: the oracle restatement against the reference's own outputs (golden
vectors, and the reference routines themselves when they were built here),
plus known-answer cases."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import golden


def f16(a):
    return np.asarray(a, np.float32).astype(np.float16)


@pytest.mark.parametrize("name", ["int4_sep_g64", "int4_sep_g32", "int4_sep_g128"])
def test_int4_sep_matches_reference_golden(name):
    g = golden(name)
    M, K, G = (int(v) for v in g["shape"])
    y = oracle.gemv_int4_sep(g["W"], g["S"], g["B"], g["x"], G)
    # the reference rounds its fp64 sum to fp32 (int4-gemv/src/main.mm:77): bit-exact
    assert np.array_equal(y.astype(np.float32), g["y"])


def test_int4_sb_matches_reference_golden():
    g = golden("int4_sb_k2880")
    M, K, G = (int(v) for v in g["shape"])
    y = oracle.gemv_int4_sb(g["W"], g["SB"], g["x"], G)
    assert np.array_equal(y.astype(np.float32), g["y"])


def test_vq_matches_reference_golden():
    g = golden("vq_s32")
    y = oracle.gemv_vq(g["IDX"], g["C"], g["S"], 32, g["x"])
    assert np.array_equal(y.astype(np.float32), g["y"])


def test_moe_block_matches_reference_golden():
    import kernels_b200 as kb
    g = golden("moe_small")
    P = kb.MoEParams(*[int(v) for v in g["params"]])
    cfg = oracle.moe_cfg(P, scale_bf16=True, has_bias_out=True, router_f16=False)
    idx, wgt, logits, h, y = oracle.moe_block(cfg, g["pool"], g["R"], g["x"])
    assert np.array_equal(idx, g["idx"])          # top-k: exact
    assert np.array_equal(logits, g["logits"])
    assert np.array_equal(wgt, g["wgt"])
    assert np.array_equal(y, g["y"])


def test_oracle_equals_reference_on_fresh_inputs():
    """Beyond the committed goldens: when the reference routines are built here,
    oracle and reference agree bit for bit on new random shapes."""
    if oracle.ref_lib() is None:
        pytest.skip("reference routines not built on this machine")
    rng = np.random.default_rng(7)
    for M, K, G in [(33, 256, 32), (65, 768, 64), (19, 1024, 256), (40, 2880, 64)]:
        W = rng.integers(0, 2**32, size=(M, K // 8), dtype=np.uint64).astype(np.uint32)
        S = f16(rng.uniform(-1, 1, (M, K // G)) * 0.02)
        B = f16(rng.uniform(-1, 1, (M, K // G)) * 0.15)
        x = f16(rng.normal(0, 1, K))
        assert np.array_equal(oracle.gemv_int4_sep(W, S, B, x, G).astype(np.float32),
                              oracle.ref_int4_cpuRef(W, S, B, x, G))
        SB = np.stack([S, B], -1)
        assert np.array_equal(oracle.gemv_int4_sb(W, SB, x, G).astype(np.float32),
                              oracle.ref_int4_sb(W, SB, x, G))
        IDX = rng.integers(0, 256, size=(M, K // 2), dtype=np.uint8)
        Cb = f16(rng.normal(0, 0.5, (256, 2)))
        Sv = f16(rng.uniform(0.5, 1.5, (M, K // 32)))
        assert np.array_equal(oracle.gemv_vq(IDX, Cb, Sv, 32, x).astype(np.float32),
                              oracle.ref_vq(IDX, Cb, Sv, x))


# ------------------------------------------------------- known answers --
def test_int4_zero_codes_unit_bias_gives_sum_x():
    K, G = 512, 64
    W = np.zeros((3, K // 8), np.uint32)
    S = f16(np.full((3, K // G), 0.5))
    B = f16(np.ones((3, K // G)))
    x = f16(np.linspace(-2, 2, K))
    y = oracle.gemv_int4_sep(W, S, B, x, G)
    assert np.allclose(y, x.astype(np.float64).sum(), rtol=0, atol=1e-12)


def test_int4_one_hot_code_gives_scaled_x():
    K, G = 256, 32
    for k in (0, 1, 7, 8, 100, 255):
        W = np.zeros((1, K // 8), np.uint32)
        W[0, k // 8] = np.uint32(1) << np.uint32(4 * (k % 8))
        S = f16(np.full((1, K // G), 0.25))
        B = f16(np.zeros((1, K // G)))
        x = f16(np.arange(K) / 64.0)
        y = oracle.gemv_int4_sep(W, S, B, x, G)
        assert y[0] == 0.25 * float(x[k])


def test_vq_identity_codebook():
    K = 64
    Cb = f16(np.stack([np.arange(256) / 256.0, -np.arange(256) / 512.0], -1))
    IDX = np.arange(K // 2, dtype=np.uint8).reshape(1, -1)
    S = f16(np.ones((1, 1)))
    x = f16(np.ones(K))
    y = oracle.gemv_vq(IDX, Cb, S, K, x)
    assert y[0] == sum(i / 256.0 - i / 512.0 for i in range(K // 2))
    dec = oracle.vq_decode(IDX, Cb)
    assert np.array_equal(dec, Cb.view(np.uint16)[IDX.reshape(-1)].reshape(-1))


def test_xsum32_order():
    x = f16(np.random.default_rng(3).normal(0, 1, 1024))
    xs = oracle.xsum32(x)
    xf = x.astype(np.float32).reshape(-1, 8, 4)
    want = np.zeros(32, np.float32)
    for i in range(8):
        t = (xf[:, i, 0] + xf[:, i, 1]) + xf[:, i, 2]
        want = want + (t + xf[:, i, 3])
    assert np.array_equal(xs, want)


def test_moe_router_tie_lowest_index_wins():
    import kernels_b200 as kb
    P = kb.moe_params(64, 64, 8, 2)
    pool = np.zeros(P.n_experts * P.blob, np.uint8)
    R = np.zeros((8, 64), np.float32)
    R[5] = R[2] = 1.0      # tie for the top logit
    R[6] = 0.5
    x = np.ones(64, np.float32)
    cfg = oracle.moe_cfg(P, scale_bf16=True, has_bias_out=True)
    idx, wgt, logits, h, y = oracle.moe_block(cfg, pool, R, x)
    assert list(idx) == [2, 5]
    assert np.allclose(wgt, [0.5, 0.5])


def test_cpu_fast_baseline_agrees_with_oracle():
    rng = np.random.default_rng(11)
    M, K, G = 256, 2048, 64
    W = rng.integers(0, 2**32, size=(M, K // 8), dtype=np.uint64).astype(np.uint32)
    S = f16(np.abs(rng.normal(0, 0.02, (M, K // G))))
    SB = np.stack([S, f16(-8 * S.astype(np.float32))], -1)
    x = f16(rng.normal(0, 1, K))
    y, n = oracle.cpu_fast_gemv_int4_sb(W, SB, x, G, nthreads=4)
    ref = oracle.gemv_int4_sb(W, SB, x, G)
    assert n >= 1
    assert np.max(np.abs(y - ref)) / np.max(np.abs(ref)) < 1e-5
