"""The VQ quantiser's CPU checker (oracle/vq_quant.py, a restatement of
vq-gemv/quant/pq_quantize.py): its steps against their definitions, and its
output format against the VQ GEMV oracle."""
from __future__ import annotations

import numpy as np

import oracle
from oracle import vq_quant as vq


def test_scales_are_group_max_abs_and_zero_groups_divide_by_one():
    rng = np.random.default_rng(1)
    W = rng.normal(0, 1, (3, 96)).astype(np.float32)
    W[1, 32:64] = 0.0
    s, safe = vq.scales(W)
    assert s.shape == (3, 3)
    for m in range(3):
        for j in range(3):
            assert s[m, j] == np.abs(W[m, 32 * j:32 * j + 32]).max()
    assert s[1, 1] == 0.0 and safe[1, 1] == 1.0
    # normalised pairs lie in [-1, 1], with a +-1 in every non-zero group
    P = vq.pairs(W, safe, np.arange(3 * 48))
    assert np.abs(P).max() <= 1.0
    assert np.all(P.reshape(3, 3, 32)[[0, 2]].__abs__().max(axis=2) == 1.0)


def test_draws_are_counter_based():
    a = vq.draws(7, 0, 100)
    b = vq.draws(7, 0, 200)
    assert np.array_equal(a, b[:100])            # draw j does not depend on n
    assert not np.array_equal(a, vq.draws(7, 1, 100))
    assert not np.array_equal(a, vq.draws(8, 0, 100))
    assert len(np.unique(a)) == 100


def test_lloyd_pass_moves_to_means_and_keeps_empty_centroids():
    rng = np.random.default_rng(2)
    centres = np.array([[0.5, 0.5], [-0.5, 0.5], [0.5, -0.5], [-0.5, -0.5]], np.float32)
    S = (centres[rng.integers(0, 4, 4000)] + rng.normal(0, 0.05, (4000, 2))).astype(np.float32)
    Q = np.rint(S.astype(np.float64) * 2.0 ** vq.FIX).astype(np.int64)
    C = np.full((vq.N_CODES, 2), 5.0, np.float32)      # far away: stays empty
    C[:4] = centres * 0.9
    for _ in range(3):
        C = vq.lloyd_pass(S, Q, C)
    a = vq.assign(S, C)
    for k in range(4):
        assert np.allclose(C[k], S[a == k].mean(axis=0), atol=1e-6)
        assert np.allclose(C[k], centres[k], atol=0.01)
    assert np.all(C[4:] == 5.0)


def test_assign_takes_the_first_maximum():
    C = np.zeros((vq.N_CODES, 2), np.float32)
    C[3] = C[9] = [0.25, 0.25]
    P = np.array([[1.0, 1.0]], np.float32)
    assert vq.assign(P, C)[0] == 3


def test_quantize_is_deterministic_and_accurate():
    rng = np.random.default_rng(3)
    W = rng.normal(0, 0.02, (64, 512)).astype(np.float32)
    a = vq.quantize(W, sub=4096, seed=5)
    b = vq.quantize(W, sub=4096, seed=5)
    for x, y in zip(a, b):
        assert np.array_equal(x, y)
    idx, C16, S16, _ = a
    assert idx.dtype == np.uint8 and idx.shape == (64, 256)
    assert C16.shape == (256, 2) and S16.shape == (64, 16)
    Wq = vq.dequantize(idx, C16, S16)
    nmse = ((Wq - W) ** 2).sum() / (W ** 2).sum()
    assert nmse < 0.012, nmse          # 4.5 bits/weight on Gaussian weights: ~0.007
    assert len(np.unique(idx)) > 200


def test_quantised_format_is_what_the_vq_gemv_reads():
    """dequantize(quantize(W)) . x equals the VQ GEMV oracle on the same
    IDX, C, S with scale group 32 (vq-gemv/src/main.mm:51-65)."""
    rng = np.random.default_rng(4)
    W = rng.normal(0, 0.02, (48, 256)).astype(np.float32)
    idx, C16, S16, _ = vq.quantize(W, sub=1 << 20, seed=0)     # all pairs sampled
    x = rng.normal(0, 1, 256).astype(np.float16)
    ref = vq.dequantize(idx, C16, S16).astype(np.float64) @ x.astype(np.float64)
    got = oracle.gemv_vq(idx, C16, S16, 32, x.view(np.uint16))
    assert np.allclose(got, ref, rtol=1e-5, atol=1e-6)
