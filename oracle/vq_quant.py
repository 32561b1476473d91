"""TEST INFRASTRUCTURE ONLY -- numpy restatement of the VQ quantiser
(vq-gemv/quant/pq_quantize.py), the checker for graft_vq_quantize.

The reference's algorithm, step by step:
  * per-32 max-abs scales of W, and W normalised by them (zero groups
    divided by 1) -- quantize_matrix, pq_quantize.py:50-60;
  * the normalised weight pairs as 2-D points; Lloyd's k-means with 256
    centroids on a subsample of them: centroids start at sampled points,
    each pass assigns every point to argmax_c (p.c - |c|^2/2) and moves each
    centroid to its points' mean, a centroid with no points stays where it
    was; a fixed number of passes (25) -- _kmeans, :28-47;
  * every pair assigned to the final fp32 centroids (same argmax), codebook
    and scales rounded to fp16 -- :62-75; reconstruction
    w = scale * C[idx][t] -- dequantize, :78-83.

The reference draws its subsample and initial centroids with MLX's random
generator, which does not exist here, so this build defines its own draws
(splitmix64, below) and its own exact centroid arithmetic; the numbers
therefore match the CUDA quantiser bit for bit, not MLX's. Parity with the
reference itself is unpinned (MLX is absent); the algorithm is.

Arithmetic contract shared with kernels_b200/csrc/vq_quant.cu:
  * u = w / safe in fp32 (IEEE division);
  * h_c = 0.5 * (c0*c0 + c1*c1) and score = (p0*c0 + p1*c1) - h_c, every
    operation a separately rounded fp32 op; argmax takes the first maximum;
  * centroid sums in 2^-40 fixed point (int64, exact in any order):
    q = rint(u * 2^40); c = fp32((double(sum) * 2^-40) / double(count)).
"""
from __future__ import annotations

import numpy as np

GROUP = 32
N_CODES = 256
FIX = 40
_GOLDEN = np.uint64(0x9E3779B97F4A7C15)
_M1 = np.uint64(0xBF58476D1CE4E5B9)
_M2 = np.uint64(0x94D049BB133111EB)


def _mix(z: np.ndarray) -> np.ndarray:
    """splitmix64's finaliser on uint64 (wrapping arithmetic)."""
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * _M1
        z = (z ^ (z >> np.uint64(27))) * _M2
    return z ^ (z >> np.uint64(31))


def draws(seed: int, stream: int, n: int) -> np.ndarray:
    """The j-th draw (j < n) of a stream: mix(mix(seed + G*(stream+1)) + G*(j+1))."""
    with np.errstate(over="ignore"):
        base = _mix(np.array([seed], np.uint64) + _GOLDEN * np.uint64(stream + 1))[0]
        j = np.arange(1, n + 1, dtype=np.uint64)
        return _mix(base + _GOLDEN * j)


def scales(W: np.ndarray):
    """Per-32 max |w| (fp32, exact) and the divisor (1 where the group is all zero)."""
    M, K = W.shape
    s = np.abs(W.reshape(M, K // GROUP, GROUP)).max(axis=2).astype(np.float32)
    safe = np.where(s > 0, s, np.float32(1.0)).astype(np.float32)
    return s, safe


def pairs(W: np.ndarray, safe: np.ndarray, pts: np.ndarray) -> np.ndarray:
    """Normalised pairs [n, 2] fp32 of the flat pair indices pts."""
    K = W.shape[1]
    m, i = pts // (K // 2), pts % (K // 2)
    s = safe[m, i // (GROUP // 2)]
    return np.stack([W[m, 2 * i] / s, W[m, 2 * i + 1] / s], axis=-1).astype(np.float32)


def assign(P: np.ndarray, C: np.ndarray, block: int = 16384) -> np.ndarray:
    """argmax_c (p.c - |c|^2/2), first maximum, in the shared fp32 op order."""
    C = C.astype(np.float32)
    h = np.float32(0.5) * (C[:, 0] * C[:, 0] + C[:, 1] * C[:, 1])
    out = np.empty(P.shape[0], np.int64)
    for a in range(0, P.shape[0], block):
        p = P[a:a + block]
        score = (p[:, 0:1] * C[None, :, 0] + p[:, 1:2] * C[None, :, 1]) - h[None, :]
        out[a:a + block] = np.argmax(score, axis=1)
    return out


def lloyd_pass(S: np.ndarray, Q: np.ndarray, C: np.ndarray) -> np.ndarray:
    """One assignment + update pass; empty clusters keep their centroid."""
    a = assign(S, C)
    sums = np.zeros((N_CODES, 2), np.int64)
    np.add.at(sums, a, Q)
    cnt = np.bincount(a, minlength=N_CODES)
    new = C.copy()
    live = cnt > 0
    new[live] = ((sums[live].astype(np.float64) * 2.0 ** -FIX) /
                 cnt[live, None].astype(np.float64)).astype(np.float32)
    return new


def quantize(W: np.ndarray, iters: int = 25, sub: int = 200_000, seed: int = 0):
    """W fp32 [M, K] -> (IDX uint8 [M, K/2], C fp16 bits [256, 2] as uint16,
    S fp16 bits [M, K/32] as uint16, C fp32 [256, 2])."""
    W = np.ascontiguousarray(W, np.float32)
    M, K = W.shape
    assert K % GROUP == 0
    s, safe = scales(W)
    N = M * K // 2
    if N <= sub:
        pts = np.arange(N, dtype=np.int64)
    else:
        pts = (draws(seed, 0, sub) % np.uint64(N)).astype(np.int64)
    S = pairs(W, safe, pts)
    Q = np.rint(S.astype(np.float64) * 2.0 ** FIX).astype(np.int64)
    init = (draws(seed, 1, N_CODES) % np.uint64(S.shape[0])).astype(np.int64)
    C = S[init].copy()
    for _ in range(iters):
        C = lloyd_pass(S, Q, C)
    idx = assign(pairs(W, safe, np.arange(N, dtype=np.int64)), C).astype(np.uint8)
    return (idx.reshape(M, K // 2), C.astype(np.float16).view(np.uint16),
            s.astype(np.float16).view(np.uint16), C)


def dequantize(idx: np.ndarray, C16: np.ndarray, S16: np.ndarray) -> np.ndarray:
    """w[m, 2i+t] = S[m, 2i/32] * C[idx[m, i]][t] in fp32 (pq_quantize.py:78-83)."""
    M, half = idx.shape
    cw = C16.view(np.float16).astype(np.float32)[idx.astype(np.int64)]     # [M, K/2, 2]
    s = S16.view(np.float16).astype(np.float32)
    return (cw.reshape(M, 2 * half // GROUP, GROUP) * s[:, :, None]).reshape(M, 2 * half)
