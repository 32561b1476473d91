"""Runs the reference's own VQ quantiser (vq-gemv/quant/pq_quantize.py,
unmodified) under the numpy stand-in for mlx.core (tests/golden/mlx_np.py) on
seeded matrices, and saves what it returns as golden vectors:

    python tests/golden/make_vq_quant_golden.py <reference checkout>

The sample size of its k-means is passed through _kmeans's own `sub`
parameter so that the fixtures stay small; everything else is its default
(256 codewords, 25 passes, seed 0).  Writes tests/golden/vq_quant_ref_*.npz.
"""
from __future__ import annotations

import functools
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))
sys.path.insert(0, str(HERE))

# (name, M, K, sub): the sample is drawn from more pairs than it holds
CASES = [("s4096", 64, 512, 4096), ("s8192", 96, 1024, 8192)]


def weights(M: int, K: int, seed: int) -> np.ndarray:
    """N(0, 0.02) fp32 weights with a few all-zero groups (the divide-by-1 rule)."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    W[1, 32:64] = 0.0
    W[M - 1, :32] = 0.0
    return W


def run_reference(ref_root: str, W: np.ndarray, sub: int):
    import mlx_np
    mx = mlx_np.install()
    spec = importlib.util.spec_from_file_location(
        "pq_quantize", Path(ref_root) / "vq-gemv" / "quant" / "pq_quantize.py")
    pq = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(pq)
    pq._kmeans = functools.partial(pq._kmeans, sub=sub)
    idx, C16, S16 = pq.quantize_matrix(mx.array(W))
    return np.asarray(idx, np.uint8), np.asarray(C16, np.float16), np.asarray(S16, np.float16)


def main() -> None:
    ref_root = sys.argv[1]
    for name, M, K, sub in CASES:
        W = weights(M, K, seed=M + K)
        idx, C16, S16 = run_reference(ref_root, W, sub)
        np.savez_compressed(HERE / f"vq_quant_ref_{name}.npz", shape=np.array([M, K, sub]),
                            idx=idx, C=C16.view(np.uint16), S=S16.view(np.uint16))
        print(name, idx.shape, C16.shape, S16.shape)


if __name__ == "__main__":
    main()
