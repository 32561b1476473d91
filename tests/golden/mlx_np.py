"""TEST INFRASTRUCTURE ONLY -- a numpy stand-in for the few `mlx.core` calls of
the reference's VQ quantiser (vq-gemv/quant/pq_quantize.py), so that its
unmodified code can run here (MLX itself needs Apple silicon).

Arrays are numpy arrays kept in float32 where MLX keeps float32.  The one
place MLX's behaviour cannot be reproduced is its random generator: here
`random.randint(lo, hi, shape, key=k)` returns the counter-based draws of
oracle/vq_quant.py, the n-th call on a key taking stream n -- the same sample
and initial centroids the repository's quantiser and its checker draw.  With
those fixed, what remains is the reference's own arithmetic: its matmul
scores, argmax, one-hot centroid sums and empty-cluster rule.
"""
from __future__ import annotations

import sys
import types

import numpy as np


class _Key:
    def __init__(self, seed: int):
        self.seed, self.calls = int(seed), 0


def _randint(lo, hi, shape, key):
    from oracle.vq_quant import draws
    n = int(np.prod(shape))
    d = draws(key.seed, key.calls, n)
    key.calls += 1
    return (int(lo) + (d % np.uint64(int(hi) - int(lo))).astype(np.int64)).reshape(shape)


def _sum(a, axis=None):
    return np.sum(a, axis=axis, dtype=a.dtype)


def install() -> types.ModuleType:
    """Registers `mlx` and `mlx.core` (this stand-in) in sys.modules."""
    core = types.ModuleType("mlx.core")
    core.float32, core.float16 = np.float32, np.float16
    core.uint8, core.uint32 = np.uint8, np.uint32
    core.array = lambda v, dtype=None: np.array(v, dtype=dtype)
    core.random = types.SimpleNamespace(key=_Key, randint=_randint)
    core.sum = _sum
    core.max = lambda a, axis=None: np.max(a, axis=axis)
    core.abs = np.abs
    core.where = np.where
    core.argmax = lambda a, axis=None: np.argmax(a, axis=axis)
    core.arange = np.arange
    core.maximum = np.maximum
    core.concatenate = np.concatenate
    core.eval = lambda *a: None
    pkg = types.ModuleType("mlx")
    pkg.core = core
    sys.modules["mlx"], sys.modules["mlx.core"] = pkg, core
    return core
