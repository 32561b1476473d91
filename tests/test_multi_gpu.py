"""GPU, 2, 4 and 8 GPUs: graft_gemv_int4_sharded, graft_gemm_int4_sharded and
graft_moe_block_ep through the C ABI against the oracle, as torchrun ranks
(tests/mp_worker.py).  Each world size is skipped on a box with fewer GPUs."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_gemv_and_ep_moe(lib, world):
    import torch
    n = torch.cuda.device_count()
    if n < world:
        pytest.skip(f"needs {world} GPUs")
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(29531 + world), str(root / "tests" / "mp_worker.py")]
    r = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "fused forms on" in r.stdout or "fused forms off" in r.stdout
