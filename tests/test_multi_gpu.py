"""GPU, 2+ GPUs: graft_gemv_int4_sharded, graft_gemm_int4_sharded and graft_moe_block_ep through the C
ABI against the oracle, as torchrun ranks (tests/mp_worker.py).  Skipped on a
single-GPU box."""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu


def test_sharded_gemv_and_ep_moe_two_ranks(lib):
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1",
           "--master-port", "29531", str(root / "tests" / "mp_worker.py")]
    r = subprocess.run(cmd, cwd=root, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "fused forms on" in r.stdout or "fused forms off" in r.stdout
