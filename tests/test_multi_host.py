"""CPU, two gloo ranks: the decomposition the multi-GPU C-ABI calls rely on
(graft_gemv_int4_sharded, graft_moe_block_ep), checked with the oracle on the
host.  Each rank builds the same seeded full problem, keeps its share -- a row
block of the GEMV, an expert range of the MoE pool -- and the collectives the
library runs over NCCL (all-gather of the row slices, sum of the partial block
outputs) are run here over gloo; the result must equal the single-rank oracle."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from conftest import norm_rel


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import kernels_b200 as kb
        import oracle
        from kernels_b200 import synth

        # row-sharded int4 GEMV: every rank holds rows [lo, hi) of the same matrix
        M, K, G = 96 * world, 512, 64
        w = synth.int4_weights(M, K, G, seed=3, device="cpu")
        x = synth.activations(K, seed=4, device="cpu")
        lo, hi = kb.shard_rows(M, world, rank)
        W, SB = w["W"].numpy().view(np.uint32), w["SB"].numpy()
        xn = x.numpy()
        y_local = torch.from_numpy(oracle.gemv_int4_sb(W[lo:hi], SB[lo:hi], xn, G))
        parts = [torch.empty_like(y_local) for _ in range(world)]
        dist.all_gather(parts, y_local)
        y_full = torch.cat(parts).numpy()
        ref = oracle.gemv_int4_sb(W, SB, xn, G)
        gemv_err = float(np.max(np.abs(y_full - ref)))

        # expert-parallel MoE block: partial outputs of each rank's experts sum to the block
        P = kb.moe_params(256, 192, 8 * world, 4)
        pool, R = synth.moe_pool(P, scale_f16=True, has_bias_out=False, act_f16=True, seed=6,
                                 device="cpu")
        xm = synth.activations(256, seed=7, device="cpu").numpy()
        e_lo, e_hi = kb.expert_range(P.n_experts, world, rank)
        Rn = R.numpy().view(np.uint16)
        cfg = oracle.moe_cfg(P, scale_bf16=False, has_bias_out=False, router_f16=True,
                             expert_lo=e_lo, expert_hi=e_hi)
        idx, _, _, _, part = oracle.moe_block(cfg, pool.numpy(), Rn, xm)
        tot = torch.from_numpy(np.ascontiguousarray(part))
        dist.all_reduce(tot)
        full = oracle.moe_block(oracle.moe_cfg(P, scale_bf16=False, has_bias_out=False,
                                               router_f16=True), pool.numpy(), Rn, xm)
        out[rank] = (gemv_err, float(np.max(np.abs(ref))), norm_rel(tot.numpy(), full[4]),
                     list(map(int, idx)), list(map(int, full[0])))
    finally:
        dist.destroy_process_group()


def test_two_rank_decomposition_matches_single_rank_oracle(lib):
    import torch.multiprocessing as mp
    world = 2
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    for rank in range(world):
        gemv_err, scale, moe_rel, idx, idx_full = res[rank]
        assert gemv_err <= 1e-12 * max(scale, 1.0)       # concatenated slices == full rows
        assert moe_rel <= 1e-12                           # sum of partials == full block
        assert idx == idx_full                            # router replicated and identical


@pytest.mark.parametrize("M,world", [(201088, 2), (201088, 4), (201088, 8)])
def test_shard_and_expert_ranges(lib, M, world):
    import kernels_b200 as kb
    blocks = [kb.shard_rows(M, world, r) for r in range(world)]
    assert blocks[0][0] == 0 and blocks[-1][1] == M
    assert all(a[1] == b[0] for a, b in zip(blocks, blocks[1:]))
    ranges = [kb.expert_range(128, world, r) for r in range(world)]
    assert sum(hi - lo for lo, hi in ranges) == 128
    with pytest.raises(ValueError):
        kb.shard_rows(M + 1, world, 0)
