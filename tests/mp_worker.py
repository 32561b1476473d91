"""Worker for tests/test_multi_gpu.py, run under torchrun (one rank per GPU):
the C-ABI multi-GPU calls against the oracle, at any world size.  Every
output is held to the 1e-3 tolerance of the single-GPU tests, both as
max|d|/max|ref| and per element.  Exits non-zero on a mismatch.  Not collected
by pytest (no test_ prefix)."""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np


TOL = 1e-3
TOL_ELEM = 2e-3   # per element: the reference's tolerance (tests/conftest.py explains)


def rels(got, ref):
    """max|d|/max|ref| and the largest per-element relative error over the
    outputs with |ref| >= 1e-2 max|ref| (tests/conftest.py's two metrics)."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    m = max(float(np.max(np.abs(ref))), 1e-30)
    d = np.abs(got - ref)
    keep = np.abs(ref) >= 1e-2 * m
    return float(np.max(d) / m), float(np.max(d[keep] / np.abs(ref[keep])))


def main() -> int:
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import kernels_b200 as kb
    import oracle
    from kernels_b200 import synth

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    # the id travels over gloo; the work runs on the library's own NCCL communicator
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    box = [kb.comm_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    comm = kb.Comm(box[0], world, rank)
    ok = True
    try:
        # row-sharded GEMV: rank r holds rows [r*M, (r+1)*M) of the full matrix
        Mt, K, G = 2048 * world, 2880, 64
        full = synth.int4_weights(Mt, K, G, seed=11, device="cpu")
        lo, hi = kb.shard_rows(Mt, world, rank)
        W = full["W"][lo:hi].cuda()
        SB = full["SB"][lo:hi].contiguous().cuda()
        x = synth.activations(K, seed=12, device="cpu").cuda()
        y = torch.full((Mt,), float("nan"), dtype=torch.float16, device="cuda")
        kb.gemv_int4_sharded(comm, W, SB, x, y, kb.gemv_params(hi - lo, K, G))
        torch.cuda.synchronize()
        ref = oracle.gemv_int4_sb(full["W"].numpy().view(np.uint32), full["SB"].numpy(),
                                  x.cpu().numpy(), G)
        got = y.cpu().numpy().astype(np.float64)
        rel, erel = rels(got, ref)
        print(f"rank {rank}: sharded gemv max|d|/max|ref| = {rel:.2e} elem {erel:.2e}", flush=True)
        ok &= bool(np.isfinite(got).all()) and rel <= TOL and erel <= TOL_ELEM

        # the same through a symmetric buffer: the gather runs inside the GEMV
        ys = comm.alloc((Mt,), torch.float16)
        print(f"rank {rank}: fused forms {'on' if comm.fused else 'off'}", flush=True)
        for it in range(4):        # back to back: epochs must advance in lockstep
            xi = synth.activations(K, seed=40 + it, device="cpu").cuda()
            kb.gemv_int4_sharded(comm, W, SB, xi, ys, kb.gemv_params(hi - lo, K, G))
        torch.cuda.synchronize()
        comm.status()
        ref3 = oracle.gemv_int4_sb(full["W"].numpy().view(np.uint32), full["SB"].numpy(),
                                   xi.cpu().numpy(), G)
        got3 = ys.cpu().numpy().astype(np.float64)
        rel3, erel3 = rels(got3, ref3)
        print(f"rank {rank}: fused sharded gemv (4th call) max|d|/max|ref| = {rel3:.2e} "
              f"elem {erel3:.2e}", flush=True)
        ok &= bool(np.isfinite(got3).all()) and rel3 <= TOL and erel3 <= TOL_ELEM

        # B tokens through the row shards (config 4's batch probe): NCCL, then fused
        for B, fused in ((8, False), (8, True), (12, True)):
            X = torch.stack([synth.activations(K, seed=60 + b, device="cpu") for b in range(B)]).cuda()
            if fused:
                Y = comm.alloc((B, Mt), torch.float16)
                Y.fill_(float("nan"))
                for _ in range(3):      # back to back: epochs advance in lockstep
                    kb.gemm_int4_sharded(comm, W, SB, X, Y, B, kb.gemv_params(hi - lo, K, G))
            else:
                Y = torch.full((B, Mt), float("nan"), dtype=torch.float16, device="cuda")
                kb.gemm_int4_sharded(comm, W, SB, X, Y, B, kb.gemv_params(hi - lo, K, G))
            torch.cuda.synchronize()
            comm.status()
            got = Y.cpu().numpy().astype(np.float64)
            worst, eworst = 0.0, 0.0
            for b in range(B):
                rb = oracle.gemv_int4_sb(full["W"].numpy().view(np.uint32), full["SB"].numpy(),
                                         X[b].cpu().numpy(), G)
                r1, r2 = rels(got[b], rb)
                worst, eworst = max(worst, r1), max(eworst, r2)
            print(f"rank {rank}: sharded gemm B={B} {'fused' if fused else 'nccl'} "
                  f"max|d|/max|ref| = {worst:.2e} elem {eworst:.2e}", flush=True)
            ok &= bool(np.isfinite(got).all()) and worst <= TOL and eworst <= TOL_ELEM

        # expert-parallel MoE: rank r's pool holds experts [r*E/n, (r+1)*E/n)
        P = kb.moe_params(2880, 2880, 16 * world, 4)
        e_lo, e_hi = kb.expert_range(P.n_experts, world, rank)
        pool, R = synth.moe_pool(P, scale_f16=True, has_bias_out=False, act_f16=True, seed=13,
                                 experts=range(e_lo, e_hi))
        shard = pool[e_lo * P.blob:e_hi * P.blob]
        # the oracle needs the whole pool: gather every rank's experts on the host
        mine = shard.cpu()
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        whole = torch.cat(parts).numpy()
        cfg = oracle.moe_cfg(P, scale_bf16=False, has_bias_out=False, router_f16=True)
        Rn = R.cpu().numpy().view(np.uint16)
        ws = kb.MoEWorkspace(P)
        # three tokens back to back (the reduce slots and counts are reused call after
        # call), fp32 y, then one with fp16 y (the epilogue's conversion branch); as
        # three launches, as one launch per rank (the one-launch block), and as three
        # launches with the cluster-free down pass (split tiles handed on, a rank
        # without a selected expert sending zero rows)
        for it, (y_f16, one, split) in enumerate([
                (False, 0, 0), (False, 0, 0), (False, 0, 0), (True, 0, 0),
                (False, 2, 0), (False, 2, 0), (True, 2, 0),
                (False, 0, 1), (False, 0, 1), (True, 0, 1)]):
            kb.moe_set_one_launch(one)
            kb.moe_set_down_pass(bool(split))
            xm = synth.activations(2880, seed=14 + it)
            fmt = kb.moe_format(scale_f16=True, has_bias_out=False, act_f16=True, y_f16=y_f16,
                                n_experts=P.n_experts)
            ym = torch.full((2880,), float("nan"), dtype=torch.float16 if y_f16 else torch.float32,
                            device="cuda")
            kb.moe_block_ep(comm, shard, R, xm, ym, P, fmt, ws)
            torch.cuda.synchronize()
            comm.status()
            idx, _, _, _, yref = oracle.moe_block(cfg, whole, Rn, xm.cpu().numpy().view(np.uint16))
            got_idx = ws.tensor("idx", torch.int32, P.top_k).cpu().numpy().view(np.uint32)
            gm = ym.float().cpu().numpy()
            r1, r2 = rels(gm, yref)
            print(f"rank {rank}: ep moe token {it} ({'f16' if y_f16 else 'f32'} y, "
                  f"{'one launch' if one else 'three launches'}"
                  f"{', cluster-free down' if split else ''}) "
                  f"max|d|/max|ref| = {r1:.2e} elem {r2:.2e} top-k {list(got_idx)}", flush=True)
            # max-norm for the block, as the reference checks it (moe-fused/src/main.mm:336-376):
            # h is fp16 in the kernels, as in the reference's, and fp64 in the oracle
            ok &= (bool(np.isfinite(gm).all()) and r1 <= TOL
                   and np.array_equal(np.sort(got_idx), np.sort(idx)))
        kb.moe_set_one_launch(0)
        kb.moe_set_down_pass(False)
    finally:
        torch.cuda.synchronize()
        comm.close()
        dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
