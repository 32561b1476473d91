"""Runs one hot-path kernel on seeded synthetic data and prints its timing --
the counterpart of the reference harness binaries' flags (int4gemv --M --K --G
--iters, vqgemv --M --K, moefused --experts), without the round-robin tables.

    python -m kernels_b200.run int4 --M 128256 --K 4096 [--G 64] [--iters 5] [--copies 2]
    python -m kernels_b200.run vq --M 14336 --K 4096 [--s32]
    python -m kernels_b200.run moe [--experts 128] [--top-k 4] [--one-launch 1]
    python -m kernels_b200.run stream --mbytes 1024
    python -m kernels_b200.run batch --M 128256 --K 4096 --B 8 [--tcgen05]
    python -m kernels_b200.run vqquant --M 4096 --K 4096
    python -m kernels_b200.run expert [--copies 4]     # one gpt-oss expert (bf16 format)

Each iteration is one launch on a rotating weight copy, timed with CUDA events;
use it for small profiler captures (a few launches, a few GB).  --graph N
instead times N launches (copies rotating) captured in one CUDA graph and
replayed back to back, as the bench times its steps, and reports the mean
time per launch (the launch overhead of a lone call excluded).
"""
from __future__ import annotations

import argparse
import json


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("kernel", choices=["int4", "vq", "moe", "stream", "batch", "vqquant",
                                       "expert"])
    ap.add_argument("--M", type=int, default=4096)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--G", type=int, default=64)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--copies", type=int, default=2)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--top-k", type=int, default=4)
    ap.add_argument("--mbytes", type=int, default=1024)
    ap.add_argument("--B", type=int, default=8, help="batch: tokens per call")
    ap.add_argument("--f32out", action="store_true")
    ap.add_argument("--s32", action="store_true", help="vq: per-32 scales (the reference's form)")
    ap.add_argument("--tcgen05", action="store_true",
                    help="batch: 9..16 tokens on the tcgen05 kernel (graft_gemm_set_tcgen05)")
    ap.add_argument("--one-launch", type=int, default=0,
                    help="moe: graft_moe_set_one_launch bits (1: the whole block in one launch)")
    ap.add_argument("--graph", type=int, default=0,
                    help="time N launches captured in one CUDA graph (mean per launch)")
    a = ap.parse_args()

    import torch
    import kernels_b200 as kb
    from kernels_b200 import synth

    torch.cuda.set_device(0)
    if a.kernel == "int4":
        ws = [synth.int4_weights(a.M, a.K, a.G, seed=c) for c in range(a.copies)]
        x = synth.activations(a.K)
        P = kb.gemv_params(a.M, a.K, a.G)
        nbytes = a.M * a.K // 2 + 4 * a.M * (a.K // a.G) + 2 * a.K + (4 if a.f32out else 2) * a.M
        if a.f32out:
            y = torch.empty(a.M, dtype=torch.float32, device="cuda")
            xs = torch.empty(a.K // 32, dtype=torch.float32, device="cuda")
            kb.xsum32(x, xs, P)
            f = lambda i: kb.gemv_int4_wide_unroll(ws[i % a.copies]["W"], ws[i % a.copies]["SB"],  # noqa
                                                   None, x, y, xs, P)
        else:
            y = torch.empty(a.M, dtype=torch.float16, device="cuda")
            f = lambda i: kb.gemv_int4_sb_f16out(ws[i % a.copies]["W"], ws[i % a.copies]["SB"],  # noqa
                                                 x, y, P)
    elif a.kernel == "vq":
        sg = 32 if a.s32 else a.K
        ws = [synth.vq_weights(a.M, a.K, seed=c, scale_group=sg) for c in range(a.copies)]
        x = synth.activations(a.K)
        y = torch.empty(a.M, dtype=torch.float16, device="cuda")
        P = kb.vq_params(a.M, a.K)
        nbytes = a.M * a.K // 2 + ws[0]["S"].numel() * 2 + 1024 + 2 * a.K + 2 * a.M
        f = lambda i: kb.gemv_vq_ex(ws[i % a.copies]["IDX"], ws[i % a.copies]["C"],  # noqa
                                    ws[i % a.copies]["S"], sg, x, y, P)
    elif a.kernel == "batch":
        kb.gemm_set_tcgen05(a.tcgen05)
        ws = [synth.int4_weights(a.M, a.K, a.G, seed=c) for c in range(a.copies)]
        X = torch.stack([synth.activations(a.K, seed=50 + b) for b in range(a.B)])
        Y = torch.empty((a.B, a.M), dtype=torch.float16, device="cuda")
        P = kb.gemv_params(a.M, a.K, a.G)
        nbytes = a.M * a.K // 2 + 4 * a.M * (a.K // a.G) + 2 * a.B * (a.K + a.M)
        f = lambda i: kb.gemm_int4_sb_f16(ws[i % a.copies]["W"], ws[i % a.copies]["SB"],  # noqa
                                          X, Y, a.B, P)
    elif a.kernel == "vqquant":
        g = torch.Generator(device="cuda").manual_seed(0)
        W = torch.randn((a.M, a.K), generator=g, device="cuda", dtype=torch.float32) * 0.02
        nbytes = a.M * a.K * 4
        f = lambda i: kb.vq_quantize(W)  # noqa
    elif a.kernel == "expert":
        # moe-pipeline's per-expert forward: xsum32 (fp32 x), gemv_int4_bf16 (gate, up),
        # SwiGLU, xsum32, gemv_int4_bf16 (down); rotating resident experts
        P = kb.moe_params(2880, 2880, a.copies, 4)
        pool, _ = synth.moe_pool(P, scale_f16=False, has_bias_out=True, act_f16=False, seed=11)
        scratch = kb.ExpertScratchBuffers(P)
        x = synth.activations(2880, seed=3).float()
        y = torch.empty(2880, dtype=torch.float32, device="cuda")
        nbytes = P.blob
        f = lambda i: kb.expert_forward(pool[(i % a.copies) * P.blob:], x, y, P, scratch)  # noqa
    elif a.kernel == "moe":
        kb.moe_set_one_launch(a.one_launch)
        P = kb.moe_params(2880, 2880, a.experts, a.top_k)
        pool, R = synth.moe_pool(P, scale_f16=True, has_bias_out=False, act_f16=True)
        xs_ = [synth.activations(2880, seed=s) for s in range(8)]
        y = torch.empty(2880, dtype=torch.float16, device="cuda")
        wsp = kb.MoEWorkspace(P)
        fmt = kb.moe_format(scale_f16=True, has_bias_out=False, act_f16=True, y_f16=True,
                            n_experts=a.experts)
        nbytes = a.top_k * 3 * (2880 * 1440 + 2 * 2 * 2880 * 45) + a.experts * 2880 * 2 + 6 * 2880 \
            + 4 * a.top_k * 2880
        f = lambda i: kb.moe_block_ex(pool, R, xs_[i % 8], y, P, fmt, wsp)  # noqa
    else:
        n = a.mbytes << 20
        bufs = [torch.empty(n, dtype=torch.uint8, device="cuda") for _ in range(a.copies)]
        sink = torch.zeros(1, dtype=torch.int32, device="cuda")
        nbytes = n
        f = lambda i: kb.stream_read(bufs[i % a.copies], sink, n // 16)  # noqa

    f(0)
    torch.cuda.synchronize()
    times = []
    for i in range(a.iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        f(i + 1)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e3)
    best = min(times)
    out = {"kernel": a.kernel, "M": a.M, "K": a.K, "best_us": round(best, 3),
           "gbs": round(nbytes / best / 1e3, 1), "bytes": nbytes,
           "times_us": [round(t, 2) for t in times]}
    if a.graph > 0:
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            for i in range(a.graph):
                f(i)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
        reps = []
        for _ in range(max(a.iters, 1)):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize()
            reps.append(e0.elapsed_time(e1) * 1e3 / a.graph)
        per = sorted(reps)[len(reps) // 2]
        out.update({"graph_launches": a.graph, "graph_us_per_launch": round(per, 3),
                    "graph_gbs": round(nbytes / per / 1e3, 1)})
        del g
    print(json.dumps(out))


if __name__ == "__main__":
    main()
