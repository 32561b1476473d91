"""Generates the golden vectors under tests/golden/ from the reference itself.

Runs the reference's own CPU reference routines (cpuRef, int4RefRows,
vqRefRows, and the fp64 MoE block of moe-fused/src/main.mm:303-333), compiled
from the reference sources by oracle/ref_build.sh, on small seeded inputs, and
stores inputs and outputs as .npz files.  The tests check both the oracle
restatement (CPU) and the CUDA kernels (GPU) against these files; neither needs
the reference checkout at run time.

    python tests/golden/make_golden.py      # needs the reference checkout

The input distributions follow the reference harnesses: W uniform uint32
(codes U{0..15}), scale U(-1,1)*0.02, bias U(-1,1)*0.15, x U(-1,1)
(int4-gemv/src/main.mm:187-207); VQ indices U{0..255}, codebook U(-1,1), scale
U(-1,1)*0.05 (vq-gemv/src/main.mm:155-172).  Values are drawn with numpy's
PCG64 generator, not the reference's mt19937, and rounded to fp16 with numpy.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402


def f16(a) -> np.ndarray:
    return np.asarray(a, np.float32).astype(np.float16)


def bf16(a) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (uint16)."""
    u = np.asarray(a, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def int4_case(rng, M, K, G):
    W = rng.integers(0, 2**32, size=(M, K // 8), dtype=np.uint64).astype(np.uint32)
    S = f16(rng.uniform(-1, 1, (M, K // G)) * 0.02)
    B = f16(rng.uniform(-1, 1, (M, K // G)) * 0.15)
    x = f16(rng.uniform(-1, 1, K))
    return W, S, B, x


def moe_small(rng, P):
    """A small pool in the reference's blob layout: bf16 S/B/BI, fp32 R and x."""
    pool = np.zeros(P.n_experts * P.blob, np.uint8)
    H, I = P.hidden, P.inter
    for e in range(P.n_experts):
        base = e * P.blob
        for off, rows, K in ((P.off_gate, I, H), (P.off_up, I, H), (P.off_down, H, I)):
            p = base + off
            W = rng.integers(0, 2**32, size=(rows, K // 8), dtype=np.uint64).astype(np.uint32)
            pool[p + P.sub_w: p + P.sub_w + W.nbytes] = W.view(np.uint8).reshape(-1)
            S = bf16(np.abs(rng.normal(0, 0.02, (rows, K // 64))))
            Bv = bf16(rng.normal(0, 0.15, (rows, K // 64)) * 0.1)
            BI = bf16(rng.normal(0, 0.1, rows))
            for sub, arr in ((P.sub_s, S), (P.sub_b, Bv), (P.sub_bi, BI)):
                pool[p + sub: p + sub + arr.nbytes] = arr.view(np.uint8).reshape(-1)
    R = (rng.normal(0, 0.3, (P.n_experts, H))).astype(np.float32)
    x = rng.normal(0, 1, H).astype(np.float32)
    return pool, R, x


def main() -> None:
    if oracle.ref_lib() is None:
        oracle.build(ref=True)
    if oracle.ref_lib() is None:
        raise SystemExit("reference routines not built (no reference checkout?)")
    rng = np.random.default_rng(20261201)
    out = {}

    for name, (M, K, G) in {"int4_sep_g64": (96, 1024, 64), "int4_sep_g32": (77, 512, 32),
                            "int4_sep_g128": (77, 512, 128)}.items():
        W, S, B, x = int4_case(rng, M, K, G)
        y = oracle.ref_int4_cpuRef(W, S, B, x, G)
        out[name] = dict(W=W, S=S.view(np.uint16), B=B.view(np.uint16), x=x.view(np.uint16),
                         y=y, shape=np.array([M, K, G], np.uint32),
                         source=np.array("int4-gemv/src/main.mm:64-92 cpuRef"))

    M, K, G = 80, 2880, 64          # K = 2880: 90 chunks, not a multiple of 512
    W, S, B, x = int4_case(rng, M, K, G)
    SB = np.stack([S, B], axis=-1)
    y = oracle.ref_int4_sb(W, SB, x, G)
    out["int4_sb_k2880"] = dict(W=W, SB=SB.view(np.uint16), x=x.view(np.uint16), y=y,
                                shape=np.array([M, K, G], np.uint32),
                                source=np.array("vq-gemv/src/main.mm:66-90 int4RefRows"))

    M, K = 64, 1024
    IDX = rng.integers(0, 256, size=(M, K // 2), dtype=np.uint8)
    Cb = f16(rng.uniform(-1, 1, (256, 2)))
    S = f16(rng.uniform(-1, 1, (M, K // 32)) * 0.05)
    x = f16(rng.uniform(-1, 1, K))
    y = oracle.ref_vq(IDX, Cb, S, x)
    out["vq_s32"] = dict(IDX=IDX, C=Cb.view(np.uint16), S=S.view(np.uint16),
                         x=x.view(np.uint16), y=y, shape=np.array([M, K], np.uint32),
                         source=np.array("vq-gemv/src/main.mm:51-65 vqRefRows"))

    import kernels_b200 as kb
    P = kb.moe_params(128, 128, 8, 4)
    for attempt in range(100):
        pool, R, x = moe_small(rng, P)
        idx, wgt, logits, y = oracle.ref_moe_block(P, pool, R, x)
        srt = np.sort(logits)[::-1]
        gaps = -np.diff(srt[:P.top_k + 1])
        if gaps.min() > 1e-3 * max(1.0, abs(srt[0])):   # top-k resolvable in fp32
            break
    else:
        raise SystemExit("could not draw a router with separated logits")
    fields = {k: getattr(P, k) for k, _ in P._fields_}
    out["moe_small"] = dict(pool=pool, R=R, x=x, idx=idx, wgt=wgt, logits=logits, y=y,
                            params=np.array([fields[k] for k, _ in P._fields_], np.uint64),
                            source=np.array("moe-fused/src/main.mm:46-62, 303-333"))

    for name, d in out.items():
        np.savez_compressed(HERE / f"{name}.npz", **d)
        print(f"wrote {name}.npz ({(HERE / f'{name}.npz').stat().st_size} B)")


if __name__ == "__main__":
    main()
