"""Seeded synthetic inputs with the shapes and value distributions of the
BASELINE configurations, generated directly in device memory.

The reference measures on no public dataset for this path; these generators
stand in for its weights and activations:
  int4 (config 0/1/4): codes U{0..15} packed 8 per uint32 along K, group 64,
      scale fp16(|N(0, 0.02)|), bias fp16(-8 * scale), x fp16(N(0, 1));
  VQ   (config 2): indices U{0..255}, codebook 256 x 2 fp16 N(0, 0.02),
      scale fp16 U(0.5, 1.5) per row (or per 32 weights), x fp16 N(0, 1);
  MoE  (config 3): router fp16 N(0, 0.02) [n_experts][hidden], experts with
      int4 group-64 gate/up/down and fp16 scale/bias as above, x fp16 N(0, 1).
"""
from __future__ import annotations

import torch


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def codes(shape, g, device) -> torch.Tensor:
    """Uniform 32-bit words: 8 codes U{0..15} each."""
    return torch.randint(-2**31, 2**31, shape, dtype=torch.int32, device=device, generator=g)


def int4_weights(M: int, K: int, G: int = 64, seed: int = 0, device="cuda", dtype=torch.float16):
    """W int32 [M, K/8], S and B [M, K/G] (B = -8 S), SB [M, K/G, 2] interleaved."""
    g = _gen(seed, device)
    W = codes((M, K // 8), g, device)
    S = torch.randn((M, K // G), generator=g, device=device).mul_(0.02).abs_().to(dtype)
    B = (S.float() * -8.0).to(dtype)
    SB = torch.stack([S, B], dim=-1).contiguous()
    return {"W": W, "S": S, "B": B, "SB": SB}


def activations(K: int, seed: int = 0, device="cuda", dtype=torch.float16) -> torch.Tensor:
    g = _gen(seed + 0x9E3779B9, device)
    return torch.randn(K, generator=g, device=device).to(dtype)


def vq_weights(M: int, K: int, seed: int = 0, device="cuda", scale_group: int | None = None):
    """IDX uint8 [M, K/2], C fp16 [256, 2], S fp16 [M] (scale_group None/K) or [M, K/32]."""
    g = _gen(seed, device)
    IDX = torch.randint(0, 256, (M, K // 2), dtype=torch.uint8, device=device, generator=g)
    C = torch.randn((256, 2), generator=g, device=device).mul_(0.02).half()
    if scale_group in (None, K):
        S = torch.rand(M, generator=g, device=device).add_(0.5).half()
    else:
        S = torch.rand((M, K // scale_group), generator=g, device=device).add_(0.5).half()
    return {"IDX": IDX, "C": C, "S": S}


def moe_pool(P, scale_f16: bool = True, has_bias_out: bool = False, act_f16: bool = True,
             seed: int = 0, device="cuda", experts=None):
    """Expert pool (uint8, n_experts * blob) in the MoEParams blob layout, plus the
    router R ([n_experts, hidden], fp16 or fp32).  `experts` limits which expert
    blobs are filled (the rest stay zero), for expert-parallel shards.  The router
    and every expert draw from their own seeded generator, so a shard's experts
    and the router are the same whichever experts are filled."""
    sdt = torch.float16 if scale_f16 else torch.bfloat16
    pool = torch.zeros(P.n_experts * P.blob, dtype=torch.uint8, device=device)
    H, I = P.hidden, P.inter
    for e in (range(P.n_experts) if experts is None else experts):
        g = _gen(seed * 1000003 + 1 + e, device)
        base = e * P.blob
        for off, rows, K in ((P.off_gate, I, H), (P.off_up, I, H), (P.off_down, H, I)):
            p = base + off
            w = pool[p + P.sub_w: p + P.sub_w + rows * K // 2].view(torch.int32)
            w.copy_(codes((rows * K // 8,), g, device))
            ng = rows * (K // 64)
            s = torch.randn(ng, generator=g, device=device).mul_(0.02).abs_().to(sdt)
            pool[p + P.sub_s: p + P.sub_s + 2 * ng].view(sdt).copy_(s)
            pool[p + P.sub_b: p + P.sub_b + 2 * ng].view(sdt).copy_((s.float() * -8.0).to(sdt))
            if has_bias_out:
                bi = torch.randn(rows, generator=g, device=device).mul_(0.02).to(sdt)
                pool[p + P.sub_bi: p + P.sub_bi + 2 * rows].view(sdt).copy_(bi)
    R = torch.randn((P.n_experts, H), generator=_gen(seed, device), device=device).mul_(0.02)
    R = R.half() if act_f16 else R.float()
    return pool, R
