"""GPU parity of the expert path of moe-pipeline: gemv_int4_bf16 (bf16 scales,
per-row output bias, fp32 x), xsum32 over fp32 x, and experts streamed from
pinned host memory into device slots and computed there (graft_expert_*),
against the fp64 oracle."""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import TOL, norm_rel

pytestmark = pytest.mark.gpu


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("engine", ["tensor", "cuda-core"])
@pytest.mark.parametrize("M,K,G", [(2880, 2880, 64), (300, 1024, 32), (77, 2048, 128)])
def test_gemv_int4_bf16(lib, engine, M, K, G):
    import torch
    import kernels_b200 as kb
    rng = np.random.default_rng(M + K + G)
    W = rng.integers(0, 2**32, size=(M, K // 8), dtype=np.uint64).astype(np.uint32)
    S = np.abs(rng.normal(0, 0.02, (M, K // G))).astype(np.float32)
    B = (-8.0 * S).astype(np.float32)
    BI = rng.normal(0, 0.02, M).astype(np.float32)
    x = rng.normal(0, 1, K).astype(np.float32)
    Sb, Bb, BIb = bf16(S), bf16(B), bf16(BI)
    d = {k: v.cuda() for k, v in dict(W=torch.from_numpy(W.view(np.int32)), S=Sb, B=Bb,
                                       BI=BIb, x=torch.from_numpy(x)).items()}
    P = kb.expert_params(M, K, G)
    xs = torch.empty(K // 32, dtype=torch.float32, device="cuda")
    y = torch.full((M,), float("nan"), dtype=torch.float32, device="cuda")
    kb.set_gemv_engine(engine)
    try:
        kb.xsum32_f32(d["x"], xs, P)
        kb.gemv_int4_bf16(d["W"], d["S"], d["B"], d["BI"], d["x"], y, xs, P)
    finally:
        kb.set_gemv_engine("tensor")
    # xsum32 in the reference's order is bit-exact
    ref_xs = np.array([np.float32(0)] * (K // 32), np.float32)
    for j in range(K // 32):
        s = np.float32(0)
        for i in range(8):
            v = x[32 * j + 4 * i: 32 * j + 4 * i + 4]
            t = np.float32(v[0] + v[1])
            t = np.float32(t + v[2])
            t = np.float32(t + v[3])
            s = np.float32(s + t)
        ref_xs[j] = s
    assert np.array_equal(host(xs), ref_xs)
    ref = oracle.gemv_int4_bf16(W, Sb.view(torch.int16).numpy().view(np.uint16),
                                Bb.view(torch.int16).numpy().view(np.uint16),
                                BIb.view(torch.int16).numpy().view(np.uint16), x, G)
    assert norm_rel(host(y), ref) <= TOL


@pytest.mark.parametrize("depth,n_slots", [(1, 2), (2, 3)])
def test_expert_stream_pipeline(lib, depth, n_slots):
    """Experts copied from pinned host memory on the side stream, refilled before
    compute, each computed from its slot: every expert's y matches the oracle."""
    import torch
    import kernels_b200 as kb
    from kernels_b200 import synth
    E, H = 7, 512
    P = kb.moe_params(H, H, E, 2)
    pool, _ = synth.moe_pool(P, scale_f16=False, has_bias_out=True, act_f16=False, seed=9)
    host_pool = torch.empty(pool.numel(), dtype=torch.uint8, pin_memory=True)
    host_pool.copy_(pool)
    blob = P.blob
    slots = torch.empty(n_slots * blob, dtype=torch.uint8, device="cuda")
    es = kb.ExpertStream(slots, n_slots, blob)
    scratch = kb.ExpertScratchBuffers(P)
    rng = np.random.default_rng(3)
    xs = [torch.from_numpy(rng.normal(0, 1, H).astype(np.float32)).cuda() for _ in range(E)]
    ys = [torch.full((H,), float("nan"), dtype=torch.float32, device="cuda") for _ in range(E)]
    st = torch.cuda.current_stream()
    hp = host_pool.data_ptr()
    for i in range(min(depth, E)):
        es.fetch(i % n_slots, hp + i * blob)
    for i in range(E):
        s = i % n_slots
        es.acquire(s, st)
        if i + depth < E:   # refill before compute
            es.fetch((i + depth) % n_slots, hp + (i + depth) * blob)
        kb.expert_forward(es.slot(s), xs[i], ys[i], P, scratch, st)
        es.release(s, st)
    es.sync()
    torch.cuda.synchronize()
    cfg = oracle.moe_cfg(P, scale_bf16=True, has_bias_out=True)
    hp_np = host_pool.numpy()
    for i in range(E):
        ref = oracle.expert_forward(cfg, hp_np[i * blob:(i + 1) * blob], host(xs[i]))
        assert norm_rel(host(ys[i]), ref) <= TOL, i
    es.close()


def test_expert_stream_rejects_pageable(lib):
    import torch
    import kernels_b200 as kb
    slots = torch.empty(2 * 4096, dtype=torch.uint8, device="cuda")
    es = kb.ExpertStream(slots, 2, 4096)
    pageable = np.zeros(4096, np.uint8)
    with pytest.raises(kb.GraftError):
        es.fetch(0, pageable.ctypes.data)
    with pytest.raises(kb.GraftError):
        es.fetch(2, pageable.ctypes.data)   # slot out of range
    es.close()
