"""GPU: the MoE block as one launch (graft_moe_set_one_launch(1)) against the
fp64 oracle -- the BASELINE format and the reference format, consecutive calls
(the tagged words of one call must never be taken for the next call's), CUDA
graph replays (the epoch advances on the device, replay after replay), a
workspace first used inside a capture (the three-kernel block runs), and the
expert-range partials the multi-GPU path sums."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import TOL, norm_rel
from test_moe_gpu import assert_separated, baseline_block, host, oracle_block

pytestmark = pytest.mark.gpu


@pytest.fixture
def one_launch(lib):
    import kernels_b200 as kb
    was = kb.moe_set_one_launch(3)   # the whole block and expert ranges
    yield kb
    kb.moe_set_one_launch(was)


def fmt16(kb, P, **kw):
    return kb.moe_format(scale_f16=True, has_bias_out=False, act_f16=True, y_f16=True,
                         n_experts=P.n_experts, **kw)


def test_one_launch_config3_consecutive_calls(one_launch):
    import torch
    from kernels_b200 import synth
    kb = one_launch
    P, pool, R, x0 = baseline_block(kb, seed=0)
    ws = kb.MoEWorkspace(P)
    y = torch.empty(P.hidden, dtype=torch.float16, device="cuda")
    for s in range(3):
        x = x0 if s == 0 else synth.activations(P.hidden, seed=10 + s)
        y.fill_(float("nan"))
        kb.moe_block_ex(pool, R, x, y, P, fmt16(kb, P), ws)
        idx, wgt, logits, _, yref = oracle_block(P, pool, R, x)
        assert_separated(logits, P.top_k)
        assert np.array_equal(host(ws.tensor("idx", torch.int32, P.top_k)).view(np.uint32), idx)
        assert np.allclose(host(ws.tensor("wgt", torch.float32, P.top_k)), wgt, rtol=1e-5,
                           atol=1e-6)
        assert norm_rel(host(y).astype(np.float32), yref) <= TOL, s
    assert kb.device_errors(clear=True)["moe"] == 0


def test_one_launch_reference_format_with_bias(one_launch):
    """bf16 scales, fp32 router/x/y, output biases; 32 experts, top-4."""
    import torch
    from kernels_b200 import synth
    kb = one_launch
    P = kb.moe_params(2880, 2880, 32, 4)
    pool, R = synth.moe_pool(P, scale_f16=False, has_bias_out=True, act_f16=False, seed=5)
    x = torch.randn(P.hidden, generator=torch.Generator().manual_seed(5)).cuda()
    ws = kb.MoEWorkspace(P)
    y = torch.full((P.hidden,), float("nan"), dtype=torch.float32, device="cuda")
    kb.moe_block(pool, R, x, y, P, ws)
    idx, _, logits, _, yref = oracle_block(P, pool, R, x, f16=False, bias=True)
    assert_separated(logits, P.top_k)
    assert np.array_equal(host(ws.tensor("idx", torch.int32, P.top_k)).view(np.uint32), idx)
    assert norm_rel(host(y), yref) <= TOL


def test_one_launch_graph_replays(one_launch):
    """Two calls captured in a graph, replayed three times: every replay gives
    the eager outputs (the call number lives in the scratch, not in the graph)."""
    import torch
    from kernels_b200 import synth
    kb = one_launch
    P, pool, R, _ = baseline_block(kb, seed=3)
    xs = [synth.activations(P.hidden, seed=20 + i) for i in range(2)]
    ws = kb.MoEWorkspace(P)
    ys = [torch.empty(P.hidden, dtype=torch.float16, device="cuda") for _ in range(2)]
    want = []
    for x, y in zip(xs, ys):
        kb.moe_block_ex(pool, R, x, y, P, fmt16(kb, P), ws)
        want.append(host(y).copy())
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=st):
        for x, y in zip(xs, ys):
            kb.moe_block_ex(pool, R, x, y, P, fmt16(kb, P), ws, stream=st)
    for _ in range(3):
        for y in ys:
            y.fill_(float("nan"))
        g.replay()
        for y, w in zip(ys, want):
            assert np.array_equal(host(y).view(np.uint16), w.view(np.uint16))
    del g
    assert kb.device_errors(clear=True)["moe"] == 0


def test_first_use_inside_capture_takes_three_launches(one_launch):
    """A scratch the library has not zeroed yet, first used inside a capture:
    the block runs as three launches there (a zeroing node would reset the
    call number on every replay) and is still right."""
    import torch
    kb = one_launch
    P, pool, R, x = baseline_block(kb, seed=4)
    n = kb.load().graft_moe_scratch_bytes(__import__("ctypes").byref(P))
    buf = torch.empty(n + 256, dtype=torch.uint8, device="cuda")
    s = kb.MoEScratch()
    base = (buf.data_ptr() + 255) & ~255
    kb.call("graft_moe_scratch_carve", base, n, __import__("ctypes").byref(P),
            __import__("ctypes").byref(s))
    y = torch.empty(P.hidden, dtype=torch.float16, device="cuda")
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    ctypes = __import__("ctypes")
    fmt = fmt16(kb, P)
    with torch.cuda.graph(g, stream=st):
        kb.call("graft_moe_block_ex", pool.data_ptr(), R.data_ptr(), x.data_ptr(), y.data_ptr(),
                ctypes.byref(P), ctypes.byref(fmt), ctypes.byref(s), st.cuda_stream)
    y.fill_(float("nan"))
    g.replay()
    yref = oracle_block(P, pool, R, x)[4]
    assert norm_rel(host(y).astype(np.float32), yref) <= TOL
    del g


def test_one_launch_expert_ranges_sum_to_block(one_launch):
    """Expert-parallel partials on one GPU (4 ranges, some selecting none of the
    token's experts): each partial matches the oracle's, the sum the block."""
    import torch
    kb = one_launch
    P, pool, R, x = baseline_block(kb, seed=6)
    ws = kb.MoEWorkspace(P)
    per = P.n_experts // 4
    total = np.zeros(P.hidden, np.float64)
    for r in range(4):
        fmt = kb.moe_format(scale_f16=True, has_bias_out=False, act_f16=True, y_f16=False,
                            expert_lo=r * per, expert_hi=(r + 1) * per)
        y = torch.full((P.hidden,), float("nan"), dtype=torch.float32, device="cuda")
        kb.moe_block_ex(pool[r * per * P.blob:(r + 1) * per * P.blob], R, x, y, P, fmt, ws)
        part = oracle_block(P, pool, R, x, lo=r * per, hi=(r + 1) * per)[4]
        got = host(y)
        assert norm_rel(got, part) <= TOL if np.any(part) else not np.any(got)
        total += got
    assert norm_rel(total, oracle_block(P, pool, R, x)[4]) <= TOL


def test_cluster_free_down_pass_matches_clusters(lib):
    """graft_moe_set_down_pass(1): the down + combine pass without clusters gives
    the cluster pass's bits (same sums, same order) on config 3, call after call."""
    import torch
    import kernels_b200 as kb
    from kernels_b200 import synth
    P, pool, R, _ = baseline_block(kb, seed=8)
    ws = kb.MoEWorkspace(P)
    y = torch.empty(P.hidden, dtype=torch.float16, device="cuda")
    was = kb.moe_set_down_pass(False)
    try:
        for s in range(3):
            x = synth.activations(P.hidden, seed=30 + s)
            outs = []
            for split in (False, True):
                kb.moe_set_down_pass(split)
                y.fill_(float("nan"))
                kb.moe_block_ex(pool, R, x, y, P, fmt16(kb, P), ws)
                outs.append(host(y).copy())
            assert np.array_equal(outs[0].view(np.uint16), outs[1].view(np.uint16)), s
        assert kb.device_errors(clear=True)["moe"] == 0
    finally:
        kb.moe_set_down_pass(was)
