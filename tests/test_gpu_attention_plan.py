"""The longest-first order of the sequences (pkv_paged_attention_plan_dev)
only changes which grid slot runs which sequence, so attention after a plan
must equal attention in batch order bit for bit: for bf16, f16 and fp8
pools, one and several query tokens, long contexts of several splits, empty
and out-of-range lengths, a plan made before the lengths changed, a plan
made for another call shape (which the call does not use), and a plan and
its attention calls replayed from a CUDA graph."""

import numpy as np
import pytest

from pagedkv.workloads import Stream
from tests.test_gpu_attention import setup as setup_pool
from tests.test_gpu_attention import tables_for
from tests.test_gpu_attention_fp8 import setup_fp8

pytestmark = pytest.mark.gpu


def attend(cuda, b, q, tab, ctx, max_ctx, layer, q_len=1, plan=False):
    import torch

    out = torch.full(q.shape, float("nan"), device=cuda, dtype=q.dtype)
    lse = torch.full(q.shape[:2], float("nan"), device=cuda, dtype=torch.float32)
    if plan:
        b.paged_attention_plan(ctx, max_ctx)
    b.paged_attention(q, tab, ctx, max_ctx, out, layer, lse=lse, q_len=q_len)
    torch.cuda.synchronize()
    return out, lse


def contexts(st, n, hi):
    return st.integers(n, 1, hi).astype(np.int64)


@pytest.mark.parametrize("pool,q_len,group", [("bf16", 1, 7), ("f16", 1, 4), ("bf16", 2, 7),
                                              ("fp8", 1, 7), ("fp8", 2, 4)])
def test_planned_attention_equals_batch_order(cuda, pool, q_len, group):
    import torch

    if pool == "fp8":
        cfg, b, _, _ = setup_fp8(cuda, kv_heads=2, num_blocks=16000, seed=7)
        tdt = torch.bfloat16
    else:
        cfg, b, tdt = setup_pool(cuda, dtype=pool, kv_heads=2, num_blocks=16000, seed=7)
    st = Stream(300 + q_len * 10 + group)
    ctx = np.maximum(contexts(st, 48, 5000), q_len)  # up to 3 splits of 128 blocks
    ctx[:3] = [q_len, 2048, 2049]  # split boundaries
    tables = tables_for(st, cfg, ctx)
    hq = cfg.num_kv_heads * group
    q = torch.from_numpy(st.normal(len(ctx) * q_len * hq * 128).reshape(len(ctx) * q_len, hq, 128)
                         .astype(np.float32)).to(cuda).to(tdt)
    tab = torch.from_numpy(tables).to(cuda)
    d_ctx = torch.from_numpy(ctx.astype(np.int32)).to(cuda)
    mx = int(ctx.max())
    ref = attend(cuda, b, q, tab, d_ctx, mx, 1, q_len)
    got = attend(cuda, b, q, tab, d_ctx, mx, 1, q_len, plan=True)
    assert b.device_error() is None
    assert torch.equal(ref[0], got[0]) and torch.equal(ref[1], got[1])
    # Another layer on the same plan.
    ref0 = attend(cuda, b, q, tab, d_ctx.clone(), mx, 0, q_len)  # another buffer: no plan applies
    got0 = attend(cuda, b, q, tab, d_ctx, mx, 0, q_len)
    assert torch.equal(ref0[0], got0[0]) and torch.equal(ref0[1], got0[1])


def test_stale_and_mismatched_plans_keep_results(cuda):
    import torch

    cfg, b, tdt = setup_pool(cuda, kv_heads=2, num_blocks=10500)
    st = Stream(11)
    ctx = contexts(st, 40, 4000)
    ctx[5] = 0       # empty
    ctx[6] = 99999   # past max_context_len: recorded, zeros
    tables = tables_for(st, cfg, np.minimum(ctx, 4000), stride=250)
    q = torch.from_numpy(st.normal(40 * 8 * 128).reshape(40, 8, 128).astype(np.float32)).to(cuda).to(tdt)
    tab = torch.from_numpy(tables).to(cuda)
    d_ctx = torch.from_numpy(ctx.astype(np.int32)).to(cuda)
    ref = attend(cuda, b, q, tab, d_ctx, 4000, 0)
    err = b.device_error()
    assert err is not None and err[1] == 6
    got = attend(cuda, b, q, tab, d_ctx, 4000, 0, plan=True)
    assert b.device_error() is not None
    assert torch.equal(ref[0], got[0]) and torch.equal(ref[1], got[1])
    # The lengths change after the plan (same buffer): the stale order is
    # still a permutation of the sequences, so the results are those of the
    # new lengths.
    ctx2 = contexts(st, 40, 4000)
    b.paged_attention_plan(d_ctx, 4000)
    d_ctx.copy_(torch.from_numpy(ctx2.astype(np.int32)).to(cuda))
    tab = torch.from_numpy(tables_for(st, cfg, ctx2, stride=250)).to(cuda)
    got2 = attend(cuda, b, q, tab, d_ctx, 4000, 0)
    ref2 = attend(cuda, b, q, tab, d_ctx.clone(), 4000, 0)
    assert b.device_error() is None
    assert torch.equal(ref2[0], got2[0]) and torch.equal(ref2[1], got2[1])
    # A plan for another shape (fewer sequences, another max length) is not used.
    b.paged_attention_plan(d_ctx[:10], 4000)
    got3 = attend(cuda, b, q, tab, d_ctx, 4000, 0)
    b.paged_attention_plan(d_ctx, 300)
    got4 = attend(cuda, b, q, tab, d_ctx, 4000, 0)
    assert torch.equal(ref2[0], got3[0]) and torch.equal(ref2[0], got4[0])


def test_plan_and_attention_in_a_cuda_graph(cuda):
    import torch

    cfg, b, tdt = setup_pool(cuda, kv_heads=2, num_blocks=12100)
    st = Stream(12)
    ctx = contexts(st, 64, 3000)
    tables = tables_for(st, cfg, ctx, stride=188)  # max_context_len 3000 fits 188 blocks
    q = torch.from_numpy(st.normal(64 * 14 * 128).reshape(64, 14, 128).astype(np.float32)).to(cuda).to(tdt)
    tab = torch.from_numpy(tables).to(cuda)
    d_ctx = torch.from_numpy(ctx.astype(np.int32)).to(cuda)
    ref = [attend(cuda, b, q, tab, d_ctx, 3000, layer) for layer in (0, 1)]
    outs = [torch.empty_like(q) for _ in range(2)]
    lses = [torch.empty(q.shape[:2], device=cuda, dtype=torch.float32) for _ in range(2)]
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):  # allocations happen before the capture
        b.paged_attention_plan(d_ctx, 3000, stream=stream)
        for layer in (0, 1):
            b.paged_attention(q, tab, d_ctx, 3000, outs[layer], layer, lse=lses[layer], stream=stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        b.paged_attention_plan(d_ctx, 3000, stream=stream)
        for layer in (0, 1):
            b.paged_attention(q, tab, d_ctx, 3000, outs[layer], layer, lse=lses[layer], stream=stream)
    for o in outs:
        o.fill_(float("nan"))
    graph.replay()
    torch.cuda.synchronize()
    assert b.device_error() is None
    for layer in (0, 1):
        assert torch.equal(outs[layer], ref[layer][0]) and torch.equal(lses[layer], ref[layer][1])
    del graph
