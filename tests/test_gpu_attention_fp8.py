"""Paged decode attention over an fp8 (E4M3) pool against the float64 oracle
(oracle/attention.py) on the dequantised cache.

The pool holds E4M3 codes with one K and one V scale per (layer, kv head);
the cache the attention reads is code * scale. The oracle takes those values
in float64; the kernel takes the codes as f16 (exact), the queries as f16
(bf16 queries scaled by a power of two into f16 range), accumulates in f32
and applies the scales to the scores and the output. Tolerance, as for the
bf16/f16 pools: every output element within 1e-2 + 1e-2 * |reference|
(bf16 output; 4e-3 for f16) of the float64 result, and the log-sum-exp
within 1e-3 relative.
"""

import numpy as np
import pytest

from oracle.attention import paged_attention as ref_attention
from pagedkv import B200Backend, CacheConfig
from pagedkv.errors import CacheError
from pagedkv.workloads import Stream

from test_gpu_attention import tables_for

pytestmark = pytest.mark.gpu

TOL = {"bf16": 1e-2, "f16": 4e-3}


def setup_fp8(cuda, kv_heads=2, head_dim=128, layers=2, num_blocks=600, seed=0, shard=(0, 1)):
    """An fp8 pool filled with codes of N(0, 3) values and seeded scales in
    [0.2, 0.5] per (layer, kv head)."""
    import torch

    cfg = CacheConfig(num_blocks, 16, kv_heads, head_dim, layers, 1)
    b = B200Backend(cfg, dtype="fp8_e4m3", shard_rank=shard[0], num_shards=shard[1])
    g = torch.Generator(device=cuda).manual_seed(seed)
    for p in b.planes():
        p.copy_((torch.randn(p.shape, generator=g, device=cuda) * 3).to(torch.float8_e4m3fn))
    st = Stream(1000 + seed)
    ks = st.uniform(layers * kv_heads, 0.2, 0.5).astype(np.float32).reshape(layers, kv_heads)
    vs = st.uniform(layers * kv_heads, 0.2, 0.5).astype(np.float32).reshape(layers, kv_heads)
    b.set_kv_scales(ks, vs)
    return cfg, b, ks, vs


def dequantised(b, ks, vs, head_dim):
    """The cache the attention reads: code * scale, [L][NB][bs][entry] float64,
    for the kv heads this backend holds."""
    h0 = b.elem_offset // head_dim
    out = []
    for p, sc in zip(b.planes(), (ks, vs)):
        x = p.float().cpu().numpy().astype(np.float64)
        L, nb, bs, e = x.shape
        x = x.reshape(L, nb, bs, e // head_dim, head_dim)
        s = sc[:, h0:h0 + e // head_dim].astype(np.float64)
        out.append((x * s[:, None, None, :, None]).reshape(L, nb, bs, e))
    return out


def run(cuda, b, qdt, q_np, tables, ctx, max_ctx, layer, scale=None):
    import torch

    tdt = torch.bfloat16 if qdt == "bf16" else torch.float16
    q = torch.from_numpy(q_np).to(cuda).to(tdt)
    out = torch.full(q.shape, float("nan"), device=cuda, dtype=tdt)
    lse = torch.full(q.shape[:2], float("nan"), device=cuda, dtype=torch.float32)
    b.paged_attention(q, torch.from_numpy(tables).to(cuda),
                      torch.from_numpy(ctx.astype(np.int32)).to(cuda), max_ctx, out, layer,
                      softmax_scale=scale, lse=lse)
    torch.cuda.synchronize()
    return q, out, lse


def check(b, ks, vs, q, out, lse, tables, ctx, layer, scale, tol):
    d = q.shape[2]
    kp, vp = dequantised(b, ks, vs, d)
    want, want_lse = ref_attention(kp, vp, layer, q.double().cpu().numpy(), tables, ctx,
                                   scale if scale is not None else d ** -0.5, d)
    got = out.double().cpu().numpy()
    np.testing.assert_allclose(got, want, rtol=tol, atol=tol)
    gl = lse.cpu().numpy()
    fin = np.isfinite(want_lse)
    assert (np.isneginf(gl) == ~fin).all()
    np.testing.assert_allclose(gl[fin], want_lse[fin], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("qdt", ["bf16", "f16"])
@pytest.mark.parametrize("head_dim", [64, 128, 256])
def test_fp8_decode_attention_matches_oracle(cuda, qdt, head_dim):
    """Many splits and one, empty and one-token contexts, a 7-head group."""
    cfg, b, ks, vs = setup_fp8(cuda, head_dim=head_dim, seed=head_dim)
    st = Stream(head_dim + 1)
    ctx = np.array([1, 15, 16, 17, 31, 33, 64, 100, 255, 0, 700, 2000, 3, 512, 513])
    tables = tables_for(st, cfg, ctx)
    hq = cfg.num_kv_heads * 7
    q_np = st.normal(len(ctx) * hq * head_dim).reshape(len(ctx), hq, head_dim).astype(np.float32)
    q, out, lse = run(cuda, b, qdt, q_np, tables, ctx, int(ctx.max()), 1)
    assert b.device_error() is None
    check(b, ks, vs, q, out, lse, tables, ctx, 1, None, TOL[qdt])


@pytest.mark.parametrize("group", [1, 8, 16])
def test_fp8_gqa_groups_and_single_split(cuda, group):
    cfg, b, ks, vs = setup_fp8(cuda, kv_heads=4, num_blocks=300, seed=group)
    st = Stream(60 + group)
    ctx = st.integers(30, 1, 120)
    tables = tables_for(st, cfg, ctx)
    hq = 4 * group
    q_np = st.normal(30 * hq * 128).reshape(30, hq, 128).astype(np.float32)
    q, out, lse = run(cuda, b, "bf16", q_np, tables, ctx, int(ctx.max()), 0)
    assert b.device_error() is None
    check(b, ks, vs, q, out, lse, tables, ctx, 0, None, TOL["bf16"])


def test_fp8_queries_beyond_f16_range(cuda):
    """bf16 queries up to 3e6 (past f16's 65504): the kernel scales them by a
    power of two into f16 range and folds it back into the softmax scale."""
    cfg, b, ks, vs = setup_fp8(cuda, num_blocks=200, seed=11)
    st = Stream(12)
    ctx = np.array([40, 300, 9])
    tables = tables_for(st, cfg, ctx)
    q_np = (st.normal(3 * 14 * 128) * 1e6).reshape(3, 14, 128).astype(np.float32)
    q, out, lse = run(cuda, b, "bf16", q_np, tables, ctx, 300, 0, scale=1e-6)
    assert b.device_error() is None
    assert np.isfinite(out.float().cpu().numpy()).all()
    check(b, ks, vs, q, out, lse, tables, ctx, 0, 1e-6, TOL["bf16"])


def test_fp8_unused_slots_holding_nan_do_not_leak(cuda):
    """E4M3 NaN codes in the tail of a sequence's last block are never weighted."""
    import torch

    cfg, b, ks, vs = setup_fp8(cuda, num_blocks=64, seed=5)
    st = Stream(5)
    ctx = np.array([17, 40, 8])
    tables = tables_for(st, cfg, ctx)
    kp, vp = b.planes()
    for s, n in enumerate(ctx):
        last = tables[s, (n - 1) // 16]
        for p in (kp, vp):
            p.view(torch.uint8)[:, last, n % 16 or 16:] = 0x7F  # E4M3 NaN
    q_np = st.normal(3 * 14 * 128).reshape(3, 14, 128).astype(np.float32)
    q, out, lse = run(cuda, b, "bf16", q_np, tables, ctx, 48, 0)
    assert torch.isfinite(out).all()
    for p in (kp, vp):
        p.view(torch.uint8)[p.view(torch.uint8) == 0x7F] = 0
    check(b, ks, vs, q, out, lse, tables, ctx, 0, None, TOL["bf16"])


def test_fp8_kv_head_shards_give_the_full_result(cuda):
    """Two shards of 4 kv heads hold their slices of the codes and use their
    heads' scales: each computes its query heads bit for bit as the whole pool."""
    import torch

    cfg = CacheConfig(128, 16, 4, 64, 2, 1)
    full = B200Backend(cfg, dtype="fp8_e4m3")
    shards = [B200Backend(cfg, dtype="fp8_e4m3", shard_rank=r, num_shards=2) for r in range(2)]
    g = torch.Generator(device=cuda).manual_seed(9)
    fk, fv = full.planes()
    fk.copy_((torch.randn(fk.shape, generator=g, device=cuda) * 3).to(torch.float8_e4m3fn))
    fv.copy_((torch.randn(fv.shape, generator=g, device=cuda) * 3).to(torch.float8_e4m3fn))
    st = Stream(10)
    ks = st.uniform(8, 0.2, 0.5).astype(np.float32).reshape(2, 4)
    vs = st.uniform(8, 0.2, 0.5).astype(np.float32).reshape(2, 4)
    full.set_kv_scales(ks, vs)
    for r, sb in enumerate(shards):
        sk, sv = sb.planes()
        sk.view(torch.uint8).copy_(fk.view(torch.uint8)[..., r * 128:(r + 1) * 128])
        sv.view(torch.uint8).copy_(fv.view(torch.uint8)[..., r * 128:(r + 1) * 128])
        sb.set_kv_scales(ks, vs)
    ctx = np.array([100, 7, 600])
    tables = tables_for(st, cfg, ctx)
    q = torch.from_numpy(st.normal(3 * 16 * 64).reshape(3, 16, 64).astype(np.float32)).to(cuda).to(torch.bfloat16)
    dt, dc = torch.from_numpy(tables).to(cuda), torch.from_numpy(ctx.astype(np.int32)).to(cuda)
    out = torch.empty_like(q)
    full.paged_attention(q, dt, dc, 600, out, 1)
    for r, sb in enumerate(shards):
        o = torch.empty((3, 8, 64), device=cuda, dtype=torch.bfloat16)
        sb.paged_attention(q[:, r * 8:(r + 1) * 8], dt, dc, 600, o, 1)
        torch.cuda.synchronize()
        assert torch.equal(o, out[:, r * 8:(r + 1) * 8])


def test_fp8_rejected_query_types(cuda):
    import torch

    t = torch.zeros((1, 4), dtype=torch.int32, device=cuda)
    c = torch.ones(1, dtype=torch.int32, device=cuda)
    fp8 = B200Backend(CacheConfig(8, 16, 1, 128, 1, 1), dtype="fp8_e4m3")
    q32 = torch.zeros((1, 2, 128), device=cuda, dtype=torch.float32)
    with pytest.raises(CacheError):  # f32 queries over an fp8 pool
        fp8.paged_attention(q32, t, c, 16, q32.clone(), 0)
    bf = B200Backend(CacheConfig(8, 16, 1, 128, 1, 2), dtype="bf16")
    q16 = torch.zeros((1, 2, 128), device=cuda, dtype=torch.float16)
    with pytest.raises(CacheError):  # f16 queries over a bf16 pool
        bf.paged_attention(q16, t, c, 16, q16.clone(), 0)
