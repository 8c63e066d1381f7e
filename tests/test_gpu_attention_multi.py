"""Paged attention with several query tokens per sequence (the verification
step of speculative decoding) against the float64 oracle: token i of a
sequence with ctx cached tokens sits at position ctx - q_len + i and attends
keys 0 .. that position.

Tolerances as for decode attention: bf16 1e-2, f16 4e-3 (absolute plus
relative to the float64 result), the log-sum-exp within 1e-3; an fp8 pool
is compared with the oracle run on its dequantised contents.
"""

import numpy as np
import pytest

from oracle.attention import paged_attention as ref_attention
from pagedkv import B200Backend, CacheConfig
from pagedkv.errors import CacheError, ShapeMismatch
from pagedkv.workloads import Stream
from tests.test_gpu_attention import TOL, tables_for
from tests.test_gpu_attention import setup as setup_pool
from tests.test_gpu_attention_fp8 import dequantised, setup_fp8

pytestmark = pytest.mark.gpu


def run_multi(cuda, b, tdt, q_np, tables, ctx, max_ctx, layer, q_len, scale=None):
    import torch

    q = torch.from_numpy(q_np).to(cuda).to(tdt)
    out = torch.full(q.shape, float("nan"), device=cuda, dtype=tdt)
    lse = torch.full(q.shape[:2], float("nan"), device=cuda, dtype=torch.float32)
    b.paged_attention(q, torch.from_numpy(tables).to(cuda),
                      torch.from_numpy(ctx.astype(np.int32)).to(cuda), max_ctx, out, layer,
                      softmax_scale=scale, lse=lse, q_len=q_len)
    torch.cuda.synchronize()
    return q, out, lse


def check_multi(kp, vp, q, out, lse, tables, ctx, layer, q_len, scale, tol):
    d = q.shape[2]
    want, want_lse = ref_attention(kp, vp, layer, q.double().cpu().numpy(), tables, ctx,
                                   scale if scale is not None else d ** -0.5, d, q_len=q_len)
    np.testing.assert_allclose(out.double().cpu().numpy(), want, rtol=tol, atol=tol)
    gl = lse.cpu().numpy()
    assert np.isfinite(want_lse).all()
    np.testing.assert_allclose(gl, want_lse, rtol=1e-3, atol=1e-3)


# Contexts where the query tokens sit inside one block, straddle a block
# boundary, fill the first block exactly, and (2050, 4097 with the 128-block
# splits of a long context) straddle a split boundary.
CTX = [16, 17, 18, 19, 31, 32, 33, 100, 255, 2050, 4097, 700]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("q_len,group", [(2, 4), (4, 2), (3, 5), (16, 1), (8, 2)])
def test_multi_query_matches_oracle(cuda, dtype, head_dim, q_len, group):
    cfg, b, tdt = setup_pool(cuda, dtype=dtype, head_dim=head_dim, num_blocks=900)
    st = Stream(head_dim * 100 + q_len * 10 + group)
    ctx = np.array([max(c, q_len) for c in CTX] + [q_len])
    tables = tables_for(st, cfg, ctx)
    hq = cfg.num_kv_heads * group
    q_np = st.normal(len(ctx) * q_len * hq * head_dim).reshape(len(ctx) * q_len, hq,
                                                               head_dim).astype(np.float32)
    q, out, lse = run_multi(cuda, b, tdt, q_np, tables, ctx, int(ctx.max()), 1, q_len)
    assert b.device_error() is None
    kp, vp = (p.float().cpu().numpy() for p in b.planes())
    check_multi(kp, vp, q, out, lse, tables, ctx, 1, q_len, None, TOL[dtype])


@pytest.mark.parametrize("head_dim", [64, 128, 256])
@pytest.mark.parametrize("q_len,group", [(2, 4), (4, 4), (5, 3)])
def test_fp8_multi_query_matches_oracle(cuda, head_dim, q_len, group):
    import torch

    cfg, b, ks, vs = setup_fp8(cuda, head_dim=head_dim, num_blocks=900, seed=head_dim + q_len)
    st = Stream(7 * head_dim + q_len)
    ctx = np.array([max(c, q_len) for c in CTX])
    tables = tables_for(st, cfg, ctx)
    hq = cfg.num_kv_heads * group
    q_np = st.normal(len(ctx) * q_len * hq * head_dim).reshape(len(ctx) * q_len, hq,
                                                               head_dim).astype(np.float32)
    q, out, lse = run_multi(cuda, b, torch.bfloat16, q_np, tables, ctx, int(ctx.max()), 0, q_len)
    assert b.device_error() is None
    kp, vp = dequantised(b, ks, vs, head_dim)
    check_multi(kp, vp, q, out, lse, tables, ctx, 0, q_len, None, TOL["bf16"])


@pytest.mark.parametrize("q_len,group", [(3, 5), (2, 4)])
def test_fp8_multi_query_with_f16_queries(cuda, q_len, group):
    """f16 queries over an fp8 pool (held to the f16 tolerance), the 16-row
    and the 8-row form."""
    import torch

    cfg, b, ks, vs = setup_fp8(cuda, head_dim=128, num_blocks=900, seed=40 + q_len)
    st = Stream(900 + q_len)
    ctx = np.array([max(c, q_len) for c in CTX])
    tables = tables_for(st, cfg, ctx)
    hq = cfg.num_kv_heads * group
    q_np = st.normal(len(ctx) * q_len * hq * 128).reshape(len(ctx) * q_len, hq,
                                                          128).astype(np.float32)
    q, out, lse = run_multi(cuda, b, torch.float16, q_np, tables, ctx, int(ctx.max()), 1, q_len)
    assert b.device_error() is None
    kp, vp = dequantised(b, ks, vs, 128)
    check_multi(kp, vp, q, out, lse, tables, ctx, 1, q_len, None, TOL["f16"])


def test_one_token_through_the_multi_entry_is_decode(cuda):
    """q_len 1 on pkv_paged_attention_multi_dev gives decode's bits."""
    import ctypes as C

    import torch
    from pagedkv import _lib

    cfg, b, tdt = setup_pool(cuda, num_blocks=400)
    st = Stream(21)
    ctx = np.array([1, 16, 17, 300, 2100, 45])
    tables = tables_for(st, cfg, ctx)
    q_np = st.normal(6 * 8 * 128).reshape(6, 8, 128).astype(np.float32)
    q, out, lse = run_multi(cuda, b, tdt, q_np, tables, ctx, 2100, 0, 1)
    out2 = torch.empty_like(out)
    lse2 = torch.empty_like(lse)
    dt = torch.from_numpy(tables).to(cuda)
    dc = torch.from_numpy(ctx.astype(np.int32)).to(cuda)
    rc = _lib.lib.pkv_paged_attention_multi_dev(
        b._h, 0, C.c_void_p(q.data_ptr()), b.dtype_tag, 1, 0, 6, 8, C.c_void_p(dt.data_ptr()),
        tables.shape[1], C.c_void_p(dc.data_ptr()), 2100, 128 ** -0.5, C.c_void_p(out2.data_ptr()),
        C.c_void_p(lse2.data_ptr()), None)
    assert rc == 0
    torch.cuda.synchronize()
    assert torch.equal(out, out2) and torch.equal(lse, lse2)


def test_masked_tail_keys_holding_nan_do_not_leak(cuda):
    """Slots past a sequence's end hold NaN; the keys a query token must not
    see (its successors among the q_len tokens) are finite but never weighted."""
    import torch

    cfg, b, tdt = setup_pool(cuda, num_blocks=64)
    st = Stream(6)
    q_len = 4
    ctx = np.array([17, 40, 8, 4])
    tables = tables_for(st, cfg, ctx)
    kp, vp = b.planes()
    for s, n in enumerate(ctx):
        last = tables[s, (n - 1) // 16]
        kp[:, last, n % 16 or 16:] = float("nan")
        vp[:, last, n % 16 or 16:] = float("nan")
    q_np = st.normal(4 * q_len * 6 * 128).reshape(4 * q_len, 6, 128).astype(np.float32)
    q, out, lse = run_multi(cuda, b, tdt, q_np, tables, ctx, 48, 0, q_len)
    assert torch.isfinite(out).all()
    kp2, vp2 = kp.float().cpu().numpy(), vp.float().cpu().numpy()
    kp2[np.isnan(kp2)] = 0
    vp2[np.isnan(vp2)] = 0
    check_multi(kp2, vp2, q, out, lse, tables, ctx, 0, q_len, None, TOL["bf16"])


def test_context_shorter_than_the_query_tokens_is_recorded(cuda):
    import torch

    cfg, b, tdt = setup_pool(cuda, num_blocks=32)
    st = Stream(8)
    q_len = 4
    ctx = np.array([20, 3, 9])
    tables = tables_for(st, cfg, ctx)
    q_np = st.normal(3 * q_len * 2 * 128).reshape(3 * q_len, 2, 128).astype(np.float32)
    q, out, lse = run_multi(cuda, b, tdt, q_np, tables, ctx, 32, 0, q_len)
    err = b.device_error()
    assert err is not None and isinstance(err[0], ShapeMismatch) and err[1] == 1
    assert (out[q_len:2 * q_len] == 0).all() and torch.isneginf(lse[q_len:2 * q_len]).all()
    kp, vp = (p.float().cpu().numpy() for p in b.planes())
    keep = np.r_[0:q_len, 2 * q_len:3 * q_len]
    check_multi(kp, vp, q[keep], out[keep], lse[keep], tables[[0, 2]], ctx[[0, 2]], 0, q_len,
                None, TOL["bf16"])


def test_multi_query_rejections(cuda):
    import torch

    ok = B200Backend(CacheConfig(8, 16, 1, 128, 1, 2), dtype="bf16")
    t = torch.zeros((2, 4), dtype=torch.int32, device=cuda)
    c = torch.full((2,), 8, dtype=torch.int32, device=cuda)
    q = torch.zeros((2 * 3, 6, 128), device=cuda, dtype=torch.bfloat16)
    with pytest.raises(CacheError):  # q_len * group = 18 > 16
        ok.paged_attention(q, t, c, 16, q.clone(), 0, q_len=3)
    with pytest.raises(ValueError):  # rows not a multiple of q_len
        ok.paged_attention(q[:5], t, c, 16, q[:5].clone(), 0, q_len=2)
