"""The float64 attention oracle (oracle/attention.py) against an independent
dense formulation on the CPU: torch's scaled_dot_product_attention over the
gathered K/V rows, kv heads repeated for the query-head groups."""

import numpy as np
import pytest
import torch

from oracle.attention import paged_attention
from pagedkv.workloads import Stream


@pytest.mark.parametrize("group", [1, 4, 7])
def test_oracle_matches_dense_sdpa(group):
    st = Stream(group)
    L, nb, bs, kvh, d = 2, 40, 16, 2, 16
    k = st.normal(L * nb * bs * kvh * d).reshape(L, nb, bs, kvh * d)
    v = st.normal(L * nb * bs * kvh * d).reshape(L, nb, bs, kvh * d)
    s_n, hq = 5, kvh * group
    ctx = np.array([1, 16, 17, 50, 0])
    tables = st.permutation(nb)[: s_n * 8].reshape(s_n, 8)
    q = st.normal(s_n * hq * d).reshape(s_n, hq, d)
    out, lse = paged_attention(k, v, 1, q, tables, ctx, 0.3, d)
    for s in range(s_n):
        n = int(ctx[s])
        if n == 0:
            assert (out[s] == 0).all() and np.isneginf(lse[s]).all()
            continue
        t = np.arange(n)
        kk = torch.from_numpy(k[1, tables[s][t // bs], t % bs].reshape(n, kvh, d)).transpose(0, 1)
        vv = torch.from_numpy(v[1, tables[s][t // bs], t % bs].reshape(n, kvh, d)).transpose(0, 1)
        kk = kk.repeat_interleave(group, 0)
        vv = vv.repeat_interleave(group, 0)
        qq = torch.from_numpy(q[s]).unsqueeze(1)  # [hq][1][d]
        want = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, scale=0.3)[:, 0]
        np.testing.assert_allclose(out[s], want.numpy(), rtol=1e-12, atol=1e-12)
        sc = torch.einsum("hd,htd->ht", qq[:, 0], kk) * 0.3
        np.testing.assert_allclose(lse[s], torch.logsumexp(sc, -1).numpy(), rtol=1e-12)


@pytest.mark.parametrize("q_len", [2, 4, 16])
def test_multi_query_oracle_matches_causal_sdpa(q_len):
    """q_len query tokens per sequence, the last q_len tokens of its context:
    torch SDPA with the causal mask of those positions over all keys."""
    st = Stream(100 + q_len)
    L, nb, bs, kvh, d = 1, 40, 16, 2, 16
    group = 1 if q_len == 16 else 2  # q_len x group up to the kernel's 16 rows
    k = st.normal(L * nb * bs * kvh * d).reshape(L, nb, bs, kvh * d)
    v = st.normal(L * nb * bs * kvh * d).reshape(L, nb, bs, kvh * d)
    s_n, hq = 3, kvh * group
    ctx = np.array([q_len, 37, 64])
    tables = st.permutation(nb)[: s_n * 8].reshape(s_n, 8)
    q = st.normal(s_n * q_len * hq * d).reshape(s_n * q_len, hq, d)
    out, lse = paged_attention(k, v, 0, q, tables, ctx, 0.25, d, q_len=q_len)
    for s in range(s_n):
        n = int(ctx[s])
        t = np.arange(n)
        kk = torch.from_numpy(k[0, tables[s][t // bs], t % bs].reshape(n, kvh, d)).transpose(0, 1)
        vv = torch.from_numpy(v[0, tables[s][t // bs], t % bs].reshape(n, kvh, d)).transpose(0, 1)
        kk = kk.repeat_interleave(group, 0)
        vv = vv.repeat_interleave(group, 0)
        qq = torch.from_numpy(q[s * q_len:(s + 1) * q_len]).transpose(0, 1)  # [hq][q_len][d]
        pos = n - q_len + torch.arange(q_len)
        mask = torch.arange(n)[None, :] <= pos[:, None]  # [q_len][n]
        want = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask, scale=0.25)
        np.testing.assert_allclose(out[s * q_len:(s + 1) * q_len], want.transpose(0, 1).numpy(),
                                   rtol=1e-12, atol=1e-12)
