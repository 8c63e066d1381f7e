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
