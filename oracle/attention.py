"""TEST INFRASTRUCTURE ONLY -- float64 restatement of decode attention over
the paged pool, the checker of pkv_paged_attention_dev.

The reference has no attention kernel: its trait leaves `paged_attention`
for later (crates/paged-kv-core/src/backend.rs:18-22) and its README lists it
as the next kernel. This restates plain softmax attention over the pool's
layout (crates/paged-kv-core/src/cpu.rs:13-21): token t of sequence s is
slot t % block_size of block table[s][t // block_size]; query head h reads
kv head h // (num_q_heads // num_kv_heads).
"""

from __future__ import annotations

import numpy as np


def paged_attention(k_plane, v_plane, layer: int, q, tables, ctx, scale: float, head_dim: int,
                    q_len: int = 1):
    """k_plane, v_plane: [L][num_blocks][block_size][entry] (this backend's
    heads); q: [S][Hq][D], or [S * q_len][Hq][D] with q_len query tokens per
    sequence: query i of sequence s sits at position ctx[s] - q_len + i and
    attends to the keys at positions 0 .. ctx[s] - q_len + i (causal over the
    sequence's last q_len tokens). Returns (out f64 shaped as q, lse [rows][Hq]
    f64, natural log, -inf for an empty context)."""
    if q_len > 1:
        q = np.asarray(q, dtype=np.float64)
        out = np.zeros(q.shape)
        lse = np.full(q.shape[:2], -np.inf)
        for i in range(q_len):
            lim = np.maximum(np.asarray(ctx) - q_len + i + 1, 0)
            o, l = paged_attention(k_plane, v_plane, layer, q[i::q_len], tables, lim, scale,
                                   head_dim)
            out[i::q_len], lse[i::q_len] = o, l
        return out, lse
    k_plane = np.asarray(k_plane)
    bs = k_plane.shape[2]
    kvh = k_plane.shape[3] // head_dim
    q = np.asarray(q, dtype=np.float64)
    s_n, hq, d = q.shape
    group = hq // kvh
    out = np.zeros((s_n, hq, d))
    lse = np.full((s_n, hq), -np.inf)
    for s in range(s_n):
        n = int(ctx[s])
        if n == 0:
            continue
        t = np.arange(n)
        blocks = np.asarray(tables[s])[t // bs]
        kk = k_plane[layer, blocks, t % bs].astype(np.float64).reshape(n, kvh, d)
        vv = np.asarray(v_plane)[layer, blocks, t % bs].astype(np.float64).reshape(n, kvh, d)
        for h in range(hq):
            sc = kk[:, h // group] @ q[s, h] * scale
            m = sc.max()
            p = np.exp(sc - m)
            l = p.sum()
            out[s, h] = (p @ vv[:, h // group]) / l
            lse[s, h] = m + np.log(l)
    return out, lse
