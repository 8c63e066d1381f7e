"""Seeded cases for the golden fixtures of the reference's own CUDA kernels.

Each case is a sequence of reshape_and_cache batches (distinct slots within
a batch, as the reference kernel needs), copy_blocks lists (no chains) and
zero_block calls on an f32 pool (the only type the reference kernels take).
Both the fixture generator (make_ref_golden.py, on a GPU) and the CPU test
(tests/test_golden_ref.py) build the operations from here.
"""

from __future__ import annotations

import numpy as np

from pagedkv import CacheConfig
from pagedkv.workloads import Stream, config1

CASES = {
    # name: (num_blocks, block_size, heads, head_dim, layers, seed, batches)
    "config1": None,
    "odd_geometry": (40, 8, 3, 20, 3, 11, 6),
    "many_layers": (24, 16, 2, 64, 12, 12, 5),
    "one_slot_blocks": (64, 1, 4, 32, 2, 13, 4),
}


def ops(name: str):
    """(CacheConfig, [op]) where op is ("write", layer, slots int64, k [n][E] f32, v),
    ("copy", pairs int64 [P][2]) or ("zero", block)."""
    if name == "config1":
        w = config1(seed=0)
        out = [("write", l, w.slots.astype(np.int64), w.k[l], w.v[l]) for l in range(w.cfg.num_layers)]
        out.append(("copy", w.pairs.astype(np.int64)))
        out += [("zero", int(z)) for z in w.zero]
        return w.cfg, out
    nb, bs, h, d, L, seed, batches = CASES[name]
    cfg = CacheConfig(nb, bs, h, d, L, 4)
    e = h * d
    st = Stream(seed)
    out = []
    for b in range(batches):
        for l in range(L):
            n = int(st.integers(1, 1, nb * bs // 2)[0])
            slots = st.permutation(nb * bs)[:n].astype(np.int64)
            k = st.uniform(n * e, -1.0, 1.0).astype(np.float32).reshape(n, e)
            v = st.uniform(n * e, -1.0, 1.0).astype(np.float32).reshape(n, e)
            out.append(("write", l, slots, k, v))
        ids = st.permutation(nb)
        p = int(st.integers(1, 1, nb // 3)[0])
        out.append(("copy", np.stack([ids[:p], ids[p:2 * p]], 1).astype(np.int64)))
        out.append(("zero", int(ids[2 * p])))
    return cfg, out


def entry_hashes(k_plane: np.ndarray, v_plane: np.ndarray, cfg) -> np.ndarray:
    """uint64 [2][L][num_blocks][block_size]: a splitmix64-based hash of each
    entry's f32 bit patterns, K plane then V plane."""
    e = cfg.num_kv_heads * cfg.head_dim
    out = []
    for p in (k_plane, v_plane):
        bits = np.ascontiguousarray(p, dtype=np.float32).reshape(-1, e).view(np.uint32).astype(np.uint64)
        with np.errstate(over="ignore"):
            z = bits + np.arange(e, dtype=np.uint64)[None, :] * np.uint64(0x9E3779B97F4A7C15)
            z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
            z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
            z = z ^ (z >> np.uint64(31))
            out.append(z.sum(axis=1, dtype=np.uint64).reshape(cfg.num_layers, cfg.num_blocks,
                                                              cfg.block_size))
    return np.stack(out)
